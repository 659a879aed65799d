// k_gemv.cu — skinny GEMV kernels of the decode step (M = streams x beams rows).
//
// Replaces the reference's M=1 matrix-vector paths:
//   Linear.forward (nn/Linear.java:23-26) -> Tensor.matmul (tensor/Tensor.java:403-422)
//   -> matmulVec (:383-398) -> VectorSimdOps.matmulVecAccumulate (java26 VectorSimdOps.java:114-133),
// with the LayerNorm before it (nn/LayerNorm.java:28-30, Tensor.java:592-619), the GELU
// after mlp.0 (Tensor.java:524-538) and the residual adds (ResidualAttentionBlock.java:48-59)
// fused into prologue / epilogue, and the vocabulary projection
// (WhisperDecoder.java:102-103 -> Tensor.matmulTransB, Tensor.java:316-340) fused with the
// logit processors (WhisperDecoder.java:450-564) and the reductions that argmax / log-softmax /
// top-k need (:566-574, :397-431, :614-626).
//
// Design (HBM-bound, M small): weights stay in their GGML (N, K) row layout; a warp owns R
// rows and its lanes walk K in 16-byte chunks (8 f16 or 16 int8), loading each weight byte
// exactly once with 128-bit non-allocating loads and dequantising in registers.  The M
// activation rows sit in shared memory as f32 (LayerNorm applied on the way in), every
// weight chunk is reused for all M rows, and the R x M partial sums are reduced across the
// warp with a butterfly that ends with one finished sum per lane.  Under programmatic
// dependent launch each block first asks L2 to prefetch its weight rows (bulk prefetch),
// then waits for the previous kernel; the weight stream therefore overlaps the tail of the
// kernel before it.
#include <float.h>

#include "w4j_internal.cuh"

namespace w4j {

// ---------------------------------------------------------------------------
// helpers
// ---------------------------------------------------------------------------

// Reduce NV per-lane partial sums over the warp.  Afterwards lane l holds the full sum of
// value index (l >> (5 - log2 NV)); the lanes with (l & (32/NV - 1)) == 0 own distinct indices.
template <int NV>
__device__ __forceinline__ float warp_reduce_multi(float (&v)[NV], int lane) {
    static_assert(NV >= 1 && NV <= 32 && (NV & (NV - 1)) == 0, "NV must be a power of two <= 32");
#pragma unroll
    for (int s = 0; s < 5; ++s) {
        const int o = 16 >> s;
        const int n = NV >> s;
        if (n >= 2) {
            const bool upper = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < NV / 2; ++i) {
                if (i < n / 2) {
                    const float send = upper ? v[i] : v[i + n / 2];
                    const float keep = upper ? v[i + n / 2] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
        }
    }
    return v[0];
}

template <int NV>
__device__ __forceinline__ int reduced_index(int lane) {
    constexpr int lg = NV >= 32 ? 5 : NV >= 16 ? 4 : NV >= 8 ? 3 : NV >= 4 ? 2 : NV >= 2 ? 1 : 0;
    return lane >> (5 - lg);
}
template <int NV>
__device__ __forceinline__ bool reduced_owner(int lane) {
    return (lane & ((32 / NV) - 1)) == 0;
}

__device__ __forceinline__ float row_value(const DMat &m, int row, int k) {
    if (m.type == WT_F16) return __half2float(m.h[(size_t)row * m.K + k]);
    const float s = __half2float(m.s[(size_t)row * (m.K / 32) + k / 32]);
    return (float)m.q[(size_t)row * m.K + k] * s;
}

// Fill act_s[mm][k] (mm < MT) for rows m0.. of the pass: plain copy, LayerNorm of x, or
// token + positional embedding then LayerNorm.  8 warps, one row per warp at a time.
template <int MT>
__device__ void load_activations(const GemvArgs &a, int m0, int K, float *act_s, int warp, int lane) {
    for (int mm = warp; mm < MT; mm += kGemvThreads / 32) {
        const int m = m0 + mm;
        float *dst = act_s + (size_t)mm * K;
        if (m >= a.M) {
            for (int k = lane; k < K; k += 32) dst[k] = 0.f;
            continue;
        }
        if (a.in_mode == IN_ACT) {
            const float4 *src = reinterpret_cast<const float4 *>(a.act + (size_t)m * K);
            for (int k4 = lane; k4 < K / 4; k4 += 32) reinterpret_cast<float4 *>(dst)[k4] = src[k4];
            continue;
        }
        // residual stream row -> shared (embedding first when asked)
        if (a.in_mode == IN_EMBED_LN) {
            const int tok = a.tok[m];
            const int p = a.pos[m];
            for (int k = lane; k < K; k += 32) {
                const float v = row_value(a.E, tok, k) + a.pos_emb[(size_t)p * K + k];
                dst[k] = v;
                if (blockIdx.x == 0 && a.x_out) a.x_out[(size_t)m * K + k] = v;
            }
        } else {
            const float *src = a.act + (size_t)m * K;
            for (int k = lane; k < K; k += 32) dst[k] = src[k];
        }
        __syncwarp();
        // Tensor.layerNorm (Tensor.java:592-619): two-pass mean / variance, eps 1e-5,
        // invStd = 1 / sqrt(var / n + eps), y = (x - mean) * invStd * g + b.
        float s = 0.f;
        for (int k = lane; k < K; k += 32) s += dst[k];
        const float mean = warp_sum(s) / (float)K;
        float v2 = 0.f;
        for (int k = lane; k < K; k += 32) {
            const float dd = dst[k] - mean;
            v2 += dd * dd;
        }
        const float var = warp_sum(v2);
        const float inv_std = 1.0f / sqrtf(var / (float)K + 1e-5f);
        __syncwarp();
        for (int k = lane; k < K; k += 32) dst[k] = (dst[k] - mean) * inv_std * a.ln_g[k] + a.ln_b[k];
    }
}

// acc[r][mm] += W[row r, chunk c] . act[mm][chunk c]
template <int MT, int R, int WT>
struct Chunk {
    static constexpr int CE = WT == WT_F16 ? 8 : 16;  // elements per 16-byte chunk
};

template <int MT, int R>
__device__ __forceinline__ void fma_chunk_f16(const uint4 (&w)[R], const float *act_s, int K, int k0,
                                              float (&acc)[R * MT]) {
    float wf[R][8];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const __half2 *h = reinterpret_cast<const __half2 *>(&w[r]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(h[j]);
            wf[r][2 * j] = f.x;
            wf[r][2 * j + 1] = f.y;
        }
    }
#pragma unroll
    for (int mm = 0; mm < MT; ++mm) {
        const float4 a0 = *reinterpret_cast<const float4 *>(act_s + (size_t)mm * K + k0);
        const float4 a1 = *reinterpret_cast<const float4 *>(act_s + (size_t)mm * K + k0 + 4);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            float t = acc[r * MT + mm];
            t = fmaf(wf[r][0], a0.x, t);
            t = fmaf(wf[r][1], a0.y, t);
            t = fmaf(wf[r][2], a0.z, t);
            t = fmaf(wf[r][3], a0.w, t);
            t = fmaf(wf[r][4], a1.x, t);
            t = fmaf(wf[r][5], a1.y, t);
            t = fmaf(wf[r][6], a1.z, t);
            t = fmaf(wf[r][7], a1.w, t);
            acc[r * MT + mm] = t;
        }
    }
}

template <int MT, int R>
__device__ __forceinline__ void fma_chunk_q8(const uint4 (&w)[R], const float (&sc)[R], const float *act_s,
                                             int K, int k0, float (&acc)[R * MT]) {
    float wf[R][16];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const uint32_t u[4] = {w[r].x, w[r].y, w[r].z, w[r].w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int b = 0; b < 4; ++b) wf[r][4 * j + b] = (float)(int8_t)((u[j] >> (8 * b)) & 0xffu);
    }
#pragma unroll
    for (int mm = 0; mm < MT; ++mm) {
        float part[R];
#pragma unroll
        for (int r = 0; r < R; ++r) part[r] = 0.f;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
            const float4 a = *reinterpret_cast<const float4 *>(act_s + (size_t)mm * K + k0 + 4 * q4);
#pragma unroll
            for (int r = 0; r < R; ++r) {
                float t = part[r];
                t = fmaf(wf[r][4 * q4 + 0], a.x, t);
                t = fmaf(wf[r][4 * q4 + 1], a.y, t);
                t = fmaf(wf[r][4 * q4 + 2], a.z, t);
                t = fmaf(wf[r][4 * q4 + 3], a.w, t);
                part[r] = t;
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r * MT + mm] = fmaf(part[r], sc[r], acc[r * MT + mm]);
    }
}

// Dot products of rows [row0, row0+R) with the MT activation rows; result reduced over the warp.
template <int MT, int R, int WT>
__device__ __forceinline__ void warp_rows(const DMat &W, int row0, const float *act_s, float (&acc)[R * MT],
                                          int lane) {
    constexpr int CE = WT == WT_F16 ? 8 : 16;
    const int K = W.K;
    const int nchunk = K / CE;
#pragma unroll
    for (int i = 0; i < R * MT; ++i) acc[i] = 0.f;
    bool ok[R];
#pragma unroll
    for (int r = 0; r < R; ++r) ok[r] = row0 + r < W.N;
    constexpr int U = (R * 2 >= 8) ? 2 : 4;  // chunks per batch: keep ~8 loads in flight per lane
    for (int c0 = lane; c0 < nchunk; c0 += 32 * U) {
        uint4 w[U][R];
        float sc[U][R];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = c0 + 32 * u;
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (ok[r] && c < nchunk) {
                    if (WT == WT_F16) {
                        w[u][r] = ld_nc_v4(W.h + (size_t)(row0 + r) * K + (size_t)c * CE);
                        sc[u][r] = 0.f;
                    } else {
                        w[u][r] = ld_nc_v4(W.q + (size_t)(row0 + r) * K + (size_t)c * CE);
                        sc[u][r] = __half2float(W.s[(size_t)(row0 + r) * (K / 32) + (c * CE) / 32]);
                    }
                } else {
                    w[u][r] = make_uint4(0, 0, 0, 0);
                    sc[u][r] = 0.f;
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = c0 + 32 * u;
            if (c < nchunk) {
                if (WT == WT_F16)
                    fma_chunk_f16<MT, R>(w[u], act_s, K, c * CE, acc);
                else
                    fma_chunk_q8<MT, R>(w[u], sc[u], act_s, K, c * CE, acc);
            }
        }
    }
}

__device__ __forceinline__ void prefetch_rows(const DMat &W, int row0, int rows) {
    if (row0 >= W.N) return;
    rows = min(rows, W.N - row0);
    if (W.type == WT_F16) {
        prefetch_l2(W.h + (size_t)row0 * W.K, (unsigned)((size_t)rows * W.K * 2));
    } else {
        prefetch_l2(W.q + (size_t)row0 * W.K, (unsigned)((size_t)rows * W.K));
        const size_t sb = (size_t)rows * (W.K / 32) * 2;
        if (sb % 16 == 0 && (((size_t)row0 * (W.K / 32) * 2) % 16) == 0)
            prefetch_l2(W.s + (size_t)row0 * (W.K / 32), (unsigned)sb);
    }
}

// ---------------------------------------------------------------------------
// GEMV kernel
// ---------------------------------------------------------------------------
template <int MT, int R, int WT>
__global__ void __launch_bounds__(kGemvThreads) k_gemv(GemvArgs a) {
    extern __shared__ float4 smem_f4[];
    float *act_s = reinterpret_cast<float *>(smem_f4);
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int N = a.W.N, K = a.W.K;
    const int n_groups = (N + R - 1) / R;
    const int total_warps = gridDim.x * (kGemvThreads / 32);
    const int gw = blockIdx.x * (kGemvThreads / 32) + warp;
    // weights do not depend on the previous kernel: start their trip to L2 now
    if (lane == 0)
        for (int g = gw; g < n_groups; g += total_warps) prefetch_rows(a.W, g * R, R);
    pdl_wait();

    for (int m0 = 0; m0 < a.M; m0 += MT) {
        load_activations<MT>(a, m0, K, act_s, warp, lane);
        __syncthreads();
        for (int g = gw; g < n_groups; g += total_warps) {
            float acc[R * MT];
            warp_rows<MT, R, WT>(a.W, g * R, act_s, acc, lane);
            const float v = warp_reduce_multi<R * MT>(acc, lane);
            if (!reduced_owner<R * MT>(lane)) continue;
            const int idx = reduced_index<R * MT>(lane);
            const int r = idx / MT, mm = idx % MT;
            const int n = g * R + r, m = m0 + mm;
            if (n >= N || m >= a.M) continue;
            if (a.active && !a.active[m]) continue;
            const float val = v + (a.bias ? a.bias[n] : 0.f);
            switch (a.out_mode) {
                case OUT_STORE:
                    a.y[(size_t)m * N + n] = val;
                    break;
                case OUT_GELU:  // Tensor.geluInPlace: table lookup at the f16 rounding of x
                    a.y[(size_t)m * N + n] = a.gelu_lut[__half_as_ushort(__float2half_rn(val))];
                    break;
                case OUT_RESIDUAL:
                    a.y[(size_t)m * N + n] += val;
                    break;
                case OUT_QKV: {
                    const int dm = N / 3;
                    const int part = n / dm, c = n - part * dm;
                    if (part == 0) {
                        a.y[(size_t)m * dm + c] = val;
                    } else {
                        const int head = c / kHeadDim, dd = c % kHeadDim;
                        const size_t row = (((size_t)a.seq_slot[m] * a.n_layer + a.layer) * a.n_head + head) *
                                               (size_t)a.n_ctx + (size_t)a.pos[m];
                        __half *dst = part == 1 ? a.kcache : a.vcache;
                        dst[row * kHeadDim + dd] = __float2half_rn(val);
                    }
                    break;
                }
            }
        }
        __syncthreads();
    }
}

template <int MT, int R, int WT>
static cudaError_t launch_gemv_t(const GemvArgs &a, cudaStream_t s, bool pdl, int sm_count) {
    const int n_groups = (a.W.N + R - 1) / R;
    int blocks = (n_groups + 7) / 8;
    blocks = blocks < 4 * sm_count ? blocks : 4 * sm_count;
    if (blocks < 1) blocks = 1;
    const size_t smem = (size_t)MT * a.W.K * sizeof(float);
    auto kern = k_gemv<MT, R, WT>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

static int g_sm_count = 0;
static int sm_count() {
    if (!g_sm_count) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev);
        if (g_sm_count <= 0) g_sm_count = 148;
    }
    return g_sm_count;
}

// Rows of activations kept in shared memory per pass: bounded by 96 KB of f32.
static int pick_mt(int M, int K) {
    const int cap = 24576 / K;  // MT * K * 4 <= 96 KB
    int mt = 1;
    while (mt < M && mt * 2 <= cap && mt < 16) mt *= 2;
    return mt;
}

template <int WT>
static cudaError_t dispatch_gemv(const GemvArgs &a, cudaStream_t s, bool pdl) {
    const int mt = pick_mt(a.M, a.W.K);
    const int sms = sm_count();
    switch (mt) {
        case 1: return launch_gemv_t<1, 4, WT>(a, s, pdl, sms);
        case 2: return launch_gemv_t<2, 4, WT>(a, s, pdl, sms);
        case 4: return launch_gemv_t<4, 4, WT>(a, s, pdl, sms);
        case 8: return launch_gemv_t<8, 2, WT>(a, s, pdl, sms);
        default: return launch_gemv_t<16, 2, WT>(a, s, pdl, sms);
    }
}

cudaError_t launch_gemv(const GemvArgs &a, cudaStream_t s, bool pdl) {
    if (a.M <= 0) return cudaSuccess;
    if (a.W.type == WT_F16) return dispatch_gemv<WT_F16>(a, s, pdl);
    if (a.W.type == WT_Q8) return dispatch_gemv<WT_Q8>(a, s, pdl);
    return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------
// vocabulary logits + logit processors + block partials
// ---------------------------------------------------------------------------

__device__ __forceinline__ bool better(float v1, int i1, float v2, int i2) {
    return v1 > v2 || (v1 == v2 && i1 < i2);
}

// LayerNorm of the residual rows into act_s (shared by all blocks, recomputed per block).
template <int MT>
__device__ void load_ln_rows(const LogitsArgs &a, int m0, float *act_s, int warp, int lane) {
    GemvArgs g;
    g.M = a.M;
    g.in_mode = IN_LN;
    g.act = a.x;
    g.ln_g = a.ln_g;
    g.ln_b = a.ln_b;
    load_activations<MT>(g, m0, a.d, act_s, warp, lane);
}

template <int MT, int R, int WT>
__global__ void __launch_bounds__(kGemvThreads) k_logits(LogitsArgs a) {
    extern __shared__ float4 smem_f4[];
    float *act_s = reinterpret_cast<float *>(smem_f4);
    const int P = gridDim.x;
    const int lo = (int)(((long long)blockIdx.x * a.V) / P);
    const int hi = (int)(((long long)(blockIdx.x + 1) * a.V) / P);
    const int CH = (a.V + P - 1) / P + 1;
    float *tile = act_s + (size_t)MT * a.d;  // [MT][CH]
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // the vocabulary matrix is larger than L2 for big models: warm only the head of this block's rows
    if (threadIdx.x == 0) {
        const int row_bytes = a.E.type == WT_F16 ? a.d * 2 : a.d;
        const int rows = min(hi - lo, max(4, (32 * 1024 / row_bytes) & ~3));
        prefetch_rows(a.E, lo, rows);
    }
    pdl_wait();

    for (int m0 = 0; m0 < a.M; m0 += MT) {
        load_ln_rows<MT>(a, m0, act_s, warp, lane);
        __syncthreads();
        const int n_groups = (hi - lo + R - 1) / R;
        for (int g = warp; g < n_groups; g += kGemvThreads / 32) {
            float acc[R * MT];
            const int row0 = lo + g * R;
            DMat E = a.E;
            E.N = hi;  // rows beyond this block's range are left to the next block
            warp_rows<MT, R, WT>(E, row0, act_s, acc, lane);
            const float v = warp_reduce_multi<R * MT>(acc, lane);
            if (reduced_owner<R * MT>(lane)) {
                const int idx = reduced_index<R * MT>(lane);
                const int r = idx / MT, mm = idx % MT;
                const int n = row0 + r;
                if (n < hi) {
                    tile[(size_t)mm * CH + (n - lo)] = v;
                    const int m = m0 + mm;
                    if (a.raw_out && m < a.M) a.raw_out[(size_t)m * a.V + n] = v;
                }
            }
        }
        __syncthreads();
        // one warp per sequence: processors, then the reductions
        for (int mm = warp; mm < MT; mm += kGemvThreads / 32) {
            const int m = m0 + mm;
            if (m >= a.M) continue;
            if (a.active && !a.active[m]) continue;
            float *row = tile + (size_t)mm * CH;
            const int n = hi - lo;
            if (a.ns_token >= 0) {  // unmasked statistics of this row (no-speech probability)
                float mx = -INFINITY;
                for (int i = lane; i < n; i += 32) mx = fmaxf(mx, row[i]);
                mx = warp_max(mx);
                float sm = 0.f;
                for (int i = lane; i < n; i += 32) sm += (mx == -INFINITY) ? 0.f : __expf(row[i] - mx);
                sm = warp_sum(sm);
                if (lane == 0) {
                    float *np = a.ns_part + ((size_t)m * P + blockIdx.x) * 2;
                    np[0] = mx;
                    np[1] = sm;
                }
                if (a.ns_token >= lo && a.ns_token < hi && lane == 0) a.ns_value[m] = row[a.ns_token - lo];
                __syncwarp();
            }
            if (a.use_mask) {
                const MaskArgs &mk = a.mask;
                for (int r = 0; r < mk.n_ranges[m]; ++r) {
                    const int2 rg = mk.ranges[(size_t)m * kMaxRanges + r];
                    const int b0 = max(rg.x, lo), b1 = min(rg.y, hi);
                    for (int i = b0 + lane; i < b1; i += 32) row[i - lo] = -INFINITY;
                }
                for (int i = lane; i < mk.n_static; i += 32) {
                    const int t = mk.static_list[i];
                    if (t >= lo && t < hi) row[t - lo] = -INFINITY;
                }
                const int nd = mk.dyn_count[m];
                for (int i = lane; i < nd; i += 32) {
                    const int t = mk.dyn_list[(size_t)m * mk.dyn_stride + i];
                    if (t >= lo && t < hi) row[t - lo] = -INFINITY;
                }
                __syncwarp();
            }
            if (a.masked_out)
                for (int i = lane; i < n; i += 32) a.masked_out[(size_t)m * a.V + lo + i] = row[i];
            // max + first argmax
            float bv = -INFINITY;
            int bi = INT_MAX;
            for (int i = lane; i < n; i += 32)
                if (better(row[i], lo + i, bv, bi)) {
                    bv = row[i];
                    bi = lo + i;
                }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (better(ov, oi, bv, bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            float sm = 0.f;
            if (bv != -INFINITY)
                for (int i = lane; i < n; i += 32) sm += __expf(row[i] - bv);
            sm = warp_sum(sm);
            float *pp = a.part + ((size_t)m * P + blockIdx.x) * kPartStride;
            if (lane == 0) {
                pp[0] = bv;
                pp[1] = sm;
                pp[2] = __int_as_float(bi == INT_MAX ? lo : bi);
            }
            // top-k candidates of this block (value desc, index asc); unfilled: (-inf, 0)
            for (int k = 0; k < a.topk; ++k) {
                float kv = -INFINITY;
                int ki = INT_MAX;
                for (int i = lane; i < n; i += 32)
                    if (row[i] != -INFINITY && better(row[i], lo + i, kv, ki)) {
                        kv = row[i];
                        ki = lo + i;
                    }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, kv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, ki, o);
                    if (better(ov, oi, kv, ki)) {
                        kv = ov;
                        ki = oi;
                    }
                }
                if (lane == 0) {
                    pp[4 + k] = kv;
                    pp[4 + kMaxTopK + k] = __int_as_float(ki == INT_MAX ? 0 : ki);
                }
                if (ki != INT_MAX && ki - lo >= 0 && ki - lo < n && lane == ((ki - lo) & 31))
                    row[ki - lo] = -INFINITY;
                __syncwarp();
            }
        }
        __syncthreads();
    }
}

int logits_parts_for(int V, int sms) {
    int p = 2 * sms;
    if (p > V) p = V;
    return p < 1 ? 1 : p;
}

static int pick_mt_logits(int M, int d) {
    int mt = pick_mt(M, d);
    return mt > 8 ? 8 : mt;
}

size_t logits_smem_bytes(int M, int V, int d, int P) {
    const int mt = pick_mt_logits(M, d);
    const int CH = (V + P - 1) / P + 1;
    return ((size_t)mt * d + (size_t)mt * CH) * sizeof(float);
}

template <int MT, int R, int WT>
static cudaError_t launch_logits_t(const LogitsArgs &a, int P, cudaStream_t s, bool pdl) {
    const int CH = (a.V + P - 1) / P + 1;
    const size_t smem = ((size_t)MT * a.d + (size_t)MT * CH) * sizeof(float);
    auto kern = k_logits<MT, R, WT>;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(P);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int WT>
static cudaError_t dispatch_logits(const LogitsArgs &a, int P, cudaStream_t s, bool pdl) {
    switch (pick_mt_logits(a.M, a.d)) {
        case 1: return launch_logits_t<1, 4, WT>(a, P, s, pdl);
        case 2: return launch_logits_t<2, 4, WT>(a, P, s, pdl);
        case 4: return launch_logits_t<4, 4, WT>(a, P, s, pdl);
        default: return launch_logits_t<8, 2, WT>(a, P, s, pdl);
    }
}

// Raise the dynamic shared-memory limit of every instantiation once (outside any graph capture).
template <int WT>
static cudaError_t prepare_wt() {
    const int lim = 160 * 1024;
    cudaError_t e = cudaSuccess;
#define W4J_SET(kern) \
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, lim)
    W4J_SET((k_gemv<1, 4, WT>));
    W4J_SET((k_gemv<2, 4, WT>));
    W4J_SET((k_gemv<4, 4, WT>));
    W4J_SET((k_gemv<8, 2, WT>));
    W4J_SET((k_gemv<16, 2, WT>));
    W4J_SET((k_logits<1, 4, WT>));
    W4J_SET((k_logits<2, 4, WT>));
    W4J_SET((k_logits<4, 4, WT>));
    W4J_SET((k_logits<8, 2, WT>));
#undef W4J_SET
    return e;
}

cudaError_t gemv_prepare() {
    cudaError_t e = prepare_wt<WT_F16>();
    if (e == cudaSuccess) e = prepare_wt<WT_Q8>();
    return e;
}

cudaError_t launch_logits(const LogitsArgs &a, int P, cudaStream_t s, bool pdl) {
    if (a.M <= 0) return cudaSuccess;
    if (a.topk > kMaxTopK) return cudaErrorInvalidValue;
    if (a.E.type == WT_F16) return dispatch_logits<WT_F16>(a, P, s, pdl);
    if (a.E.type == WT_Q8) return dispatch_logits<WT_Q8>(a, P, s, pdl);
    return cudaErrorInvalidValue;
}

}  // namespace w4j
