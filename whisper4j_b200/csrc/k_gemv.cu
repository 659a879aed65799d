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
// Design (HBM-bound, M small).  Weights stay in their GGML (N, K) row layout.  Each block
// owns a contiguous range of rows, so its weight bytes are one contiguous run that a single
// thread moves into shared memory with TMA bulk copies (cp.async.bulk + mbarrier).  Under
// programmatic dependent launch those copies are issued *before* griddepcontrol.wait: the
// weight stream of kernel i+1 overlaps kernel i, and after the wait only the activations
// (a few KB from L2) stand between the previous kernel and this one's result.  A warp owns R
// rows at a time and its lanes walk K in 16-byte chunks (8 f16 or 16 int8), dequantising in
// registers; the M activation rows sit in shared memory as f32 (LayerNorm applied on the way
// in), every weight chunk is reused for all M rows, and the R x M partial sums are reduced
// across the warp with a butterfly that leaves one finished sum per lane.  The vocabulary
// projection streams its rows through a ring of shared-memory stages, the first stages again
// issued before the wait.
#include <float.h>

#include "logits_epilogue.cuh"
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

// Accumulators are laid out acc[r * P2 + mm] with P2 the power of two >= MT, so the
// butterfly reduction works on a power-of-two count; entries mm >= MT stay zero.
template <int MT>
struct P2 {
    static constexpr int v = MT <= 1 ? 1 : MT <= 2 ? 2 : MT <= 4 ? 4 : MT <= 8 ? 8 : 16;
};


// Fill act_s[mm][k] (mm < MT) for rows m0.. of the pass: plain copy, LayerNorm of x, or
// token + positional embedding then LayerNorm.  All threads cooperate on the loads with
// eight independent 16-byte loads in flight each (one L2 round trip for a few KB), then
// one warp per row normalises in shared memory.
template <int MT, int NT>
__device__ void load_activations(const GemvArgs &a, int m0, int K, float *act_s, const float *ln_s, int warp,
                                 int lane, const int *tok_s = nullptr, const int *pos_s = nullptr) {
    const int K4 = K / 4;
    const int total = MT * K4;
    // LayerNorm inputs with K a multiple of 128 up to 1280 (every Whisper width): one warp per
    // row loads the row straight into registers (all loads in flight), reduces mean and
    // variance there, and writes the normalised row once
    constexpr int kLnF4 = 10;  // float4 per lane
    const bool embed_f16 = a.in_mode == IN_EMBED_LN && a.E.type == WT_F16;
    if ((a.in_mode == IN_LN || embed_f16) && K % 128 == 0 && K <= 128 * kLnF4) {
        const int nf4 = K / 128;
        for (int mm = warp; mm < MT; mm += (NT / 32)) {
            float4 *dst = reinterpret_cast<float4 *>(act_s + (size_t)mm * K);
            const int m = m0 + mm;
            if (m >= a.M) {
                for (int c = lane; c < K4; c += 32) dst[c] = make_float4(0.f, 0.f, 0.f, 0.f);
                continue;
            }
            float4 v[kLnF4];
            if (a.in_mode == IN_LN) {
                const float4 *src = reinterpret_cast<const float4 *>(a.act + (size_t)m * K);
#pragma unroll
                for (int j = 0; j < kLnF4; ++j) v[j] = j < nf4 ? src[lane + 32 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
            } else {  // x = E[tok] + P[pos] (WhisperDecoder.java:66-80), kept in x_out by block 0
                const int tok = tok_s ? tok_s[m] : a.tok[m], pos = pos_s ? pos_s[m] : pe_row(a, m);
                const uint2 *e = reinterpret_cast<const uint2 *>(a.E.h + (size_t)tok * K);
                const float4 *pe = reinterpret_cast<const float4 *>(a.pos_emb + (size_t)pos * K);
                uint2 eu[kLnF4];
#pragma unroll
                for (int j = 0; j < kLnF4; ++j) {
                    eu[j] = j < nf4 ? e[lane + 32 * j] : make_uint2(0u, 0u);
                    v[j] = j < nf4 ? pe[lane + 32 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int j = 0; j < kLnF4; ++j) {
                    const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&eu[j].x));
                    const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&eu[j].y));
                    v[j] = make_float4(lo.x + v[j].x, lo.y + v[j].y, hi.x + v[j].z, hi.y + v[j].w);
                    if (j < nf4 && blockIdx.x == 0 && a.x_out)
                        reinterpret_cast<float4 *>(a.x_out)[(size_t)m * K4 + lane + 32 * j] = v[j];
                }
            }
            // Tensor.layerNorm (Tensor.java:592-619): two-pass mean / variance, eps 1e-5,
            // invStd = 1 / sqrt(var / n + eps), y = (x - mean) * invStd * g + b.
            float s = 0.f;
#pragma unroll
            for (int j = 0; j < kLnF4; ++j)
                if (j < nf4) s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
            const float mean = warp_sum(s) / (float)K;
            float v2 = 0.f;
#pragma unroll
            for (int j = 0; j < kLnF4; ++j)
                if (j < nf4) {
                    const float dx = v[j].x - mean, dy = v[j].y - mean, dz = v[j].z - mean, dw = v[j].w - mean;
                    v2 += (dx * dx + dy * dy) + (dz * dz + dw * dw);
                }
            const float inv_std = 1.0f / sqrtf(warp_sum(v2) / (float)K + 1e-5f);
            const float4 *g4 = reinterpret_cast<const float4 *>(ln_s);
            const float4 *b4 = reinterpret_cast<const float4 *>(ln_s + K);
#pragma unroll
            for (int j = 0; j < kLnF4; ++j)
                if (j < nf4) {
                    const int c = lane + 32 * j;
                    const float4 g = g4[c], b = b4[c];
                    dst[c] = make_float4((v[j].x - mean) * inv_std * g.x + b.x, (v[j].y - mean) * inv_std * g.y + b.y,
                                         (v[j].z - mean) * inv_std * g.z + b.z, (v[j].w - mean) * inv_std * g.w + b.w);
                }
        }
        return;
    }
    if (a.in_mode == IN_EMBED_LN) {
        const bool f16 = a.E.type == WT_F16;
        for (int i0 = threadIdx.x; i0 < total; i0 += NT * 8) {
            float4 e[8], p[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = i0 + NT * j;
                const int mm = i / K4, k = (i - mm * K4) * 4;
                const int m = m0 + mm;
                e[j] = p[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (i < total && m < a.M) {
                    const int tok = tok_s ? tok_s[m] : a.tok[m], pos = pos_s ? pos_s[m] : pe_row(a, m);
                    p[j] = *reinterpret_cast<const float4 *>(a.pos_emb + (size_t)pos * K + k);
                    if (f16) {
                        const uint2 u = *reinterpret_cast<const uint2 *>(a.E.h + (size_t)tok * K + k);
                        const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
                        const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
                        e[j] = make_float4(lo.x, lo.y, hi.x, hi.y);
                    } else {
                        const float sc = __half2float(a.E.s[(size_t)tok * (K / 32) + k / 32]);
                        const char4 q = *reinterpret_cast<const char4 *>(a.E.q + (size_t)tok * K + k);
                        e[j] = make_float4(q.x * sc, q.y * sc, q.z * sc, q.w * sc);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = i0 + NT * j;
                if (i >= total) continue;
                const float4 v = make_float4(e[j].x + p[j].x, e[j].y + p[j].y, e[j].z + p[j].z, e[j].w + p[j].w);
                reinterpret_cast<float4 *>(act_s)[i] = v;
                const int mm = i / K4, m = m0 + mm;
                if (blockIdx.x == 0 && a.x_out && m < a.M)
                    reinterpret_cast<float4 *>(a.x_out)[(size_t)m * K4 + (i - mm * K4)] = v;
            }
        }
    } else {
        // rows m0.. are contiguous in `act`: one flat copy of the live rows (rows past M: zero)
        const int live = (a.M - m0 < MT ? a.M - m0 : MT) * K4;
        const float4 *src = reinterpret_cast<const float4 *>(a.act) + (size_t)m0 * K4;
        constexpr int kB = 16;  // 16 x 16 B in flight per thread: 64 KB per block per round trip
        for (int i0 = threadIdx.x; i0 < total; i0 += NT * kB) {
            float4 v[kB];
#pragma unroll
            for (int j = 0; j < kB; ++j) {
                const int i = i0 + NT * j;
                v[j] = i < live ? src[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int j = 0; j < kB; ++j)
                if (i0 + NT * j < total) reinterpret_cast<float4 *>(act_s)[i0 + NT * j] = v[j];
        }
    }
    if (a.in_mode == IN_ACT) return;
    __syncthreads();
    for (int mm = warp; mm < MT; mm += (NT / 32)) {
        if (m0 + mm >= a.M) continue;
        float *dst = act_s + (size_t)mm * K;
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
        for (int k = lane; k < K; k += 32) dst[k] = (dst[k] - mean) * inv_std * ln_s[k] + ln_s[K + k];
    }
}

// gamma / beta of the LayerNorm into shared memory (constant: done before the grid wait)
template <int NT>
__device__ __forceinline__ void stage_ln(const float *g, const float *b, int K, float *ln_s) {
    for (int i0 = threadIdx.x; i0 < 2 * K; i0 += NT * 8) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = i0 + NT * j;
            v[j] = i < K ? g[i] : i < 2 * K ? b[i - K] : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (i0 + NT * j < 2 * K) ln_s[i0 + NT * j] = v[j];
    }
}

template <int MT, int R>
__device__ __forceinline__ void fma_chunk_f16(const uint4 (&w)[R], const float *act_s, int K, int k0,
                                              float (&acc)[R * P2<MT>::v]) {
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
            float t = acc[r * P2<MT>::v + mm];
            t = fmaf(wf[r][0], a0.x, t);
            t = fmaf(wf[r][1], a0.y, t);
            t = fmaf(wf[r][2], a0.z, t);
            t = fmaf(wf[r][3], a0.w, t);
            t = fmaf(wf[r][4], a1.x, t);
            t = fmaf(wf[r][5], a1.y, t);
            t = fmaf(wf[r][6], a1.z, t);
            t = fmaf(wf[r][7], a1.w, t);
            acc[r * P2<MT>::v + mm] = t;
        }
    }
}

template <int MT, int R>
__device__ __forceinline__ void fma_chunk_q8(const uint4 (&w)[R], const float (&sc)[R], const float *act_s, int K,
                                             int k0, float (&acc)[R * P2<MT>::v]) {
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
        for (int r = 0; r < R; ++r) acc[r * P2<MT>::v + mm] = fmaf(part[r], sc[r], acc[r * P2<MT>::v + mm]);
    }
}

// Dot products of R rows staged in shared memory (row stride `row_bytes`; Q8 scales in
// `sc_s` with K/32 per row, or read from global when sc_s is null) with the MT activation rows.
template <int MT, int R, int WT>
__device__ __forceinline__ void smem_rows(const unsigned char *w_s, int row_bytes, int nrows, const __half *sc_s,
                                          const __half *sc_g, int K, const float *act_s,
                                          float (&acc)[R * P2<MT>::v], int lane, int c0, int cstep) {
    constexpr int CE = WT == WT_F16 ? 8 : 16;
    const int nchunk = K / CE;
#pragma unroll
    for (int i = 0; i < R * P2<MT>::v; ++i) acc[i] = 0.f;
    for (int c = c0; c < nchunk; c += cstep) {
        uint4 w[R];
        float sc[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            if (r < nrows) {
                w[r] = *reinterpret_cast<const uint4 *>(w_s + (size_t)r * row_bytes + (size_t)c * 16);
                if (WT == WT_Q8)
                    sc[r] = __half2float(sc_s ? sc_s[(size_t)r * (K / 32) + (c * CE) / 32]
                                              : sc_g[(size_t)r * (K / 32) + (c * CE) / 32]);
                else
                    sc[r] = 0.f;
            } else {
                w[r] = make_uint4(0, 0, 0, 0);
                sc[r] = 0.f;
            }
        }
        if (WT == WT_F16)
            fma_chunk_f16<MT, R>(w, act_s, K, c * CE, acc);
        else
            fma_chunk_q8<MT, R>(w, sc, act_s, K, c * CE, acc);
    }
}

__device__ __forceinline__ void drain(uint64_t *bar, unsigned parity) {
    // a wait that timed out: give the copy in flight a second bounded chance to land
    for (long long it = 0; it < (1ll << 22); ++it)
        if (mbar_test(bar, parity)) return;
}

// ---------------------------------------------------------------------------
// GEMV kernel: block = rows [r0, r0 + rows_per_block) of W, staged whole in shared memory
// ---------------------------------------------------------------------------
// Threads of a k_gemv block.  Q8_0 rows carry more arithmetic per weight byte (dequantisation),
// so sixteen warps split each row group's K; f16 blocks stay at eight warps, which keeps them
// small enough for blocks of consecutive kernels to be co-resident and prefetch their weights.
__host__ __device__ constexpr int gemv_threads(int wt) { return wt == WT_Q8 ? 512 : 256; }

struct GemvLaunch {
    int rows_per_block;
    size_t w_bytes, s_bytes;  // staging capacity for weights / Q8 scales (16-byte multiples)
};

template <int MT, int R, int WT>
__global__ void __launch_bounds__(gemv_threads(WT)) k_gemv(GemvArgs a, GemvLaunch L) {
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int NT = gemv_threads(WT);
    const int N = a.W.N, K = a.W.K;
    const int r0 = blockIdx.x * L.rows_per_block;
    const int nr = min(N, r0 + L.rows_per_block) - r0;
    unsigned char *w_s = smem;
    __half *sc_s = reinterpret_cast<__half *>(smem + L.w_bytes);
    float *act_s = reinterpret_cast<float *>(smem + L.w_bytes + L.s_bytes);
    float *ln_s = act_s + (size_t)MT * K;  // [gamma | beta]
    uint64_t *bar = reinterpret_cast<uint64_t *>(ln_s + (a.in_mode != IN_ACT ? 2 * (size_t)K : 0));
    // epilogue operands: bias of the block's rows, per-sequence liveness / cache slot / position /
    // token, and (residual epilogue) the residual values of the pass
    float *bias_s = reinterpret_cast<float *>(bar + 2);                        // [rows_per_block]
    int *mi_s = reinterpret_cast<int *>(bias_s + L.rows_per_block);           // [5][M]
    float *res_s = reinterpret_cast<float *>(mi_s + 5 * (size_t)a.M);         // [MT][rows_per_block]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row_bytes = WT == WT_F16 ? K * 2 : K;
    const int M = a.M;
    // --- independent of the previous kernel: the weight rows ---
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
        const unsigned bytes = (unsigned)((size_t)nr * row_bytes);
        mbar_expect_tx(bar, bytes);
        const unsigned char *src = WT == WT_F16 ? reinterpret_cast<const unsigned char *>(a.W.h + (size_t)r0 * K)
                                                : reinterpret_cast<const unsigned char *>(a.W.q + (size_t)r0 * K);
        for (unsigned off = 0; off < bytes; off += 65536u) bulk_g2s(w_s + off, src + off, min(65536u, bytes - off), bar);
        l2_ahead(a.pf, blockIdx.x, gridDim.x);
    }
    if (WT == WT_Q8)
        for (int i = tid; i < nr * (K / 32); i += NT) sc_s[i] = a.W.s[(size_t)r0 * (K / 32) + i];
    if (a.in_mode != IN_ACT) stage_ln<NT>(a.ln_g, a.ln_b, K, ln_s);
    // Biases are weights; liveness, cache slots, positions and tokens were written by the host
    // or by an earlier graph launch, never by a kernel of this launch's chain: read them now.
    for (int i = tid; i < nr; i += NT) bias_s[i] = a.bias ? a.bias[r0 + i] : 0.f;
    for (int i = tid; i < M; i += NT) {
        mi_s[i] = a.active ? a.active[i] : 1;
        if (a.out_mode == OUT_QKV) {
            mi_s[M + i] = a.seq_slot[i];
            mi_s[2 * M + i] = a.pos[i];
        }
        if (a.in_mode == IN_EMBED_LN) {
            mi_s[3 * M + i] = a.tok[i];
            mi_s[4 * M + i] = pe_row(a, i);
        }
    }
    pdl_wait();

    bool ok = true;
    for (int m0 = 0; m0 < a.M; m0 += MT) {
        // residual values of the pass (rows r0 + tid): loaded into registers now, stored to
        // shared memory after the activation loads were issued, so both are in flight together
        float resv[MT];
        const bool has_res = a.out_mode == OUT_RESIDUAL && tid < nr;
        if (has_res)
#pragma unroll
            for (int mm = 0; mm < MT; ++mm) resv[mm] = m0 + mm < M ? a.y[(size_t)(m0 + mm) * N + r0 + tid] : 0.f;
        if (m0 == 0) __syncthreads();  // mi_s
        load_activations<MT, NT>(a, m0, K, act_s, ln_s, warp, lane, mi_s + 3 * M, mi_s + 4 * M);
        if (has_res)
#pragma unroll
            for (int mm = 0; mm < MT; ++mm) res_s[mm * L.rows_per_block + tid] = resv[mm];
        if (a.out_mode == OUT_RESIDUAL)  // blocks of more than NT rows (op-level calls)
            for (int r = tid + NT; r < nr; r += NT)
#pragma unroll
                for (int mm = 0; mm < MT; ++mm)
                    res_s[mm * L.rows_per_block + r] = m0 + mm < M ? a.y[(size_t)(m0 + mm) * N + r0 + r] : 0.f;
        __syncthreads();
        // The next kernel may launch (and start its own weight copies) only now: its copies no
        // longer queue ahead of this block's activation loads, which are on the critical path.
        if (m0 == 0) pdl_trigger();
        if (m0 == 0) ok = __syncthreads_and(mbar_wait(bar, 0, a.err));  // block-uniform: a barrier follows
        if (ok) {
            constexpr int PM = P2<MT>::v;
            // output (row lr of the block, sequence m0 + mm) with its epilogue
            auto emit = [&](float v, int lr, int mm) {
                const int n = r0 + lr, m = m0 + mm;
                if (mm >= MT || lr >= nr || m >= a.M || !mi_s[m]) return;
                const float val = v + bias_s[lr];
                switch (a.out_mode) {
                    case OUT_STORE:
                        a.y[(size_t)m * N + n] = val;
                        break;
                    case OUT_GELU:  // Tensor.geluInPlace: table lookup at the f16 rounding of x
                        a.y[(size_t)m * N + n] = a.gelu_lut[__half_as_ushort(__float2half_rn(val))];
                        break;
                    case OUT_RESIDUAL:
                        a.y[(size_t)m * N + n] = res_s[mm * L.rows_per_block + lr] + val;
                        break;
                    case OUT_QKV: {
                        const int dm = N / 3;
                        const int part = n / dm, c = n - part * dm;
                        if (part == 0) {
                            a.y[(size_t)m * dm + c] = val;
                        } else {
                            const int head = c / kHeadDim, dd = c % kHeadDim;
                            const size_t row = (((size_t)mi_s[M + m] * a.n_layer + a.layer) * a.n_head + head) *
                                                   (size_t)a.n_ctx + (size_t)mi_s[2 * M + m];
                            __half *dst = part == 1 ? a.kcache : a.vcache;
                            dst[row * kHeadDim + dd] = __float2half_rn(val);
                        }
                        break;
                    }
                }
            };
            // G groups of R rows; with fewer groups than warps, KS warps share a group's K
            // chunks and their sums meet in shared memory (added in warp order)
            const int G = (nr + R - 1) / R;
            // G * KS <= warps
            const int KS = NT == 256 ? (G >= 5 ? 1 : G >= 3 ? 2 : G == 2 ? 4 : 8) : (G >= NT / 32 ? 1 : (NT / 32) / G);
            if (KS == 1) {
                for (int g = warp; g < G; g += NT / 32) {
                    float acc[R * PM];
                    smem_rows<MT, R, WT>(w_s + (size_t)g * R * row_bytes, row_bytes, min(R, nr - g * R),
                                         sc_s + (size_t)g * R * (K / 32), nullptr, K, act_s, acc, lane, lane, 32);
                    const float v = warp_reduce_multi<R * PM>(acc, lane);
                    if (!reduced_owner<R * PM>(lane)) continue;
                    const int idx = reduced_index<R * PM>(lane);
                    emit(v, g * R + idx / PM, idx % PM);
                }
            } else {
                __shared__ float red_s[NT / 32][32];
                const int g = warp / KS, kp = warp % KS;
                if (g < G) {
                    float acc[R * PM];
                    smem_rows<MT, R, WT>(w_s + (size_t)g * R * row_bytes, row_bytes, min(R, nr - g * R),
                                         sc_s + (size_t)g * R * (K / 32), nullptr, K, act_s, acc, lane,
                                         lane + 32 * kp, 32 * KS);
                    const float v = warp_reduce_multi<R * PM>(acc, lane);
                    if (reduced_owner<R * PM>(lane)) red_s[warp][reduced_index<R * PM>(lane)] = v;
                }
                __syncthreads();
                if (g < G && kp == 0 && reduced_owner<R * PM>(lane)) {
                    const int idx = reduced_index<R * PM>(lane);
                    float v = 0.f;
                    for (int q = 0; q < KS; ++q) v += red_s[warp + q][idx];
                    emit(v, g * R + idx / PM, idx % PM);
                }
            }
        }
        __syncthreads();
    }
    if (!ok) drain(bar, 0);
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

constexpr size_t kSmemBudget = 220 * 1024;  // of the 227 KB a block may use

static size_t align16(size_t x) { return (x + 15) & ~(size_t)15; }

// Activation rows per pass (exact, up to 8) and the weight staging of one block.
static void plan_gemv(int M, int N, int K, int type, int sms, int &mt, GemvLaunch &L, int &blocks) {
    const size_t row_bytes = type == WT_F16 ? (size_t)K * 2 : (size_t)K;
    const size_t srow = type == WT_F16 ? 0 : (size_t)(K / 32) * 2;
    int rpb = (N + sms - 1) / sms;
    // keep the weight slice within ~160 KB so activations fit beside it
    const size_t wcap = 160 * 1024;
    if ((size_t)rpb * (row_bytes + srow) > wcap) rpb = (int)(wcap / (row_bytes + srow));
    if (rpb < 1) rpb = 1;
    blocks = (N + rpb - 1) / rpb;
    L.rows_per_block = rpb;
    L.w_bytes = align16((size_t)rpb * row_bytes);
    L.s_bytes = align16((size_t)rpb * srow);
    // epilogue staging: bias, 5 ints per sequence, up to 8 residual rows
    const size_t epi = ((size_t)rpb * 9 + 5 * (size_t)M) * 4;
    const size_t left = kSmemBudget - L.w_bytes - L.s_bytes - 64 - 2 * (size_t)K * 4 - epi;
    int cap = (int)(left / ((size_t)K * 4));
    mt = M < 8 ? M : 8;
    if (mt > cap) mt = cap;
    if (mt < 1) mt = 1;
    if (M > mt) {
        const int passes = (M + mt - 1) / mt;
        mt = (M + passes - 1) / passes;
    }
}

template <int MT, int R, int WT>
static cudaError_t launch_gemv_t(const GemvArgs &a, const GemvLaunch &L, int blocks, cudaStream_t s, bool pdl) {
    const size_t smem = L.w_bytes + L.s_bytes + ((size_t)MT + (a.in_mode != IN_ACT ? 2 : 0)) * a.W.K * sizeof(float) + 16 +
                        ((size_t)L.rows_per_block * (1 + MT) + 5 * (size_t)a.M) * 4;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(gemv_threads(WT));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_gemv<MT, R, WT>, a, L);
}

template <int MT, int WT>
static cudaError_t launch_gemv_r(const GemvArgs &a, const GemvLaunch &L, int blocks, cudaStream_t s, bool pdl) {
    // few rows per block: one row per warp keeps all warps busy; many rows: 4 rows share
    // each activation read
    if (L.rows_per_block <= 8) return launch_gemv_t<MT, 1, WT>(a, L, blocks, s, pdl);
    if constexpr (MT == 1 || (MT == 2 && WT == WT_F16)) {  // > 32 rows: 8 rows per warp keeps every row group within one round
        if (L.rows_per_block > 32) return launch_gemv_t<MT, 8, WT>(a, L, blocks, s, pdl);
    }
    if constexpr (MT <= 4) return launch_gemv_t<MT, 4, WT>(a, L, blocks, s, pdl);
    else
    return launch_gemv_t<MT, 2, WT>(a, L, blocks, s, pdl);
}

template <int WT>
static cudaError_t dispatch_gemv(const GemvArgs &a, cudaStream_t s, bool pdl) {
    int mt, blocks;
    GemvLaunch L;
    plan_gemv(a.M, a.W.N, a.W.K, WT, sm_count(), mt, L, blocks);
    switch (mt) {
        case 1: return launch_gemv_r<1, WT>(a, L, blocks, s, pdl);
        case 2: return launch_gemv_r<2, WT>(a, L, blocks, s, pdl);
        case 3: return launch_gemv_r<3, WT>(a, L, blocks, s, pdl);
        case 4: return launch_gemv_r<4, WT>(a, L, blocks, s, pdl);
        case 5: return launch_gemv_r<5, WT>(a, L, blocks, s, pdl);
        case 6: return launch_gemv_r<6, WT>(a, L, blocks, s, pdl);
        case 7: return launch_gemv_r<7, WT>(a, L, blocks, s, pdl);
        default: return launch_gemv_r<8, WT>(a, L, blocks, s, pdl);
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

struct LogitsLaunch {
    int stage_rows;      // rows per ring stage (8 * R)
    int n_stages;
    size_t stage_bytes;  // 16-byte multiple
    int ch;              // max rows per block (+1)
};

template <int MT, int R, int WT>
__global__ void __launch_bounds__(kGemvThreads) k_logits(LogitsArgs a, LogitsLaunch L) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int P = gridDim.x;
    const int lo = (int)(((long long)blockIdx.x * a.V) / P);
    const int hi = (int)(((long long)(blockIdx.x + 1) * a.V) / P);
    const int nrows = hi - lo;
    const int d = a.d;
    const int row_bytes = WT == WT_F16 ? d * 2 : d;
    const int SR = L.stage_rows, NS = L.n_stages;
    unsigned char *ring = smem;
    float *act_s = reinterpret_cast<float *>(smem + (size_t)NS * L.stage_bytes);
    float *ln_s = act_s + (size_t)MT * d;  // [gamma | beta]
    float *tile = ln_s + 2 * (size_t)d;     // [MT][ch]
    uint64_t *bars = reinterpret_cast<uint64_t *>((reinterpret_cast<uintptr_t>(tile + (size_t)MT * L.ch) + 15) &
                                                  ~(uintptr_t)15);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_tiles = (nrows + SR - 1) / SR;
    const int passes = (a.M + MT - 1) / MT;
    const int total = n_tiles * passes;
    const unsigned char *base = WT == WT_F16 ? reinterpret_cast<const unsigned char *>(a.E.h + (size_t)lo * d)
                                             : reinterpret_cast<const unsigned char *>(a.E.q + (size_t)lo * d);
    auto issue = [&](int gidx) {  // thread 0: stream tile (gidx % n_tiles) into stage gidx % NS
        const int t = gidx % n_tiles;
        const int rows = min(SR, nrows - t * SR);
        const unsigned bytes = (unsigned)rows * row_bytes;
        uint64_t *b = bars + (gidx % NS);
        mbar_expect_tx(b, bytes);
        bulk_g2s(ring + (size_t)(gidx % NS) * L.stage_bytes, base + (size_t)t * SR * row_bytes, bytes, b);
    };
    // --- independent of the previous kernel: the first stages of this block's rows ---
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) mbar_init(bars + i, 1);
        fence_mbar_init();
        for (int g = 0; g < NS && g < total; ++g) issue(g);
    }
    stage_ln<kGemvThreads>(a.ln_g, a.ln_b, d, ln_s);
    pdl_trigger();
    pdl_wait();

    bool ok = true;
    for (int pass = 0; pass < passes; ++pass) {
        const int m0 = pass * MT;
        GemvArgs g;
        g.M = a.M;
        g.in_mode = IN_LN;
        g.act = a.x;
        g.ln_g = a.ln_g;
        g.ln_b = a.ln_b;
        load_activations<MT, kGemvThreads>(g, m0, d, act_s, ln_s, warp, lane);
        __syncthreads();
        for (int t = 0; t < n_tiles; ++t) {
            const int gidx = pass * n_tiles + t;
            if (ok) ok = mbar_wait(bars + (gidx % NS), (unsigned)((gidx / NS) & 1), a.err);
            const int rows = min(SR, nrows - t * SR);
            const unsigned char *st = ring + (size_t)(gidx % NS) * L.stage_bytes;
            constexpr int PM = P2<MT>::v;
            if (ok && warp * R < rows) {
                float acc[R * PM];
                const int rloc = warp * R;
                smem_rows<MT, R, WT>(st + (size_t)rloc * row_bytes, row_bytes, min(R, rows - rloc), nullptr,
                                     WT == WT_Q8 ? a.E.s + (size_t)(lo + t * SR + rloc) * (d / 32) : nullptr, d,
                                     act_s, acc, lane, lane, 32);
                const float v = warp_reduce_multi<R * PM>(acc, lane);
                if (reduced_owner<R * PM>(lane)) {
                    const int idx = reduced_index<R * PM>(lane);
                    const int r = idx / PM, mm = idx % PM;
                    const int local = t * SR + rloc + r;
                    if (mm < MT && rloc + r < rows) {
                        tile[(size_t)mm * L.ch + local] = v;
                        const int m = m0 + mm;
                        if (a.raw_out && m < a.M) a.raw_out[(size_t)m * a.V + lo + local] = v;
                    }
                }
            }
            __syncthreads();  // stage consumed by every warp
            if (tid == 0 && ok && gidx + NS < total) issue(gidx + NS);
        }
        logits_rows_epilogue(a, tile, L.ch, MT, m0, lo, hi, ok);
        __syncthreads();
    }
    if (!ok)
        for (int i = 0; i < NS; ++i) drain(bars + i, 0), drain(bars + i, 1);
}

int logits_parts_for(int V, int sms) {
    int p = sms;
    if (p > V) p = V;
    return p < 1 ? 1 : p;
}

static void plan_logits(int M, int V, int d, int type, int P, int &mt, int &R, LogitsLaunch &L) {
    const int row_bytes = type == WT_F16 ? d * 2 : d;
    mt = M < 8 ? M : 8;
    if (M > mt) {
        const int passes = (M + mt - 1) / mt;
        mt = (M + passes - 1) / passes;
    }
    R = mt <= 4 ? 4 : 2;
    if (mt <= 2 && d <= 512) R = 4;
    L.stage_rows = 8 * R;
    L.stage_bytes = align16((size_t)L.stage_rows * row_bytes);
    L.ch = (V + P - 1) / P + 1;
    const size_t fixed = ((size_t)mt + 2) * d * 4 + (size_t)mt * L.ch * 4 + 16 * 8 + 64;
    int ns = (int)((kSmemBudget - fixed) / L.stage_bytes);
    L.n_stages = ns < 2 ? 2 : ns > 8 ? 8 : ns;
}

size_t logits_smem_bytes(int M, int V, int d, int P) {
    int mt, R;
    LogitsLaunch L;
    plan_logits(M, V, d, WT_F16, P, mt, R, L);
    return (size_t)L.n_stages * L.stage_bytes + ((size_t)mt + 2) * d * 4 + (size_t)mt * L.ch * 4 + 8 * L.n_stages + 16;
}

template <int MT, int R, int WT>
static cudaError_t launch_logits_t(const LogitsArgs &a, const LogitsLaunch &L, int P, cudaStream_t s, bool pdl) {
    const size_t smem =
        (size_t)L.n_stages * L.stage_bytes + ((size_t)MT + 2) * a.d * 4 + (size_t)MT * L.ch * 4 + 8 * (size_t)L.n_stages + 16;
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
    return cudaLaunchKernelEx(&cfg, k_logits<MT, R, WT>, a, L);
}

template <int WT>
static cudaError_t dispatch_logits(const LogitsArgs &a, int P, cudaStream_t s, bool pdl) {
    int mt, R;
    LogitsLaunch L;
    plan_logits(a.M, a.V, a.d, WT, P, mt, R, L);
    if (R == 4) {
        switch (mt) {
            case 1: return launch_logits_t<1, 4, WT>(a, L, P, s, pdl);
            case 2: return launch_logits_t<2, 4, WT>(a, L, P, s, pdl);
            case 3: return launch_logits_t<3, 4, WT>(a, L, P, s, pdl);
            default: return launch_logits_t<4, 4, WT>(a, L, P, s, pdl);
        }
    }
    switch (mt) {
        case 5: return launch_logits_t<5, 2, WT>(a, L, P, s, pdl);
        case 6: return launch_logits_t<6, 2, WT>(a, L, P, s, pdl);
        case 7: return launch_logits_t<7, 2, WT>(a, L, P, s, pdl);
        default: return launch_logits_t<8, 2, WT>(a, L, P, s, pdl);
    }
}

// Raise the dynamic shared-memory limit of every instantiation once (outside any graph capture).
template <int WT>
static cudaError_t prepare_wt() {
    cudaError_t e = cudaSuccess;
#define W4J_SET(...) \
    if (e == cudaSuccess) e = allow_dynamic_smem(__VA_ARGS__)
#define W4J_SET_MT(MT)                  \
    W4J_SET(k_gemv<MT, 1, WT>);         \
    W4J_SET(k_gemv<MT, (MT <= 4 ? 4 : 2), WT>)
    W4J_SET(k_gemv<1, 8, WT>);
    W4J_SET(k_gemv<2, 8, WT>);
    W4J_SET_MT(1);
    W4J_SET_MT(2);
    W4J_SET_MT(3);
    W4J_SET_MT(4);
    W4J_SET_MT(5);
    W4J_SET_MT(6);
    W4J_SET_MT(7);
    W4J_SET_MT(8);
    W4J_SET(k_logits<1, 4, WT>);
    W4J_SET(k_logits<2, 4, WT>);
    W4J_SET(k_logits<3, 4, WT>);
    W4J_SET(k_logits<4, 4, WT>);
    W4J_SET(k_logits<5, 2, WT>);
    W4J_SET(k_logits<6, 2, WT>);
    W4J_SET(k_logits<7, 2, WT>);
    W4J_SET(k_logits<8, 2, WT>);
#undef W4J_SET_MT
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
    if (a.topk > kLaneTopK) return cudaErrorInvalidValue;
    if (a.E.type == WT_F16) return dispatch_logits<WT_F16>(a, P, s, pdl);
    if (a.E.type == WT_Q8) return dispatch_logits<WT_Q8>(a, P, s, pdl);
    return cudaErrorInvalidValue;
}

}  // namespace w4j
