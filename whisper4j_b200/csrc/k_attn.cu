// k_attn.cu — single-query attention of the decode step over the device KV caches.
//
// Replaces MultiHeadAttention.fusedSingleTokenAttention (nn/MultiHeadAttention.java:110-132)
// -> fusedAttentionHead (java26 VectorSimdOps.java:137-203, scalar SimdOps.java:182-226):
//   s_j = (q . k_j) * (1/sqrt(64)),  p = softmax(s),  out = sum_j p_j v_j   per head,
// for self-attention over the growing cache and cross-attention over the encoder states
// (kvLen = n_audio_ctx), and the cache append of appendHeadsCache (:140-164), which here is
// an in-place row write done by the QKV kernel's epilogue.
//
// Flash-decoding: block (split, head, group) streams keys [j0, j1) of one head through
// shared memory in tiles of 128 rows with an online softmax, for every query of the group
// (cross-attention: all beams of one stream share its encoder K/V, so those bytes are read
// once per stream, not once per beam).  Per-split partial (max, sum, o[64]) go to scratch;
// the last split block of a (group, head) to finish combines them in split order, so the
// result is deterministic.  Self-attention rows are gathered through the beam table
// (position -> physical slot), which replaces the reference's per-beam cache copies
// (WhisperDecoder.java:343-361).
#include "w4j_internal.cuh"

namespace w4j {

constexpr int kRowPad = 72;  // halves per shared K/V row (144 B: conflict-free 16-byte reads)
constexpr int kMaxNq = 8;
constexpr int kWarps = kAttnThreads / 32;

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// NQ queries per group (self-attention: 1; cross-attention: the beams of one stream).
template <int NQ>
__global__ void __launch_bounds__(kAttnThreads) k_attn(AttnArgs a) {
    __shared__ __align__(16) __half skv[2 * kAttnKeyTile * kRowPad];  // K tile, V tile; reduction and combine staging
    __half *sk = skv, *sv = skv + kAttnKeyTile * kRowPad;
    __shared__ __align__(16) float sq[NQ][kHeadDim];
    __shared__ float sp[NQ][kAttnKeyTile];
    __shared__ float s_m[NQ], s_l[NQ], s_alpha[NQ];
    __shared__ int s_last;

    const int split = blockIdx.x, head = blockIdx.y, group = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // Positions, beam tables and liveness were written by the host or by an earlier graph
    // launch, never by a kernel of this launch's chain, so they are read before the wait.
    const bool live = !a.active || a.active[group];
    const __half *kbase = nullptr, *vbase = nullptr;
    if (a.cross) {
        const int stream = a.stream_of_group[group];
        const size_t off = (((size_t)stream * a.n_layer + a.layer) * a.n_head + head) * (size_t)a.n_audio * kHeadDim;
        kbase = a.kc + off;
        vbase = a.vc + off;
    }
    const int len = a.cross ? a.n_audio : a.pos[group] + 1;
    const int newest = a.cross ? -1 : len - 1;  // the row the previous kernel (QKV) writes
    // splits in use: one key tile each while the context is short (the grid is sized for the
    // longest context); blocks past them have nothing to do
    const int ns = a.cross ? a.nsplit : min(a.nsplit, max(1, (len + kAttnKeyTile - 1) / kAttnKeyTile));
    if (split >= ns) return;
    const int j0 = (int)(((long long)split * len) / ns), j1 = (int)(((long long)(split + 1) * len) / ns);
    const float scale = 0.125f;  // (float)(1 / sqrt(64))

    // stage K and V rows [t0, t0 + nk) (128 B each = 8 x 16 B); which: 0 all, 1 all but the
    // newest self row, 2 only the newest
    auto stage = [&](int t0, int nk, int which) {
        for (int c = tid; c < nk * 8; c += kAttnThreads) {
            const int r = c >> 3, part = c & 7;
            const int p = t0 + r;
            if ((which == 1 && p == newest) || (which == 2 && p != newest)) continue;
            const __half *krow, *vrow;
            if (a.cross) {
                krow = kbase + (size_t)p * kHeadDim;
                vrow = vbase + (size_t)p * kHeadDim;
            } else {
                const int slot = a.table ? a.table[(size_t)group * a.n_ctx + p] : a.seq_slot[group];
                const size_t off = ((((size_t)slot * a.n_layer + a.layer) * a.n_head + head) * (size_t)a.n_ctx + p) * kHeadDim;
                krow = a.kc + off;
                vrow = a.vc + off;
            }
            cp_async16(&sk[r * kRowPad + part * 8], krow + part * 8);
            cp_async16(&sv[r * kRowPad + part * 8], vrow + part * 8);
        }
    };
    // Encoder K/V never change during a decode, and self rows older than the newest were
    // written by an earlier graph launch (a.self_prefetch): stage the first tile now, so it
    // streams in while the previous kernel finishes.
    const bool pre = live && j1 > j0 && (a.cross || a.self_prefetch);
    if (pre) stage(j0, min(kAttnKeyTile, j1 - j0), a.cross ? 0 : 1);
    pdl_trigger();
    pdl_wait();
    if (!live) {
        cp_async_wait_all();
        return;
    }
    // the newest self row (written by the previous kernel) streams in with the queries
    if (pre && !a.cross) stage(j0, min(kAttnKeyTile, j1 - j0), 2);
    if (tid < NQ * kHeadDim / 4) {  // queries: one 16-byte load per thread
        const int i = tid / (kHeadDim / 4), c = tid % (kHeadDim / 4);
        reinterpret_cast<float4 *>(sq[i])[c] =
            reinterpret_cast<const float4 *>(a.q + (size_t)(group * NQ + i) * a.d + head * kHeadDim)[c];
    }
    if (tid < NQ) {
        s_m[tid] = -INFINITY;
        s_l[tid] = 0.f;
    }
    // output accumulators: warp w sums the keys j = w (mod kWarps) of every tile for dims
    // 2*lane, 2*lane+1 of every query; the warp shares are added at the end
    float ow[NQ][2];
#pragma unroll
    for (int i = 0; i < NQ; ++i) ow[i][0] = ow[i][1] = 0.f;
    __syncthreads();

    for (int t0 = j0; t0 < j1; t0 += kAttnKeyTile) {
        const int nk = min(kAttnKeyTile, j1 - t0);
        if (t0 != j0 || !pre) stage(t0, nk, 0);
        cp_async_wait_all();
        __syncthreads();
        {  // scores: two threads per key, 32 dims each
            const int key = tid >> 1, hf = tid & 1;
            float acc[NQ];
#pragma unroll
            for (int i = 0; i < NQ; ++i) acc[i] = 0.f;
            if (key < nk) {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint4 u = *reinterpret_cast<const uint4 *>(&sk[key * kRowPad + hf * 32 + c * 8]);
                    const __half2 *h = reinterpret_cast<const __half2 *>(&u);
                    float kf[8];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 f = __half22float2(h[j]);
                        kf[2 * j] = f.x;
                        kf[2 * j + 1] = f.y;
                    }
#pragma unroll
                    for (int i = 0; i < NQ; ++i) {
                        const float4 q0 = *reinterpret_cast<const float4 *>(&sq[i][hf * 32 + c * 8]);
                        const float4 q1 = *reinterpret_cast<const float4 *>(&sq[i][hf * 32 + c * 8 + 4]);
                        acc[i] = fmaf(q0.x, kf[0], acc[i]);
                        acc[i] = fmaf(q0.y, kf[1], acc[i]);
                        acc[i] = fmaf(q0.z, kf[2], acc[i]);
                        acc[i] = fmaf(q0.w, kf[3], acc[i]);
                        acc[i] = fmaf(q1.x, kf[4], acc[i]);
                        acc[i] = fmaf(q1.y, kf[5], acc[i]);
                        acc[i] = fmaf(q1.z, kf[6], acc[i]);
                        acc[i] = fmaf(q1.w, kf[7], acc[i]);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < NQ; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], 1);
            if (key < nk && hf == 0)
#pragma unroll
                for (int i = 0; i < NQ; ++i) sp[i][key] = acc[i] * scale;
        }
        __syncthreads();
        // online softmax bookkeeping: warp i takes query i
        for (int i = warp; i < NQ; i += kWarps) {
            float mx = -INFINITY;
            for (int j = lane; j < nk; j += 32) mx = fmaxf(mx, sp[i][j]);
            mx = warp_max(mx);
            const float m_old = s_m[i];
            const float m_new = fmaxf(m_old, mx);
            float sum = 0.f;
            for (int j = lane; j < nk; j += 32) {
                const float e = __expf(sp[i][j] - m_new);
                sp[i][j] = e;
                sum += e;
            }
            sum = warp_sum(sum);
            if (lane == 0) {
                const float alpha = m_old == -INFINITY ? 0.f : __expf(m_old - m_new);
                s_alpha[i] = alpha;
                s_l[i] = s_l[i] * alpha + sum;
                s_m[i] = m_new;
            }
        }
        __syncthreads();
        // o = o * alpha + p . V  (this warp's keys, two dims per lane)
#pragma unroll
        for (int i = 0; i < NQ; ++i) {
            const float al = s_alpha[i];
            ow[i][0] *= al;
            ow[i][1] *= al;
        }
        for (int j = warp; j < nk; j += kWarps) {
            const float2 v = __half22float2(*reinterpret_cast<const __half2 *>(&sv[j * kRowPad + 2 * lane]));
#pragma unroll
            for (int i = 0; i < NQ; ++i) {
                const float p = sp[i][j];
                ow[i][0] = fmaf(p, v.x, ow[i][0]);
                ow[i][1] = fmaf(p, v.y, ow[i][1]);
            }
        }
        __syncthreads();
    }
    // add the warp shares (through the K/V tiles' shared memory, no longer needed)
    float *red = reinterpret_cast<float *>(skv);  // [kWarps][NQ][64]
#pragma unroll
    for (int i = 0; i < NQ; ++i)
        *reinterpret_cast<float2 *>(&red[((size_t)warp * NQ + i) * kHeadDim + 2 * lane]) = make_float2(ow[i][0], ow[i][1]);
    __syncthreads();
    constexpr int kPer = (NQ * kHeadDim + kAttnThreads - 1) / kAttnThreads;  // (query, dim) pairs per thread
    float o[kPer];
#pragma unroll
    for (int t = 0; t < kPer; ++t) {
        const int pidx = tid + kAttnThreads * t;
        o[t] = 0.f;
        if (pidx < NQ * kHeadDim)
#pragma unroll
            for (int w = 0; w < kWarps; ++w) o[t] += red[(size_t)w * NQ * kHeadDim + pidx];
    }
    if (ns == 1) {
#pragma unroll
        for (int t = 0; t < kPer; ++t) {
            const int pidx = tid + kAttnThreads * t;
            const int i = pidx / kHeadDim, dd = pidx % kHeadDim;
            if (pidx < NQ * kHeadDim) a.out[(size_t)(group * NQ + i) * a.d + head * kHeadDim + dd] = o[t] / s_l[i];
        }
        return;
    }
    // partial record (m, l, o[64], pad) of this split
    auto rec = [&](int i, int sp_) {
        return a.part + ((((size_t)(group * NQ + i)) * a.n_head + head) * a.nsplit + sp_) * kAttnRec;
    };
#pragma unroll
    for (int t = 0; t < kPer; ++t) {
        const int pidx = tid + kAttnThreads * t;
        const int i = pidx / kHeadDim, dd = pidx % kHeadDim;
        if (pidx < NQ * kHeadDim) {
            float *pp = rec(i, split);
            pp[4 + dd] = o[t];
            if (dd == 0) {
                pp[0] = s_m[i];
                pp[1] = s_l[i];
            }
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        unsigned *ctr = a.counters + (size_t)group * a.n_head + head;
        const unsigned prev = atomicAdd(ctr, 1u);
        s_last = prev == (unsigned)(ns - 1);
        if (s_last) *ctr = 0u;  // ready for the next use of the counter
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // every split's record of this (group, head): one round of independent 16-byte L2 loads
    float *stg = reinterpret_cast<float *>(skv);  // [NQ][ns][kAttnRec]
    constexpr int kR4 = kAttnRec / 4;
    const int n4 = ns * kR4;
    for (int e0 = tid; e0 < n4; e0 += kAttnThreads * 2) {
        float4 v[NQ][2];
#pragma unroll
        for (int i = 0; i < NQ; ++i)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int e = e0 + kAttnThreads * j;
                if (e < n4) v[i][j] = __ldcg(reinterpret_cast<const float4 *>(rec(i, 0)) + e);
            }
#pragma unroll
        for (int i = 0; i < NQ; ++i)
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int e = e0 + kAttnThreads * j;
                if (e < n4) reinterpret_cast<float4 *>(stg + (size_t)i * ns * kAttnRec)[e] = v[i][j];
            }
    }
    __syncthreads();
    // per query: the split weights exp(m_s - M) (in split order) and the denominator, once
    float *wts = stg + (size_t)NQ * ns * kAttnRec;  // [NQ][ns + 1]
    for (int i = warp; i < NQ; i += kWarps) {
        const float *base = stg + (size_t)i * ns * kAttnRec;
        float M = -INFINITY;
        for (int s2 = lane; s2 < ns; s2 += 32) M = fmaxf(M, base[s2 * kAttnRec]);
        M = warp_max(M);
        float den = 0.f;
        for (int s2 = lane; s2 < ns; s2 += 32) {
            const float ms = base[s2 * kAttnRec];
            const float w = ms == -INFINITY ? 0.f : __expf(ms - M);
            wts[i * (ns + 1) + s2] = w;
            den = fmaf(w, base[s2 * kAttnRec + 1], den);
        }
        den = warp_sum(den);
        if (lane == 0) wts[i * (ns + 1) + ns] = den;
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < kPer; ++t) {
        const int pidx = tid + kAttnThreads * t;
        const int i = pidx / kHeadDim, dd = pidx % kHeadDim;
        if (pidx >= NQ * kHeadDim) continue;
        const float *base = stg + (size_t)i * ns * kAttnRec;
        const float *w = wts + i * (ns + 1);
        float num = 0.f;
        for (int s2 = 0; s2 < ns; ++s2) num = fmaf(w[s2], base[s2 * kAttnRec + 4 + dd], num);
        a.out[(size_t)(group * NQ + i) * a.d + head * kHeadDim + dd] = num / w[ns];
    }
}

cudaError_t attn_prepare() {
    cudaError_t e = prefer_max_smem(k_attn<1>);
    if (e == cudaSuccess) e = prefer_max_smem(k_attn<2>);
    if (e == cudaSuccess) e = prefer_max_smem(k_attn<3>);
    if (e == cudaSuccess) e = prefer_max_smem(k_attn<4>);
    if (e == cudaSuccess) e = prefer_max_smem(k_attn<5>);
    if (e == cudaSuccess) e = prefer_max_smem(k_attn<6>);
    if (e == cudaSuccess) e = prefer_max_smem(k_attn<7>);
    if (e == cudaSuccess) e = prefer_max_smem(k_attn<8>);
    return e;
}

// Splits whose records (and the per-query weights) fit the combine's staging in the K/V tiles.
int attn_max_splits(int nq) {
    return (int)((2 * kAttnKeyTile * kRowPad * sizeof(__half) / sizeof(float)) / (nq * (kAttnRec + 1) + 1));
}

cudaError_t launch_attn(const AttnArgs &a, cudaStream_t s, bool pdl) {
    if (a.groups <= 0) return cudaSuccess;
    if (a.nq < 1 || a.nq > kMaxNq || a.nsplit > attn_max_splits(a.nq)) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.nsplit, a.n_head, a.groups);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    switch (a.nq) {
        case 1: return cudaLaunchKernelEx(&cfg, k_attn<1>, a);
        case 2: return cudaLaunchKernelEx(&cfg, k_attn<2>, a);
        case 3: return cudaLaunchKernelEx(&cfg, k_attn<3>, a);
        case 4: return cudaLaunchKernelEx(&cfg, k_attn<4>, a);
        case 5: return cudaLaunchKernelEx(&cfg, k_attn<5>, a);
        case 6: return cudaLaunchKernelEx(&cfg, k_attn<6>, a);
        case 7: return cudaLaunchKernelEx(&cfg, k_attn<7>, a);
        default: return cudaLaunchKernelEx(&cfg, k_attn<8>, a);
    }
}

}  // namespace w4j
