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

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__global__ void __launch_bounds__(kAttnThreads) k_attn(AttnArgs a) {
    __shared__ __align__(16) __half skv[2 * kAttnKeyTile * kRowPad];  // K tile, V tile; combine staging
    __half *sk = skv, *sv = skv + kAttnKeyTile * kRowPad;
    __shared__ __align__(16) float sq[kMaxNq][kHeadDim];
    __shared__ float sp[kMaxNq][kAttnKeyTile];
    __shared__ float s_m[kMaxNq], s_l[kMaxNq], s_alpha[kMaxNq];
    __shared__ int s_last;

    const int split = blockIdx.x, head = blockIdx.y, group = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nq = a.nq;

    // Positions, beam tables and liveness were written by the host or by an earlier graph
    // launch, never by the kernel this one waits on, so they are read before the wait.
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
    const int j0 = (int)(((long long)split * len) / a.nsplit), j1 = (int)(((long long)(split + 1) * len) / a.nsplit);
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

    {  // queries: all loads issued before any is used
        constexpr int kQ = kMaxNq * kHeadDim / kAttnThreads;
        float qv[kQ];
#pragma unroll
        for (int t = 0; t < kQ; ++t) {
            const int i = tid + kAttnThreads * t;
            qv[t] = i < nq * kHeadDim
                        ? a.q[(size_t)(group * nq + i / kHeadDim) * a.d + head * kHeadDim + i % kHeadDim]
                        : 0.f;
        }
#pragma unroll
        for (int t = 0; t < kQ; ++t) {
            const int i = tid + kAttnThreads * t;
            if (i < nq * kHeadDim) sq[i / kHeadDim][i % kHeadDim] = qv[t];
        }
    }
    if (tid < kMaxNq) {
        s_m[tid] = -INFINITY;
        s_l[tid] = 0.f;
    }
    // output accumulators: warp w sums the keys j = w (mod 4) of every tile for dims
    // 2*lane, 2*lane+1 of every query; the four warp shares are added at the end
    float ow[kMaxNq][2];
#pragma unroll
    for (int i = 0; i < kMaxNq; ++i) ow[i][0] = ow[i][1] = 0.f;
    constexpr int kPairsPerThread = kMaxNq * kHeadDim / kAttnThreads;
    __syncthreads();

    for (int t0 = j0; t0 < j1; t0 += kAttnKeyTile) {
        const int nk = min(kAttnKeyTile, j1 - t0);
        if (t0 == j0 && pre) {
            if (!a.cross) stage(t0, nk, 2);  // the newest row, now written
        } else {
            stage(t0, nk, 0);
        }
        cp_async_wait_all();
        __syncthreads();
        // scores: thread per key
        if (tid < nk) {
            float kf[kHeadDim];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint4 u = *reinterpret_cast<const uint4 *>(&sk[tid * kRowPad + c * 8]);
                const __half2 *h = reinterpret_cast<const __half2 *>(&u);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 f = __half22float2(h[j]);
                    kf[c * 8 + 2 * j] = f.x;
                    kf[c * 8 + 2 * j + 1] = f.y;
                }
            }
            float acc[kMaxNq];
#pragma unroll
            for (int i = 0; i < kMaxNq; ++i) acc[i] = 0.f;
#pragma unroll
            for (int dd = 0; dd < kHeadDim; dd += 4) {
#pragma unroll
                for (int i = 0; i < kMaxNq; ++i) {
                    if (i < nq) {  // independent chains per query
                        const float4 q4 = *reinterpret_cast<const float4 *>(&sq[i][dd]);
                        acc[i] = fmaf(q4.x, kf[dd], acc[i]);
                        acc[i] = fmaf(q4.y, kf[dd + 1], acc[i]);
                        acc[i] = fmaf(q4.z, kf[dd + 2], acc[i]);
                        acc[i] = fmaf(q4.w, kf[dd + 3], acc[i]);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < kMaxNq; ++i)
                if (i < nq) sp[i][tid] = acc[i] * scale;
        }
        __syncthreads();
        // online softmax bookkeeping: warp w takes queries w, w+4
        for (int i = warp; i < nq; i += kAttnThreads / 32) {
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
        for (int i = 0; i < kMaxNq; ++i) {
            const float al = i < nq ? s_alpha[i] : 0.f;
            ow[i][0] *= al;
            ow[i][1] *= al;
        }
        for (int j = warp; j < nk; j += kAttnThreads / 32) {
            const float2 v = __half22float2(*reinterpret_cast<const __half2 *>(&sv[j * kRowPad + 2 * lane]));
#pragma unroll
            for (int i = 0; i < kMaxNq; ++i) {
                if (i < nq) {
                    const float p = sp[i][j];
                    ow[i][0] = fmaf(p, v.x, ow[i][0]);
                    ow[i][1] = fmaf(p, v.y, ow[i][1]);
                }
            }
        }
        __syncthreads();
    }
    // add the four warp shares (through the K tile's shared memory, no longer needed)
    float *red = reinterpret_cast<float *>(sk);  // [4][kMaxNq][64]
#pragma unroll
    for (int i = 0; i < kMaxNq; ++i) {
        if (i < nq) {
            red[((size_t)warp * kMaxNq + i) * kHeadDim + 2 * lane] = ow[i][0];
            red[((size_t)warp * kMaxNq + i) * kHeadDim + 2 * lane + 1] = ow[i][1];
        }
    }
    __syncthreads();
    float o[kPairsPerThread];
#pragma unroll
    for (int t = 0; t < kPairsPerThread; ++t) {
        const int pidx = tid + kAttnThreads * t;
        const int i = pidx / kHeadDim, dd = pidx % kHeadDim;
        o[t] = 0.f;
        if (i < nq)
#pragma unroll
            for (int w = 0; w < kAttnThreads / 32; ++w) o[t] += red[((size_t)w * kMaxNq + i) * kHeadDim + dd];
    }
    __syncthreads();  // `red` aliases the staging area used by the combine below

    if (a.nsplit == 1) {
#pragma unroll
        for (int t = 0; t < kPairsPerThread; ++t) {
            const int pidx = tid + kAttnThreads * t;
            const int i = pidx / kHeadDim, dd = pidx % kHeadDim;
            if (i < nq) a.out[(size_t)(group * nq + i) * a.d + head * kHeadDim + dd] = o[t] / s_l[i];
        }
        return;
    }
    // partial (m, l, o[64]) of this split
#pragma unroll
    for (int t = 0; t < kPairsPerThread; ++t) {
        const int pidx = tid + kAttnThreads * t;
        const int i = pidx / kHeadDim, dd = pidx % kHeadDim;
        if (i < nq) {
            float *pp = a.part + ((((size_t)(group * nq + i)) * a.n_head + head) * a.nsplit + split) * (2 + kHeadDim);
            pp[2 + dd] = o[t];
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
        s_last = prev == (unsigned)(a.nsplit - 1);
        if (s_last) *ctr = 0u;  // ready for the next use of the counter
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // stage every split's partial of this (group, head) in shared memory with one round of
    // independent L2 loads, then combine in split order
    constexpr int per = 2 + kHeadDim;
    float *stg = reinterpret_cast<float *>(skv);
    const int span = a.nsplit * per;
    for (int e = tid; e < nq * span; e += kAttnThreads) {
        const int i = e / span, rest = e - i * span;
        stg[e] = __ldcg(a.part + ((((size_t)(group * nq + i)) * a.n_head + head) * a.nsplit) * per + rest);
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < kPairsPerThread; ++t) {
        const int pidx = tid + kAttnThreads * t;
        const int i = pidx / kHeadDim, dd = pidx % kHeadDim;
        if (i >= nq) continue;
        const float *base = stg + (size_t)i * span;
        float M = -INFINITY;
        for (int s = 0; s < a.nsplit; ++s) M = fmaxf(M, base[s * per]);
        float num = 0.f, den = 0.f;
        for (int s = 0; s < a.nsplit; ++s) {
            const float *pp = base + s * per;
            const float ms = pp[0];
            if (ms == -INFINITY) continue;
            const float w = __expf(ms - M);
            num = fmaf(w, pp[2 + dd], num);
            den = fmaf(w, pp[1], den);
        }
        a.out[(size_t)(group * nq + i) * a.d + head * kHeadDim + dd] = num / den;
    }
}

int attn_max_splits(int nq) { return (2 * kAttnKeyTile * kRowPad * 2 / 4) / ((2 + kHeadDim) * nq); }

cudaError_t launch_attn(const AttnArgs &a, cudaStream_t s, bool pdl) {
    if (a.groups <= 0) return cudaSuccess;
    if (a.nq < 1 || a.nq > kMaxNq) return cudaErrorInvalidValue;
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
    return cudaLaunchKernelEx(&cfg, k_attn, a);
}

}  // namespace w4j
