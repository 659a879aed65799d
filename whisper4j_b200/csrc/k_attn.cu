// k_attn.cu — single-query attention of the decode step over the device KV caches.
//
// Replaces MultiHeadAttention.fusedSingleTokenAttention (nn/MultiHeadAttention.java:110-132)
// -> fusedAttentionHead (java26 VectorSimdOps.java:137-203, scalar SimdOps.java:182-226):
//   s_j = (q . k_j) * (1/sqrt(64)),  p = softmax(s),  out = sum_j p_j v_j   per head,
// for self-attention over the growing cache and cross-attention over the encoder states
// (kvLen = n_audio_ctx), and the cache append of appendHeadsCache (:140-164), which here is
// an in-place row write done by the QKV kernel's epilogue.
//
// Flash-decoding: block (split, head, group) stages keys [j0, j1) of one head in shared memory
// (every tile before griddepcontrol.wait where the rows are already final) and runs an online
// softmax over them for every query of the group (cross-attention: all beams of one stream
// share its encoder K/V, so those bytes are read once per stream, not once per beam).  The
// split blocks of one (group, head) form a thread-block cluster: each leaves its partial
// (max, sum, o[64] per query) in its own shared memory and, after a cluster barrier, combines
// a slice of the output from all partials through distributed shared memory, in split order,
// so the result is deterministic and no partial goes through global memory.  Self-attention
// rows are gathered through the beam table (position -> physical slot), which replaces the
// reference's per-beam cache copies (WhisperDecoder.java:343-361).
#include "w4j_internal.cuh"

namespace w4j {

constexpr int kRowPad = 72;  // halves per shared K/V row (144 B: conflict-free 16-byte reads)
constexpr int kMaxNq = 8;
constexpr int kWarps = kAttnThreads / 32;
constexpr int kMaxSplits = 8;  // portable cluster size
constexpr int kTileHalves = 2 * kAttnKeyTile * kRowPad;  // one K tile + one V tile

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_cluster_f32(const float *local, unsigned rank) {
    unsigned remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}

// Dynamic shared memory: `tiles` K/V tile pairs of the block's key range.
// NQ queries per group (self-attention: 1; cross-attention: the beams of one stream).
template <int NQ>
__global__ void __launch_bounds__(kAttnThreads) k_attn(AttnArgs a) {
    extern __shared__ __align__(16) __half skv[];  // [tiles][K tile | V tile]; then reused for the reduction
    __shared__ __align__(16) float sq[NQ][kHeadDim];
    __shared__ float sp[NQ][kAttnKeyTile];
    __shared__ float s_m[NQ], s_l[NQ], s_alpha[NQ];
    __shared__ __align__(16) float s_part[NQ][kHeadDim];  // this split's unnormalised output (cluster mode)

    const int split = blockIdx.x, head = blockIdx.y, group = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // Positions, beam tables and liveness were written by the host or by an earlier graph
    // launch, never by a kernel of this launch's chain, so they are read before the wait.
    const bool live = !a.active || a.active[group];
    if (!live) return;  // uniform over the cluster (one group)
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
    // longest context); with a single one, the other blocks have nothing to do
    const int ns = a.cross ? a.nsplit : min(a.nsplit, max(1, (len + kAttnKeyTile - 1) / kAttnKeyTile));
    if (ns == 1 && split > 0) return;  // uniform over the cluster: no cluster barrier is reached
    const int j0 = split < ns ? (int)(((long long)split * len) / ns) : len;
    const int j1 = split < ns ? (int)(((long long)(split + 1) * len) / ns) : len;
    const float scale = 0.125f;  // (float)(1 / sqrt(64))

    // stage K and V rows [t0, t0 + nk) into tile pair `ti` (128 B each = 8 x 16 B); which: 0 all,
    // 1 all but the newest self row, 2 only the newest
    auto stage = [&](int ti, int t0, int nk, int which) {
        __half *tk = skv + (size_t)ti * kTileHalves, *tv = tk + kAttnKeyTile * kRowPad;
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
            cp_async16(&tk[r * kRowPad + part * 8], krow + part * 8);
            cp_async16(&tv[r * kRowPad + part * 8], vrow + part * 8);
        }
    };
    // Encoder K/V never change during a decode, and self rows older than the newest were
    // written by an earlier graph launch (a.self_prefetch): stage them now, so they stream in
    // while the previous kernel finishes.
    const int nt = (j1 - j0 + kAttnKeyTile - 1) / kAttnKeyTile;
    const bool pre = a.cross || a.self_prefetch;
    if (pre)
        for (int ti = 0; ti < nt; ++ti) stage(ti, j0 + ti * kAttnKeyTile, min(kAttnKeyTile, j1 - j0 - ti * kAttnKeyTile), a.cross ? 0 : 1);
    pdl_trigger();
    pdl_wait();
    for (int ti = 0; ti < nt; ++ti)  // the newest self row (written by the previous kernel), or everything
        stage(ti, j0 + ti * kAttnKeyTile, min(kAttnKeyTile, j1 - j0 - ti * kAttnKeyTile), pre ? 2 : 0);
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
    cp_async_wait_all();
    __syncthreads();

    for (int ti = 0; ti < nt; ++ti) {
        const int nk = min(kAttnKeyTile, j1 - j0 - ti * kAttnKeyTile);
        const __half *sk = skv + (size_t)ti * kTileHalves, *sv = sk + kAttnKeyTile * kRowPad;
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
    // cluster combine: this split's (max, sum, o) stay in shared memory; after the barrier,
    // block r produces the outputs (query, dim) with index = r (mod cluster size) from the
    // partials of all splits, read through distributed shared memory in split order
#pragma unroll
    for (int t = 0; t < kPer; ++t) {
        const int pidx = tid + kAttnThreads * t;
        if (pidx < NQ * kHeadDim) s_part[pidx / kHeadDim][pidx % kHeadDim] = o[t];
    }
    cluster_sync();
    const int cs = a.nsplit;  // cluster size = blocks along x
    for (int pidx = split + cs * tid; pidx < NQ * kHeadDim; pidx += cs * kAttnThreads) {
        const int i = pidx / kHeadDim, dd = pidx % kHeadDim;
        float ms[kMaxSplits], ls[kMaxSplits], os[kMaxSplits];
#pragma unroll
        for (int r = 0; r < kMaxSplits; ++r)
            if (r < ns) {
                ms[r] = ld_cluster_f32(&s_m[i], (unsigned)r);
                ls[r] = ld_cluster_f32(&s_l[i], (unsigned)r);
                os[r] = ld_cluster_f32(&s_part[i][dd], (unsigned)r);
            }
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < kMaxSplits; ++r)
            if (r < ns) M = fmaxf(M, ms[r]);
        float num = 0.f, den = 0.f;
#pragma unroll
        for (int r = 0; r < kMaxSplits; ++r)
            if (r < ns && ms[r] != -INFINITY) {
                const float w = __expf(ms[r] - M);
                num = fmaf(w, os[r], num);
                den = fmaf(w, ls[r], den);
            }
        a.out[(size_t)(group * NQ + i) * a.d + head * kHeadDim + dd] = num / den;
    }
    cluster_sync();  // no block leaves while its partial may still be read
}

// Key splits of one launch: up to kMaxSplits (one cluster); tiles each block stages.
int attn_max_splits(int) { return kMaxSplits; }
static int attn_tiles(const AttnArgs &a) {
    const int len_max = a.cross ? a.n_audio : a.n_ctx;
    const int per = (len_max + a.nsplit - 1) / a.nsplit;
    return (per + kAttnKeyTile - 1) / kAttnKeyTile;
}

template <int NQ>
static cudaError_t prep_nq() {
    return allow_dynamic_smem(k_attn<NQ>);
}

cudaError_t attn_prepare() {
    cudaError_t e = prep_nq<1>();
    if (e == cudaSuccess) e = prep_nq<2>();
    if (e == cudaSuccess) e = prep_nq<3>();
    if (e == cudaSuccess) e = prep_nq<4>();
    if (e == cudaSuccess) e = prep_nq<5>();
    if (e == cudaSuccess) e = prep_nq<6>();
    if (e == cudaSuccess) e = prep_nq<7>();
    if (e == cudaSuccess) e = prep_nq<8>();
    return e;
}

cudaError_t launch_attn(const AttnArgs &a, cudaStream_t s, bool pdl) {
    if (a.groups <= 0) return cudaSuccess;
    if (a.nq < 1 || a.nq > kMaxNq || a.nsplit < 1 || a.nsplit > kMaxSplits) return cudaErrorInvalidValue;
    const int tiles = attn_tiles(a);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.nsplit, a.n_head, a.groups);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = (size_t)tiles * kTileHalves * sizeof(__half);
    if (cfg.dynamicSmemBytes < (size_t)kWarps * kMaxNq * kHeadDim * sizeof(float))
        cfg.dynamicSmemBytes = (size_t)kWarps * kMaxNq * kHeadDim * sizeof(float);  // the reduction reuses it
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (a.nsplit > 1) {  // the split blocks of one (head, group) combine through a cluster
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = a.nsplit;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
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
