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
#include "attn_tile.cuh"
#include "tc_common.cuh"
#include "w4j_internal.cuh"

namespace w4j {

constexpr int kRowPad = 72;  // halves per shared K/V row (144 B: conflict-free 16-byte reads)
constexpr int kMaxNq = 8;
constexpr int kWarps = kAttnThreads / 32;
constexpr int kMaxSplits = 8;  // portable cluster size
constexpr int kTileHalves = 2 * kAttnKeyTile * kRowPad;  // one K tile + one V tile

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

// One key tile of the online softmax for NQ queries: scores S^T = K . Q^T and O^T += V^T . P^T on
// warp-level tensor cores (warp w owns keys [16 w, 16 w + 16) of the tile); s_m / s_l carry the
// running max and denominator per query, of[4][4] this warp's O^T fragments.
struct AttnShared {
    __half (*qh)[kHeadDim + 8];       // queries (f16; rows >= NQ zero): MMA B operand
    __half (*ps)[kAttnKeyTile + 8];   // probabilities of the tile (f16): MMA B operand
    float (*w_max)[8], (*w_sum)[8];   // per-warp max / sum per query
    float *s_m, *s_l;                 // running max / denominator per query
};

// Barrier of the 256 threads that run one tile: the block (id 0) or a named barrier of one
// warpgroup pair (ids 1, 2).
__device__ __forceinline__ void group_sync(int bar) {
    if (bar == 0) __syncthreads();
    else asm volatile("bar.sync %0, %1;" ::"r"(bar), "n"(kAttnThreads) : "memory");
}

// gtid: the thread's index among the kAttnThreads threads running the tile; bar: their barrier.
// kpos0: position of the tile's first key; keys with mk.x <= position < mk.y are masked.
template <int NQ>
__device__ __forceinline__ void attn_tile(const AttnShared &sh, const __half *sk, const __half *sv, int nk,
                                          float (&of)[4][4], int gtid, int bar, int kpos0, int2 mk) {
    const int tid = gtid, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, tq = lane & 3;
    const float scale = 0.125f;  // (float)(1 / sqrt(64))
    __half (*qh)[kHeadDim + 8] = sh.qh;
    __half (*ps)[kAttnKeyTile + 8] = sh.ps;
    float (*w_max)[8] = sh.w_max, (*w_sum)[8] = sh.w_sum;
    float *s_m = sh.s_m, *s_l = sh.s_l;
    const int kb = 16 * warp;  // this warp's first key of the tile
    // scores S^T (16 keys x 8 queries) = K (16 x 64) . Q^T (64 x 8): four k16 steps
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
    if (kb < nk) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t af[4], bf[2];
            ldsm_x4(af, &sk[(kb + (lane & 15)) * kRowPad + 16 * kk + (lane >> 4) * 8]);
            ldsm_x2(bf, &qh[lane & 7][16 * kk + ((lane >> 3) & 1) * 8]);
            mma_16816(sc, af, bf);
        }
    }
    // c0: (key kb+g, query 2tq), c1: (kb+g, 2tq+1), c2: (kb+g+8, 2tq), c3: (kb+g+8, 2tq+1)
    const int q0 = 2 * tq, q1 = 2 * tq + 1;
    const int kp0 = kpos0 + kb + g, kp1 = kp0 + 8;
    const bool k0ok = kb + g < nk && !(kp0 >= mk.x && kp0 < mk.y);
    const bool k1ok = kb + g + 8 < nk && !(kp1 >= mk.x && kp1 < mk.y);
    sc[0] = (k0ok && q0 < NQ) ? sc[0] * scale : -INFINITY;
    sc[1] = (k0ok && q1 < NQ) ? sc[1] * scale : -INFINITY;
    sc[2] = (k1ok && q0 < NQ) ? sc[2] * scale : -INFINITY;
    sc[3] = (k1ok && q1 < NQ) ? sc[3] * scale : -INFINITY;
    // online softmax over the tile's keys, per query (lanes with the same tq share queries)
    float mx0 = fmaxf(sc[0], sc[2]), mx1 = fmaxf(sc[1], sc[3]);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    if (g == 0) {
        w_max[warp][q0] = mx0;
        w_max[warp][q1] = mx1;
    }
    group_sync(bar);
    float tm0 = -INFINITY, tm1 = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
        tm0 = fmaxf(tm0, w_max[w][q0]);
        tm1 = fmaxf(tm1, w_max[w][q1]);
    }
    const float mo0 = s_m[q0], mo1 = s_m[q1];
    const float mn0 = fmaxf(mo0, tm0), mn1 = fmaxf(mo1, tm1);
    const float p0 = sc[0] == -INFINITY ? 0.f : __expf(sc[0] - mn0);
    const float p1 = sc[1] == -INFINITY ? 0.f : __expf(sc[1] - mn1);
    const float p2 = sc[2] == -INFINITY ? 0.f : __expf(sc[2] - mn0);
    const float p3 = sc[3] == -INFINITY ? 0.f : __expf(sc[3] - mn1);
    float sm0 = p0 + p2, sm1 = p1 + p3;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        sm0 += __shfl_xor_sync(0xffffffffu, sm0, o);
        sm1 += __shfl_xor_sync(0xffffffffu, sm1, o);
    }
    if (g == 0) {
        w_sum[warp][q0] = sm0;
        w_sum[warp][q1] = sm1;
    }
    // P^T of this warp's keys for the P.V step (read back only by this warp)
    ps[q0][kb + g] = __float2half_rn(p0);
    ps[q1][kb + g] = __float2half_rn(p1);
    ps[q0][kb + g + 8] = __float2half_rn(p2);
    ps[q1][kb + g + 8] = __float2half_rn(p3);
    const float al0 = mo0 == -INFINITY ? 0.f : __expf(mo0 - mn0);
    const float al1 = mo1 == -INFINITY ? 0.f : __expf(mo1 - mn1);
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
        of[mt][0] *= al0;
        of[mt][1] *= al1;
        of[mt][2] *= al0;
        of[mt][3] *= al1;
    }
    __syncwarp();
    // O^T (16 dims x 8 queries, 4 tiles) += V^T (16 dims x 16 keys) . P^T (16 keys x 8 queries)
    if (kb < nk) {
        uint32_t bf[2];
        ldsm_x2(bf, &ps[lane & 7][kb + ((lane >> 3) & 1) * 8]);
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
            uint32_t af[4];
            ldsm_x4_t(af, &sv[(kb + (lane & 7) + ((lane >> 4) & 1) * 8) * kRowPad + 16 * mt + ((lane >> 3) & 1) * 8]);
            mma_16816(of[mt], af, bf);
        }
    }
    group_sync(bar);  // w_max / w_sum read; s_m read by every thread
    if (tid < 8) {    // running max and denominator per query
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) tot += w_sum[w][tid];
        const float mo = s_m[tid];
        float tmx = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) tmx = fmaxf(tmx, w_max[w][tid]);
        const float mn = fmaxf(mo, tmx);
        s_l[tid] = s_l[tid] * (mo == -INFINITY ? 0.f : __expf(mo - mn)) + tot;
        s_m[tid] = mn;
    }
    group_sync(bar);
}

// Dynamic shared memory: `tiles` K/V tile pairs of the block's key range.
// NQ queries per group (self-attention: 1; cross-attention: the beams of one stream).
template <int NQ>
__global__ void __launch_bounds__(kAttnThreads) k_attn(AttnArgs a) {
    extern __shared__ __align__(16) __half skv[];  // [tiles][K tile | V tile]; then reused for the reduction
    constexpr int kQPad = kHeadDim + 8, kPPad = kAttnKeyTile + 8;  // halves per row (16-byte aligned rows)
    __shared__ __align__(16) __half qh[8][kQPad];        // queries (f16; rows >= NQ zero): MMA B operand
    __shared__ __align__(16) __half ps[8][kPPad];        // probabilities of the tile (f16): MMA B operand
    __shared__ float w_max[kWarps][8], w_sum[kWarps][8];
    __shared__ float s_m[8], s_l[8];
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
    const int len = a.cross ? a.n_audio : a.kv_len ? a.kv_len[group] : a.pos[group] + 1;
    // a multi-token pass masks keys [lo, hi) of this query (the causal mask from key column 0)
    const int2 mk = (!a.cross && a.mask) ? a.mask[group] : make_int2(0, 0);
    const int newest = a.cross ? -1 : len - 1;  // the row the previous kernel (QKV) writes
    // splits in use: one key tile each while the context is short (the grid is sized for the
    // longest context); with a single one, the other blocks have nothing to do
    const int ns = a.cross ? a.nsplit : min(a.nsplit, max(1, (len + kAttnKeyTile - 1) / kAttnKeyTile));
    if (ns == 1 && split > 0) return;  // uniform over the cluster: no cluster barrier is reached
    const int j0 = split < ns ? (int)(((long long)split * len) / ns) : len;
    const int j1 = split < ns ? (int)(((long long)(split + 1) * len) / ns) : len;

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
    if (tid < 8 * kHeadDim / 4) {  // queries as f16, one 16-byte load per thread; rows >= NQ are zero
        const int i = tid / (kHeadDim / 4), c = tid % (kHeadDim / 4);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < NQ) v = reinterpret_cast<const float4 *>(a.q + (size_t)(group * NQ + i) * a.d + head * kHeadDim)[c];
        const __half2 h0 = __floats2half2_rn(v.x, v.y), h1 = __floats2half2_rn(v.z, v.w);
        *reinterpret_cast<uint2 *>(&qh[i][4 * c]) =
            make_uint2(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1));
    }
    if (tid < 8) {
        s_m[tid] = -INFINITY;
        s_l[tid] = 0.f;
    }
    // warp w owns keys [16 w, 16 w + 16) of every tile; MMA fragment coordinates
    const int g = lane >> 2, tq = lane & 3;
    // O^T accumulators: 4 tiles of 16 dims x 8 queries (c0/c1: dim 16 mt + g, queries 2 tq / 2 tq + 1;
    // c2/c3: dim 16 mt + g + 8)
    float of[4][4];
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) of[mt][0] = of[mt][1] = of[mt][2] = of[mt][3] = 0.f;
    // V rows past the keys of a partial tile are zeroed: the P.V product multiplies them by
    // zero probabilities, which must not meet stale (possibly non-finite) shared memory
    for (int ti = 0; ti < nt; ++ti) {
        const int nk = min(kAttnKeyTile, j1 - j0 - ti * kAttnKeyTile);
        __half *tv = skv + (size_t)ti * kTileHalves + kAttnKeyTile * kRowPad;
        for (int c = tid; c < (kAttnKeyTile - nk) * 8; c += kAttnThreads)
            *reinterpret_cast<uint4 *>(&tv[(nk + (c >> 3)) * kRowPad + (c & 7) * 8]) = make_uint4(0u, 0u, 0u, 0u);
    }
    cp_async_wait_all();
    __syncthreads();

    const AttnShared sh{qh, ps, w_max, w_sum, s_m, s_l};
    for (int ti = 0; ti < nt; ++ti) {
        const int nk = min(kAttnKeyTile, j1 - j0 - ti * kAttnKeyTile);
        const __half *sk = skv + (size_t)ti * kTileHalves, *sv = sk + kAttnKeyTile * kRowPad;
        attn_tile<NQ>(sh, sk, sv, nk, of, tid, 0, j0 + ti * kAttnKeyTile, mk);
    }
    // add the warp shares (through the K/V tiles' shared memory, no longer needed)
    float *red = reinterpret_cast<float *>(skv);  // [kWarps][NQ][64]
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
        const int q0 = 2 * tq, q1 = 2 * tq + 1, d0 = 16 * mt + g;
        if (q0 < NQ) {
            red[((size_t)warp * NQ + q0) * kHeadDim + d0] = of[mt][0];
            red[((size_t)warp * NQ + q0) * kHeadDim + d0 + 8] = of[mt][2];
        }
        if (q1 < NQ) {
            red[((size_t)warp * NQ + q1) * kHeadDim + d0] = of[mt][1];
            red[((size_t)warp * NQ + q1) * kHeadDim + d0 + 8] = of[mt][3];
        }
    }
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

// ---------------------------------------------------------------------------
// Streaming cross-attention for many (group, head) pairs (batched greedy / beam decoding).
// One block per SM walks the pairs round-robin.  Its two warpgroups of 256 threads take the
// even and the odd 128-key tiles of a pair.  Each warpgroup streams its tiles through three
// buffers with TMA (cp.async.bulk.tensor.2d over the cross K and V caches viewed as
// [rows][64] f16, 128-byte swizzle: chunk c of row r lands at c ^ (r & 7), so ldmatrix reads are
// conflict-free), completed through an mbarrier per buffer and released through a second one
// that every warp arrives on; the first three tiles are requested before griddepcontrol.wait,
// then one thread refills a buffer as soon as all eight warps are done with it, so two tiles
// are in flight while one is computed, across pair boundaries.  Every warp keeps its own
// online-softmax state over its 16 keys of each tile; at the end of a pair the 16 warp states
// are combined in shared memory in a fixed order, so no partial leaves the SM and the result does
// not depend on timing.  Needs n_audio > 128 (a tile for each warpgroup in every pair: both meet
// at the block barrier that ends a pair).
// ---------------------------------------------------------------------------
template <int NQ>
__global__ void __launch_bounds__(kStreamThreads, 1)
    k_attn_stream(AttnArgs a, const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap) {
    extern __shared__ __align__(1024) unsigned char sraw[];
    // [warpgroup][kStreamBufs][K tile | V tile], 1024-byte aligned for the 128-byte swizzle
    __half *sbuf = reinterpret_cast<__half *>(sraw + ((1024u - (smem_u32(sraw) & 1023u)) & 1023u));
    __shared__ __align__(8) uint64_t full[2][kStreamBufs], empty[2][kStreamBufs];
    __shared__ __align__(16) __half qh[2][8][kHeadDim + 8];
    __shared__ __align__(16) __half pw[2 * kWarps][8][kPwPad];
    __shared__ float wm[2 * kWarps][8], wl[2 * kWarps][8];
    __shared__ __align__(16) float red[2 * kWarps][NQ * kHeadDim];
    const int tid = threadIdx.x, wg = tid / kAttnThreads, gtid = tid % kAttnThreads;
    const int warp = tid >> 5, gwarp = gtid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
    const int H = a.n_head, A = a.n_audio;
    const int n_pairs = a.groups * H, G = gridDim.x;
    const int n_tiles = (A + kAttnKeyTile - 1) / kAttnKeyTile;
    const int my_tiles = (n_tiles - wg + 1) / 2;  // tiles wg, wg + 2, ... of every pair
    const int my_pairs = blockIdx.x < n_pairs ? (n_pairs - 1 - blockIdx.x) / G + 1 : 0;
    const int n_items = my_pairs * my_tiles;
    __half *wbuf = sbuf + (size_t)wg * kStreamBufs * kStreamTile;
    const bool producer = gwarp == 0 && lane == 0;  // one thread per warpgroup requests its tiles

    // stream liveness and stream of each group: written by the host or an earlier graph launch
    auto live = [&](int pair) { return !a.active || a.active[pair / H] != 0; };
    // item i of this warpgroup -> buffer i % 3 (a finished stream's buffer completes empty)
    auto issue = [&](int i) {
        const int pair = blockIdx.x + (i / my_tiles) * G, t = wg + 2 * (i % my_tiles), b = i % kStreamBufs;
        if (live(pair)) {
            const int group = pair / H, head = pair - group * H;
            const int y = (((a.stream_of_group[group] * a.n_layer + a.layer) * H + head) * A) + t * kAttnKeyTile;
            __half *tk = wbuf + (size_t)b * kStreamTile;
            mbar_expect_tx(&full[wg][b], 2 * kHalfTileBytes);
            tma_load_2d(tk, &kmap, 0, y, &full[wg][b]);
            tma_load_2d(tk + kAttnKeyTile * kHeadDim, &vmap, 0, y, &full[wg][b]);
        } else {
            mbar_arrive(&full[wg][b]);
        }
    };
    // a pair's queries (f32 registers; converted into qh when the pair starts)
    auto load_q = [&](int pair, float4 &v) {
        v = make_float4(0.f, 0.f, 0.f, 0.f);
        const int i = gtid / (kHeadDim / 4), c = gtid % (kHeadDim / 4);
        if (gtid < 8 * kHeadDim / 4 && i < NQ && pair < n_pairs && live(pair)) {
            const int group = pair / H, head = pair - group * H;
            v = reinterpret_cast<const float4 *>(a.q + (size_t)(group * NQ + i) * a.d + head * kHeadDim)[c];
        }
    };

    if (tid < 2 * kStreamBufs) {
        mbar_init(&full[tid / kStreamBufs][tid % kStreamBufs], 1);
        mbar_init(&empty[tid / kStreamBufs][tid % kStreamBufs], kWarps);
    }
    fence_mbar_init();
    __syncthreads();
    if (producer)
        for (int i = 0; i < kStreamBufs && i < n_items; ++i) issue(i);
    pdl_trigger();
    pdl_wait();
    float4 qn;
    load_q(blockIdx.x, qn);
    float m[2], l[2], of[4][4];
    bool ok = true;
    for (int i = 0; i < n_items; ++i) {
        const int k = i / my_tiles, j = i - k * my_tiles;
        const int pair = blockIdx.x + k * G, t = wg + 2 * j, b = i % kStreamBufs;
        const bool lv = live(pair);
        const int nk = min(kAttnKeyTile, A - t * kAttnKeyTile);
        __half *sk = wbuf + (size_t)b * kStreamTile, *sv = sk + kAttnKeyTile * kHeadDim;
        if (j == 0) {  // a new pair: queries and state; the next pair's queries start loading
            if (gtid < 8 * kHeadDim / 4) {
                const int qi = gtid / (kHeadDim / 4), c = gtid % (kHeadDim / 4);
                const __half2 h0 = __floats2half2_rn(qn.x, qn.y), h1 = __floats2half2_rn(qn.z, qn.w);
                *reinterpret_cast<uint2 *>(&qh[wg][qi][4 * c]) =
                    make_uint2(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1));
            }
            load_q(pair + G, qn);
            m[0] = m[1] = -INFINITY;
            l[0] = l[1] = 0.f;
#pragma unroll
            for (int mt = 0; mt < 4; ++mt) of[mt][0] = of[mt][1] = of[mt][2] = of[mt][3] = 0.f;
            group_sync(1 + wg);  // qh is read by every warp of the warpgroup
        }
        ok = mbar_wait(&full[wg][b], (unsigned)((i / kStreamBufs) & 1), a.err) && ok;
        if (lv && ok) {
            // a short last tile: V rows past its keys meet zero probabilities and must be finite;
            // each warp clears the rows of its own 16 keys (the TMA copy has completed)
            const int kb = 16 * gwarp;
            if (nk < kAttnKeyTile && kb < nk && kb + 16 > nk) {
                for (int c = lane; c < (kb + 16 - nk) * 8; c += 32)
                    *reinterpret_cast<uint4 *>(&sv[(nk + (c >> 3)) * kHeadDim + (c & 7) * 8]) = make_uint4(0u, 0u, 0u, 0u);
                __syncwarp();
            }
            tile_warp<NQ>(sk, sv, nk, qh[wg], pw[warp], m, l, of, gwarp, lane);
        }
        fence_proxy_async();  // this warp's generic accesses to the buffer precede the next copy into it
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[wg][b]);
        if (producer && i + kStreamBufs < n_items) {
            // refill buffer b once all eight warps are done with tile i
            if (mbar_wait(&empty[wg][b], (unsigned)((i / kStreamBufs) & 1), a.err)) issue(i + kStreamBufs);
            else ok = false;
        }
        __syncwarp();  // warp 0 reconverges before the next tile's ldmatrix / mma
        if (j == my_tiles - 1) {
            // end of the pair: the 16 warp states, combined in warp order
            if (lv) {
                if (g == 0) {
                    wm[warp][2 * tq] = m[0];
                    wm[warp][2 * tq + 1] = m[1];
                    wl[warp][2 * tq] = l[0];
                    wl[warp][2 * tq + 1] = l[1];
                }
#pragma unroll
                for (int mt = 0; mt < 4; ++mt) {
                    const int q0 = 2 * tq, q1 = 2 * tq + 1, d0 = 16 * mt + g;
                    if (q0 < NQ) {
                        red[warp][q0 * kHeadDim + d0] = of[mt][0];
                        red[warp][q0 * kHeadDim + d0 + 8] = of[mt][2];
                    }
                    if (q1 < NQ) {
                        red[warp][q1 * kHeadDim + d0] = of[mt][1];
                        red[warp][q1 * kHeadDim + d0 + 8] = of[mt][3];
                    }
                }
            }
            __syncthreads();
            if (lv) {
                const int group = pair / H, head = pair - group * H;
                for (int pidx = tid; pidx < NQ * kHeadDim; pidx += kStreamThreads) {
                    const int qi = pidx / kHeadDim, dd = pidx % kHeadDim;
                    float M = -INFINITY;
#pragma unroll
                    for (int w = 0; w < 2 * kWarps; ++w) M = fmaxf(M, wm[w][qi]);
                    float num = 0.f, den = 0.f;
#pragma unroll
                    for (int w = 0; w < 2 * kWarps; ++w)
                        if (wm[w][qi] != -INFINITY) {
                            const float wt = __expf(wm[w][qi] - M);
                            num = fmaf(wt, red[w][pidx], num);
                            den = fmaf(wt, wl[w][qi], den);
                        }
                    a.out[(size_t)(group * NQ + qi) * a.d + head * kHeadDim + dd] = num / den;
                }
            }
            __syncthreads();  // wm, wl, red and qh of both warpgroups are free
        }
    }
    // after a wait that ran out: the copies still in flight land before the block exits
    if (!ok && producer)
        for (int i = n_items > kStreamBufs ? n_items - kStreamBufs : 0; i < n_items; ++i)
            mbar_wait(&full[wg][i % kStreamBufs], (unsigned)((i / kStreamBufs) & 1), nullptr);
}

// ---------------------------------------------------------------------------
// Streaming self-attention for many sequences without beam tables (batched greedy steps): each
// warpgroup owns whole (sequence, head) pairs — pairs wg + 2 b, wg + 2 b + 2 G, ... of block b —
// and streams their 128-key tiles of the self cache (viewed as [rows][64] f16: one contiguous
// run of n_ctx rows per (slot, layer, head)) through three buffers with TMA, one thread of the
// warpgroup requesting the next tile as soon as all eight warps released a buffer.  The pairs
// of a step all have the same length, so the round-robin split is balanced.  The newest row of
// every sequence is written by the kernel before, so the copies start after the grid wait.
// Warp states (16 keys of each tile) are combined per pair in a fixed order, as in the
// cross-attention kernel.  Needs no mask and no explicit key counts (the decode step's case).
// ---------------------------------------------------------------------------
// CROSS: the same over the encoder K / V (n_audio keys per pair, NQ queries: the beams of a stream);
// those rows are constant during the decode, so the first copies start before the grid wait.
template <int NQ, bool CROSS>
__global__ void __launch_bounds__(kStreamThreads, 1)
    k_attn_pairs(AttnArgs a, const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap) {
    extern __shared__ __align__(1024) unsigned char sraw[];
    __half *sbuf = reinterpret_cast<__half *>(sraw + ((1024u - (smem_u32(sraw) & 1023u)) & 1023u));
    __shared__ __align__(8) uint64_t full[2][kStreamBufs], empty[2][kStreamBufs];
    __shared__ __align__(16) __half qh[2][8][kHeadDim + 8];
    __shared__ __align__(16) __half pw[2 * kWarps][8][kPwPad];
    __shared__ float wm[2 * kWarps][8], wl[2 * kWarps][8];
    __shared__ __align__(16) float red[2 * kWarps][NQ * kHeadDim];
    constexpr int kLocal = 64;  // pairs of one warpgroup whose key counts are kept in shared memory
    __shared__ short plen[2][kLocal];
    const int tid = threadIdx.x, wg = tid / kAttnThreads, gtid = tid % kAttnThreads;
    const int warp = tid >> 5, gwarp = gtid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
    const int H = a.n_head, n_pairs = a.groups * H;
    const int stride = 2 * (int)gridDim.x, first = 2 * (int)blockIdx.x + wg;
    __half *wbuf = sbuf + (size_t)wg * kStreamBufs * kStreamTile;
    const bool producer = gwarp == 0 && lane == 0;
    // keys of a pair's group: the encoder rows, or the sequence's positions 0 .. pos
    auto len_of = [&](int grp) { return CROSS ? a.n_audio : a.pos[grp] + 1; };
    auto len_global = [&](int pair) {
        const int grp = pair / H;
        return (a.active && !a.active[grp]) ? 0 : len_of(grp);
    };
    // the warpgroup's pairs first, first + stride, ...: their key counts (0 for finished sequences) read
    // once into shared memory, so that neither the producer nor a pair's start waits on a global load
    const bool local = (n_pairs - first + stride - 1) / stride <= kLocal;
    auto keys_of = [&](int pair) { return local ? (int)plen[wg][(pair - first) / stride] : len_global(pair); };
    auto tiles_of = [&](int pair) { return (keys_of(pair) + kAttnKeyTile - 1) / kAttnKeyTile; };
    auto fill_local = [&]() {
        if (local)
            for (int i = gtid; first + i * stride < n_pairs; i += kAttnThreads)
                plen[wg][i] = (short)len_global(first + i * stride);
        group_sync(1 + wg);
    };
    if (tid < 2 * kStreamBufs) {
        mbar_init(&full[tid / kStreamBufs][tid % kStreamBufs], 1);
        mbar_init(&empty[tid / kStreamBufs][tid % kStreamBufs], kWarps);
    }
    fence_mbar_init();
    __syncthreads();
    if (!CROSS) {
        pdl_trigger();
        pdl_wait();
    }
    fill_local();
    // producer cursor: the next (pair, tile) to request, in the consumers' order
    int ppair = first, ptile = 0, pn = ppair < n_pairs ? tiles_of(ppair) : 0;
    auto skip_empty = [&]() {
        while (ppair < n_pairs && ptile >= pn) {
            ppair += stride;
            ptile = 0;
            pn = ppair < n_pairs ? tiles_of(ppair) : 0;
        }
    };
    int issued = 0;
    auto issue = [&]() {  // request the cursor's tile into buffer issued % 3
        const int grp = ppair / H, head = ppair - grp * H, b = issued % kStreamBufs;
        const int y = CROSS ? ((a.stream_of_group[grp] * a.n_layer + a.layer) * H + head) * a.n_audio + ptile * kAttnKeyTile
                            : ((a.seq_slot[grp] * a.n_layer + a.layer) * H + head) * a.n_ctx + ptile * kAttnKeyTile;
        __half *tk = wbuf + (size_t)b * kStreamTile;
        mbar_expect_tx(&full[wg][b], 2 * kHalfTileBytes);
        tma_load_2d(tk, &kmap, 0, y, &full[wg][b]);
        tma_load_2d(tk + kAttnKeyTile * kHeadDim, &vmap, 0, y, &full[wg][b]);
        ++issued;
        ++ptile;
        skip_empty();
    };
    if (producer) {
        skip_empty();
        for (int i = 0; i < kStreamBufs && ppair < n_pairs; ++i) issue();
    }
    if (CROSS) {  // the queries come from the kernel before
        pdl_trigger();
        pdl_wait();
    }
    float m[2], l[2], of[4][4];
    bool ok = true;
    int item = 0;
    // the queries of the warpgroup's next pair are loaded while the current one is computed
    const int qi_l = gtid / (kHeadDim / 4), qc_l = gtid % (kHeadDim / 4);
    auto q_load = [&](int pair) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (gtid < 8 * kHeadDim / 4 && qi_l < NQ && pair < n_pairs) {
            const int grp = pair / H, head = pair - grp * H;
            v = reinterpret_cast<const float4 *>(a.q + (size_t)(grp * NQ + qi_l) * a.d + head * kHeadDim)[qc_l];
        }
        return v;
    };
    auto next_live = [&](int pair) {
        while (pair < n_pairs && tiles_of(pair) == 0) pair += stride;
        return pair;
    };
    int qpair = next_live(first);
    float4 qnext = q_load(qpair);
    for (int pair = first; pair < n_pairs; pair += stride) {
        const int nt = tiles_of(pair);
        if (nt == 0) continue;
        const int grp = pair / H, head = pair - grp * H, len = keys_of(pair);
        const float4 qcur = qpair == pair ? qnext : q_load(pair);
        qpair = next_live(pair + stride);
        qnext = q_load(qpair);
        if (gtid < 8 * kHeadDim / 4) {  // this pair's queries as f16; rows >= NQ zero
            const int qi = qi_l, c = qc_l;
            const float4 v = qcur;
            const __half2 h0 = __floats2half2_rn(v.x, v.y), h1 = __floats2half2_rn(v.z, v.w);
            *reinterpret_cast<uint2 *>(&qh[wg][qi][4 * c]) =
                make_uint2(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1));
        }
        m[0] = m[1] = -INFINITY;
        l[0] = l[1] = 0.f;
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) of[mt][0] = of[mt][1] = of[mt][2] = of[mt][3] = 0.f;
        group_sync(1 + wg);  // qh is read by every warp of the warpgroup
        for (int j = 0; j < nt; ++j, ++item) {
            const int b = item % kStreamBufs;
            const int nk = min(kAttnKeyTile, len - j * kAttnKeyTile);
            __half *sk = wbuf + (size_t)b * kStreamTile, *sv = sk + kAttnKeyTile * kHeadDim;
            ok = mbar_wait(&full[wg][b], (unsigned)((item / kStreamBufs) & 1), a.err) && ok;
            if (ok) {
                // rows past the keys meet zero probabilities in P.V and must be finite: each warp
                // clears the V rows of its own 16 keys past nk (the copy has completed)
                const int kb = 16 * gwarp;
                if (nk < kAttnKeyTile && kb < nk && kb + 16 > nk) {
                    for (int c = lane; c < (kb + 16 - nk) * 8; c += 32)
                        *reinterpret_cast<uint4 *>(&sv[(nk + (c >> 3)) * kHeadDim + (c & 7) * 8]) = make_uint4(0u, 0u, 0u, 0u);
                    __syncwarp();
                }
                tile_warp<NQ>(sk, sv, nk, qh[wg], pw[warp], m, l, of, gwarp, lane);
            }
            fence_proxy_async();  // this warp's generic accesses to the buffer precede the next copy into it
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[wg][b]);
            if (producer && ppair < n_pairs) {
                if (mbar_wait(&empty[wg][b], (unsigned)((item / kStreamBufs) & 1), a.err)) issue();
                else {
                    ok = false;
                    ppair = n_pairs;  // request nothing more
                }
            }
            __syncwarp();
        }
        // the pair's eight warp states, combined in warp order
        if (g == 0) {
            wm[warp][2 * tq] = m[0];
            wm[warp][2 * tq + 1] = m[1];
            wl[warp][2 * tq] = l[0];
            wl[warp][2 * tq + 1] = l[1];
        }
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
            const int q0 = 2 * tq, q1 = 2 * tq + 1, d0 = 16 * mt + g;
            if (q0 < NQ) {
                red[warp][q0 * kHeadDim + d0] = of[mt][0];
                red[warp][q0 * kHeadDim + d0 + 8] = of[mt][2];
            }
            if (q1 < NQ) {
                red[warp][q1 * kHeadDim + d0] = of[mt][1];
                red[warp][q1 * kHeadDim + d0 + 8] = of[mt][3];
            }
        }
        group_sync(1 + wg);
        for (int pidx = gtid; pidx < NQ * kHeadDim; pidx += kAttnThreads) {
            const int qi = pidx / kHeadDim, dd = pidx % kHeadDim;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) M = fmaxf(M, wm[wg * kWarps + w][qi]);
            float num = 0.f, den = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w)
                if (wm[wg * kWarps + w][qi] != -INFINITY) {
                    const float wt = __expf(wm[wg * kWarps + w][qi] - M);
                    num = fmaf(wt, red[wg * kWarps + w][pidx], num);
                    den = fmaf(wt, wl[wg * kWarps + w][qi], den);
                }
            if (ok) a.out[(size_t)(grp * NQ + qi) * a.d + head * kHeadDim + dd] = num / den;
        }
        group_sync(1 + wg);  // wm, wl, red and qh of this warpgroup are free
    }
    // after a wait that ran out: the copies still in flight land before the block exits
    if (!ok && producer)
        for (int i = issued > kStreamBufs ? issued - kStreamBufs : 0; i < issued; ++i)
            mbar_wait(&full[wg][i % kStreamBufs], (unsigned)((i / kStreamBufs) & 1), nullptr);
}

bool attn_self_stream_pays(const AttnArgs &a, int sms) {
    return !a.cross && !a.table && !a.mask && !a.kv_len && a.nq == 1 && (long long)a.groups * a.n_head > 2LL * sms;
}

// Cross-attention with a warpgroup per pair pays once every warpgroup has several pairs (the
// pair-end block barrier of k_attn_stream then costs more than the last round's imbalance).
bool attn_pairs_pays(const AttnArgs &a, int sms) {
    // (up to 5 queries per pair: the warp sums of 8 would not fit beside the six tile buffers)
    return a.cross && a.nq <= 5 && a.n_audio > kAttnKeyTile && (long long)a.groups * a.n_head >= 8LL * sms;
}

cudaError_t launch_attn_pairs(const AttnArgs &a, const void *kmap, const void *vmap, int sms, cudaStream_t s, bool pdl) {
    if (a.groups <= 0) return cudaSuccess;
    if (!a.cross || a.nq < 1 || a.nq > 5 || !kmap || !vmap) return cudaErrorInvalidValue;
    const long long pairs = (long long)a.groups * a.n_head;
    const long long want = (pairs + 1) / 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(want < sms ? want : sms));
    cfg.blockDim = dim3(kStreamThreads);
    cfg.dynamicSmemBytes = 2 * kStreamBufs * (size_t)kStreamTile * sizeof(__half) + 1024;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    const CUtensorMap &km = *reinterpret_cast<const CUtensorMap *>(kmap), &vm = *reinterpret_cast<const CUtensorMap *>(vmap);
    switch (a.nq) {
        case 1: return cudaLaunchKernelEx(&cfg, k_attn_pairs<1, true>, a, km, vm);
        case 2: return cudaLaunchKernelEx(&cfg, k_attn_pairs<2, true>, a, km, vm);
        case 3: return cudaLaunchKernelEx(&cfg, k_attn_pairs<3, true>, a, km, vm);
        case 4: return cudaLaunchKernelEx(&cfg, k_attn_pairs<4, true>, a, km, vm);
        default: return cudaLaunchKernelEx(&cfg, k_attn_pairs<5, true>, a, km, vm);
    }
}

cudaError_t launch_attn_self_stream(const AttnArgs &a, const void *kmap, const void *vmap, int sms, cudaStream_t s,
                                    bool pdl) {
    if (a.groups <= 0) return cudaSuccess;
    if (a.cross || a.table || a.mask || a.kv_len || a.nq != 1 || !kmap || !vmap) return cudaErrorInvalidValue;
    const long long pairs = (long long)a.groups * a.n_head;
    const long long want = (pairs + 1) / 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(want < sms ? want : sms));
    cfg.blockDim = dim3(kStreamThreads);
    cfg.dynamicSmemBytes = 2 * kStreamBufs * (size_t)kStreamTile * sizeof(__half) + 1024;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_attn_pairs<1, false>, a, *reinterpret_cast<const CUtensorMap *>(kmap),
                              *reinterpret_cast<const CUtensorMap *>(vmap));
}

// ---------------------------------------------------------------------------
// k_attn_self_warps: self-attention of many sequences (one query each, keys 0 .. pos) with one
// warp per (sequence, head) pair and no step that involves more than one warp: each warp streams its
// pair's keys in 32-key tiles through its own two-buffer TMA ring (128-byte swizzle, the layout
// tile_warp reads), runs tile_warp over both 16-key halves of a tile, and writes its output row.
// Twelve warps per SM, each with a tile in flight while it computes the other, replace the
// warpgroup-wide combine of k_attn_pairs, whose per-pair barriers dominated at ~120 keys per pair.
// ---------------------------------------------------------------------------
constexpr int kSwWarps = 12, kSwKeys = 32, kSwBufs = 2;
constexpr unsigned kSwHalf = kSwKeys * kHeadDim * 2;  // K (or V) of one tile: 4 KB

__global__ void __launch_bounds__(kSwWarps * 32, 1)
    k_attn_self_warps(AttnArgs a, const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap) {
    extern __shared__ __align__(1024) unsigned char sraw[];
    unsigned char *base = sraw + ((1024u - (smem_u32(sraw) & 1023u)) & 1023u);
    __shared__ __align__(8) uint64_t full[kSwWarps][kSwBufs];
    __shared__ __align__(16) __half qh[kSwWarps][8][kHeadDim + 8];
    __shared__ __align__(16) __half pw[kSwWarps][8][kPwPad];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
    const int H = a.n_head, n_pairs = a.groups * H;
    const int stride = kSwWarps * (int)gridDim.x, first = (int)blockIdx.x * kSwWarps + warp;
    unsigned char *wb = base + (size_t)warp * kSwBufs * 2 * kSwHalf;
    if (lane < kSwBufs) mbar_init(&full[warp][lane], 1);
    fence_mbar_init();
    __syncwarp();
    pdl_trigger();
    pdl_wait();  // positions, slots, queries and this step's K / V rows come from the kernels before
    auto keys_of = [&](int pair) {
        const int grp = pair / H;
        return (a.active && !a.active[grp]) ? 0 : a.pos[grp] + 1;
    };
    // lane 0's cursor: the next (pair, tile) to request, in the order the warp consumes them
    int ppair = first, ptile = 0, pn = ppair < n_pairs ? (keys_of(ppair) + kSwKeys - 1) / kSwKeys : 0;
    int issued = 0;
    auto skip = [&]() {
        while (ppair < n_pairs && ptile >= pn) {
            ppair += stride;
            ptile = 0;
            pn = ppair < n_pairs ? (keys_of(ppair) + kSwKeys - 1) / kSwKeys : 0;
        }
    };
    auto issue = [&]() {
        const int grp = ppair / H, head = ppair - grp * H, b = issued % kSwBufs;
        const int y = ((a.seq_slot[grp] * a.n_layer + a.layer) * H + head) * a.n_ctx + ptile * kSwKeys;
        unsigned char *dst = wb + (size_t)b * 2 * kSwHalf;
        mbar_expect_tx(&full[warp][b], 2 * kSwHalf);
        tma_load_2d(dst, &kmap, 0, y, &full[warp][b]);
        tma_load_2d(dst + kSwHalf, &vmap, 0, y, &full[warp][b]);
        ++issued;
        ++ptile;
        skip();
    };
    if (lane == 0) {
        skip();
        for (int i = 0; i < kSwBufs && ppair < n_pairs; ++i) issue();
    }
    bool ok = true;
    int item = 0;
    for (int pair = first; pair < n_pairs; pair += stride) {
        const int len = keys_of(pair);
        if (len == 0) continue;
        const int grp = pair / H, head = pair - grp * H;
        for (int i = lane; i < 8 * kHeadDim / 4; i += 32) {  // the query as row 0 of the B tile, rows 1-7 zero
            const int qi = i / (kHeadDim / 4), c = i % (kHeadDim / 4);
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (qi == 0) v = reinterpret_cast<const float4 *>(a.q + (size_t)grp * a.d + head * kHeadDim)[c];
            const __half2 h0 = __floats2half2_rn(v.x, v.y), h1 = __floats2half2_rn(v.z, v.w);
            *reinterpret_cast<uint2 *>(&qh[warp][qi][4 * c]) =
                make_uint2(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1));
        }
        __syncwarp();
        float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f}, of[4][4];
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) of[mt][0] = of[mt][1] = of[mt][2] = of[mt][3] = 0.f;
        const int nt = (len + kSwKeys - 1) / kSwKeys;
        for (int t = 0; t < nt; ++t, ++item) {
            const int b = item % kSwBufs, nk = min(kSwKeys, len - t * kSwKeys);
            __half *sk = reinterpret_cast<__half *>(wb + (size_t)b * 2 * kSwHalf), *sv = sk + kSwKeys * kHeadDim;
            ok = ok && mbar_wait(&full[warp][b], (unsigned)((item / kSwBufs) & 1), a.err);
            if (ok) {
                // V rows past the keys meet zero probabilities in P.V and must be finite (whole rows:
                // the swizzle only permutes chunks within a row)
                for (int c = lane; c < (kSwKeys - nk) * 8; c += 32)
                    *reinterpret_cast<uint4 *>(&sv[(nk + (c >> 3)) * kHeadDim + (c & 7) * 8]) = make_uint4(0u, 0u, 0u, 0u);
                __syncwarp();
                tile_warp<1>(sk, sv, nk, qh[warp], pw[warp], m, l, of, 0, lane);
                tile_warp<1>(sk, sv, nk, qh[warp], pw[warp], m, l, of, 1, lane);
            }
            fence_proxy_async();  // the warp's generic accesses to the buffer precede the next copy into it
            __syncwarp();
            if (lane == 0 && ok && ppair < n_pairs) issue();
        }
        if (ok && tq == 0) {  // query 0's O: dims 16 mt + g and 16 mt + g + 8 on the lanes with tq = 0
            const float inv = 1.0f / l[0];
            float *o = a.out + (size_t)grp * a.d + head * kHeadDim;
#pragma unroll
            for (int mt = 0; mt < 4; ++mt) {
                o[16 * mt + g] = of[mt][0] * inv;
                o[16 * mt + g + 8] = of[mt][2] * inv;
            }
        }
        __syncwarp();  // qh and pw are rewritten by the next pair
    }
    // after a wait that ran out: the copies still in flight land before the warp exits
    if (!ok && lane == 0)
        for (int i = issued > kSwBufs ? issued - kSwBufs : 0; i < issued; ++i)
            mbar_wait(&full[warp][i % kSwBufs], (unsigned)((i / kSwBufs) & 1), nullptr);
}

cudaError_t launch_attn_self_warps(const AttnArgs &a, const void *kmap32, const void *vmap32, int sms, cudaStream_t s,
                                   bool pdl) {
    if (a.groups <= 0) return cudaSuccess;
    if (a.cross || a.table || a.mask || a.kv_len || a.nq != 1 || !kmap32 || !vmap32) return cudaErrorInvalidValue;
    const long long pairs = (long long)a.groups * a.n_head;
    const long long want = (pairs + kSwWarps - 1) / kSwWarps;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(want < sms ? want : sms));
    cfg.blockDim = dim3(kSwWarps * 32);
    cfg.dynamicSmemBytes = (size_t)kSwWarps * kSwBufs * 2 * kSwHalf + 1024;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_attn_self_warps, a, *reinterpret_cast<const CUtensorMap *>(kmap32),
                              *reinterpret_cast<const CUtensorMap *>(vmap32));
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
    cudaError_t e = allow_dynamic_smem(k_attn_pairs<1, false>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_attn_self_warps);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_attn_pairs<1, true>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_attn_pairs<2, true>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_attn_pairs<3, true>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_attn_pairs<4, true>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_attn_pairs<5, true>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_attn_stream<1>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_attn_stream<2>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_attn_stream<3>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_attn_stream<4>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_attn_stream<5>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_attn_stream<6>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_attn_stream<7>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_attn_stream<8>);
    if (e != cudaSuccess) return e;
    e = prep_nq<1>();
    if (e == cudaSuccess) e = prep_nq<2>();
    if (e == cudaSuccess) e = prep_nq<3>();
    if (e == cudaSuccess) e = prep_nq<4>();
    if (e == cudaSuccess) e = prep_nq<5>();
    if (e == cudaSuccess) e = prep_nq<6>();
    if (e == cudaSuccess) e = prep_nq<7>();
    if (e == cudaSuccess) e = prep_nq<8>();
    return e;
}

bool attn_stream_pays(const AttnArgs &a, int sms) {
    // more (split, head, group) blocks than one resident wave of the cluster kernel; both
    // warpgroups need a tile of every pair
    // (up to 5 queries: the warp sums of more would not fit beside the six tile buffers)
    return a.cross && a.nq <= 5 && a.n_audio > kAttnKeyTile && (long long)a.nsplit * a.n_head * a.groups > 2LL * sms;
}

static size_t stream_smem() { return 2 * kStreamBufs * (size_t)kStreamTile * sizeof(__half) + 1024; }

cudaError_t launch_attn_stream(const AttnArgs &a, const void *kmap, const void *vmap, int sms, cudaStream_t s, bool pdl) {
    if (a.groups <= 0) return cudaSuccess;
    if (!a.cross || a.nq < 1 || a.nq > kMaxNq || a.n_audio <= kAttnKeyTile || !kmap || !vmap)
        return cudaErrorInvalidValue;
    const long long pairs = (long long)a.groups * a.n_head;
    const CUtensorMap &km = *reinterpret_cast<const CUtensorMap *>(kmap);
    const CUtensorMap &vm = *reinterpret_cast<const CUtensorMap *>(vmap);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(pairs < sms ? pairs : sms));
    cfg.blockDim = dim3(kStreamThreads);
    cfg.dynamicSmemBytes = stream_smem();
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
    }
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    switch (a.nq) {
        case 1: return cudaLaunchKernelEx(&cfg, k_attn_stream<1>, a, km, vm);
        case 2: return cudaLaunchKernelEx(&cfg, k_attn_stream<2>, a, km, vm);
        case 3: return cudaLaunchKernelEx(&cfg, k_attn_stream<3>, a, km, vm);
        case 4: return cudaLaunchKernelEx(&cfg, k_attn_stream<4>, a, km, vm);
        case 5: return cudaLaunchKernelEx(&cfg, k_attn_stream<5>, a, km, vm);
        case 6: return cudaLaunchKernelEx(&cfg, k_attn_stream<6>, a, km, vm);
        case 7: return cudaLaunchKernelEx(&cfg, k_attn_stream<7>, a, km, vm);
        default: return cudaLaunchKernelEx(&cfg, k_attn_stream<8>, a, km, vm);
    }
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
