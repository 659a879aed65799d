// k_gemm_tc.cu — the decoder projections on the 5th-generation tensor cores (tcgen05 + TMEM +
// TMA) once streams x beams give M >= 16 rows: y[m][n] = LN?(x[m]) . W[n]^T + b with the
// epilogues of the GEMV kernel (store, GELU table, residual add, Q/K/V with the self-cache
// scatter).  Same computation as k_gemv (Linear.forward, nn/Linear.java:23-26, with the
// LayerNorm of ResidualAttentionBlock.java:48-59 before it), for batched decoding.
//
// Grid (split, tile): a block owns 128 rows of W (one UMMA M tile) and a range of K.
//   * TMA (cp.async.bulk.tensor.2d, 128-byte swizzle) streams its [128 x 64] weight tiles through
//     a ring of shared-memory stages, the first stages before griddepcontrol.wait.
//   * With a LayerNorm prologue and a split K, block q of the tile's cluster computes the
//     two-pass statistics of rows q, q + ks, ... over the full row and stores (mean, 1/std)
//     into every block of the cluster, so each block then reads only its K range of the rows.
//   * The activations (LayerNorm-ed when the projection has one) of the block's K range are
//     written as the f16 B operand, K-major with the same swizzle, each f32
//     value x as two f16 rows: hi = f16(x) and lo = f16(x - hi).  hi + lo carries x to about 22
//     bits, so with f16 weights and f32 accumulation the product keeps the f32 activations of
//     the reference instead of rounding them to f16.  Rows hold the NU sequence slots (NU = M
//     padded to 16, 32, 64 or 128; slots >= M are zero): hi in rows [0, NU), lo in [NU, 2 NU).
//   * One thread issues tcgen05.mma.kind::f16 (M 128, N 2 NU, K 16) into an f32 accumulator in
//     tensor memory; eight warps read it back with tcgen05.ld and add the hi and lo columns.
//   * With a split K the split blocks of a tile form a thread-block cluster.  Block q owns rows
//     [q * 128 / ks, (q + 1) * 128 / ks) of the tile: every block stores its partial of those
//     rows into the owner's shared memory (distributed shared memory stores), and after one
//     cluster barrier the owner adds the partials in split order, so the result is
//     deterministic, then applies the epilogue.
// Every wait on a copy is bounded; a time-out raises the device error word.
#include "tc_common.cuh"
#include "w4j_internal.cuh"

namespace w4j {

constexpr int kGemmThreads = 512, kGemmWarps = kGemmThreads / 32;
// Q8_0 weights: a raw stage holds the [128 x 64] int8 tile (TMA) and its 128 x 2 f16 scales (bulk
// copy from the tiled scale layout); eight converter warps dequantise it into an A stage of two
// swizzled f16 tiles, hi = f16(q * s) and lo = f16(q * s - hi), so the product keeps the
// reference's exact f32 weight q * s (GgmlLoader.java:292-300)
constexpr unsigned kRawBytes = kTileRows * kKB;                  // int8 tile: 8 KB
constexpr unsigned kRawStage = kRawBytes + kTileRows * 2 * 2;    // + its scales: 8704 B
constexpr unsigned kAStage = 2 * kStageBytes;                    // hi and lo f16 tiles: 32 KB
constexpr int kConvWarps = 8;                                    // warps 8 .. 15

struct GemmTcLaunch {
    int mchunk;      // sequence rows per block (grid z walks the chunks of M > 128 rows)
    int KB;          // 64-wide k-blocks in K
    int ks;          // K splits (cluster size)
    int nkb_max;     // k-blocks of the largest split
    int n_stages;    // weight ring stages
    int rmax;        // most tile rows a split block owns: ceil(128 / ks)
    int recv_alias;  // 1: the partials land in the weight ring (free once every block's MMAs are done)
    unsigned ring_off;  // weight ring (Q8_0: raw stages after the two dequantised A stages at 0)
    unsigned b_off, ln_off, bias_off, mi_off, stat_off, recv_off, bar_off;  // shared-memory layout (bytes)
};

__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ unsigned cluster_map(const void *local, unsigned rank) {
    unsigned remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
    return remote;
}
__device__ __forceinline__ void st_cluster_f32(unsigned addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_f32x2(unsigned addr, float x, float y) {
    asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(x), "f"(y) : "memory");
}

// Rows [m0, m0 + n) of a projection: every per-sequence pointer advanced by m0 rows.
__device__ __forceinline__ GemvArgs rows_of(const GemvArgs &g, int m0, int n) {
    GemvArgs a = g;
    const int K = g.W.K, N = g.W.N;
    a.M = n;
    if (a.act) a.act += (size_t)m0 * K;
    if (a.tok) a.tok += m0;
    if (a.pos) a.pos += m0;
    if (a.pe_pos) a.pe_pos += m0;
    if (a.seq_slot) a.seq_slot += m0;
    if (a.active) a.active += m0;
    if (a.x_out) a.x_out += (size_t)m0 * K;
    a.y += (size_t)m0 * (a.out_mode == OUT_QKV ? N / 3 : N);
    return a;
}

// BT: the B operand comes from a staged f16 hi / lo activation buffer (k_act_hilo) through TMA, one
// [256 rows x 64] tile per ring stage beside the weight tile, instead of being built in shared memory
// for the block's whole K range (more than 128 rows: NU = 128, f16 weights)
template <int NU, int WT, bool BT>
__global__ void __launch_bounds__(kGemmThreads, 1) k_gemm_tc(GemvArgs a_all, const __grid_constant__ CUtensorMap tmap,
                                                              const __grid_constant__ CUtensorMap bmap, GemmTcLaunch L) {
    static_assert(!BT || WT == WT_F16, "staged B: f16 projections");
    constexpr bool kQ8 = WT == WT_Q8;
    constexpr unsigned kBTile = 2u * NU * 128u;  // one k-block of B: hi and lo rows of 128 bytes
    constexpr unsigned SB = kQ8 ? kRawStage : BT ? (unsigned)kStageBytes + kBTile : (unsigned)kStageBytes;
    // grid z: chunks of at most 128 sequence rows; every chunk's blocks stream the same weight
    // tiles at about the same time, so the chunks after the first mostly read them from L2
    const int mc0 = blockIdx.z * L.mchunk;
    const GemvArgs a = rows_of(a_all, mc0, min(L.mchunk, a_all.M - mc0));
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int N = a.W.N, K = a.W.K, M = a.M;
    const int split = blockIdx.x, ks = L.ks;
    const int n0 = blockIdx.y * kTileRows;
    const int kb0 = (split * L.KB) / ks, kb1 = ((split + 1) * L.KB) / ks, nkb = kb1 - kb0;
    const int NS = L.n_stages;
    unsigned char *ring = smem + L.ring_off;
    unsigned char *aring = smem;  // Q8_0: two dequantised A stages
    constexpr int NB = 2 * NU;             // B rows: hi, then lo parts of the NU slots
    unsigned char *bop = smem + L.b_off;  // [nkb][NB rows][128 B]
    float *ln_s = reinterpret_cast<float *>(smem + L.ln_off);      // gamma, beta of the K range
    float *bias_s = reinterpret_cast<float *>(smem + L.bias_off);  // [128]
    int *mi_s = reinterpret_cast<int *>(smem + L.mi_off);          // [5][M] active, slot, row, token, pe row
    float2 *stat_s = reinterpret_cast<float2 *>(smem + L.stat_off); // [M] LayerNorm mean, 1/std (split K)
    // split-K partials of the rows this block owns: [split][M][rmax], written by the cluster
    float *recv = reinterpret_cast<float *>(smem + (L.recv_alias ? 0u : L.recv_off));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bar_off);
    uint64_t *empty = full + NS;
    uint64_t *afull = empty + NS;  // Q8_0: A stage converted (one arrival per converter warp)
    uint64_t *aempty = afull + 2;  // Q8_0: A stage read by the MMAs (commit)
    uint64_t *accf = aempty + 2;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(accf + 1);
    volatile int *fail = reinterpret_cast<volatile int *>(tslot + 1);
    volatile int *issued = fail + 1;  // weight tiles whose copy has been started
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr uint32_t kCols = NB;  // 32 .. 256 f32 columns
    const int kr = nkb * kKB;  // K range of this block: [kb0 * 64, kb0 * 64 + kr)

    // ---- independent of the previous kernel: barriers, TMEM, first weight tiles, parameters ----
    // copy of weight k-block i of this block's range into ring stage i % NS
    auto issue = [&](int i) {
        const int st = i % NS;
        unsigned char *dst = ring + (size_t)st * SB;
        if (kQ8) {
            mbar_expect_tx(full + st, kRawStage);
            tma_load_2d(dst, &tmap, (kb0 + i) * kKB, n0, full + st);
            bulk_g2s(dst + kRawBytes, a.W.st + ((size_t)blockIdx.y * L.KB + kb0 + i) * (kTileRows * 2),
                     kRawStage - kRawBytes, full + st);
        } else if (BT) {
            mbar_expect_tx(full + st, kStageBytes + kBTile);
            tma_load_2d(dst, &tmap, (kb0 + i) * kKB, n0, full + st);
            tma_load_2d(dst + kStageBytes, &bmap, (kb0 + i) * kKB, (int)blockIdx.z * 2 * NU, full + st);
        } else {
            mbar_expect_tx(full + st, kStageBytes);
            tma_load_2d(dst, &tmap, (kb0 + i) * kKB, n0, full + st);
        }
    };
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, kQ8 ? kConvWarps : 1);  // Q8_0: released by the converters
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(afull + i, kConvWarps);
            mbar_init(aempty + i, 1);
        }
        mbar_init(accf, 1);
        *fail = 0;
        fence_mbar_init();
        // the first stages' weight tiles now; staged B tiles are written by the previous kernel, so
        // their copies into the same stages follow the wait (each stage's barrier expects both)
        for (int i = 0; i < NS && i < nkb; ++i) {
            if (BT) {
                mbar_expect_tx(full + i, kStageBytes + kBTile);
                tma_load_2d(ring + (size_t)i * SB, &tmap, (kb0 + i) * kKB, n0, full + i);
            } else {
                issue(i);
            }
        }
        *issued = NS < nkb ? NS : nkb;
    }
    if (warp == 1) {
        tmem_alloc(tslot, kCols);
        tmem_relinquish();
    }
    // LayerNorm parameters of the K range (2 kr <= 2560 floats: at most 5 per thread), biases,
    // liveness, cache slots, positions and tokens (written by the host or an earlier graph
    // launch): every load of a thread is issued before the first store, so they overlap
    {
        const int nln = (a.in_mode != IN_ACT && !BT) ? 2 * kr : 0;
        float lnv[5];
#pragma unroll
        for (int j = 0; j < 5; ++j) {
            const int i = tid + j * kGemmThreads;
            lnv[j] = i < nln ? (i < kr ? a.ln_g[kb0 * kKB + i] : a.ln_b[kb0 * kKB + i - kr]) : 0.f;
        }
        const float bv = (tid < kTileRows && a.bias && n0 + tid < N) ? a.bias[n0 + tid] : 0.f;
        int mv0 = 1, mv1 = 0, mv2 = 0, mv3 = 0, mv4 = 0;
        if (tid < M) {
            if (a.active) mv0 = a.active[tid];
            if (a.out_mode == OUT_QKV) mv1 = a.seq_slot[tid];
            if (a.out_mode == OUT_QKV) mv2 = a.pos[tid];
            if (a.in_mode == IN_EMBED_LN) {
                mv3 = a.tok[tid];
                mv4 = pe_row(a, tid);
            }
        }
#pragma unroll
        for (int j = 0; j < 5; ++j) {
            const int i = tid + j * kGemmThreads;
            if (i < nln) ln_s[i] = lnv[j];
        }
        if (tid < kTileRows) bias_s[tid] = bv;
        if (tid < M) {
            mi_s[tid] = mv0;
            mi_s[M + tid] = mv1;
            mi_s[2 * M + tid] = mv2;
            mi_s[3 * M + tid] = mv3;
            mi_s[4 * M + tid] = mv4;
        }
    }
    for (int i = tid; !BT && i < 2 * (NU - M) * nkb * 8; i += blockDim.x) {  // slots M .. NU are zero
        const int j = i / (nkb * 8), c = i % (nkb * 8);
        const int m = j < NU - M ? M + j : NU + M + (j - (NU - M));
        const int kb = c / 8, cc = c % 8;
        *reinterpret_cast<uint4 *>(bop + (size_t)kb * NB * 128 + (size_t)m * 128 + ((cc ^ (m & 7)) * 16)) =
            make_uint4(0, 0, 0, 0);
    }
    // the cluster's blocks must all have started before one stores into another's shared memory:
    // every thread arrives here and waits before its first distributed store
    if (ks > 1) cluster_arrive_relaxed();
    bool started = ks == 1;
    pdl_trigger();
    pdl_wait();
    if (BT && tid == 0)
        for (int i = 0; i < NS && i < nkb; ++i)
            tma_load_2d(ring + (size_t)i * SB + kStageBytes, &bmap, (kb0 + i) * kKB, (int)blockIdx.z * 2 * NU, full + i);
    __syncthreads();

    if constexpr (!BT) {
    // ---- B operand: the rows' K range as f16 hi / lo pairs, K-major, 128-byte swizzle ----
    // 4 consecutive elements k .. k+3 of slot m (k inside the K range) go to their 8-byte half of
    // the 16-byte chunk of row m (hi) and of row NU + m (lo)
    auto put4 = [&](int m, int kk, float4 v) {
        const int kb = kk / kKB, cc = (kk % kKB) / 8, half = (kk % 8) / 4;
        const __half2 h0 = __floats2half2_rn(v.x, v.y), h1 = __floats2half2_rn(v.z, v.w);
        const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
        const __half2 l0 = __floats2half2_rn(v.x - f0.x, v.y - f0.y), l1 = __floats2half2_rn(v.z - f1.x, v.w - f1.y);
        unsigned char *row = bop + (size_t)kb * NB * 128 + half * 8;
        const int ml = NU + m;
        *reinterpret_cast<uint2 *>(row + (size_t)m * 128 + ((cc ^ (m & 7)) * 16)) =
            make_uint2(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1));
        *reinterpret_cast<uint2 *>(row + (size_t)ml * 128 + ((cc ^ (ml & 7)) * 16)) =
            make_uint2(*reinterpret_cast<const uint32_t *>(&l0), *reinterpret_cast<const uint32_t *>(&l1));
    };
    if (a.in_mode != IN_ACT && ks > 1) {
        // LayerNorm statistics over the full rows (Tensor.java:592-619: two-pass mean / variance,
        // eps 1e-5), shared by the split blocks: block `split` computes rows split, split + ks, ...
        // (one warp per row, the row in registers) and stores (mean, 1/std) into every block of
        // the cluster; then each block reads only its K range of the rows
        constexpr int kLnF4 = 10;  // K <= 1280
        const int nf4 = K / 128;
        __syncwarp();
        cluster_wait_acquire();
        started = true;
        for (int m = split + ks * warp; m < M; m += ks * kGemmWarps) {
            float4 v[kLnF4];
            if (a.in_mode == IN_LN) {
                const float4 *src = reinterpret_cast<const float4 *>(a.act + (size_t)m * K);
#pragma unroll
                for (int j = 0; j < kLnF4; ++j) v[j] = j < nf4 ? src[lane + 32 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
            } else {  // x = E[tok] + P[pos] (WhisperDecoder.java:66-80); the first tile's owner keeps it
                const uint2 *e = reinterpret_cast<const uint2 *>(a.E.h + (size_t)mi_s[3 * M + m] * K);
                const float4 *pe = reinterpret_cast<const float4 *>(a.pos_emb + (size_t)mi_s[4 * M + m] * K);
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
                    if (j < nf4 && blockIdx.y == 0 && a.x_out)
                        reinterpret_cast<float4 *>(a.x_out)[(size_t)m * (K / 4) + lane + 32 * j] = v[j];
                }
            }
            float sm = 0.f;
#pragma unroll
            for (int j = 0; j < kLnF4; ++j)
                if (j < nf4) sm += (v[j].x + v[j].y) + (v[j].z + v[j].w);
            const float mean = warp_sum(sm) / (float)K;
            float v2 = 0.f;
#pragma unroll
            for (int j = 0; j < kLnF4; ++j)
                if (j < nf4) {
                    const float dx = v[j].x - mean, dy = v[j].y - mean, dz = v[j].z - mean, dw = v[j].w - mean;
                    v2 += (dx * dx + dy * dy) + (dz * dz + dw * dw);
                }
            const float inv_std = 1.0f / sqrtf(warp_sum(v2) / (float)K + 1e-5f);
            if (lane < ks) st_cluster_f32x2(cluster_map(&stat_s[m], (unsigned)lane), mean, inv_std);
        }
        __syncwarp();
        cluster_arrive_release();
        cluster_wait_acquire();
        // the K range of every row, normalised: 8 float4 (and for the embedding 8 f16 quads) in flight
        const int r4 = kr / 4;
        const int total = M * r4;
        for (int i0 = tid; i0 < total; i0 += kGemmThreads * 8) {
            float4 v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = i0 + kGemmThreads * j;
                if (i < total) {
                    const int m = i / r4, c4 = i - m * r4;
                    if (a.in_mode == IN_LN) {
                        v[j] = reinterpret_cast<const float4 *>(a.act + (size_t)m * K + kb0 * kKB)[c4];
                    } else {
                        const uint2 eu =
                            reinterpret_cast<const uint2 *>(a.E.h + (size_t)mi_s[3 * M + m] * K + kb0 * kKB)[c4];
                        const float4 p =
                            reinterpret_cast<const float4 *>(a.pos_emb + (size_t)mi_s[4 * M + m] * K + kb0 * kKB)[c4];
                        const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&eu.x));
                        const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&eu.y));
                        v[j] = make_float4(lo.x + p.x, lo.y + p.y, hi.x + p.z, hi.y + p.w);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = i0 + kGemmThreads * j;
                if (i < total) {
                    const int m = i / r4, c4 = i - m * r4, kk = 4 * c4;
                    const float2 st = stat_s[m];
                    const float4 g = *reinterpret_cast<const float4 *>(ln_s + kk);
                    const float4 b = *reinterpret_cast<const float4 *>(ln_s + kr + kk);
                    put4(m, kk, make_float4((v[j].x - st.x) * st.y * g.x + b.x, (v[j].y - st.x) * st.y * g.y + b.y,
                                            (v[j].z - st.x) * st.y * g.z + b.z, (v[j].w - st.x) * st.y * g.w + b.w));
                }
            }
        }
    } else if (a.in_mode == IN_ACT) {
        // the K range of every row, 16 float4 loads in flight per thread
        const int r4 = kr / 4;  // float4 per row in the K range
        const int total = M * r4;
        for (int i0 = tid; i0 < total; i0 += kGemmThreads * 16) {
            float4 v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int i = i0 + kGemmThreads * j;
                if (i < total) {
                    const int m = i / r4, c4 = i - m * r4;
                    v[j] = reinterpret_cast<const float4 *>(a.act + (size_t)m * K + kb0 * kKB)[c4];
                }
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int i = i0 + kGemmThreads * j;
                if (i < total) {
                    const int m = i / r4, c4 = i - m * r4;
                    put4(m, 4 * c4, v[j]);
                }
            }
        }
    } else {
        // LayerNorm over the full row (Tensor.java:592-619: two-pass mean / variance, eps 1e-5),
        // one warp per row with the row in registers; then the K range is written
        constexpr int kLnF4 = 10;  // K <= 1280
        const int nf4 = K / 128;
        auto ln_put = [&](int m, float4 (&v)[kLnF4]) {
            float sm = 0.f;
#pragma unroll
            for (int j = 0; j < kLnF4; ++j)
                if (j < nf4) sm += (v[j].x + v[j].y) + (v[j].z + v[j].w);
            const float mean = warp_sum(sm) / (float)K;
            float v2 = 0.f;
#pragma unroll
            for (int j = 0; j < kLnF4; ++j)
                if (j < nf4) {
                    const float dx = v[j].x - mean, dy = v[j].y - mean, dz = v[j].z - mean, dw = v[j].w - mean;
                    v2 += (dx * dx + dy * dy) + (dz * dz + dw * dw);
                }
            const float inv_std = 1.0f / sqrtf(warp_sum(v2) / (float)K + 1e-5f);
#pragma unroll
            for (int j = 0; j < kLnF4; ++j) {
                const int k = 4 * (lane + 32 * j), kk = k - kb0 * kKB;
                if (j < nf4 && kk >= 0 && kk < kr) {
                    const float4 g = *reinterpret_cast<const float4 *>(ln_s + kk);
                    const float4 b = *reinterpret_cast<const float4 *>(ln_s + kr + kk);
                    put4(m, kk, make_float4((v[j].x - mean) * inv_std * g.x + b.x, (v[j].y - mean) * inv_std * g.y + b.y,
                                            (v[j].z - mean) * inv_std * g.z + b.z, (v[j].w - mean) * inv_std * g.w + b.w));
                }
            }
        };
        if (a.in_mode == IN_LN) {
            // two rows per warp in flight: rows m0 and m0 + 16
            for (int m0 = warp; m0 < M; m0 += 2 * kGemmWarps) {
                const int m1 = m0 + kGemmWarps;
                const float4 *s0 = reinterpret_cast<const float4 *>(a.act + (size_t)m0 * K);
                const float4 *s1 = reinterpret_cast<const float4 *>(a.act + (size_t)(m1 < M ? m1 : m0) * K);
                float4 v0[kLnF4], v1[kLnF4];
#pragma unroll
                for (int j = 0; j < kLnF4; ++j) v0[j] = j < nf4 ? s0[lane + 32 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int j = 0; j < kLnF4; ++j) v1[j] = j < nf4 ? s1[lane + 32 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
                ln_put(m0, v0);
                if (m1 < M) ln_put(m1, v1);
            }
        } else {  // x = E[tok] + P[pos] (WhisperDecoder.java:66-80), kept in x_out by one block
            for (int m = warp; m < M; m += kGemmWarps) {
                const int tok = mi_s[3 * M + m], pos = mi_s[4 * M + m];
                const uint2 *e = reinterpret_cast<const uint2 *>(a.E.h + (size_t)tok * K);
                const float4 *pe = reinterpret_cast<const float4 *>(a.pos_emb + (size_t)pos * K);
                float4 v[kLnF4];
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
                    if (j < nf4 && blockIdx.x == 0 && blockIdx.y == 0 && a.x_out)
                        reinterpret_cast<float4 *>(a.x_out)[(size_t)m * (K / 4) + lane + 32 * j] = v[j];
                }
                ln_put(m, v);
            }
        }
    }
    }
    fence_proxy_async();  // generic-proxy writes of B visible to the tensor core
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = *tslot;
    const uint32_t idesc = idesc_f16(kTileRows, NB);

    // output (row r of the tile, sequence m) with the GEMV epilogues
    auto emit = [&](float v, int r, int m) {
        const int n = n0 + r;
        if (n >= N || m >= M || !mi_s[m]) return;
        const float val = v + bias_s[r];
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
                const int part_ = n / dm, c = n - part_ * dm;
                if (part_ == 0) {
                    a.y[(size_t)m * dm + c] = val;
                } else {
                    const int head = c / kHeadDim, dd = c % kHeadDim;
                    const size_t row = (((size_t)mi_s[M + m] * a.n_layer + a.layer) * a.n_head + head) * (size_t)a.n_ctx +
                                       (size_t)mi_s[2 * M + m];
                    __half *dst = part_ == 1 ? a.kcache : a.vcache;
                    dst[row * kHeadDim + dd] = __float2half_rn(val);
                }
                break;
            }
        }
    };
    // The residual and GELU epilogues for 16 outputs at once (m < 0: none): their global loads are
    // all issued before the first store, one L2 round trip for the batch instead of one per output.
    const bool batched = a.out_mode == OUT_GELU || a.out_mode == OUT_RESIDUAL;
    auto emit16 = [&](const float (&v)[16], const int (&rr)[16], const int (&mm)[16]) {
        float val[16], g[16];
        bool live[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            const int n = n0 + rr[e], m = mm[e];
            live[e] = m >= 0 && n < N && m < M && mi_s[m];
            val[e] = live[e] ? v[e] + bias_s[rr[e]] : 0.f;
        }
        if (a.out_mode == OUT_GELU) {
#pragma unroll
            for (int e = 0; e < 16; ++e)
                g[e] = live[e] ? __ldg(a.gelu_lut + __half_as_ushort(__float2half_rn(val[e]))) : 0.f;
        } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) g[e] = live[e] ? a.y[(size_t)mm[e] * N + n0 + rr[e]] : 0.f;
        }
#pragma unroll
        for (int e = 0; e < 16; ++e)
            if (live[e]) a.y[(size_t)mm[e] * N + n0 + rr[e]] = a.out_mode == OUT_GELU ? g[e] : g[e] + val[e];
    };

    if (warp == 0 && lane == 0) {
        // ---- producer: the remaining weight tiles as stages free up ----
        for (int i = NS; i < nkb && !*fail; ++i) {
            const int st = i % NS;
            if (!mbar_wait(empty + st, (unsigned)((i / NS - 1) & 1), a.err)) {
                *fail = 1;
                break;
            }
            issue(i);
            *issued = i + 1;
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer ----
        const uint32_t ring_a = smem_u32(ring), aring_a = smem_u32(aring), b_a = smem_u32(bop);
        for (int i = 0; i < nkb && !*fail; ++i) {
            const int st = i % NS;
            if (!mbar_wait(kQ8 ? afull + (i & 1) : full + st, (unsigned)((kQ8 ? i >> 1 : i / NS) & 1), a.err)) {
                *fail = 1;
                break;
            }
            tc_fence_after();
            if (kQ8) {
                // W = hi + lo: both dequantised tiles against the same B columns, one accumulator
                const uint32_t ahi = aring_a + (uint32_t)(i & 1) * kAStage, alo = ahi + kStageBytes;
#pragma unroll
                for (int j = 0; j < kKB / 16; ++j) {
                    const uint64_t bd = sw128_desc(b_a + (uint32_t)i * NB * 128 + j * 32);
                    umma_f16(taddr, sw128_desc(ahi + j * 32), bd, idesc, (i | j) != 0);
                    umma_f16(taddr, sw128_desc(alo + j * 32), bd, idesc, 1u);
                }
                umma_commit(aempty + (i & 1));  // the A stage is free once these MMAs have read it
            } else {
#pragma unroll
                for (int j = 0; j < kKB / 16; ++j) {
                    const uint32_t sa = ring_a + (uint32_t)st * SB;
                    const uint64_t ad = sw128_desc(sa + j * 32);
                    const uint64_t bd = BT ? sw128_desc(sa + kStageBytes + j * 32)
                                           : sw128_desc(b_a + (uint32_t)i * NB * 128 + j * 32);
                    umma_f16(taddr, ad, bd, idesc, (i | j) != 0);
                }
                umma_commit(empty + st);  // the stage is free once these MMAs have read it
            }
        }
        umma_commit(accf);  // the accumulator is complete (or nothing was issued)
    } else if (kQ8 && warp >= 16 - kConvWarps) {
        // ---- Q8_0 converters: raw stage i -> A stage i % 2 (thread: row r, scale group h) ----
        const int ct = tid - (16 - kConvWarps) * 32, r = ct >> 1, h = ct & 1;
        for (int i = 0; i < nkb && !*fail; ++i) {
            const int st = i % NS;
            if (!mbar_wait(full + st, (unsigned)((i / NS) & 1), a.err) ||
                (i >= 2 && !mbar_wait(aempty + (i & 1), (unsigned)(((i >> 1) - 1) & 1), a.err))) {
                *fail = 1;
                break;
            }
            const unsigned char *raw = ring + (size_t)st * SB;
            const uint4 q0 = *reinterpret_cast<const uint4 *>(raw + r * kKB + h * 32);
            const uint4 q1 = *reinterpret_cast<const uint4 *>(raw + r * kKB + h * 32 + 16);
            const float sc = __half2float(reinterpret_cast<const __half *>(raw + kRawBytes)[r * 2 + h]);
            unsigned char *ahi = aring + (size_t)(i & 1) * kAStage, *alo = ahi + kStageBytes;
            const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
            for (int c = 0; c < 4; ++c) {  // 8 weights per 16-byte chunk: chunk 4 h + c of row r
                uint32_t hv[4], lv[4];
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const uint32_t wd = qw[2 * c + (p >> 1)];
                    const int b0 = (p & 1) * 16;
                    const float w0 = (float)(int8_t)((wd >> b0) & 0xffu) * sc;
                    const float w1 = (float)(int8_t)((wd >> (b0 + 8)) & 0xffu) * sc;
                    const __half2 hh = __floats2half2_rn(w0, w1);
                    const float2 hf = __half22float2(hh);
                    const __half2 ll = __floats2half2_rn(w0 - hf.x, w1 - hf.y);
                    hv[p] = *reinterpret_cast<const uint32_t *>(&hh);
                    lv[p] = *reinterpret_cast<const uint32_t *>(&ll);
                }
                const int off = r * 128 + (((4 * h + c) ^ (r & 7)) * 16);
                *reinterpret_cast<uint4 *>(ahi + off) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
                *reinterpret_cast<uint4 *>(alo + off) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
            }
            fence_proxy_async();  // A visible to the tensor core; raw reads done before the refill
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(empty + st);
                mbar_arrive(afull + (i & 1));
            }
        }
    }
    __syncthreads();
    // ---- epilogue, all sixteen warps (their roles above are done): warp w reads TMEM lanes
    // 32 (w % 4) .. and the 16-column groups cg, cg + 4, ... of its column set cg = w / 4 ----
    const bool epi = true;
    const int q4 = warp & 3, cg = warp >> 2, r = q4 * 32 + lane;
    bool ok = true;
    if (epi) {
        ok = !*fail && mbar_wait(accf, 0u, a.err);
        if (!ok) *fail = 1;
        tc_fence_after();
    }
    if (ks == 1) {
        if (epi)
            for (int c0 = 16 * cg; c0 < NU; c0 += 64) {
                // slot m = hi column m + lo column NU + m
                float v[16], lo[16];
                tmem_ld16(taddr + ((uint32_t)(q4 * 32) << 16) + (uint32_t)c0, v);
                tmem_ld16(taddr + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(NU + c0), lo);
                if (ok && batched) {
                    int rr[16], mm[16];
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        v[e] += lo[e];
                        rr[e] = r;
                        mm[e] = c0 + e;
                    }
                    emit16(v, rr, mm);
                } else if (ok) {
#pragma unroll
                    for (int e = 0; e < 16; ++e) emit(v[e] + lo[e], r, c0 + e);
                }
            }
        if (epi) tc_fence_before();
    } else {
        const int R = L.rmax;
        if (!started) {  // every block of the cluster has started
            __syncwarp();
            cluster_wait_acquire();
        }
        if (L.recv_alias) {
            // the partials go into the weight ring: every block of the cluster must be past its
            // MMAs (its epilogue warps saw the accumulator complete) before any of them stores
            __syncwarp();
            cluster_arrive_relaxed();
            __syncwarp();
            cluster_wait_acquire();
        }
        if (epi) {
            // row r belongs to block o: partial -> o's recv[split][m][r - r0(o)]
            int o = 0;
            while (o + 1 < ks && ((o + 1) * kTileRows) / ks <= r) ++o;
            const int rr = r - (o * kTileRows) / ks;
            const unsigned dst = cluster_map(recv, (unsigned)o) + (unsigned)((split * M * R + rr) * 4);
            for (int c0 = 16 * cg; c0 < NU; c0 += 64) {
                float v[16], lo[16];
                tmem_ld16(taddr + ((uint32_t)(q4 * 32) << 16) + (uint32_t)c0, v);
                tmem_ld16(taddr + ((uint32_t)(q4 * 32) << 16) + (uint32_t)(NU + c0), lo);
#pragma unroll
                for (int e = 0; e < 16; ++e)
                    if (c0 + e < M) st_cluster_f32(dst + (unsigned)((c0 + e) * R * 4), v[e] + lo[e]);
            }
            tc_fence_before();
        }
        // the owned rows [r0, r0 + nr): thread t adds up output row rr = t mod nr for the sequences
        // m = t / nr + j * per (neighbouring threads: neighbouring outputs), so the row's index
        // arithmetic and bias are done once; residual values load while the partials arrive
        const int r0 = (split * kTileRows) / ks, nr = ((split + 1) * kTileRows) / ks - r0;
        const int per = kGemmThreads / nr, rr = tid % nr, mt0 = tid / nr, n = n0 + r0 + rr;
        const bool own = tid < per * nr && n < N;
        constexpr int kResPer = 8;
        const bool res_pre = a.out_mode == OUT_RESIDUAL && (M + per - 1) / per <= kResPer;
        float resv[kResPer];
#pragma unroll
        for (int j = 0; j < kResPer; ++j) {
            const int m = mt0 + j * per;
            resv[j] = res_pre && own && !*fail && m < M ? a.y[(size_t)m * N + n] : 0.f;
        }
        __syncwarp();
        cluster_arrive_release();
        cluster_wait_acquire();
        // add the ks partials in split order, then the epilogue
        if (!*fail && own) {
            const float b = bias_s[r0 + rr];
            if (res_pre) {
#pragma unroll
                for (int j = 0; j < kResPer; ++j) {
                    const int m = mt0 + j * per;
                    if (m >= M) break;
                    float acc = 0.f;
                    for (int q = 0; q < ks; ++q) acc += recv[(q * M + m) * R + rr];
                    if (mi_s[m]) a.y[(size_t)m * N + n] = resv[j] + (acc + b);
                }
            } else if (a.out_mode == OUT_QKV) {
                const int dm = N / 3, part_ = n / dm, c = n - part_ * dm;
                const int head = c / kHeadDim, dd = c % kHeadDim;
                __half *dst = part_ == 1 ? a.kcache : a.vcache;
                for (int m = mt0; m < M; m += per) {
                    float acc = 0.f;
                    for (int q = 0; q < ks; ++q) acc += recv[(q * M + m) * R + rr];
                    if (!mi_s[m]) continue;
                    const float val = acc + b;
                    if (part_ == 0) {
                        a.y[(size_t)m * dm + c] = val;
                    } else {
                        const size_t row = (((size_t)mi_s[M + m] * a.n_layer + a.layer) * a.n_head + head) * (size_t)a.n_ctx +
                                           (size_t)mi_s[2 * M + m];
                        dst[row * kHeadDim + dd] = __float2half_rn(val);
                    }
                }
            } else {
                for (int m = mt0; m < M; m += per) {
                    float acc = 0.f;
                    for (int q = 0; q < ks; ++q) acc += recv[(q * M + m) * R + rr];
                    emit(acc, r0 + rr, m);
                }
            }
        }
    }
    __syncthreads();
    if (*fail && tid == 0) drain_ring(full, NS, *issued);
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(taddr, kCols);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static int nu_for(int M) { return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128; }

// Clusters of each size that can be resident at once (a cluster's blocks share one GPC, so
// fewer clusters of 8 fit than 148 / 8); 0 = not queried.  A launch keeps its tiles within one
// wave of clusters.
static int g_max_clusters[9];

static bool plan_gemm_tc(const GemvArgs &a, int sms, int &nu, GemmTcLaunch &L, int &tiles, int &chunks, bool &bt) {
    const int N = a.W.N, K = a.W.K;
    const bool q8 = a.W.type == WT_Q8;
    if (a.M < 16 || K % kKB != 0 || N < 1) return false;
    if (!(a.W.type == WT_F16 || (q8 && a.W.st && N % kTileRows == 0))) return false;
    // more than 128 rows (f16): the activations come staged as f16 hi / lo rows (k_act_hilo)
    bt = gemm_tc_staged(a);
    if (q8 && a.M > 128) return false;
    if (!bt && a.in_mode != IN_ACT && (K % 128 != 0 || K > 1280)) return false;
    if (!bt && a.in_mode == IN_EMBED_LN && a.E.type != WT_F16) return false;
    chunks = (a.M + 127) / 128;
    L.mchunk = (a.M + chunks - 1) / chunks;
    const int M = L.mchunk;  // rows of one block
    nu = nu_for(M);
    tiles = (N + kTileRows - 1) / kTileRows;
    L.KB = K / kKB;
    int ks = sms / (tiles * chunks);
    ks = ks < 1 ? 1 : ks > 8 ? 8 : ks;
    if (ks > L.KB) ks = L.KB;
    while (ks > 1 && g_max_clusters[ks] > 0 && g_max_clusters[ks] < tiles * chunks) --ks;
    L.ks = ks;
    L.nkb_max = (L.KB + ks - 1) / ks;
    const size_t bbytes = bt ? 0 : (size_t)L.nkb_max * 2 * nu * 128;  // hi and lo rows
    const size_t lnbytes = (a.in_mode == IN_ACT || bt) ? 0 : (size_t)2 * L.nkb_max * kKB * 4;
    const size_t mibytes = ((size_t)5 * M * 4 + 15) & ~(size_t)15;
    L.rmax = (kTileRows + ks - 1) / ks;
    const size_t recvbytes = ks > 1 ? (((size_t)ks * M * L.rmax * 4 + 15) & ~(size_t)15) : 0;
    const size_t statbytes = (size_t)M * 8;  // 8-byte multiple: keeps recv / barriers aligned
    const size_t fixed = bbytes + lnbytes + 512 + mibytes + statbytes + 256 + (q8 ? 1024 : 0);
    const size_t budget = 220 * 1024;
    // weight ring: f16 tiles straight from TMA; Q8_0 raw int8 + scale stages after the two
    // dequantised A stages (the A stages come first, 1024-aligned for the swizzle)
    const size_t sb = q8 ? kRawStage : bt ? (size_t)kStageBytes + 2 * (size_t)nu * 128 : (size_t)kStageBytes;
    const size_t front = q8 ? 2 * (size_t)kAStage : 0;
    // the partials get their own buffer when it fits beside two stages, else they reuse the ring
    L.recv_alias = fixed + front + recvbytes + 2 * sb > budget;
    const size_t own = L.recv_alias ? 0 : recvbytes;
    int ns_need = 2;
    if (L.recv_alias && recvbytes > front) ns_need = (int)((recvbytes - front + sb - 1) / sb);
    if (ns_need < 2) ns_need = 2;
    if (fixed + front + own + (size_t)ns_need * sb > budget) return false;
    int ns = (int)((budget - fixed - front - own) / sb);  // as many stages as fit, up to the k-blocks
    if (ns > (q8 ? 12 : 8)) ns = q8 ? 12 : 8;
    if (ns > L.nkb_max) ns = L.nkb_max;
    if (ns < ns_need) ns = ns_need;
    L.n_stages = ns;
    L.ring_off = (unsigned)front;
    // B after the ring, 1024-aligned (2 nu * 128 B per k-block keeps the k-blocks so)
    L.b_off = (unsigned)((front + ns * sb + 1023) & ~(size_t)1023);
    L.ln_off = L.b_off + (unsigned)bbytes;
    L.bias_off = L.ln_off + (unsigned)lnbytes;
    L.mi_off = L.bias_off + 512;
    L.stat_off = L.mi_off + (unsigned)mibytes;
    L.recv_off = L.stat_off + (unsigned)statbytes;
    L.bar_off = L.recv_off + (unsigned)own;
    return true;
}

// Dynamic shared memory of a launch.  A block holds 2 nu tensor-memory columns of the SM's 512
// from before griddepcontrol.wait to its exit, and split blocks wait for one another at the
// cluster barrier, so no more blocks may be resident on an SM than its columns serve: from
// 128 columns on, the request is raised until 228 KB of shared memory per SM admits no more.
static size_t gemm_tc_smem(const GemmTcLaunch &L, int nu) {
    size_t bytes = (size_t)L.bar_off + (2 * L.n_stages + 5) * 8 + 16 + 1024;
    const int cols = 2 * nu;
    if (cols >= 128) {
        const size_t per_sm = 228 * 1024, fit = 512 / cols;
        const size_t floor_bytes = per_sm / (fit + 1) + 1;
        if (bytes < floor_bytes) bytes = floor_bytes;
    }
    return bytes;
}

template <int NU, int WT, bool BT>
static cudaError_t launch_gemm_tc_t(const GemvArgs &a, const CUtensorMap &map, const CUtensorMap &bmap,
                                    const GemmTcLaunch &L, int tiles, int chunks, cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(L.ks, tiles, chunks);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = gemm_tc_smem(L, NU);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (L.ks > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = L.ks;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, k_gemm_tc<NU, WT, BT>, a, map, bmap, L);
}

template <int WT>
static cudaError_t prep_wt() {
    cudaError_t e = allow_dynamic_smem(k_gemm_tc<16, WT, false>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_gemm_tc<32, WT, false>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_gemm_tc<64, WT, false>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_gemm_tc<128, WT, false>);
    return e;
}

cudaError_t gemm_tc_prepare() {
    cudaError_t e = prep_wt<WT_F16>();
    if (e == cudaSuccess) e = prep_wt<WT_Q8>();
    if (e == cudaSuccess) e = allow_dynamic_smem(k_gemm_tc<16, WT_F16, true>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_gemm_tc<32, WT_F16, true>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_gemm_tc<64, WT_F16, true>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_gemm_tc<128, WT_F16, true>);
    if (e != cudaSuccess) return e;
    // one block per SM (the register file), so the count does not depend on shared memory
    for (int ks = 2; ks <= 8; ++ks) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(ks);
        cfg.blockDim = dim3(kGemmThreads);
        cfg.dynamicSmemBytes = 100 * 1024;
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = ks;
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, k_gemm_tc<32, WT_F16, false>, &cfg) == cudaSuccess) g_max_clusters[ks] = n;
        else cudaGetLastError();
    }
    return cudaSuccess;
}

// f16 projections of at least this many rows take their activations staged as f16 hi / lo rows
// (k_act_hilo) instead of building the B operand in every block (W4J_STAGED_MIN_ROWS overrides).
// Measured at 224-token turbo decodes: staged from 65 rows is 2.1x faster at 128 rows per GPU and
// equal at 64; below that the extra launch costs more than the in-block build (32 rows: -10 %).
static int staged_min_rows() {
    static const int v = [] {
        const char *e = getenv("W4J_STAGED_MIN_ROWS");
        const int r = e ? atoi(e) : 65;
        return r < 16 ? 16 : r;
    }();
    return v;
}

// cudaErrorNotSupported when the projection is outside the tensor-core kernel's range.
bool gemm_tc_staged(const GemvArgs &a) { return a.W.type == WT_F16 && (a.M > 128 || a.M >= staged_min_rows()); }

bool gemm_tc_supported(const GemvArgs &a, int sms) {
    int nu, tiles, chunks;
    bool bt;
    GemmTcLaunch L;
    return plan_gemm_tc(a, sms, nu, L, tiles, chunks, bt);
}

cudaError_t launch_gemm_tc(const GemvArgs &a, const void *tmap, const void *bmap, int sms, cudaStream_t s, bool pdl) {
    int nu, tiles, chunks;
    bool bt = false;
    GemmTcLaunch L;
    if (!tmap || !plan_gemm_tc(a, sms, nu, L, tiles, chunks, bt) || (bt && !bmap)) return cudaErrorNotSupported;
    const CUtensorMap &map = *reinterpret_cast<const CUtensorMap *>(tmap);
    const CUtensorMap &bm = bt ? *reinterpret_cast<const CUtensorMap *>(bmap) : map;
    if (bt) switch (nu) {  // staged B tiles of 2 nu rows (hi, lo)
            case 16: return launch_gemm_tc_t<16, WT_F16, true>(a, map, bm, L, tiles, chunks, s, pdl);
            case 32: return launch_gemm_tc_t<32, WT_F16, true>(a, map, bm, L, tiles, chunks, s, pdl);
            case 64: return launch_gemm_tc_t<64, WT_F16, true>(a, map, bm, L, tiles, chunks, s, pdl);
            default: return launch_gemm_tc_t<128, WT_F16, true>(a, map, bm, L, tiles, chunks, s, pdl);
        }
    if (a.W.type == WT_Q8) switch (nu) {
            case 16: return launch_gemm_tc_t<16, WT_Q8, false>(a, map, bm, L, tiles, chunks, s, pdl);
            case 32: return launch_gemm_tc_t<32, WT_Q8, false>(a, map, bm, L, tiles, chunks, s, pdl);
            case 64: return launch_gemm_tc_t<64, WT_Q8, false>(a, map, bm, L, tiles, chunks, s, pdl);
            default: return launch_gemm_tc_t<128, WT_Q8, false>(a, map, bm, L, tiles, chunks, s, pdl);
        }
    switch (nu) {
        case 16: return launch_gemm_tc_t<16, WT_F16, false>(a, map, bm, L, tiles, chunks, s, pdl);
        case 32: return launch_gemm_tc_t<32, WT_F16, false>(a, map, bm, L, tiles, chunks, s, pdl);
        case 64: return launch_gemm_tc_t<64, WT_F16, false>(a, map, bm, L, tiles, chunks, s, pdl);
        default: return launch_gemm_tc_t<128, WT_F16, false>(a, map, bm, L, tiles, chunks, s, pdl);
    }
}

// ---------------------------------------------------------------------------
// k_act_hilo: the activations of a staged projection, once, as the UMMA B operand's f16 hi / lo
// rows: out[(z * 2 nu + r) * K + k] = hi, out[(z * 2 nu + nu + r) * K + k] = lo for sequence
// m = z * mchunk + r (rows past the chunk's sequences zero; nu = the GEMM's row tile), after the input mode
// (plain, LayerNorm of x, or token + positional embedding then LayerNorm, kept in x_out).
// One warp per (chunk, row, segment of K): a LayerNorm row is one segment (Tensor.java:592-619,
// two-pass, eps 1e-5); a plain row of more than 1280 values is cut into `parts` segments of at most
// 1280, a multiple of 128, so every lane has all its loads of a segment in flight at once.
// ---------------------------------------------------------------------------
static int act_hilo_parts(const GemvArgs &a) {
    const int K = a.W.K;
    if (a.in_mode != IN_ACT || K % 128 != 0 || K <= 1280) return 1;
    int p = (K + 1279) / 1280;
    while (K % (p * 128) != 0) ++p;
    return p;
}

__global__ void __launch_bounds__(256) k_act_hilo(GemvArgs a, int mchunk, int chunks, int nu, int parts, __half *out) {
    const int K = a.W.K;
    const int gw = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    pdl_trigger();
    // the LayerNorm parameters are weights: in registers before the wait
    constexpr int kLnF4 = 10;
    float4 gv[kLnF4], bv[kLnF4];
    if (a.in_mode != IN_ACT)
#pragma unroll
        for (int j = 0; j < kLnF4; ++j) {
            const bool in = j < K / 128 && K <= 128 * kLnF4;
            gv[j] = in ? reinterpret_cast<const float4 *>(a.ln_g)[lane + 32 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
            bv[j] = in ? reinterpret_cast<const float4 *>(a.ln_b)[lane + 32 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    pdl_wait();
    if (gw >= chunks * nu * parts) return;
    const int row = gw / parts, part = gw - row * parts;
    const int z = row / nu, r = row - z * nu, m = z * mchunk + r;
    __half *hi = out + ((size_t)z * 2 * nu + r) * K, *lo = hi + (size_t)nu * K;
    const bool live = r < mchunk && m < a.M;
    auto put = [&](int k, float4 v) {
        const __half2 h0 = __floats2half2_rn(v.x, v.y), h1 = __floats2half2_rn(v.z, v.w);
        const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
        const __half2 l0 = __floats2half2_rn(v.x - f0.x, v.y - f0.y), l1 = __floats2half2_rn(v.z - f1.x, v.w - f1.y);
        *reinterpret_cast<uint2 *>(hi + k) =
            make_uint2(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1));
        *reinterpret_cast<uint2 *>(lo + k) =
            make_uint2(*reinterpret_cast<const uint32_t *>(&l0), *reinterpret_cast<const uint32_t *>(&l1));
    };
    const int seg = K / parts, k0 = part * seg;
    if (!live) {
        for (int k = k0 + 4 * lane; k < k0 + seg; k += 128) put(k, make_float4(0.f, 0.f, 0.f, 0.f));
        return;
    }
    if (a.in_mode == IN_ACT) {
        const float4 *src = reinterpret_cast<const float4 *>(a.act + (size_t)m * K + k0);
        if (seg % 128 == 0 && seg <= 128 * kLnF4) {  // every load of the lane issued before any store
            const int nf = seg / 128;
            float4 v[kLnF4];
#pragma unroll
            for (int j = 0; j < kLnF4; ++j) v[j] = j < nf ? src[lane + 32 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < kLnF4; ++j)
                if (j < nf) put(k0 + 4 * (lane + 32 * j), v[j]);
        } else {
            for (int c = lane; c < seg / 4; c += 32) put(k0 + 4 * c, src[c]);
        }
        return;
    }
    // LayerNorm inputs: K <= 1280, a multiple of 128 (the row in registers)
    const int nf4 = K / 128;
    float4 v[kLnF4];
    if (a.in_mode == IN_LN) {
        const float4 *src = reinterpret_cast<const float4 *>(a.act + (size_t)m * K);
#pragma unroll
        for (int j = 0; j < kLnF4; ++j) v[j] = j < nf4 ? src[lane + 32 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
    } else {  // x = E[tok] + P[pos] (WhisperDecoder.java:66-80), kept in x_out
        const uint2 *e = reinterpret_cast<const uint2 *>(a.E.h + (size_t)a.tok[m] * K);
        const float4 *pe = reinterpret_cast<const float4 *>(a.pos_emb + (size_t)pe_row(a, m) * K);
#pragma unroll
        for (int j = 0; j < kLnF4; ++j) {
            if (j < nf4) {
                const uint2 eu = e[lane + 32 * j];
                const float4 p = pe[lane + 32 * j];
                const float2 l2 = __half22float2(*reinterpret_cast<const __half2 *>(&eu.x));
                const float2 h2 = __half22float2(*reinterpret_cast<const __half2 *>(&eu.y));
                v[j] = make_float4(l2.x + p.x, l2.y + p.y, h2.x + p.z, h2.y + p.w);
                if (a.x_out) reinterpret_cast<float4 *>(a.x_out)[(size_t)m * (K / 4) + lane + 32 * j] = v[j];
            } else {
                v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    }
    float sm = 0.f;
#pragma unroll
    for (int j = 0; j < kLnF4; ++j)
        if (j < nf4) sm += (v[j].x + v[j].y) + (v[j].z + v[j].w);
    const float mean = warp_sum(sm) / (float)K;
    float v2 = 0.f;
#pragma unroll
    for (int j = 0; j < kLnF4; ++j)
        if (j < nf4) {
            const float dx = v[j].x - mean, dy = v[j].y - mean, dz = v[j].z - mean, dw = v[j].w - mean;
            v2 += (dx * dx + dy * dy) + (dz * dz + dw * dw);
        }
    const float inv_std = 1.0f / sqrtf(warp_sum(v2) / (float)K + 1e-5f);
#pragma unroll
    for (int j = 0; j < kLnF4; ++j)
        if (j < nf4) {
            const int k = 4 * (lane + 32 * j);
            const float4 g = gv[j], b = bv[j];
            put(k, make_float4((v[j].x - mean) * inv_std * g.x + b.x, (v[j].y - mean) * inv_std * g.y + b.y,
                               (v[j].z - mean) * inv_std * g.z + b.z, (v[j].w - mean) * inv_std * g.w + b.w));
        }
}

// Rows of the staged activation buffer for M sequences (at most chunks * 256), and the rows of one
// staged B tile (2 nu: the tensor map's box height)
int act_hilo_rows(int M) { return ((M + 127) / 128) * 256; }
int act_hilo_box_rows(int M) {
    const int chunks = (M + 127) / 128, mchunk = (M + chunks - 1) / chunks;
    return 2 * nu_for(mchunk);
}

cudaError_t launch_act_hilo(const GemvArgs &a, __half *out, cudaStream_t s, bool pdl) {
    const int K = a.W.K;
    if (K % 4 != 0 || (a.in_mode != IN_ACT && (K % 128 != 0 || K > 1280))) return cudaErrorNotSupported;
    const int chunks = (a.M + 127) / 128, mchunk = (a.M + chunks - 1) / chunks, nu = nu_for(mchunk);
    const int parts = act_hilo_parts(a);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(chunks * nu * parts * 32 + 255) / 256);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_act_hilo, a, mchunk, chunks, nu, parts, out);
}

}  // namespace w4j
