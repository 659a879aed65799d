// k_logits_tc.cu — vocabulary logits on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces the logits GEMV of WhisperDecoder.forwardWithAttn (nn/WhisperDecoder.java:102-103,
// Tensor.matmulTransB M=1 path, tensor/Tensor.java:316-340): logits[m][v] = LN(x[m]) . E[v]
// for the M live sequences (M <= 32), followed by the logit processors and block reductions
// of logits_rows_epilogue (shared with the SIMT kernel in k_gemv.cu).
//
// Each block owns whole 128-row tiles of the token embedding E (V x d, f16, GGML row layout).
//   * TMA (cp.async.bulk.tensor.2d, 128-byte swizzle) streams [128 rows x 64 k] tiles through a
//     ring of shared-memory stages; the first stages are issued before griddepcontrol.wait, so
//     they load while the previous kernel finishes.
//   * The activations are LayerNorm-ed once per block straight into the MMA's B operand:
//     [NU x d] f16, K-major with the same 128-byte swizzle (NU = M padded to 16 or 32).
//   * One thread issues tcgen05.mma.kind::f16 (M=128, N=NU, K=16) into a double-buffered f32
//     accumulator in tensor memory; tcgen05.commit releases ring stages and hands finished
//     tiles to four epilogue warps, which read TMEM with tcgen05.ld into a shared tile.
// Every wait is bounded; a time-out raises the device error word and the block drains.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "logits_epilogue.cuh"
#include "tc_common.cuh"
#include "w4j_internal.cuh"

namespace w4j {

// 16 warps: warp 0 produces, warp 1 issues the MMAs, warps 4-7 move tiles out of TMEM; all
// sixteen build the B operand (one LayerNorm row per warp at a time) and run the row epilogue.
constexpr int kLogitsThreads = 512;

struct LogitsBigLaunch {
    int tiles_total;  // ceil(V / 128): embedding tiles, also the records per row
    int chunks;       // chunks of rows (grid-independent: every block walks them all)
    int mchunk;       // rows per chunk
    int n_stages;
    unsigned tile_off, mk_off, bar_off;  // shared-memory layout (bytes)
};

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

struct LogitsTcLaunch {
    int tiles_total;  // ceil(V / 128)
    int ch;           // max rows of a block (tiles per block * 128)
    int n_stages;
    unsigned b_off, tile_off, ln_off, mk_off, bar_off;  // shared-memory layout (bytes)
};


template <int NU>
__global__ void __launch_bounds__(kLogitsThreads, 1) k_logits_tc(LogitsArgs a, const __grid_constant__ CUtensorMap tmap,
                                                       LogitsTcLaunch L) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // the 128-byte swizzle pattern is anchored on 1024-byte boundaries: align the base
    unsigned char *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int P = gridDim.x;
    const int t0 = (int)(((long long)blockIdx.x * L.tiles_total) / P);
    const int t1 = (int)(((long long)(blockIdx.x + 1) * L.tiles_total) / P);
    const int n_tiles = t1 - t0;
    const int lo = min(a.V, t0 * kTileRows), hi = min(a.V, t1 * kTileRows);
    const int d = a.d, KB = d / kKB, NS = L.n_stages;
    const int total = n_tiles * KB;
    unsigned char *ring = smem;
    unsigned char *bop = smem + L.b_off;  // [KB][NU rows][128 B]
    float *tile = reinterpret_cast<float *>(smem + L.tile_off);
    float *ln_s = reinterpret_cast<float *>(smem + L.ln_off);
    int2 *mk_rg = reinterpret_cast<int2 *>(smem + L.mk_off);  // 16-byte aligned: the int2 array first
    int *mk_act = reinterpret_cast<int *>(mk_rg + (size_t)a.M * kMaxRanges);
    int *mk_nr = mk_act + a.M, *mk_cnt = mk_nr + a.M;
    int *mk_dyn = mk_cnt + a.M;
    int *mk_stat = mk_dyn + (size_t)a.M * kDynStage;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bar_off);
    uint64_t *empty = full + NS;
    uint64_t *accf = empty + NS;  // [2]
    uint64_t *acce = accf + 2;    // [2]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(acce + 2);
    volatile int *fail = reinterpret_cast<volatile int *>(tslot + 1);
    volatile int *issued = fail + 1;  // weight tiles whose copy has been started
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr uint32_t kCols = NU * 2 <= 32 ? 32 : 64;

    // ---- independent of the previous kernel: barriers, TMEM, first weight stages, LN params ----
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, 1);
        }
        mbar_init(accf + 0, 1);
        mbar_init(accf + 1, 1);
        mbar_init(acce + 0, 4);
        mbar_init(acce + 1, 4);
        *fail = 0;
        fence_mbar_init();
        const int first = a.withhold ? 0 : (NS < total ? NS : total);
        for (int i = 0; i < first; ++i) {
            mbar_expect_tx(full + i, kStageBytes);
            tma_load_2d(ring + (size_t)i * kStageBytes, &tmap, (i % KB) * kKB, (t0 + i / KB) * kTileRows, full + i);
        }
        *issued = first;
    }
    if (warp == 1) {
        tmem_alloc(tslot, kCols);
        tmem_relinquish();
    }
    for (int i = tid; i < 2 * d; i += blockDim.x) ln_s[i] = i < d ? a.ln_g[i] : a.ln_b[i - d];
    // liveness and masks of the rows: written by the previous step's select kernel (an earlier
    // graph launch) or by the mask initialisation that completed before this kernel started
    if (a.active)
        for (int i = tid; i < a.M; i += blockDim.x) mk_act[i] = a.active[i];
    if (a.use_mask) {
        const MaskArgs &mk = a.mask;
        for (int i = tid; i < a.M; i += blockDim.x) {
            mk_nr[i] = mk.n_ranges[i];
            mk_cnt[i] = mk.dyn_count[i];
        }
        for (int i = tid; i < a.M * kMaxRanges; i += blockDim.x) mk_rg[i] = mk.ranges[i];
        for (int i = tid; i < min(mk.n_static, kStatStage); i += blockDim.x) mk_stat[i] = mk.static_list[i];
        __syncthreads();
        for (int i = tid; i < a.M * kDynStage; i += blockDim.x) {
            const int m = i / kDynStage, j = i - m * kDynStage;
            if (j < mk_cnt[m]) mk_dyn[i] = mk.dyn_list[(size_t)m * mk.dyn_stride + j];
        }
    }
    // rows M..NU of the B operand are zero whatever the activations are
    for (int i = tid; i < (NU - a.M) * (d / 8); i += blockDim.x) {
        const int m = a.M + i / (d / 8), c = i % (d / 8);
        const int kb = c / 8, cc = c % 8;
        *reinterpret_cast<uint4 *>(bop + (size_t)kb * NU * 128 + (size_t)m * 128 + ((cc ^ (m & 7)) * 16)) =
            make_uint4(0, 0, 0, 0);
    }
    pdl_trigger();
    pdl_wait();
    __syncthreads();  // ln_s is read across warps below

    // ---- B operand: LayerNorm(x[m]) as f16, K-major, 128-byte swizzle (rows >= M were zeroed) ----
    for (int m = warp; m < a.M; m += kLogitsThreads / 32) {
        const bool live = true;
        constexpr int kMaxChunks = 1280 / 8 / 32;  // 16-byte chunks per lane for d <= 1280
        float v[kMaxChunks][8];
        const int nch = d / 8;  // chunks of 8 along K
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < kMaxChunks; ++j) {
            const int c = lane + 32 * j;
            if (live && c < nch) {
                const float4 x0 = *reinterpret_cast<const float4 *>(a.x + (size_t)m * d + c * 8);
                const float4 x1 = *reinterpret_cast<const float4 *>(a.x + (size_t)m * d + c * 8 + 4);
                v[j][0] = x0.x; v[j][1] = x0.y; v[j][2] = x0.z; v[j][3] = x0.w;
                v[j][4] = x1.x; v[j][5] = x1.y; v[j][6] = x1.z; v[j][7] = x1.w;
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) v[j][e] = 0.f;
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) s += v[j][e];
        }
        const float mean = warp_sum(s) / (float)d;
        float s2 = 0.f;
#pragma unroll
        for (int j = 0; j < kMaxChunks; ++j)
            if (lane + 32 * j < nch)
#pragma unroll
                for (int e = 0; e < 8; ++e) s2 += (v[j][e] - mean) * (v[j][e] - mean);
        const float inv_std = 1.0f / sqrtf(warp_sum(s2) / (float)d + 1e-5f);
#pragma unroll
        for (int j = 0; j < kMaxChunks; ++j) {
            const int c = lane + 32 * j;
            if (c >= nch) continue;
            uint32_t hpk[4];
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
                const int k = c * 8 + e;
                const float y0 = live ? (v[j][e] - mean) * inv_std * ln_s[k] + ln_s[d + k] : 0.f;
                const float y1 = live ? (v[j][e + 1] - mean) * inv_std * ln_s[k + 1] + ln_s[d + k + 1] : 0.f;
                const __half2 h = __floats2half2_rn(y0, y1);
                hpk[e / 2] = *reinterpret_cast<const uint32_t *>(&h);
            }
            const int kb = c / 8, cc = c % 8;
            unsigned char *dst = bop + (size_t)kb * NU * 128 + (size_t)m * 128 + ((cc ^ (m & 7)) * 16);
            *reinterpret_cast<uint4 *>(dst) = make_uint4(hpk[0], hpk[1], hpk[2], hpk[3]);
        }
    }
    fence_proxy_async();  // generic-proxy writes of B visible to the tensor core
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = *tslot;
    const uint32_t idesc = idesc_f16(kTileRows, NU);

    if (warp == 0 && lane == 0) {
        // ---- producer: stream the remaining tiles as stages free up ----
        for (int i = NS; i < total && !*fail && !a.withhold; ++i) {
            const int st = i % NS, use = i / NS;
            if (!mbar_wait(empty + st, (unsigned)((use - 1) & 1), a.err)) {
                *fail = 1;
                break;
            }
            mbar_expect_tx(full + st, kStageBytes);
            tma_load_2d(ring + (size_t)st * kStageBytes, &tmap, (i % KB) * kKB, (t0 + i / KB) * kTileRows, full + st);
            *issued = i + 1;
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer ----
        const uint32_t ring_a = smem_u32(ring), b_a = smem_u32(bop);
        for (int lt = 0; lt < n_tiles && !*fail; ++lt) {
            const int b = lt & 1;
            if (lt >= 2 && !mbar_wait(acce + b, (unsigned)(((lt - 2) >> 1) & 1), a.err)) {
                *fail = 1;
                break;
            }
            tc_fence_after();
            for (int kb = 0; kb < KB; ++kb) {
                const int i = lt * KB + kb, st = i % NS;
                if (!mbar_wait(full + st, (unsigned)((i / NS) & 1), a.err)) {
                    *fail = 1;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int j = 0; j < kKB / 16; ++j) {
                    const uint64_t ad = sw128_desc(ring_a + (uint32_t)st * kStageBytes + j * 32);
                    const uint64_t bd = sw128_desc(b_a + (uint32_t)kb * NU * 128 + j * 32);
                    umma_f16(taddr + (uint32_t)(b * NU), ad, bd, idesc, (kb | j) != 0);
                }
                umma_commit(empty + st);  // the stage is free once these MMAs have read it
            }
            umma_commit(accf + b);  // tile lt's accumulator is complete
        }
    } else if (warp >= 4 && warp < 8) {
        // ---- epilogue: TMEM -> shared logits tile ----
        const int q = warp - 4;  // TMEM lane quarter of this warp
        for (int lt = 0; lt < n_tiles; ++lt) {
            const int b = lt & 1;
            if (*fail || !mbar_wait(accf + b, (unsigned)((lt >> 1) & 1), a.err)) {
                *fail = 1;
                break;
            }
            tc_fence_after();
            const int row = lt * kTileRows + q * 32 + lane;
#pragma unroll
            for (int c0 = 0; c0 < NU; c0 += 16) {
                float v[16];
                tmem_ld16(taddr + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * NU + c0), v);
                if (row < hi - lo)
#pragma unroll
                    for (int e = 0; e < 16; ++e)
                        if (c0 + e < a.M) tile[(size_t)(c0 + e) * L.ch + row] = v[e];
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acce + b);
        }
    }
    __syncthreads();
    const bool ok = !*fail;
    if (ok && a.raw_out)
        for (int i = tid; i < a.M * (hi - lo); i += blockDim.x) {
            const int m = i / (hi - lo), r = i - m * (hi - lo);
            a.raw_out[(size_t)m * a.V + lo + r] = tile[(size_t)m * L.ch + r];
        }
    const MaskStage ms{mk_act, mk_nr, mk_rg, mk_cnt, mk_dyn, mk_stat};
    logits_rows_epilogue(a, tile, L.ch, a.M, 0, lo, hi, ok, &ms);
    __syncthreads();
    if (!ok && tid == 0) drain_ring(full, NS, *issued);
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(taddr, kCols);
    }
}

// ---------------------------------------------------------------------------
// k_logits_big: the same vocabulary pass for 33 .. 256 rows in one launch, reading the embedding
// once.  The rows come LayerNorm-ed and rounded to f16 from the staged activation buffer (k_act_hilo's
// hi rows, K = d: the f16(LN(x)) that k_logits_tc builds in shared memory) and stream beside the
// embedding: a stage is a [128 x 64] embedding tile and the [NU x 64] tile of the rows.  Work items
// are (embedding tile, chunk of <= 128 rows) pairs, tile-major, so the second chunk of a tile finds
// the tile's bytes in L2.  Each item's logits go through the row epilogue's processors and
// reductions (logits_row_thread: one thread per row, in id order), one record per (row, embedding
// tile): P = ceil(V / 128) records per row for the greedy / sampling select.
// Warps: 0 produces, 1 issues the MMAs, 4-7 move accumulators out of TMEM, 2-15 take part in the
// epilogue (threads 64 .. 64 + rows scan the rows).
// ---------------------------------------------------------------------------
template <int NU>
__global__ void __launch_bounds__(kLogitsThreads, 1)
    k_logits_big(LogitsArgs a, const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap bmap,
                 LogitsBigLaunch L) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    constexpr unsigned kB = NU * 128, kSt = kStageBytes + kB;  // stage: embedding tile, then row tile
    constexpr uint32_t kCols = 2 * NU;                         // two accumulators
    constexpr int kEpiWarp0 = 2, kEpiWarps = kLogitsThreads / 32 - kEpiWarp0;
    const int P = gridDim.x;
    const int t0 = (int)(((long long)blockIdx.x * L.tiles_total) / P);
    const int t1 = (int)(((long long)(blockIdx.x + 1) * L.tiles_total) / P);
    const int d = a.d, KB = d / kKB, NS = L.n_stages, CH = L.chunks;
    const int items = (t1 - t0) * CH, total = items * KB;
    unsigned char *ring = smem;
    // logits of the item, column-major: tile[id * kTS + row], the odd stride keeps both the
    // accumulator copy (a thread per id) and the row scans (a thread per row) free of bank conflicts
    constexpr int kTS = NU + 1;
    float *tile = reinterpret_cast<float *>(smem + L.tile_off);
    int2 *mk_rg = reinterpret_cast<int2 *>(smem + L.mk_off);
    int *mk_act = reinterpret_cast<int *>(mk_rg + (size_t)a.M * kMaxRanges);
    int *mk_nr = mk_act + a.M, *mk_cnt = mk_nr + a.M;
    int *mk_dyn = mk_cnt + a.M;
    int *mk_stat = mk_dyn + (size_t)a.M * kDynStage;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bar_off);
    uint64_t *empty = full + NS;
    uint64_t *accf = empty + NS;  // [2]
    uint64_t *acce = accf + 2;    // [2]
    uint32_t *tslot = reinterpret_cast<uint32_t *>(acce + 2);
    volatile int *fail = reinterpret_cast<volatile int *>(tslot + 1);
    volatile int *issued = fail + 1;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    auto a_coords = [&](int i, int &x, int &y) {  // stage i: item i / KB (tile-major), k-block i % KB
        x = (i % KB) * kKB;
        y = (t0 + (i / KB) / CH) * kTileRows;
    };
    auto b_coords = [&](int i, int &x, int &y) {
        x = (i % KB) * kKB;
        y = ((i / KB) % CH) * 2 * NU;  // the chunk's hi rows in the staged buffer
    };

    // ---- independent of the previous kernel: barriers, TMEM, the first embedding tiles, masks ----
    const int first = a.withhold ? 0 : (NS < total ? NS : total);
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, 1);
        }
        mbar_init(accf + 0, 1);
        mbar_init(accf + 1, 1);
        mbar_init(acce + 0, 1);
        mbar_init(acce + 1, 1);
        *fail = 0;
        fence_mbar_init();
        for (int i = 0; i < first; ++i) {
            int x, y;
            a_coords(i, x, y);
            mbar_expect_tx(full + i, kSt);  // the row tile follows after the wait
            tma_load_2d(ring + (size_t)i * kSt, &tmap, x, y, full + i);
        }
        *issued = first;
    }
    if (warp == 1) {
        tmem_alloc(tslot, kCols);
        tmem_relinquish();
    }
    if (a.active)
        for (int i = tid; i < a.M; i += blockDim.x) mk_act[i] = a.active[i];
    if (a.use_mask) {
        const MaskArgs &mk = a.mask;
        for (int i = tid; i < a.M; i += blockDim.x) {
            mk_nr[i] = mk.n_ranges[i];
            mk_cnt[i] = mk.dyn_count[i];
        }
        for (int i = tid; i < a.M * kMaxRanges; i += blockDim.x) mk_rg[i] = mk.ranges[i];
        for (int i = tid; i < min(mk.n_static, kStatStage); i += blockDim.x) mk_stat[i] = mk.static_list[i];
        __syncthreads();
        for (int i = tid; i < a.M * kDynStage; i += blockDim.x) {
            const int m = i / kDynStage, j = i - m * kDynStage;
            if (j < mk_cnt[m]) mk_dyn[i] = mk.dyn_list[(size_t)m * mk.dyn_stride + j];
        }
    }
    pdl_trigger();
    pdl_wait();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = *tslot;

    if (warp == 0 && lane == 0) {
        // ---- producer: the row tiles of the first stages, then whole stages as they free up ----
        for (int i = 0; i < first; ++i) {
            int x, y;
            b_coords(i, x, y);
            tma_load_2d(ring + (size_t)i * kSt + kStageBytes, &bmap, x, y, full + i);
        }
        for (int i = NS; i < total && !*fail && !a.withhold; ++i) {
            const int st = i % NS, use = i / NS;
            if (!mbar_wait(empty + st, (unsigned)((use - 1) & 1), a.err)) {
                *fail = 1;
                break;
            }
            int x, y;
            mbar_expect_tx(full + st, kSt);
            a_coords(i, x, y);
            tma_load_2d(ring + (size_t)st * kSt, &tmap, x, y, full + st);
            b_coords(i, x, y);
            tma_load_2d(ring + (size_t)st * kSt + kStageBytes, &bmap, x, y, full + st);
            *issued = i + 1;
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer: item it accumulates into buffer it & 1 ----
        const uint32_t ring_a = smem_u32(ring);
        const uint32_t idesc = idesc_f16(kTileRows, NU);
        for (int it = 0; it < items && !*fail; ++it) {
            const int b = it & 1;
            if (it >= 2 && !mbar_wait(acce + b, (unsigned)(((it - 2) >> 1) & 1), a.err)) {
                *fail = 1;
                break;
            }
            tc_fence_after();
            for (int kb = 0; kb < KB; ++kb) {
                const int i = it * KB + kb, st = i % NS;
                if (!mbar_wait(full + st, (unsigned)((i / NS) & 1), a.err)) {
                    *fail = 1;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int j = 0; j < kKB / 16; ++j) {
                    const uint64_t ad = sw128_desc(ring_a + (uint32_t)st * kSt + j * 32);
                    const uint64_t bd = sw128_desc(ring_a + (uint32_t)st * kSt + kStageBytes + j * 32);
                    umma_f16(taddr + (uint32_t)(b * NU), ad, bd, idesc, (kb | j) != 0);
                }
                umma_commit(empty + st);
            }
            if (*fail) break;
            umma_commit(accf + b);
        }
    } else if (warp >= kEpiWarp0) {
        // ---- epilogue: TMEM -> column-major logits tile -> the row epilogue with one thread per
        // row, one item at a time.  Every epilogue thread passes the same barriers per item, failed
        // or not. ----
        const MaskStage ms{mk_act, mk_nr, mk_rg, mk_cnt, mk_dyn, mk_stat};
        const int etid = tid - kEpiWarp0 * 32, ecount = kEpiWarps * 32;
        for (int it = 0; it < items; ++it) {
            const int b = it & 1, lt = it / CH, z = it % CH;
            if (!*fail && !mbar_wait(accf + b, (unsigned)((it >> 1) & 1), a.err)) *fail = 1;
            tc_fence_after();
            named_bar_sync(1, ecount);
            const bool go = !*fail;
            const int lo = (t0 + lt) * kTileRows, hi = min(a.V, lo + kTileRows), n = hi - lo;
            const int m0 = z * L.mchunk, mt = min(L.mchunk, a.M - m0);
            if (go && warp >= 4 && warp < 8) {
                const int q = warp - 4, row = q * 32 + lane;
#pragma unroll
                for (int c0 = 0; c0 < NU; c0 += 16) {
                    float v[16];
                    tmem_ld16(taddr + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * NU + c0), v);
                    if (row < n)
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            if (c0 + e < mt) tile[(size_t)row * kTS + c0 + e] = v[e];
                }
            }
            tc_fence_before();
            named_bar_sync(1, ecount);
            if (etid == 0) mbar_arrive(acce + b);  // the accumulator may be overwritten
            if (go && a.raw_out)
                for (int i = etid; i < mt * n; i += ecount) {
                    const int mm = i / n, r = i - mm * n;
                    a.raw_out[(size_t)(m0 + mm) * a.V + lo + r] = tile[(size_t)r * kTS + mm];
                }
            if (a.raw_out) named_bar_sync(1, ecount);
            if (go)
                for (int mm = etid; mm < mt; mm += ecount)
                    logits_row_thread(a, tile, kTS, mm, m0, lo, hi, &ms, L.tiles_total, t0 + lt);
            named_bar_sync(1, ecount);
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
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// Tensor map of a row-major f16 matrix [rows][cols] read in [128 rows x 64 cols] boxes with
// the 128-byte swizzle the UMMA K-major operand expects.
bool make_tmap_f16_rows(void *map_out, const void *base, int rows, int cols) {
    return make_tmap_f16_box(map_out, base, rows, cols, kTileRows);
}

bool make_tmap_f16_box(void *map_out, const void *base, int rows, int cols, int box_rows) {
    auto fn = encode_fn();
    if (!fn || cols % kKB != 0 || ((uintptr_t)base & 15) || box_rows < 1 || box_rows > 256) return false;
    CUtensorMap *m = reinterpret_cast<CUtensorMap *>(map_out);
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kKB, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tensor map of a row-major int8 matrix [rows][cols] read in [128 rows x 64 cols] boxes, unswizzled
// (the Q8_0 converters read it with 16-byte loads).
bool make_tmap_i8_rows(void *map_out, const void *base, int rows, int cols) {
    auto fn = encode_fn();
    if (!fn || cols % kKB != 0 || ((uintptr_t)base & 15)) return false;
    CUtensorMap *m = reinterpret_cast<CUtensorMap *>(map_out);
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols};
    const cuuint32_t box[2] = {(cuuint32_t)kKB, (cuuint32_t)kTileRows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Staged masks: ranges (M x kMaxRanges int2), then active, n_ranges, dyn_count (M ints each),
// dyn (M x kDynStage ints), static list (kStatStage ints); a multiple of 16 bytes.
static size_t mask_stage_bytes(int M) {
    return (((size_t)M * (3 + 2 * kMaxRanges + kDynStage) + kStatStage) * 4 + 15) & ~(size_t)15;
}

static bool plan_tc(int M, int V, int d, int P, int &nu, LogitsTcLaunch &L) {
    if (M < 1 || M > 32 || d % kKB != 0 || d > 1280) return false;
    nu = M <= 16 ? 16 : 32;
    L.tiles_total = (V + kTileRows - 1) / kTileRows;
    L.ch = ((L.tiles_total + P - 1) / P) * kTileRows;
    const size_t bbytes = (size_t)nu * d * 2;
    const size_t tbytes = (size_t)M * L.ch * 4;
    const size_t lnbytes = (size_t)2 * d * 4;
    const size_t mkbytes = mask_stage_bytes(M);
    const size_t fixed = bbytes + tbytes + lnbytes + mkbytes + 256;
    const size_t budget = 220 * 1024;
    if (fixed + 2 * kStageBytes > budget) return false;
    // 7 stages (112 KB) keep ~16 MB of the embedding in flight over the GPU, enough to cover
    // DRAM latency, and leave room beside the block for the select kernel that follows
    int ns = (int)((budget - fixed) / kStageBytes);
    L.n_stages = ns > 7 ? 7 : ns;
    L.b_off = (unsigned)(L.n_stages * kStageBytes);  // 1024-byte aligned (stages are 16 KB)
    L.tile_off = L.b_off + (unsigned)bbytes;        // bbytes is a multiple of 2 KB
    L.ln_off = L.tile_off + (unsigned)((tbytes + 15) & ~(size_t)15);
    L.mk_off = L.ln_off + (unsigned)lnbytes;
    L.bar_off = L.mk_off + (unsigned)mkbytes;
    return true;
}

static size_t tc_smem(const LogitsTcLaunch &L) { return (size_t)L.bar_off + (2 * L.n_stages + 4) * 8 + 16 + 1024; }

template <int NU>
static cudaError_t launch_tc_t(const LogitsArgs &a, const CUtensorMap &map, const LogitsTcLaunch &L, int P,
                               cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(P);
    cfg.blockDim = dim3(kLogitsThreads);
    cfg.dynamicSmemBytes = tc_smem(L);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_logits_tc<NU>, a, map, L);
}

cudaError_t logits_tc_prepare() {
    cudaError_t e = allow_dynamic_smem(k_logits_tc<16>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_logits_tc<32>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_logits_big<64>);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_logits_big<128>);
    return e;
}

// The one-launch pass over M rows (33 .. 256, greedy / sampling: no per-block top-k) in chunks
// of the staged activation buffer's layout: ceil(M / 128) chunks of mchunk rows, NU = 64 or 128.
static bool plan_big(int M, int V, int d, int topk, int &nu, LogitsBigLaunch &L) {
    if (M <= 32 || M > kLogitsBigMaxRows || topk != 0 || d % 128 != 0 || d > 1280) return false;
    L.chunks = (M + 127) / 128;
    L.mchunk = (M + L.chunks - 1) / L.chunks;
    nu = L.mchunk <= 64 ? 64 : 128;
    L.tiles_total = (V + kTileRows - 1) / kTileRows;
    const size_t st = (size_t)kStageBytes + (size_t)nu * 128;
    const size_t tbytes = (((size_t)(nu + 1) * kTileRows * 4) + 15) & ~(size_t)15;
    const size_t mkbytes = mask_stage_bytes(M);
    const size_t fixed = tbytes + mkbytes + 256;
    const size_t budget = 220 * 1024;
    if (fixed + 2 * st > budget) return false;
    int ns = (int)((budget - fixed) / st);
    L.n_stages = ns > 6 ? 6 : ns;
    L.tile_off = (unsigned)(L.n_stages * st);  // 1024-byte multiple
    L.mk_off = L.tile_off + (unsigned)tbytes;
    L.bar_off = L.mk_off + (unsigned)mkbytes;
    return true;
}

int logits_big_box_rows(int M) {
    const int chunks = (M + 127) / 128, mchunk = (M + chunks - 1) / chunks;
    return mchunk <= 64 ? 64 : 128;
}

int logits_big_parts(int M, int V, int d, int topk) {
    int nu;
    LogitsBigLaunch L;
    return plan_big(M, V, d, topk, nu, L) ? L.tiles_total : 0;
}

cudaError_t launch_logits_big(const LogitsArgs &a, const void *tmap, const void *bmap, int blocks, cudaStream_t s, bool pdl) {
    int nu;
    LogitsBigLaunch L;
    if (!tmap || !bmap || a.E.type != WT_F16 || !plan_big(a.M, a.V, a.d, a.topk, nu, L)) return cudaErrorNotSupported;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(kLogitsThreads);
    cfg.dynamicSmemBytes = (size_t)L.bar_off + (2 * L.n_stages + 4) * 8 + 16 + 1024;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    const CUtensorMap &map = *reinterpret_cast<const CUtensorMap *>(tmap);
    const CUtensorMap &bm = *reinterpret_cast<const CUtensorMap *>(bmap);
    if (nu == 64) return cudaLaunchKernelEx(&cfg, k_logits_big<64>, a, map, bm, L);
    return cudaLaunchKernelEx(&cfg, k_logits_big<128>, a, map, bm, L);
}

// Returns cudaErrorNotSupported when the shape is outside the tensor-core kernel's range.
cudaError_t launch_logits_tc(const LogitsArgs &a, const void *tmap, int P, cudaStream_t s, bool pdl) {
    int nu;
    LogitsTcLaunch L;
    if (a.topk > kLaneTopK) return cudaErrorInvalidValue;
    if (!tmap || a.E.type != WT_F16 || !plan_tc(a.M, a.V, a.d, P, nu, L)) return cudaErrorNotSupported;
    const CUtensorMap &map = *reinterpret_cast<const CUtensorMap *>(tmap);
    if (nu == 16) return launch_tc_t<16>(a, map, L, P, s, pdl);
    return launch_tc_t<32>(a, map, L, P, s, pdl);
}

}  // namespace w4j
