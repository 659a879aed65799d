// k_xkv_tc.cu — the cross-attention K/V projection of one stream's encoder output on the
// 5th-generation tensor cores, once per chunk: K = xa . Wk^T (+ bk), V = xa . Wv^T + bv for one decoder
// layer (MultiHeadAttention.forward, first-call branch, nn/MultiHeadAttention.java:65-75, which
// the reference runs through Tensor.matmulTiled, tensor/Tensor.java:460-489), written straight
// into the head-major f16 cross cache [head][n_audio_ctx][64] (rearrangeToHeads, :645-659).
//
// Block (n tile, a tile): 128 rows of [Wk; Wv] (the UMMA M) x 128 encoder rows.
//   * One thread streams the weight tiles [128 x 64] f16 with TMA (128-byte swizzle) through a
//     ring of stages.
//   * Eight warps read the encoder rows' f32 values for the same 64-wide k-block and write them
//     into the stage's B operand as f16 hi / lo pairs (hi = f16(x), lo = f16(x - hi): about 22
//     bits of x, so the product keeps the reference's f32 activations): rows [0, 128) hi,
//     [128, 256) lo, K-major with the same swizzle.
//   * One thread issues tcgen05.mma.kind::f16 (M 128, N 256, K 16) into a TMEM accumulator; each
//     stage is released by tcgen05.commit.  Four of the converter warps then read the accumulator
//     (tcgen05.ld), add the hi and lo columns and the bias, and store f16 rows of the cache.
// Every wait is bounded; a time-out raises the device error word.
#include "tc_common.cuh"
#include "w4j_internal.cuh"

namespace w4j {

constexpr int kXkvThreads = 384;
constexpr int kXkvStages = 4;
constexpr int kXRows = 128;                            // encoder rows per block
constexpr unsigned kXStageB = 2u * kXRows * 128u;      // B stage: 256 rows x 64 f16 = 32 KB
constexpr int kConvWarps = 8;                          // warps 4..11 convert; warps 4..7 then drain TMEM

__global__ void __launch_bounds__(kXkvThreads, 1)
    k_xkv_tc(const float *xa, int A, int d, const __grid_constant__ CUtensorMap kmap,
             const __grid_constant__ CUtensorMap vmap, const float *bk, const float *bv, __half *kout, __half *vout,
             int *err) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    unsigned char *ring_a = smem;                                  // [stages][16 KB]
    unsigned char *ring_b = smem + kXkvStages * kStageBytes;       // [stages][32 KB]
    uint64_t *full = reinterpret_cast<uint64_t *>(ring_b + kXkvStages * kXStageB);
    uint64_t *empty = full + kXkvStages;
    uint64_t *accf = empty + kXkvStages;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(accf + 1);
    volatile int *fail = reinterpret_cast<volatile int *>(tslot + 1);
    volatile int *issued = fail + 1;  // weight tiles whose copy has been started
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool isv = (int)blockIdx.x * kTileRows >= d;
    const int n0 = (int)blockIdx.x * kTileRows - (isv ? d : 0);  // first row of Wk or Wv
    const CUtensorMap *map = isv ? &vmap : &kmap;
    const int a0 = (int)blockIdx.y * kXRows;
    const int KB = d / kKB;
    constexpr uint32_t kCols = 2 * kXRows;  // hi and lo columns

    if (tid == 0) {
        for (int i = 0; i < kXkvStages; ++i) {
            mbar_init(full + i, 1 + kConvWarps);  // the weight copy's arrival + one per converter warp
            mbar_init(empty + i, 1);              // the MMAs' commit
        }
        mbar_init(accf, 1);
        *fail = 0;
        *issued = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tslot, kCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t taddr = *tslot;

    if (warp == 0 && lane == 0) {
        // ---- weight tiles ----
        for (int i = 0; i < KB && !*fail; ++i) {
            const int st = i % kXkvStages;
            if (i >= kXkvStages && !mbar_wait(empty + st, (unsigned)((i / kXkvStages - 1) & 1), err)) {
                *fail = 1;
                break;
            }
            mbar_expect_tx(full + st, kStageBytes);
            tma_load_2d(ring_a + (size_t)st * kStageBytes, map, i * kKB, n0, full + st);
            *issued = i + 1;
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer ----
        const uint32_t idesc = idesc_f16(kTileRows, 2 * kXRows);
        const uint32_t a_s = smem_u32(ring_a), b_s = smem_u32(ring_b);
        for (int i = 0; i < KB && !*fail; ++i) {
            const int st = i % kXkvStages;
            if (!mbar_wait(full + st, (unsigned)((i / kXkvStages) & 1), err)) {
                *fail = 1;
                break;
            }
            tc_fence_after();
#pragma unroll
            for (int j = 0; j < kKB / 16; ++j)
                umma_f16(taddr, sw128_desc(a_s + (uint32_t)st * kStageBytes + j * 32),
                         sw128_desc(b_s + (uint32_t)st * kXStageB + j * 32), idesc, (i | j) != 0);
            umma_commit(empty + st);  // the stage is free once these MMAs have read it
        }
        umma_commit(accf);
    } else if (warp >= 4) {
        // ---- encoder rows -> B operand (f16 hi / lo, K-major, 128-byte swizzle) ----
        const int ct = tid - 4 * 32;  // 0 .. kConvWarps * 32 - 1
        for (int i = 0; i < KB; ++i) {
            const int st = i % kXkvStages;
            if (i >= kXkvStages && !mbar_wait(empty + st, (unsigned)((i / kXkvStages - 1) & 1), err)) {
                *fail = 1;
                break;
            }
            unsigned char *bs = ring_b + (size_t)st * kXStageB;
            // 128 rows x 16 float4 of the k-block: 8 per thread, all loads in flight
            constexpr int kPer = 2048 / (kConvWarps * 32);
            float4 v[kPer];
#pragma unroll
            for (int u = 0; u < kPer; ++u) {
                const int idx = ct + kConvWarps * 32 * u, r = idx >> 4, c4 = idx & 15;
                v[u] = a0 + r < A ? reinterpret_cast<const float4 *>(xa + (size_t)(a0 + r) * d + i * kKB)[c4]
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < kPer; ++u) {
                const int idx = ct + kConvWarps * 32 * u, r = idx >> 4, c4 = idx & 15;
                const int cc = c4 >> 1, half = c4 & 1, rl = r + kXRows;
                const __half2 h0 = __floats2half2_rn(v[u].x, v[u].y), h1 = __floats2half2_rn(v[u].z, v[u].w);
                const float2 f0 = __half22float2(h0), f1 = __half22float2(h1);
                const __half2 l0 = __floats2half2_rn(v[u].x - f0.x, v[u].y - f0.y);
                const __half2 l1 = __floats2half2_rn(v[u].z - f1.x, v[u].w - f1.y);
                *reinterpret_cast<uint2 *>(bs + (size_t)r * 128 + ((cc ^ (r & 7)) * 16) + half * 8) =
                    make_uint2(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1));
                *reinterpret_cast<uint2 *>(bs + (size_t)rl * 128 + ((cc ^ (rl & 7)) * 16) + half * 8) =
                    make_uint2(*reinterpret_cast<const uint32_t *>(&l0), *reinterpret_cast<const uint32_t *>(&l1));
            }
            fence_proxy_async();  // generic-proxy writes of B visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(full + st);
        }
    }
    __syncthreads();
    if (warp >= 4 && warp < 8) {
        // ---- TMEM -> cache: tile row r (warp w reads TMEM lanes 32 (w % 4) ..), encoder rows a0 .. ----
        const int q = warp & 3, r = q * 32 + lane;
        const bool ok = !*fail && mbar_wait(accf, 0u, err);
        tc_fence_after();
        const int n = n0 + r, head = n / kHeadDim, dd = n % kHeadDim;
        const float *bias = isv ? bv : bk;
        const float b = bias ? bias[n] : 0.f;
        __half *out = (isv ? vout : kout) + (size_t)head * A * kHeadDim + dd;
#pragma unroll 1
        for (int c0 = 0; c0 < kXRows; c0 += 16) {
            float hi[16], lo[16];
            tmem_ld16(taddr + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, hi);
            tmem_ld16(taddr + ((uint32_t)(q * 32) << 16) + (uint32_t)(kXRows + c0), lo);
            if (ok)
#pragma unroll
                for (int e = 0; e < 16; ++e)
                    if (a0 + c0 + e < A) out[(size_t)(a0 + c0 + e) * kHeadDim] = __float2half_rn(hi[e] + lo[e] + b);
        }
        tc_fence_before();
    }
    __syncthreads();
    if (*fail && tid == 0) drain_ring(full, kXkvStages, *issued);
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(taddr, kCols);
    }
}

static size_t xkv_smem() { return (size_t)kXkvStages * (kStageBytes + kXStageB) + (2 * kXkvStages + 1) * 8 + 16 + 1024; }

cudaError_t xkv_tc_prepare() { return allow_dynamic_smem(k_xkv_tc); }

// cudaErrorNotSupported when d is not a multiple of 128 or a map is missing (the SIMT kernel then runs).
cudaError_t launch_cross_kv_tc(const float *xa, int A, int d, const void *kmap, const void *vmap, const float *bk,
                               const float *bv, __half *kout, __half *vout, int *err, cudaStream_t s) {
    if (!kmap || !vmap || d % kTileRows != 0 || A < 1) return cudaErrorNotSupported;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * d / kTileRows, (A + kXRows - 1) / kXRows);
    cfg.blockDim = dim3(kXkvThreads);
    cfg.dynamicSmemBytes = xkv_smem();
    cfg.stream = s;
    return cudaLaunchKernelEx(&cfg, k_xkv_tc, xa, A, d, *reinterpret_cast<const CUtensorMap *>(kmap),
                              *reinterpret_cast<const CUtensorMap *>(vmap), bk, bv, kout, vout, err);
}

}  // namespace w4j
