// attn_tile.cuh — warp-level tensor-core attention tiles shared by the attention kernels
// (k_attn.cu) and the persistent decode-step kernel (k_step.cu): fragments of mma.sync
// m16n8k16 (f16 inputs, f32 accumulation) and the per-warp online softmax over 16 keys of a
// 128-key tile held with the 128-byte swizzle (the layout TMA writes).
#pragma once
#include "w4j_internal.cuh"

namespace w4j {

// warp-level tensor-core tiles (m16n8k16, f16 inputs, f32 accumulation) and their fragments
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
constexpr int kStreamThreads = 2 * kAttnThreads;
constexpr int kPwPad = 24;  // halves per row of a warp's P^T block (48 B: conflict-free ldmatrix)
constexpr int kStreamBufs = 3;                            // tile buffers per warpgroup
constexpr int kStreamTile = 2 * kAttnKeyTile * kHeadDim;  // halves of one K tile + one V tile
constexpr unsigned kHalfTileBytes = kAttnKeyTile * kHeadDim * 2;  // one K (or V) tile: 16 KB
// offset (halves) of 16-byte chunk c of row r in a swizzled 128-byte-row tile
__device__ __forceinline__ int swz(int r, int c) { return r * kHeadDim + ((c ^ (r & 7)) << 3); }

// One warp's 16 keys [16 w, 16 w + 16) of a 128-key tile, online softmax kept per warp: m / l
// are the running max / denominator of queries 2 tq and 2 tq + 1, of[4][4] the O^T fragments.
template <int NQ>
__device__ __forceinline__ void tile_warp(const __half *sk, const __half *sv, int nk, const __half (*qh)[kHeadDim + 8],
                                          __half (*pw)[kPwPad], float (&m)[2], float (&l)[2], float (&of)[4][4],
                                          int gwarp, int lane) {
    const int g = lane >> 2, tq = lane & 3, kb = 16 * gwarp;
    const float scale = 0.125f;  // (float)(1 / sqrt(64))
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
    if (kb < nk) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t af[4], bf[2];
            ldsm_x4(af, &sk[swz(kb + (lane & 15), 2 * kk + (lane >> 4))]);
            ldsm_x2(bf, &qh[lane & 7][16 * kk + ((lane >> 3) & 1) * 8]);
            mma_16816(sc, af, bf);
        }
    }
    // c0: (key kb+g, query 2tq), c1: (kb+g, 2tq+1), c2: (kb+g+8, 2tq), c3: (kb+g+8, 2tq+1)
    const int q0 = 2 * tq, q1 = 2 * tq + 1;
    const bool k0ok = kb + g < nk, k1ok = kb + g + 8 < nk;
    sc[0] = (k0ok && q0 < NQ) ? sc[0] * scale : -INFINITY;
    sc[1] = (k0ok && q1 < NQ) ? sc[1] * scale : -INFINITY;
    sc[2] = (k1ok && q0 < NQ) ? sc[2] * scale : -INFINITY;
    sc[3] = (k1ok && q1 < NQ) ? sc[3] * scale : -INFINITY;
    float mx0 = fmaxf(sc[0], sc[2]), mx1 = fmaxf(sc[1], sc[3]);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    const float mn0 = fmaxf(m[0], mx0), mn1 = fmaxf(m[1], mx1);
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
    const float al0 = m[0] == -INFINITY ? 0.f : __expf(m[0] - mn0);
    const float al1 = m[1] == -INFINITY ? 0.f : __expf(m[1] - mn1);
    l[0] = l[0] * al0 + sm0;
    l[1] = l[1] * al1 + sm1;
    m[0] = mn0;
    m[1] = mn1;
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
        of[mt][0] *= al0;
        of[mt][1] *= al1;
        of[mt][2] *= al0;
        of[mt][3] *= al1;
    }
    if (kb < nk) {
        // O^T (16 dims x 8 queries, 4 tiles) += V^T (16 dims x 16 keys) . P^T (16 keys x 8 queries)
        pw[q0][g] = __float2half_rn(p0);
        pw[q1][g] = __float2half_rn(p1);
        pw[q0][g + 8] = __float2half_rn(p2);
        pw[q1][g + 8] = __float2half_rn(p3);
        __syncwarp();
        uint32_t bf[2];
        ldsm_x2(bf, &pw[lane & 7][((lane >> 3) & 1) * 8]);
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
            uint32_t af[4];
            ldsm_x4_t(af, &sv[swz(kb + (lane & 7) + ((lane >> 4) & 1) * 8, 2 * mt + ((lane >> 3) & 1))]);
            mma_16816(of[mt], af, bf);
        }
        __syncwarp();  // pw is rewritten by the next tile
    }
}


}  // namespace w4j
