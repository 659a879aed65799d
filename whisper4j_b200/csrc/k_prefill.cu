// k_prefill.cu — cross-attention K/V projection of the encoder output (once per chunk),
// plus weight-format helpers used at upload.
//
// Replaces the first-call branch of MultiHeadAttention.forward for cross-attention
// (nn/MultiHeadAttention.java:65-75): K = xa . Wk^T (no key bias), V = xa . Wv^T + bv for
// every decoder layer, which the reference runs through Tensor.matmulTiled
// (tensor/Tensor.java:460-489) on Linux, then rearrangeToHeads (:645-659).  Here the product
// is written straight into the head-major f16 cross cache [head][n_audio_ctx][64].
//
// Tiled f32 GEMM: 64 x 64 output tiles, k-tiles of 32, 4 x 4 register blocks per thread,
// weights dequantised (f16 / Q8_0) while staging into shared memory.
#include "w4j_internal.cuh"

namespace w4j {

constexpr int kBM = 64, kBN = 64, kBK = 32;

__device__ __forceinline__ float mat_at(const DMat &m, int row, int k) {
    if (m.type == WT_F16) return __half2float(m.h[(size_t)row * m.K + k]);
    return (float)m.q[(size_t)row * m.K + k] * __half2float(m.s[(size_t)row * (m.K / 32) + k / 32]);
}

__global__ void __launch_bounds__(256) k_cross_kv(const float *xa, int A, int K, DMat wk, DMat wv,
                                                  const float *bk, const float *bv, __half *kout, __half *vout) {
    __shared__ float As[kBK][kBM + 4];
    __shared__ float Bs[kBK][kBN + 4];
    const int which = blockIdx.z;  // 0 = K, 1 = V
    const DMat &W = which ? wv : wk;
    const float *bias = which ? bv : bk;
    __half *out = which ? vout : kout;
    const int N = W.N;
    const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
    const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += kBK) {
        for (int e = tid; e < kBM * kBK; e += 256) {
            const int r = e / kBK, c = e % kBK;
            const int gm = m0 + r, gk = k0 + c;
            As[c][r] = (gm < A && gk < K) ? xa[(size_t)gm * K + gk] : 0.f;
        }
        for (int e = tid; e < kBN * kBK; e += 256) {
            const int r = e / kBK, c = e % kBK;
            const int gn = n0 + r, gk = k0 + c;
            Bs[c][r] = (gn < N && gk < K) ? mat_at(W, gn, gk) : 0.f;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < kBK; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int gm = m0 + ty * 4 + i;
        if (gm >= A) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gn = n0 + tx * 4 + j;
            if (gn >= N) continue;
            const float v = acc[i][j] + (bias ? bias[gn] : 0.f);
            const int h = gn / kHeadDim, dd = gn % kHeadDim;
            out[((size_t)h * A + gm) * kHeadDim + dd] = __float2half_rn(v);
        }
    }
}

cudaError_t launch_cross_kv(const float *xa, int A, int d, const DMat &wk, const DMat &wv, const float *bk,
                            const float *bv, __half *kout, __half *vout, int n_head, cudaStream_t s) {
    (void)n_head;
    dim3 grid((d + kBN - 1) / kBN, (A + kBM - 1) / kBM, 2);
    k_cross_kv<<<grid, 256, 0, s>>>(xa, A, d, wk, wv, bk, bv, kout, vout);
    return cudaGetLastError();
}

// GGML Q8_0 blocks (f16 scale + 32 int8, 34 B) -> int8 plane [N][K] then f16 scales [N][K/32]
__global__ void k_q8_repack(const uint8_t *src, int N, int K, int8_t *q, __half *sc) {
    const long long nb = (long long)N * (K / 32);
    for (long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x; b < nb; b += (long long)gridDim.x * blockDim.x) {
        const uint8_t *blk = src + b * 34;
        const unsigned short bits = (unsigned short)(blk[0] | (blk[1] << 8));
        sc[b] = __ushort_as_half(bits);
        int8_t *dst = q + b * 32;
#pragma unroll
        for (int i = 0; i < 32; ++i) dst[i] = (int8_t)blk[2 + i];
    }
}

cudaError_t launch_q8_repack(const void *src, int N, int K, int8_t *q, __half *sc, cudaStream_t s) {
    const long long nb = (long long)N * (K / 32);
    int blocks = (int)((nb + 255) / 256);
    if (blocks > 65535) blocks = 65535;
    if (blocks < 1) blocks = 1;
    k_q8_repack<<<blocks, 256, 0, s>>>(reinterpret_cast<const uint8_t *>(src), N, K, q, sc);
    return cudaGetLastError();
}

__global__ void k_f32_to_f16(const float *src, __half *dst, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = __float2half_rn(src[i]);
}

cudaError_t launch_f32_to_f16(const float *src, __half *dst, size_t n, cudaStream_t s) {
    int blocks = (int)((n + 255) / 256);
    if (blocks > 65535) blocks = 65535;
    if (blocks < 1) blocks = 1;
    k_f32_to_f16<<<blocks, 256, 0, s>>>(src, dst, n);
    return cudaGetLastError();
}

}  // namespace w4j

namespace w4j {
// st[((t * KB + kb) * 128 + r) * 2 + h] = s[(t * 128 + r) * (K / 32) + kb * 2 + h]: the two scales of row
// r in 64-wide k-block kb of 128-row tile t, contiguous per (tile, k-block) for one bulk copy
__global__ void k_q8_tile_scales(const __half *s, int N, int K, __half *st) {
    const size_t n = (size_t)N * (K / 32);
    const int KB = K / 64;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int h = (int)(i & 1), r = (int)((i >> 1) & 127);
        const size_t tk = i >> 8;
        const int kb = (int)(tk % KB), t = (int)(tk / KB);
        st[i] = s[((size_t)t * 128 + r) * (K / 32) + (size_t)kb * 2 + h];
    }
}

cudaError_t launch_q8_tile_scales(const __half *s, int N, int K, __half *st, cudaStream_t stream) {
    if (N % 128 || K % 64) return cudaErrorInvalidValue;
    k_q8_tile_scales<<<256, 256, 0, stream>>>(s, N, K, st);
    return cudaGetLastError();
}
}  // namespace w4j
