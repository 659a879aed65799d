// k_encoder.cu — the audio encoder's own kernels (WhisperEncoder.forward, WhisperEncoder.java:42-76):
// the im2col rows of the two convolutions (Conv1d.java:49-64), the positional-embedding add, the
// non-causal multi-head self-attention over all n_audio_ctx frames, and the final LayerNorm.  The
// projections and the convolutions' matrix products run on the decoder's tensor-core GEMM
// (k_gemm_tc.cu, staged activations) with its bias / GELU-table / residual epilogues.
#include <algorithm>

#include "attn_tile.cuh"
#include "w4j_internal.cuh"

namespace w4j {

// ---------------------------------------------------------------------------
// im2col of a kernel-3, padding-1 convolution: row t of the output holds, at column ic * 3 + k,
// in(ic, t * stride - 1 + k) (zero outside [0, in_len)), columns [in_ch * 3, kp) zero.
// in(ic, i) = src[ic * in_len + i] for a channel-major source (the mel input), src[i * in_ch + ic]
// for a time-major one (the first convolution's output).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_enc_im2col(const float *src, int in_ch, int in_len, bool time_major, int stride,
                                                    int out_len, int kp, float *out) {
    const long long n = (long long)out_len * kp;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / kp), r = (int)(i % kp);
        float v = 0.f;
        if (r < in_ch * 3) {
            const int ic = r / 3, k = r - 3 * ic, j = t * stride - 1 + k;
            if (j >= 0 && j < in_len) v = time_major ? src[(size_t)j * in_ch + ic] : src[(size_t)ic * in_len + j];
        }
        out[i] = v;
    }
}

cudaError_t launch_enc_im2col(const float *src, int in_ch, int in_len, bool time_major, int stride, int out_len, int kp,
                              float *out, cudaStream_t s) {
    const long long n = (long long)out_len * kp;
    const int blocks = (int)std::min<long long>((n + 255) / 256, 148LL * 16);
    k_enc_im2col<<<blocks, 256, 0, s>>>(src, in_ch, in_len, time_major, stride, out_len, kp, out);
    return cudaGetLastError();
}

// x[i] += p[i] (the encoder's positional embedding after the second convolution, :57-58)
__global__ void __launch_bounds__(256) k_enc_add(float *x, const float *p, long long n4) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
        float4 a = reinterpret_cast<float4 *>(x)[i];
        const float4 b = reinterpret_cast<const float4 *>(p)[i];
        a.x = a.x + b.x;
        a.y = a.y + b.y;
        a.z = a.z + b.z;
        a.w = a.w + b.w;
        reinterpret_cast<float4 *>(x)[i] = a;
    }
}

cudaError_t launch_enc_add(float *x, const float *p, long long n, cudaStream_t s) {
    if (n % 4) return cudaErrorInvalidValue;
    const int blocks = (int)std::min<long long>((n / 4 + 255) / 256, 148LL * 16);
    k_enc_add<<<blocks, 256, 0, s>>>(x, p, n / 4);
    return cudaGetLastError();
}

// LayerNorm of rows (Tensor.java:592-619: two-pass mean / variance, eps 1e-5), one warp per row.
__global__ void __launch_bounds__(256) k_enc_ln(const float *x, int rows, int n, const float *g, const float *b, float *y) {
    const int row = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float *xr = x + (size_t)row * n;
    float s = 0.f;
    for (int k = lane; k < n; k += 32) s += xr[k];
    const float mean = warp_sum(s) / (float)n;
    float v = 0.f;
    for (int k = lane; k < n; k += 32) {
        const float t = xr[k] - mean;
        v += t * t;
    }
    const float inv_std = 1.0f / sqrtf(warp_sum(v) / (float)n + 1e-5f);
    float *yr = y + (size_t)row * n;
    for (int k = lane; k < n; k += 32) yr[k] = (xr[k] - mean) * inv_std * g[k] + b[k];
}

cudaError_t launch_enc_ln(const float *x, int rows, int n, const float *g, const float *b, float *y, cudaStream_t s) {
    k_enc_ln<<<(rows * 32 + 255) / 256, 256, 0, s>>>(x, rows, n, g, b, y);
    return cudaGetLastError();
}

// q, k, v of a fused projection output [T][3 d] (f32) as f16 head-major tiles [3][H][T][64]: each
// head's keys and values become one contiguous run for the attention kernel's 16-byte copies.
__global__ void __launch_bounds__(256) k_enc_qkv_f16(const float *qkv, int T, int H, __half *out) {
    const int d = H * kHeadDim;
    const long long n8 = (long long)T * 3 * d / 8;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
        const long long e = i * 8;
        const int t = (int)(e / (3 * d)), c = (int)(e % (3 * d));
        const int part = c / d, h = (c % d) / kHeadDim, dd = c % kHeadDim;
        const float4 a = reinterpret_cast<const float4 *>(qkv)[2 * i], b = reinterpret_cast<const float4 *>(qkv)[2 * i + 1];
        const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
        const __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
        uint4 u;
        u.x = *reinterpret_cast<const uint32_t *>(&h0);
        u.y = *reinterpret_cast<const uint32_t *>(&h1);
        u.z = *reinterpret_cast<const uint32_t *>(&h2);
        u.w = *reinterpret_cast<const uint32_t *>(&h3);
        *reinterpret_cast<uint4 *>(out + ((((size_t)part * H + h) * T + t) * kHeadDim + dd)) = u;
    }
}

cudaError_t launch_enc_qkv_f16(const float *qkv, int T, int H, __half *out, cudaStream_t s) {
    const long long n8 = (long long)T * 3 * H * kHeadDim / 8;
    const int blocks = (int)std::min<long long>((n8 + 255) / 256, 148LL * 16);
    k_enc_qkv_f16<<<blocks, 256, 0, s>>>(qkv, T, H, out);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Encoder self-attention (MultiHeadAttention.forward without mask or cache, :84-97): per head,
// softmax(q k^T / sqrt(64)) v over all T frames.  Block = 64 queries of one head, four warps of 16
// queries; keys and values stream through two 64-key buffers (cp.async, the next tile in flight
// while the current one is computed); scores and P.V on m16n8k16 tensor-core tiles (f16 inputs, f32
// accumulation) with an online softmax per query row in f32.
// ---------------------------------------------------------------------------
constexpr int kEncQ = 64, kEncKeys = 64, kEncPad = kHeadDim + 8;  // 144-byte rows: conflict-free ldmatrix

__device__ __forceinline__ void enc_load_tile(__half (*dst)[kEncPad], const __half *src, int rows_valid) {
    // 64 rows x 8 chunks of 16 bytes; rows past the valid ones are zero
    for (int c = threadIdx.x; c < kEncKeys * 8; c += blockDim.x) {
        const int r = c >> 3, ch = c & 7;
        if (r < rows_valid)
            cp_async16(&dst[r][ch * 8], src + (size_t)r * kHeadDim + ch * 8);
        else
            *reinterpret_cast<uint4 *>(&dst[r][ch * 8]) = make_uint4(0u, 0u, 0u, 0u);
    }
}

__global__ void __launch_bounds__(128) k_enc_attn(const __half *qkvh, int T, int H, float scale, float *out) {
    __shared__ __align__(16) __half qs[kEncQ][kEncPad];
    __shared__ __align__(16) __half ks[2][kEncKeys][kEncPad];
    __shared__ __align__(16) __half vs[2][kEncKeys][kEncPad];
    const int head = blockIdx.y, q0 = blockIdx.x * kEncQ;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
    const __half *Q = qkvh + ((size_t)head * T) * kHeadDim;
    const __half *Kh = qkvh + ((size_t)(H + head) * T) * kHeadDim;
    const __half *Vh = qkvh + ((size_t)(2 * H + head) * T) * kHeadDim;
    const int ntiles = (T + kEncKeys - 1) / kEncKeys;
    enc_load_tile(qs, Q + (size_t)q0 * kHeadDim, min(kEncQ, T - q0));
    enc_load_tile(ks[0], Kh, min(kEncKeys, T));
    enc_load_tile(vs[0], Vh, min(kEncKeys, T));
    cp_async_commit();

    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    float o[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    uint32_t qa[4][4];  // the warp's 16 query rows as A fragments, 4 k-steps of 16 dims

    for (int t = 0; t < ntiles; ++t) {
        const int b = t & 1;
        if (t + 1 < ntiles) {  // next tile into the other buffer (its previous use ended at the last barrier)
            const int k1 = (t + 1) * kEncKeys;
            enc_load_tile(ks[b ^ 1], Kh + (size_t)k1 * kHeadDim, min(kEncKeys, T - k1));
            enc_load_tile(vs[b ^ 1], Vh + (size_t)k1 * kHeadDim, min(kEncKeys, T - k1));
        }
        cp_async_commit();
        cp_async_wait_group<1>();
        __syncthreads();
        if (t == 0) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) ldsm_x4(qa[kk], &qs[16 * warp + (lane & 15)][kk * 16 + 8 * (lane >> 4)]);
        }
        // S = Q K^T for 64 keys: 8 n-tiles of 8 keys
        float s[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
            for (int np = 0; np < 4; ++np) {  // n-tiles 2 np, 2 np + 1
                uint32_t r[4];
                const int mi = lane >> 3;
                ldsm_x4(r, &ks[b][16 * np + 8 * (mi >> 1) + (lane & 7)][kk * 16 + 8 * (mi & 1)]);
                const uint32_t b0[2] = {r[0], r[1]}, b1[2] = {r[2], r[3]};
                mma_16816(s[2 * np], qa[kk], b0);
                mma_16816(s[2 * np + 1], qa[kk], b1);
            }
        // scale (after the dot, as Tensor.matmulTransB(kr, scale)), mask keys past T, online softmax
        const int kbase = t * kEncKeys;
        float mx[2] = {m[0], m[1]};
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int key = kbase + 8 * n + 2 * tq + (j & 1);
                s[n][j] = key < T ? s[n][j] * scale : -INFINITY;
                mx[j >> 1] = fmaxf(mx[j >> 1], s[n][j]);
            }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
        }
        float corr[2], rs[2] = {0.f, 0.f};
#pragma unroll
        for (int h = 0; h < 2; ++h) corr[h] = m[h] == -INFINITY ? 0.f : __expf(m[h] - mx[h]);
        uint32_t pa[4][4];  // P as A fragments: k-step kk covers keys 16 kk .. 16 kk + 15
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            const float p0 = __expf(s[n][0] - mx[0]), p1 = __expf(s[n][1] - mx[0]);
            const float p2 = __expf(s[n][2] - mx[1]), p3 = __expf(s[n][3] - mx[1]);
            rs[0] += p0 + p1;
            rs[1] += p2 + p3;
            const __half2 lo = __floats2half2_rn(p0, p1), hi = __floats2half2_rn(p2, p3);
            pa[n >> 1][(n & 1) * 2] = *reinterpret_cast<const uint32_t *>(&lo);
            pa[n >> 1][(n & 1) * 2 + 1] = *reinterpret_cast<const uint32_t *>(&hi);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 1);
            rs[h] += __shfl_xor_sync(0xffffffffu, rs[h], 2);
            l[h] = l[h] * corr[h] + rs[h];
            m[h] = mx[h];
        }
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            o[n][0] *= corr[0];
            o[n][1] *= corr[0];
            o[n][2] *= corr[1];
            o[n][3] *= corr[1];
        }
        // O += P V: B fragments of V (k = key, n = dim) through transposing loads
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
            for (int np = 0; np < 4; ++np) {  // dim tiles 2 np, 2 np + 1
                uint32_t r[4];
                const int mi = lane >> 3;
                ldsm_x4_t(r, &vs[b][16 * kk + 8 * (mi & 1) + (lane & 7)][16 * np + 8 * (mi >> 1)]);
                const uint32_t b0[2] = {r[0], r[1]}, b1[2] = {r[2], r[3]};
                mma_16816(o[2 * np], pa[kk], b0);
                mma_16816(o[2 * np + 1], pa[kk], b1);
            }
        __syncthreads();  // buffer b is free for the tile after next
    }
    // out[q][head * 64 + dim] = O / l
    const int d = H * kHeadDim;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int q = q0 + 16 * warp + g + 8 * h;
        if (q >= T) continue;
        const float inv = 1.0f / l[h];
        float *row = out + (size_t)q * d + head * kHeadDim;
#pragma unroll
        for (int n = 0; n < 8; ++n)
            *reinterpret_cast<float2 *>(row + 8 * n + 2 * tq) = make_float2(o[n][2 * h] * inv, o[n][2 * h + 1] * inv);
    }
}

cudaError_t launch_enc_attn(const __half *qkvh, int T, int H, float *out, cudaStream_t s) {
    dim3 grid((T + kEncQ - 1) / kEncQ, H);
    k_enc_attn<<<grid, 128, 0, s>>>(qkvh, T, H, 0.125f, out);
    return cudaGetLastError();
}

}  // namespace w4j
