// k_logmel.cu — the log-mel front end on the device (FeatureExtractor.extract + padOrTrim,
// FeatureExtractor.java:68-160), restating the reference's arithmetic operation for operation:
// periodic Hann window, zero padding of n_fft / 2 on each side, Bluestein's algorithm for
// n_fft = 400 (chirp convolution through 1024-point radix-2 FFTs whose twiddles follow the Java
// loop's float recurrence, :248-320), |X|^2, the model's mel filters summed in bin order, log10 in
// double, the global-max floor and the (x + 4) / 4 scaling.  Products and sums use round-to-nearest
// intrinsics, so nothing is contracted into an FMA the Java code does not have.
//
// One block per frame: the frame's samples are windowed into a 1024-point complex buffer in shared
// memory, transformed, multiplied by the transformed chirp, transformed back; the n_mels log values
// of the frame and their max / min go to global memory.  A second kernel applies the floor and the
// scaling and lays the result out as n_mels x out_frames (padOrTrim).
#include <cmath>
#include <vector>

#include "w4j_internal.cuh"

namespace w4j {

constexpr int kMelFftN = 1024;  // the Bluestein convolution length for n_fft = 400 (next power of two >= 799)

// Host tables (float values computed exactly as the Java code computes them)
void logmel_tables(int n_fft, std::vector<float> &tabs) {
    const int n = n_fft, m = kMelFftN;
    // [0, n): window; [n, 3n): chirp re / im; [3n, 3n + 2m): FFT of the chirp sequence b (re / im);
    // [3n + 2m, 3n + 4m): radix-2 twiddles, stage len at index len / 2 + j (re / im)
    tabs.assign((size_t)3 * n + 4 * m, 0.f);
    float *win = tabs.data(), *cre = win + n, *cim = cre + n, *bre = cim + n, *bim = bre + m, *twr = bim + m, *twi = twr + m;
    for (int i = 0; i < n; i++) win[i] = 0.5f * (1.0f - (float)std::cos(2.0 * M_PI * i / n));  // :322-328
    for (int k = 0; k < n; k++) {                                                              // :206-211
        const double angle = -M_PI * (double)(((long long)k * k) % (2LL * n)) / n;
        cre[k] = (float)std::cos(angle);
        cim[k] = (float)std::sin(angle);
    }
    for (int len = 2; len <= m; len <<= 1) {  // :296-300 twiddle recurrence of one butterfly group
        const double angle = -2.0 * M_PI / len;
        const float wr = (float)std::cos(angle), wi = (float)std::sin(angle);
        float cr = 1.0f, ci = 0.0f;
        for (int j = 0; j < len / 2; j++) {
            twr[len / 2 + j] = cr;
            twi[len / 2 + j] = ci;
            const float p = cr * wr, q = ci * wi, r = cr * wi, s = ci * wr;
            const float ncr = p - q;
            ci = r + s;
            cr = ncr;
        }
    }
    // b (:220-226), transformed once: the same for every frame
    std::vector<float> re(m, 0.f), im(m, 0.f);
    re[0] = cre[0];
    im[0] = cim[0];
    for (int k = 1; k < n; k++) {
        re[k] = re[m - k] = cre[k];
        im[k] = im[m - k] = cim[k];
    }
    for (int i = 1, j = 0; i < m; i++) {
        int bit = m >> 1;
        while (j & bit) {
            j ^= bit;
            bit >>= 1;
        }
        j ^= bit;
        if (i < j) {
            std::swap(re[i], re[j]);
            std::swap(im[i], im[j]);
        }
    }
    for (int len = 2; len <= m; len <<= 1)
        for (int i = 0; i < m; i += len)
            for (int j = 0; j < len / 2; j++) {
                const int a = i + j, b = i + j + len / 2;
                const float c = twr[len / 2 + j], s = twi[len / 2 + j];
                const float p = re[b] * c, q = im[b] * s, r = re[b] * s, t = im[b] * c;
                const float vr = p - q, vi = r + t, ur = re[a], ui = im[a];
                re[a] = ur + vr;
                im[a] = ui + vi;
                re[b] = ur - vr;
                im[b] = ui - vi;
            }
    for (int k = 0; k < m; k++) {
        bre[k] = re[k];
        bim[k] = im[k];
    }
}

// in-place 1024-point radix-2 FFT of (re, im) in shared memory, 512 threads, Java's butterfly
// arithmetic (:286-318) with the recurrence twiddles from the table
__device__ __forceinline__ void mel_fft1024(float *re, float *im, const float *twr, const float *twi) {
    const int tid = threadIdx.x;
    for (int k = tid; k < kMelFftN; k += blockDim.x) {  // bit-reversal permutation (:288-301)
        const int r = (int)(__brev((unsigned)k) >> (32 - 10));
        if (k < r) {
            const float a = re[k], b = im[k];
            re[k] = re[r];
            im[k] = im[r];
            re[r] = a;
            im[r] = b;
        }
    }
    __syncthreads();
    for (int len = 2; len <= kMelFftN; len <<= 1) {
        const int half = len >> 1;
        for (int bf = tid; bf < kMelFftN / 2; bf += blockDim.x) {
            const int j = bf % half, a = (bf / half) * len + j, b = a + half;
            const float c = twr[half + j], s = twi[half + j];
            const float vr = __fsub_rn(__fmul_rn(re[b], c), __fmul_rn(im[b], s));
            const float vi = __fadd_rn(__fmul_rn(re[b], s), __fmul_rn(im[b], c));
            const float ur = re[a], ui = im[a];
            re[a] = __fadd_rn(ur, vr);
            im[a] = __fadd_rn(ui, vi);
            re[b] = __fsub_rn(ur, vr);
            im[b] = __fsub_rn(ui, vi);
        }
        __syncthreads();
    }
}

// Frame t: window the samples padded[t hop .. t hop + n), Bluestein DFT, |X|^2 of bins [0, n_bins),
// mel sums, log10.  spec: [n_mels][frames]; fmax / fmin: the frame's largest and smallest log value.
// The padded signal is the audio shifted by n / 2 with zeros outside [0, n_samples) (:75-84).
__global__ void __launch_bounds__(512) k_logmel_frames(const float *audio, int n_samples, int n, int hop, int frames,
                                                       const float *tabs, const float *filt, int n_mels, int n_bins,
                                                       float *spec, float *fmax_out, float *fmin_out) {
    __shared__ float re[kMelFftN], im[kMelFftN], twr[kMelFftN], twi[kMelFftN];
    __shared__ float mag[kMelFftN / 2 + 1];
    __shared__ float red[2][32];
    const int t = blockIdx.x, tid = threadIdx.x;
    const float *win = tabs, *cre = tabs + n, *cim = cre + n, *bre = cim + n, *bim = bre + kMelFftN;
    for (int k = tid; k < kMelFftN; k += blockDim.x) {
        twr[k] = tabs[3 * n + 2 * kMelFftN + k];
        twi[k] = tabs[3 * n + 3 * kMelFftN + k];
        float ar = 0.f, ai = 0.f;
        if (k < n) {  // a[k] = x[k] conj(chirp[k]) with x = windowed frame, im(x) = 0 (:213-217)
            const long long p = (long long)t * hop + k - n / 2;
            const float xs = p >= 0 && p < n_samples ? audio[p] : 0.f;
            const float x = __fmul_rn(xs, win[k]);
            ar = __fadd_rn(__fmul_rn(x, cre[k]), __fmul_rn(0.f, cim[k]));
            ai = __fsub_rn(__fmul_rn(0.f, cre[k]), __fmul_rn(x, cim[k]));
        }
        re[k] = ar;
        im[k] = ai;
    }
    __syncthreads();
    mel_fft1024(re, im, twr, twi);
    for (int k = tid; k < kMelFftN; k += blockDim.x) {  // times FFT(b), then conjugate (:229-239)
        const float ar = re[k], ai = im[k];
        const float tr = __fsub_rn(__fmul_rn(ar, bre[k]), __fmul_rn(ai, bim[k]));
        const float ti = __fadd_rn(__fmul_rn(ar, bim[k]), __fmul_rn(ai, bre[k]));
        re[k] = tr;
        im[k] = -ti;
    }
    __syncthreads();
    mel_fft1024(re, im, twr, twi);
    const float inv_m = 1.0f / kMelFftN;
    for (int k = tid; k < n_bins; k += blockDim.x) {  // scale, X[k] = conj(chirp) conv (:240-246), |X|^2 (:98-100)
        const float ar = __fmul_rn(re[k], inv_m), ai = __fmul_rn(im[k], -inv_m);
        const float xr = __fadd_rn(__fmul_rn(ar, cre[k]), __fmul_rn(ai, cim[k]));
        const float xi = __fsub_rn(__fmul_rn(ai, cre[k]), __fmul_rn(ar, cim[k]));
        mag[k] = __fadd_rn(__fmul_rn(xr, xr), __fmul_rn(xi, xi));
    }
    __syncthreads();
    // mel sums in bin order, log10 in double (:103-117)
    float vmax = -INFINITY, vmin = INFINITY;
    for (int m = tid; m < n_mels; m += blockDim.x) {
        const float *w = filt + (size_t)m * n_bins;
        float sum = 0.f;
        for (int f = 0; f < n_bins; ++f) sum = __fadd_rn(sum, __fmul_rn(w[f], mag[f]));
        const float v = (float)log10(fmax((double)sum, 1e-10));
        spec[(size_t)m * frames + t] = v;
        vmax = fmaxf(vmax, v);
        vmin = fminf(vmin, v);
    }
    vmax = warp_max(vmax);
    for (int o = 16; o > 0; o >>= 1) vmin = fminf(vmin, __shfl_xor_sync(0xffffffffu, vmin, o));
    if ((tid & 31) == 0) {
        red[0][tid >> 5] = vmax;
        red[1][tid >> 5] = vmin;
    }
    __syncthreads();
    if (tid == 0) {
        float a = red[0][0], b = red[1][0];
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
            a = fmaxf(a, red[0][w]);
            b = fminf(b, red[1][w]);
        }
        fmax_out[t] = a;
        fmin_out[t] = b;
    }
}

// floor = global max - 8, (max(v, floor) + 4) / 4 (:119-124); padOrTrim to out_frames (:130-160): the
// first frames, or the spectrogram's minimum (the scaled minimum) past its end.
__global__ void __launch_bounds__(256) k_logmel_norm(const float *spec, int n_mels, int frames, const float *fmax_in,
                                                     const float *fmin_in, int out_frames, float *out) {
    __shared__ float red[2][8];
    __shared__ float g[2];
    float a = -INFINITY, b = INFINITY;
    for (int i = threadIdx.x; i < frames; i += blockDim.x) {
        a = fmaxf(a, fmax_in[i]);
        b = fminf(b, fmin_in[i]);
    }
    a = warp_max(a);
    for (int o = 16; o > 0; o >>= 1) b = fminf(b, __shfl_xor_sync(0xffffffffu, b, o));
    if ((threadIdx.x & 31) == 0) {
        red[0][threadIdx.x >> 5] = a;
        red[1][threadIdx.x >> 5] = b;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; ++w) {
            red[0][0] = fmaxf(red[0][0], red[0][w]);
            red[1][0] = fminf(red[1][0], red[1][w]);
        }
        g[0] = red[0][0];
        g[1] = red[1][0];
    }
    __syncthreads();
    const float floor_v = __fsub_rn(g[0], 8.0f);
    const float padv = __fdiv_rn(__fadd_rn(fmaxf(g[1], floor_v), 4.0f), 4.0f);
    const long long total = (long long)n_mels * out_frames;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int m = (int)(i / out_frames), t = (int)(i % out_frames);
        float v = padv;
        if (t < frames) v = __fdiv_rn(__fadd_rn(fmaxf(spec[(size_t)m * frames + t], floor_v), 4.0f), 4.0f);
        out[i] = v;
    }
}

int logmel_frames(int n_samples, int n, int hop) {
    const int len = n_samples < n ? n : n_samples;
    return 1 + (len + 2 * (n / 2) - n) / hop;
}

// n_total samples (the spectrogram's length), of which the first n_valid are read from audio and the
// rest are zero (a chunk shorter than 30 s, as WhisperModel zero-fills its chunk array, :355-358)
cudaError_t launch_logmel(const float *audio, int n_valid, int n_total, int n, int hop, const float *tabs,
                          const float *filt, int n_mels, int n_bins, int out_frames, float *spec, float *fmx, float *fmn,
                          float *out, cudaStream_t s) {
    if (n < 2 || 2 * n - 1 > kMelFftN || n_bins != n / 2 + 1 || n_mels > 512 || n_valid > n_total) return cudaErrorInvalidValue;
    const int frames = logmel_frames(n_total, n, hop);
    k_logmel_frames<<<frames, 512, 0, s>>>(audio, n_valid, n, hop, frames, tabs, filt, n_mels, n_bins, spec, fmx, fmn);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const long long total = (long long)n_mels * out_frames;
    const int blocks = (int)std::min<long long>((total + 255) / 256, 148LL * 8);
    k_logmel_norm<<<blocks, 256, 0, s>>>(spec, n_mels, frames, fmx, fmn, out_frames, out);
    return cudaGetLastError();
}

}  // namespace w4j
