// k_select.cu — per-step token selection and decode bookkeeping, on the device.
//
// Restates the host-side policy of the reference's decode loops so that only token ids
// leave the GPU:
//   greedy / temperature  WhisperDecoder.decode            (nn/WhisperDecoder.java:161-204)
//   beam search           WhisperDecoder.decodeBeam        (:214-394), computeLogSoftmax (:397-412),
//                         topkIndices (:415-431), MaximumLikelihood pick (:379-393)
//   logit processors      suppressBlank (:450-455), applySuppress (:457-466), n-gram block
//                         n=3,4 (:472-476, :543-564), timestamp rules (:484-541)
//   log-probabilities     logSoftmax (:614-626), softmaxAt for the no-speech prob (:442-448, :600-612)
//   sampling              sample (:576-598)
// The logits kernel leaves per-block partials (max, sum of exp, first argmax, top-k); these
// kernels merge them (sums in double, ties to the lower id as the reference's loops do),
// apply the decision, update token histories / beam tables, and build the masks that the
// next step's logits kernel applies.
#include <float.h>

#include "w4j_internal.cuh"

namespace w4j {

constexpr int kSelThreads = 256;

__device__ __forceinline__ bool better_c(float v1, int i1, float v2, int i2) {
    return v1 > v2 || (v1 == v2 && i1 < i2);
}

// A 64-bit key whose unsigned order is Double.compare's order (-0.0 < 0.0, every NaN equal
// and above +inf), so a sort compares integers.
__device__ __forceinline__ unsigned long long dkey(double x) {
    if (isnan(x)) return ~0ull;
    const unsigned long long b = (unsigned long long)__double_as_longlong(x);
    return (b >> 63) ? ~b : (b | 0x8000000000000000ull);
}

// ---------------------------------------------------------------------------
// warp-level merges of the logits partials of one sequence
// ---------------------------------------------------------------------------
struct Merged {
    float max;
    int argmax;
    double sum;  // sum_i exp(l_i - max)
};

__device__ __forceinline__ void warp_best(float &v, int &i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (better_c(ov, oi, v, i)) {
            v = ov;
            i = oi;
        }
    }
}

// One warp: copy P block partials into shared memory with 8 independent 8-byte loads in
// flight per lane (one L2 round trip instead of one per partial).  A partial record starts
// [max, sum, argmax, pad, topv[0..k), topi[0..k)], which is what is copied: row c of `dst`
// holds those F = 4 + 2k floats.
__device__ void stage_partials(const float *part, int P, int k, float *dst) {
    const int lane = threadIdx.x & 31;
    const int F2 = 2 + k;  // float2 per record
    const int n = P * F2;
    for (int e0 = lane; e0 < n; e0 += 32 * 8) {
        float2 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int e = e0 + 32 * j;
            if (e < n) {
                const int c = e / F2, f = e - c * F2;
                v[j] = reinterpret_cast<const float2 *>(part + (size_t)c * kPartStride)[f];
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (e0 + 32 * j < n) reinterpret_cast<float2 *>(dst)[e0 + 32 * j] = v[j];
    }
    __syncwarp();
}

// One warp: (max, first argmax, sum of exp relative to the max) over P staged partials.
__device__ Merged merge_partials(const float *stg, int P, int F) {
    const int lane = threadIdx.x & 31;
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int c = lane; c < P; c += 32) {
        const float v = stg[c * F];
        const int i = __float_as_int(stg[c * F + 2]);
        if (better_c(v, i, bv, bi)) {
            bv = v;
            bi = i;
        }
    }
    warp_best(bv, bi);
    double s = 0.0;
    if (bv != -INFINITY)
        for (int c = lane; c < P; c += 32) {
            const float mc = stg[c * F];
            if (mc != -INFINITY) s += (double)(stg[c * F + 1] * expf(mc - bv));
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    Merged out;
    out.max = bv;
    // reference argmax: index 0 when nothing beats a[0] = -inf
    out.argmax = (bv == -INFINITY || bi == INT_MAX) ? 0 : bi;
    out.sum = s;
    return out;
}

// One warp: top-k over the staged per-block candidate lists, each sorted (value desc,
// index asc); a k-way merge where every lane keeps the current heads of the blocks it owns
// in registers and only the lane whose head won reloads it.  Unfilled entries come out as
// (-inf, 0), as topkIndices leaves them.  P <= 32 * kMaxOwned.
__device__ void merge_topk(const float *stg, int P, int F, int kk, int k, float *out_v, int *out_i) {
    const int lane = threadIdx.x & 31;
    constexpr int kMaxOwned = 8;
    int head[kMaxOwned];
    float hv[kMaxOwned];
    int hi[kMaxOwned];
#pragma unroll
    for (int j = 0; j < kMaxOwned; ++j) {
        const int c = lane + 32 * j;
        head[j] = 0;
        hv[j] = c < P && kk > 0 ? stg[c * F + 4] : -INFINITY;
        hi[j] = c < P && kk > 0 ? __float_as_int(stg[c * F + 4 + kk]) : INT_MAX;
    }
    for (int r = 0; r < k; ++r) {
        float bv = -INFINITY;
        int bi = INT_MAX, bj = -1;
#pragma unroll
        for (int j = 0; j < kMaxOwned; ++j)
            if (hv[j] != -INFINITY && better_c(hv[j], hi[j], bv, bi)) {
                bv = hv[j];
                bi = hi[j];
                bj = j;
            }
        const int mine = bi;
        warp_best(bv, bi);
        if (bi != INT_MAX && mine == bi && bj >= 0) {  // ids are unique across blocks
#pragma unroll
            for (int j = 0; j < kMaxOwned; ++j)
                if (j == bj) {
                    const int c = lane + 32 * j;
                    ++head[j];
                    hv[j] = head[j] < kk ? stg[c * F + 4 + head[j]] : -INFINITY;
                    hi[j] = head[j] < kk ? __float_as_int(stg[c * F + 4 + kk + head[j]]) : INT_MAX;
                }
        }
        if (lane == 0) {
            out_v[r] = bi == INT_MAX ? -INFINITY : bv;
            out_i[r] = bi == INT_MAX ? 0 : bi;
        }
    }
    __syncwarp();
}

// ---------------------------------------------------------------------------
// masks of the next step (one warp)
// ---------------------------------------------------------------------------
__device__ void build_masks(const DecodeState &st, int m, const int *hg, int n, bool first_ts, bool blank,
                            bool rules, int *hbuf) {
    const int lane = threadIdx.x & 31;
    // the history is scanned many times below: bring it into shared memory first
    for (int i0 = lane; hg != hbuf && i0 < n; i0 += 32 * 8) {
        int v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (i0 + 32 * j < n) v[j] = hg[i0 + 32 * j];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (i0 + 32 * j < n) hbuf[i0 + 32 * j] = v[j];
    }
    __syncwarp();
    const int *h = hbuf;
    int *list = st.dyn_list + (size_t)m * st.dyn_stride;
    int2 *rg = st.ranges + (size_t)m * kMaxRanges;
    int cnt = 0, nr = 0;
    const int V = st.V;
    if (lane == 0) {
        if (blank) {  // suppressBlank
            list[cnt++] = st.eot;
            if (220 < V) list[cnt++] = 220;
        }
        if (rules && st.ts_begin > 0) {
            const int tb = st.ts_begin;
            if (tb - 1 >= 0 && tb - 1 < V) list[cnt++] = tb - 1;
            if (first_ts) {
                rg[nr++] = make_int2(0, min(tb, V));
                rg[nr++] = make_int2(min(tb + 51, V), V);
            } else if (n > 0) {
                const bool last_ts = h[n - 1] >= tb;
                const bool pen_ts = n < 2 || h[n - 2] >= tb;
                if (last_ts) {
                    if (pen_ts)
                        rg[nr++] = make_int2(min(tb, V), V);
                    else
                        rg[nr++] = make_int2(0, min(st.eot, V));
                }
                int lts = -1;
                for (int i = n - 1; i >= 0; --i)
                    if (h[i] >= tb) {
                        lts = h[i];
                        break;
                    }
                if (lts >= 0) {
                    const int up = (last_ts && !pen_ts) ? lts + 1 : lts;
                    if (up > tb) rg[nr++] = make_int2(tb, min(up, V));
                }
            }
        }
    }
    cnt = __shfl_sync(0xffffffffu, cnt, 0);
    nr = __shfl_sync(0xffffffffu, nr, 0);
    if (rules) {
        // no-repeat n-gram block, n = 3 and 4
        for (int nn = 3; nn <= 4; ++nn) {
            if (n < nn - 1) continue;
            for (int i0 = 0; i0 <= n - nn; i0 += 32) {
                const int i = i0 + lane;
                bool hit = false;
                int blocked = 0;
                if (i <= n - nn) {
                    hit = true;
                    for (int j = 0; j < nn - 1; ++j)
                        if (h[i + j] != h[n - (nn - 1) + j]) {
                            hit = false;
                            break;
                        }
                    if (hit) {
                        blocked = h[i + nn - 1];
                        hit = blocked >= 0 && blocked < V;
                    }
                }
                const unsigned bal = __ballot_sync(0xffffffffu, hit);
                const int off = __popc(bal & ((1u << lane) - 1u));
                if (hit && cnt + off < st.dyn_stride) list[cnt + off] = blocked;
                cnt += __popc(bal);
            }
        }
    }
    if (cnt > st.dyn_stride) {
        if (lane == 0) atomicExch(st.err, 1);
        cnt = st.dyn_stride;
    }
    if (lane == 0) {
        st.dyn_count[m] = cnt;
        st.n_ranges[m] = nr;
    }
}

// splitmix64 of (seed, stream, step): the device stand-in for Math.random()
__device__ __forceinline__ double uniform01(unsigned long long seed, int stream, int step) {
    unsigned long long z = seed ^ (0x9e3779b97f4a7c15ull * (unsigned long long)(stream + 1)) ^
                           ((unsigned long long)step << 32);
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    z ^= z >> 31;
    return (double)(z >> 11) * (1.0 / 9007199254740992.0);
}

// Sampling at temperature T over one masked logits row (reference: sample, then the
// log-softmax of the array that sample overwrote with exp values).
__device__ void sample_row(float *row, int V, float T, double u, int *out_tok, double *out_lp) {
    __shared__ float r_f[kSelThreads];
    __shared__ double r_d[kSelThreads];
    __shared__ double seg[kSelThreads];
    __shared__ int s_tok;
    const int tid = threadIdx.x;
    float mx = -INFINITY;
    for (int i = tid; i < V; i += kSelThreads) mx = fmaxf(mx, row[i]);
    r_f[tid] = mx;
    __syncthreads();
    for (int o = kSelThreads / 2; o > 0; o >>= 1) {
        if (tid < o) r_f[tid] = fmaxf(r_f[tid], r_f[tid + o]);
        __syncthreads();
    }
    const float M = r_f[0];
    __syncthreads();
    // contiguous segments so that the cumulative search runs in index order
    const int per = (V + kSelThreads - 1) / kSelThreads;
    const int b0 = min(V, tid * per), b1 = min(V, b0 + per);
    double s = 0.0;
    for (int i = b0; i < b1; ++i) {
        const double p = exp((double)((row[i] - M) / T));
        row[i] = (float)p;
        s += p;
    }
    seg[tid] = s;
    __syncthreads();
    if (tid == 0) {
        double tot = 0.0;
        for (int t = 0; t < kSelThreads; ++t) tot += seg[t];
        const double r = u * tot;
        double cum = 0.0;
        int tok = V - 1;
        bool found = false;
        for (int t = 0; t < kSelThreads && !found; ++t) {
            if (cum + seg[t] >= r) {
                const int c0 = min(V, t * per), c1 = min(V, c0 + per);
                for (int i = c0; i < c1; ++i) {
                    cum += (double)row[i];
                    if (cum >= r) {
                        tok = i;
                        found = true;
                        break;
                    }
                }
            } else {
                cum += seg[t];
            }
        }
        s_tok = tok;
    }
    __syncthreads();
    // log-softmax at tok of the overwritten array
    float mp = -INFINITY;
    for (int i = tid; i < V; i += kSelThreads) mp = fmaxf(mp, row[i]);
    r_f[tid] = mp;
    __syncthreads();
    for (int o = kSelThreads / 2; o > 0; o >>= 1) {
        if (tid < o) r_f[tid] = fmaxf(r_f[tid], r_f[tid + o]);
        __syncthreads();
    }
    const float MP = r_f[0];
    double ls = 0.0;
    for (int i = tid; i < V; i += kSelThreads) ls += exp((double)(row[i] - MP));
    r_d[tid] = ls;
    __syncthreads();
    for (int o = kSelThreads / 2; o > 0; o >>= 1) {
        if (tid < o) r_d[tid] += r_d[tid + o];
        __syncthreads();
    }
    if (tid == 0) {
        *out_tok = s_tok;
        *out_lp = (double)(row[s_tok] - MP) - log(r_d[0]);
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// greedy / sampling step (one block per stream, beam = 1)
// ---------------------------------------------------------------------------
// log2 of the float4 count of a staged partial record holding 4 + 2k floats, rounded up to
// a power of two (so record and field split with shifts): k = 0 -> 0, k = 6 -> 2, k = 9 -> 3.
__host__ __device__ inline int rec_l2(int k) {
    const int f4 = (4 + 2 * k + 3) / 4;
    int l2 = 0;
    while ((1 << l2) < f4) ++l2;
    return l2;
}

// One warp: the P partial records of one sequence into shared memory, record c at
// dst + c * (4 << l2) floats (the first 4 << l2 <= kPartStride floats of the record, whose
// used prefix is 4 + 2k); 24 independent 16-byte loads in flight per lane.
__device__ void stage_partials_warp(const float *part, int P, int l2, float *dst) {
    const int lane = threadIdx.x & 31;
    const int n = P << l2;
    const int mask = (1 << l2) - 1;
    constexpr int kB = 24;
    for (int e0 = lane; e0 < n; e0 += 32 * kB) {
        float4 v[kB];
#pragma unroll
        for (int j = 0; j < kB; ++j) {
            const int e = e0 + 32 * j;
            if (e < n) v[j] = *reinterpret_cast<const float4 *>(part + (size_t)(e >> l2) * kPartStride + ((e & mask) << 2));
        }
#pragma unroll
        for (int j = 0; j < kB; ++j) {
            const int e = e0 + 32 * j;
            if (e < n) reinterpret_cast<float4 *>(dst)[e] = v[j];
        }
    }
    __syncwarp();
}

// All threads of the block: n ints from global memory into shared memory, 8 loads in flight.
__device__ __forceinline__ void stage_ints(const int *src, int n, int *dst) {
    for (int i0 = threadIdx.x; i0 < n; i0 += blockDim.x * 8) {
        int v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = i0 + blockDim.x * j;
            v[j] = i < n ? src[i] : 0;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = i0 + blockDim.x * j;
            if (i < n) dst[i] = v[j];
        }
    }
}

__global__ void __launch_bounds__(kSelThreads) k_select_greedy(DecodeState st, int mode, const float *part, int P,
                                                               float *masked, int step) {
    __shared__ int s_tok, s_len, s_done, s_pos;
    __shared__ double s_lp, s_lp0;
    extern __shared__ __align__(16) float sel_smem[];
    float *stg = sel_smem;                                   // [P][4]
    int *hbuf = reinterpret_cast<int *>(sel_smem + P * 4);   // [hs]: this sequence's history
    const int s = blockIdx.x;
    const int m = s;
    // The sequence's state was written by an earlier graph launch (or, after the prompt, by
    // kernels that completed before the logits kernel started), never by the logits kernel
    // this one waits on: read it, and stage the history, before the wait.
    if (threadIdx.x == 0) {
        s_done = st.done[s];
        s_len = st.hist_len[0][m];
        s_lp0 = st.lp[0][m];
        s_pos = st.seq_pos[m];
    }
    __syncthreads();
    const int len = s_len;
    if (!s_done) stage_ints(st.hist[0] + (size_t)m * st.hs, len, hbuf);
    pdl_trigger();
    pdl_wait();
    if (st.gbar && blockIdx.x == 0) {  // the next step kernel's barriers
        if (threadIdx.x == 0) *st.gbar = 0;
        for (int j = threadIdx.x; j < st.n_gflag; j += blockDim.x) st.gflag[32 * j] = 0;
    }
    if (s_done) return;
    if (mode == SEL_GREEDY) {
        if (threadIdx.x < 32) {
            stage_partials_warp(part + (size_t)m * P * kPartStride, P, 0, stg);
            const Merged mg = merge_partials(stg, P, 4);
            if (threadIdx.x == 0) {
                s_tok = mg.argmax;
                // logSoftmax(last, best) with last[best] == max: (max - max) - log(sum)
                s_lp = (double)(mg.max - mg.max) - log(mg.sum);
            }
        }
    } else {
        int tok;
        double lp;
        // the draw is keyed by (seed, stream, tokens so far): reproducible for a given seed
        sample_row(masked + (size_t)m * st.V, st.V, st.temperature, uniform01(st.seed, s, len), &tok, &lp);
        if (threadIdx.x == 0) {
            s_tok = tok;
            s_lp = lp;
        }
    }
    __syncthreads();
    const int tok = s_tok;
    if (threadIdx.x == 0) {
        st.lp[0][m] = s_lp0 + s_lp;
        if (tok == st.eot) {
            st.done[s] = 1;
            st.active[m] = 0;
        } else if (len < st.max_tokens) {
            st.hist[0][(size_t)m * st.hs + len] = tok;
            st.hist_len[0][m] = len + 1;
            st.tok_in[m] = tok;
            st.seq_pos[m] = s_pos + 1;
            hbuf[len] = tok;
        }
    }
    __syncthreads();
    if (threadIdx.x < 32 && tok != st.eot)
        build_masks(st, m, hbuf, min(len + 1, st.max_tokens), false, false, true, hbuf);
}

// ---------------------------------------------------------------------------
// beam search: initial expansion from the prompt logits, then one step per call
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kSelThreads) k_select_beam_init(DecodeState st, const float *part, int P) {
    __shared__ float tv[kMaxTopK];
    __shared__ int ti[kMaxTopK];
    pdl_trigger();
    pdl_wait();
    if (st.gbar && blockIdx.x == 0) {  // the next step kernel's barriers
        if (threadIdx.x == 0) *st.gbar = 0;
        for (int j = threadIdx.x; j < st.n_gflag; j += blockDim.x) st.gflag[32 * j] = 0;
    }
    const int s = blockIdx.x;
    const int B = st.beam;
    const float *pp = part + (size_t)s * P * kPartStride;
    extern __shared__ __align__(16) float sel_smem[];
    const int F = 4 + 2 * B;
    // per warp: staged partials, then a history buffer; a multiple of 4 floats keeps every
    // warp's region 16-byte aligned for the vector copies into it
    const int region = (P * F + st.hs + 3) & ~3;
    __shared__ float s_lsf;
    if (threadIdx.x < 32) {
        stage_partials(pp, P, B, sel_smem);
        const Merged mg = merge_partials(sel_smem, P, F);
        merge_topk(sel_smem, P, F, B, B, tv, ti);
        if (threadIdx.x == 0) s_lsf = (float)((double)mg.max + log(mg.sum));
    }
    const int base = st.stream_base[s];  // prompt rows were written in the stream's first slot
    __syncthreads();
    const float log_sum_f = s_lsf;
    for (int b = 0; b < B; ++b) {
        const int mb = s * B + b;
        for (int p = threadIdx.x; p < st.n_prompt; p += kSelThreads)
            st.table[0][(size_t)mb * st.n_ctx + p] = base;
        if (threadIdx.x == 0) {
            st.hist[0][(size_t)mb * st.hs] = ti[b];
            st.hist_len[0][mb] = 1;
            st.lp[0][mb] = (double)(float)(tv[b] - log_sum_f);
            st.tok_in[mb] = ti[b];
            st.seq_pos[mb] = st.n_prompt;
            st.active[mb] = 1;
            if (st.n_prompt < st.n_ctx) st.table[0][(size_t)mb * st.n_ctx + st.n_prompt] = base + b;
        }
    }
    if (threadIdx.x == 0) {
        st.fin_n[s] = 0;
        st.beam_par[s] = 0;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5;
    for (int b = warp; b < B; b += kSelThreads / 32) {
        const int mb = s * B + b;
        build_masks(st, mb, st.hist[0] + (size_t)mb * st.hs, 1, false, false, true,
                    reinterpret_cast<int *>(sel_smem + (size_t)b * region + P * F));
    }
}

constexpr int kMaxBeam = 8;  // contexts allow beam <= 8

__global__ void __launch_bounds__(kSelThreads) k_select_beam(DecodeState st, int parity, const float *part, int P) {
    constexpr int kMaxC = kMaxBeam * (kMaxBeam + 1);
    __shared__ double c_score[kMaxC], r_score[kMaxC];
    __shared__ int c_beam[kMaxC], c_tok[kMaxC], r_beam[kMaxC], r_tok[kMaxC];
    __shared__ int new_src[kMaxBeam], new_tok[kMaxBeam], fin_src[kMaxBeam];
    __shared__ double new_score[kMaxBeam], fin_score[kMaxBeam];
    __shared__ float b_tv[kMaxBeam][kMaxBeam + 1];
    __shared__ int b_ti[kMaxBeam][kMaxBeam + 1];
    __shared__ float b_lsf[kMaxBeam];
    __shared__ int b_live[kMaxBeam], b_len[kMaxBeam], b_pos[kMaxBeam], b_slot[kMaxBeam];
    __shared__ double b_lp[kMaxBeam];
    __shared__ int s_done, s_fin, s_nc, n_saved, n_fin_new;
    extern __shared__ __align__(16) float sel_smem[];
    const int s = blockIdx.x;
    const int B = st.beam, K1 = B + 1;
    const int po = parity, pn = parity ^ 1;
    const int stride = st.hs, C = st.n_ctx;
    const int l2 = rec_l2(K1), Fp = 4 << l2;
    // shared memory: per beam a region (staged partials, then the new history for the masks;
    // a multiple of 4 floats keeps every region 16-byte aligned), then the old histories and
    // beam tables of all beams
    const int region = (P * Fp + stride + 3) & ~3;
    int *h_old = reinterpret_cast<int *>(sel_smem + (size_t)B * region);  // [B][stride]
    int *t_old = h_old + (size_t)B * stride;                               // [B][C]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // The beams' state at parity po was written by an earlier graph launch (or by the initial
    // expansion, which completed before the logits kernel started), never by the logits kernel
    // this one waits on: read it, and stage histories and tables, before the wait.
    if (threadIdx.x == 0) {
        s_done = st.done[s];
        s_fin = st.fin_n[s];
        n_saved = 0;
        n_fin_new = 0;
    }
    if (threadIdx.x < B) {
        const int mb = s * B + threadIdx.x;
        b_len[threadIdx.x] = st.hist_len[po][mb];
        b_pos[threadIdx.x] = st.seq_pos[mb];
        b_lp[threadIdx.x] = st.lp[po][mb];
        b_slot[threadIdx.x] = st.seq_slot[mb];
    }
    __syncthreads();
    if (!s_done) {
        int n = 0;
        for (int b = 0; b < B; ++b) n = max(n, max(b_len[b], min(b_pos[b] + 1, C)));
        for (int r = threadIdx.x; r < n; r += kSelThreads) {  // every beam's entry r at once
            int hv[kMaxBeam], tv[kMaxBeam];
#pragma unroll
            for (int b = 0; b < kMaxBeam; ++b) {
                const int mb = s * B + b;
                hv[b] = (b < B && r < b_len[b]) ? st.hist[po][(size_t)mb * stride + r] : 0;
                tv[b] = (b < B && r <= b_pos[b] && r < C) ? st.table[po][(size_t)mb * C + r] : 0;
            }
#pragma unroll
            for (int b = 0; b < kMaxBeam; ++b) {
                if (b < B && r < b_len[b]) h_old[b * stride + r] = hv[b];
                if (b < B && r <= b_pos[b] && r < C) t_old[b * C + r] = tv[b];
            }
        }
    }
    pdl_trigger();
    pdl_wait();
    if (st.gbar && blockIdx.x == 0) {  // the next step kernel's barriers
        if (threadIdx.x == 0) *st.gbar = 0;
        for (int j = threadIdx.x; j < st.n_gflag; j += blockDim.x) st.gflag[32 * j] = 0;
    }
    if (s_done) return;
    __syncthreads();  // staged histories
    // one warp per beam: its partials, their merge and top-(beam + 1); finished beams skip
    if (warp < B) {
        const int b = warp;
        const bool live = h_old[b * stride + b_len[b] - 1] != st.eot;
        if (lane == 0) b_live[b] = live;
        if (live) {
            float *stg = sel_smem + (size_t)b * region;
            stage_partials_warp(part + (size_t)(s * B + b) * P * kPartStride, P, l2, stg);
            const Merged mg = merge_partials(stg, P, Fp);
            merge_topk(stg, P, Fp, K1, K1, b_tv[b], b_ti[b]);
            if (lane == 0) b_lsf[b] = (float)((double)mg.max + log(mg.sum));
        }
    }
    __syncthreads();
    // candidates in the reference's insertion order (live beams, then rank within the beam)
    if (threadIdx.x < B * K1) {
        const int t = threadIdx.x, b = t / K1, k = t - b * K1;
        if (b_live[b]) {
            int before = 0;
            for (int u = 0; u < b; ++u) before += b_live[u];
            const int idx = before * K1 + k;
            c_score[idx] = b_lp[b] + (double)(float)(b_tv[b][k] - b_lsf[b]);
            c_beam[idx] = b;
            c_tok[idx] = b_ti[b][k];
        }
    }
    if (threadIdx.x == 0) {
        int nl = 0;
        for (int b = 0; b < B; ++b) nl += b_live[b];
        s_nc = nl * K1;
    }
    __syncthreads();
    const int n_c = s_nc;
    // stable sort by score, descending (List.sort with Double.compare): every candidate
    // computes its own rank and moves there
    __shared__ unsigned long long c_key[kMaxC];
    if (threadIdx.x < n_c) c_key[threadIdx.x] = dkey(c_score[threadIdx.x]);
    __syncthreads();
    if (threadIdx.x < n_c) {
        const int t = threadIdx.x;
        const unsigned long long ck = c_key[t];
        int rank = 0;
#pragma unroll 8
        for (int u = 0; u < n_c; ++u) {
            const unsigned long long uk = c_key[u];
            rank += (uk > ck) | ((uk == ck) & (u < t));
        }
        r_score[rank] = c_score[t];
        r_beam[rank] = c_beam[t];
        r_tok[rank] = c_tok[t];
    }
    __syncthreads();
    // the reference walks the sorted list: an eot candidate finishes a sequence (and the walk
    // stops once fin_n reaches beam), any other continues as a new beam while fewer than beam
    // are saved.  Candidate i is reached iff fin_n + (eot candidates before i) < beam.
    if (threadIdx.x < n_c) {
        const int i = threadIdx.x;
        int eb = 0;
#pragma unroll 8
        for (int j = 0; j < i; ++j) eb += r_tok[j] == st.eot;
        if (s_fin + eb < B) {
            if (r_tok[i] == st.eot) {
                fin_src[eb] = r_beam[i];
                fin_score[eb] = r_score[i];
                atomicAdd(&n_fin_new, 1);
            } else if (i - eb < B) {
                new_src[i - eb] = r_beam[i];
                new_tok[i - eb] = r_tok[i];
                new_score[i - eb] = r_score[i];
                atomicAdd(&n_saved, 1);
            }
        }
    }
    __syncthreads();
    const int saved = n_saved, nf = n_fin_new, fin0 = s_fin;
    const bool finish = n_c == 0 || saved == 0 || fin0 + nf >= B;
    // finished sequences: the source beam's tokens (without the eot), from shared memory
    for (int f = 0; f < nf; ++f) {
        const int sb = fin_src[f];
        const int len = b_len[sb];
        int *dst = st.fin_tok + ((size_t)s * B + fin0 + f) * stride;
        for (int i = threadIdx.x; i < len; i += kSelThreads) dst[i] = h_old[sb * stride + i];
        if (threadIdx.x == 0) {
            st.fin_len[(size_t)s * B + fin0 + f] = len;
            st.fin_lp[(size_t)s * B + fin0 + f] = fin_score[f];
        }
    }
    if (threadIdx.x == 0) st.fin_n[s] = fin0 + nf;
    if (finish) {
        if (threadIdx.x == 0) {
            st.done[s] = 1;
            for (int b = 0; b < B; ++b) st.active[s * B + b] = 0;  // live beams stay at parity po
        }
        return;
    }
    // rearrange: new beam b continues source beam new_src[b] (beams past `saved` copy beam 0);
    // histories and tables at parity pn are written from the staged copies, and each new
    // history also goes to its beam's region for the masks
    for (int b = 0; b < B; ++b) {
        const int sb = new_src[b < saved ? b : 0];
        const int len = b_len[sb], pos = b_pos[sb];
        const int mb = s * B + b;
        int *hb = reinterpret_cast<int *>(sel_smem + (size_t)b * region + P * Fp);
        for (int r = threadIdx.x; r < len; r += kSelThreads) {
            const int v = h_old[sb * stride + r];
            st.hist[pn][(size_t)mb * stride + r] = v;
            hb[r] = v;
        }
        for (int r = threadIdx.x; r <= pos && r < C; r += kSelThreads)
            st.table[pn][(size_t)mb * C + r] = t_old[sb * C + r];
    }
    if (threadIdx.x < B) {
        const int b = threadIdx.x;
        const int bb = b < saved ? b : 0;
        const int sb = new_src[bb];
        const int mb = s * B + b;
        const int len = b_len[sb];
        const int pos = b_pos[sb];  // row written this step by the source beam
        st.hist[pn][(size_t)mb * stride + len] = new_tok[bb];
        reinterpret_cast<int *>(sel_smem + (size_t)b * region + P * Fp)[len] = new_tok[bb];
        st.hist_len[pn][mb] = len + 1;
        st.lp[pn][mb] = new_score[bb];
        if (pos + 1 < C) st.table[pn][(size_t)mb * C + pos + 1] = b_slot[b];
        st.tok_in[mb] = new_tok[bb];
        st.seq_pos[mb] = b_pos[0] + 1;  // beams of a stream advance in lockstep
    }
    __syncthreads();
    if (warp < B) {
        const int b = warp;
        int *hb = reinterpret_cast<int *>(sel_smem + (size_t)b * region + P * Fp);
        build_masks(st, s * B + b, hb, b_len[new_src[b < saved ? b : 0]] + 1, false, false, true, hb);
    }
    if (threadIdx.x == 0) st.beam_par[s] = pn;  // parity holding the live beams (finalize reads it)
}

// no-speech probability from the unmasked statistics of the first prompt row
__global__ void k_nsp(DecodeState st, const float *ns_part, int P, const float *ns_value) {
    __shared__ float r_v[kSelThreads];
    __shared__ double r_s[kSelThreads];
    pdl_trigger();
    pdl_wait();
    const int s = blockIdx.x;
    const int tid = threadIdx.x;
    const float *np = ns_part + (size_t)s * P * 2;
    float mx = -INFINITY;
    for (int c = tid; c < P; c += kSelThreads) mx = fmaxf(mx, np[2 * c]);
    r_v[tid] = mx;
    __syncthreads();
    for (int o = kSelThreads / 2; o > 0; o >>= 1) {
        if (tid < o) r_v[tid] = fmaxf(r_v[tid], r_v[tid + o]);
        __syncthreads();
    }
    const float M = r_v[0];
    double sm = 0.0;
    for (int c = tid; c < P; c += kSelThreads)
        if (np[2 * c] != -INFINITY) sm += (double)np[2 * c + 1] * exp((double)(np[2 * c] - M));
    r_s[tid] = sm;
    __syncthreads();
    for (int o = kSelThreads / 2; o > 0; o >>= 1) {
        if (tid < o) r_s[tid] += r_s[tid + o];
        __syncthreads();
    }
    if (tid == 0) st.nsp[s] = (float)(exp((double)(ns_value[s] - M)) / r_s[0]);
}

// masks of the first decision (step 0): suppressBlank always, timestamp first-step rules for greedy
__global__ void k_init_masks(DecodeState st, int beam_mode) {
    const int m = blockIdx.x;
    if (threadIdx.x >= 32) return;
    __shared__ int hbuf[1];  // the first decision has no history
    build_masks(st, m, st.hist[0] + (size_t)m * st.hs, 0, !beam_mode, true, !beam_mode, hbuf);
}

__global__ void k_finalize(DecodeState st, int beam_mode) {
    const int s = blockIdx.x;
    const int stride = st.hs;
    if (!beam_mode) {
        const int m = s;
        const int len = st.hist_len[0][m];
        for (int i = threadIdx.x; i < len; i += blockDim.x)
            st.out_tok[(size_t)s * st.max_tokens + i] = st.hist[0][(size_t)m * stride + i];
        if (threadIdx.x == 0) {
            st.out_len[s] = len;
            st.out_sum[s] = st.lp[0][m];
        }
        return;
    }
    __shared__ int s_best, s_par;
    const int B = st.beam;
    if (threadIdx.x == 0) {
        s_par = st.beam_par[s];
        int fin = st.fin_n[s];
        // not enough finished sequences: add the live beams in order (:370-377)
        for (int b = 0; b < B && fin < B; ++b, ++fin) {
            const int mb = s * B + b;
            const int len = st.hist_len[s_par][mb];
            int *dst = st.fin_tok + ((size_t)s * B + fin) * stride;
            for (int i = 0; i < len; ++i) dst[i] = st.hist[s_par][(size_t)mb * stride + i];
            st.fin_len[(size_t)s * B + fin] = len;
            st.fin_lp[(size_t)s * B + fin] = st.lp[s_par][mb];
        }
        st.fin_n[s] = fin;
        int best = 0;
        double best_score = -INFINITY;
        for (int i = 0; i < fin; ++i) {
            const int len = st.fin_len[(size_t)s * B + i];
            const double sc = st.fin_lp[(size_t)s * B + i] / (double)(len > 1 ? len : 1);
            if (sc > best_score) {
                best_score = sc;
                best = i;
            }
        }
        s_best = best;
    }
    __syncthreads();
    const int len = st.fin_len[(size_t)s * B + s_best];
    const int *src = st.fin_tok + ((size_t)s * B + s_best) * stride;
    const int n = len < st.max_tokens ? len : st.max_tokens;
    for (int i = threadIdx.x; i < n; i += blockDim.x) st.out_tok[(size_t)s * st.max_tokens + i] = src[i];
    if (threadIdx.x == 0) {
        st.out_len[s] = n;
        st.out_sum[s] = st.fin_lp[(size_t)s * B + s_best];
    }
}

__global__ void k_argmax_merge(const float *part, int P, int32_t *tok, double *lp) {
    const int m = blockIdx.x;
    extern __shared__ __align__(16) float sel_smem[];
    if (threadIdx.x >= 32) return;
    stage_partials(part + (size_t)m * P * kPartStride, P, 0, sel_smem);
    const Merged mg = merge_partials(sel_smem, P, 4);
    if (threadIdx.x == 0) {
        tok[m] = mg.argmax;
        lp[m] = (double)(mg.max - mg.max) - log(mg.sum);
    }
}

// One block, one warp per row: the same merge as k_argmax_merge, then the device error word.
// If a bounded wait of the logits kernel ran out, every row reports token -1 and a NaN
// log-probability, and the word is cleared so that the next call starts from zero.
__global__ void k_argmax_merge_status(const float *part, int P, int M, int32_t *tok, double *lp, int *err) {
    extern __shared__ __align__(16) float sel_smem[];
    const int warp = threadIdx.x >> 5;
    if (warp < M) {
        float *stg = sel_smem + (size_t)warp * P * 4;
        stage_partials(part + (size_t)warp * P * kPartStride, P, 0, stg);
        const Merged mg = merge_partials(stg, P, 4);
        if ((threadIdx.x & 31) == 0) {
            tok[warp] = mg.argmax;
            lp[warp] = (double)(mg.max - mg.max) - log(mg.sum);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && *err != 0) {
        for (int m = 0; m < M; ++m) {
            tok[m] = -1;
            lp[m] = __longlong_as_double(0x7ff8000000000000ll);
        }
        *err = 0;
    }
}

// After a merge of M rows: if the device error word is set (a bounded wait of the vocabulary
// pass ran out), every row reports token -1 and a NaN log-probability, and the word is cleared.
__global__ void k_err_apply(int M, int32_t *tok, double *lp, int *err) {
    __shared__ int e;
    if (threadIdx.x == 0) e = *err;
    __syncthreads();
    if (!e) return;
    for (int m = threadIdx.x; m < M; m += blockDim.x) {
        tok[m] = -1;
        lp[m] = __longlong_as_double(0x7ff8000000000000ll);
    }
    __syncthreads();
    if (threadIdx.x == 0) *err = 0;
}

// ---------------------------------------------------------------------------
static cudaLaunchConfig_t cfg_for(dim3 grid, dim3 block, cudaStream_t s, bool pdl, cudaLaunchAttribute *attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = s;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

// Dynamic shared memory of the select kernels: per working warp, the staged partials of one
// sequence (P x (3 + 2k) floats) followed by a token-history buffer (hs ints).
static size_t select_smem(const DecodeState &st, int mode, int P) {
    const int B = st.beam;
    if (mode == SEL_GREEDY || mode == SEL_SAMPLE) return ((size_t)P * 4 + st.hs) * 4;
    if (mode == SEL_BEAM_INIT) return (size_t)B * (((size_t)P * (4 + 2 * B) + st.hs + 3) & ~(size_t)3) * 4;
    const size_t fp = (size_t)4 << rec_l2(B + 1);
    return ((size_t)B * (((size_t)P * fp + st.hs + 3) & ~(size_t)3) + (size_t)B * (st.hs + st.n_ctx)) * 4;
}

size_t select_smem_bytes(const DecodeState &st, int mode, int P) { return select_smem(st, mode, P); }

cudaError_t select_prepare() {
    cudaError_t e = allow_dynamic_smem(k_select_greedy);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_select_beam_init);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_select_beam);
    if (e == cudaSuccess) e = allow_dynamic_smem(k_argmax_merge);
    if (e == cudaSuccess) e = prefer_max_smem(k_argmax_merge_status);
    if (e == cudaSuccess) e = prefer_max_smem(k_nsp);
    if (e == cudaSuccess) e = prefer_max_smem(k_init_masks);
    if (e == cudaSuccess) e = prefer_max_smem(k_finalize);
    return e;
}

cudaError_t launch_select(const DecodeState &st, int mode, int parity, const float *part, int n_parts,
                          float *masked, int step, cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = cfg_for(dim3(st.n_streams), dim3(kSelThreads), s, pdl, attr);
    cfg.dynamicSmemBytes = select_smem(st, mode, n_parts);
    // the beam merge keeps at most 256 records' heads in registers (merge_topk); greedy takes any count
    const bool beam = mode == SEL_BEAM_INIT || mode == SEL_BEAM;
    if (cfg.dynamicSmemBytes > 227 * 1024 || (beam && n_parts > 256) || st.beam > kMaxBeam) return cudaErrorInvalidValue;
    switch (mode) {
        case SEL_GREEDY:
        case SEL_SAMPLE:
            return cudaLaunchKernelEx(&cfg, k_select_greedy, st, mode, part, n_parts, masked, step);
        case SEL_BEAM_INIT:
            return cudaLaunchKernelEx(&cfg, k_select_beam_init, st, part, n_parts);
        case SEL_BEAM:
            return cudaLaunchKernelEx(&cfg, k_select_beam, st, parity, part, n_parts);
    }
    return cudaErrorInvalidValue;
}

cudaError_t launch_nsp(const DecodeState &st, const float *ns_part, int n_parts, const float *ns_value,
                       cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = cfg_for(dim3(st.n_streams), dim3(kSelThreads), s, pdl, attr);
    return cudaLaunchKernelEx(&cfg, k_nsp, st, ns_part, n_parts, ns_value);
}

cudaError_t launch_init_masks(const DecodeState &st, int beam_mode, cudaStream_t s) {
    k_init_masks<<<st.n_streams, 32, 0, s>>>(st, beam_mode);
    return cudaGetLastError();
}

cudaError_t launch_finalize(const DecodeState &st, int beam_mode, int parity, cudaStream_t s) {
    (void)parity;
    k_finalize<<<st.n_streams, 128, 0, s>>>(st, beam_mode);
    return cudaGetLastError();
}

cudaError_t launch_argmax_merge(const float *part, int n_parts, int M, int32_t *tok, double *lp, cudaStream_t s) {
    k_argmax_merge<<<M, kSelThreads, (size_t)n_parts * 4 * 4, s>>>(part, n_parts, tok, lp);
    return cudaGetLastError();
}

cudaError_t launch_err_apply(int M, int32_t *tok, double *lp, int *err, cudaStream_t s) {
    k_err_apply<<<1, 256, 0, s>>>(M, tok, lp, err);
    return cudaGetLastError();
}

// M <= 32 rows in one block; shared memory M * n_parts * 16 bytes (the caller bounds it).
cudaError_t launch_argmax_merge_status(const float *part, int n_parts, int M, int32_t *tok, double *lp, int *err,
                                       cudaStream_t s) {
    if (M < 1 || M > 32) return cudaErrorInvalidValue;
    k_argmax_merge_status<<<1, 32 * M, (size_t)M * n_parts * 4 * 4, s>>>(part, n_parts, M, tok, lp, err);
    return cudaGetLastError();
}

}  // namespace w4j
