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

// Double.compare(a, b) > 0, as the reference's candidate sort uses (-0.0 < 0.0, NaN largest).
__device__ __forceinline__ bool dgreater(double a, double b) {
    if (a > b) return true;
    if (a < b) return false;
    const bool an = isnan(a), bn = isnan(b);
    if (an || bn) return an && !bn;
    return !signbit(a) && signbit(b);
}

// ---------------------------------------------------------------------------
// block-level merge of the logits partials of one sequence
// ---------------------------------------------------------------------------
struct Merged {
    float max;
    int argmax;
    double sum;  // sum_i exp(l_i - max)
};

__device__ Merged merge_partials(const float *part, int P) {
    __shared__ float r_v[kSelThreads];
    __shared__ int r_i[kSelThreads];
    __shared__ double r_s[kSelThreads];
    const int tid = threadIdx.x;
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int c = tid; c < P; c += kSelThreads) {
        const float v = part[(size_t)c * kPartStride];
        const int i = __float_as_int(part[(size_t)c * kPartStride + 2]);
        if (better_c(v, i, bv, bi)) {
            bv = v;
            bi = i;
        }
    }
    r_v[tid] = bv;
    r_i[tid] = bi;
    __syncthreads();
    for (int o = kSelThreads / 2; o > 0; o >>= 1) {
        if (tid < o && better_c(r_v[tid + o], r_i[tid + o], r_v[tid], r_i[tid])) {
            r_v[tid] = r_v[tid + o];
            r_i[tid] = r_i[tid + o];
        }
        __syncthreads();
    }
    const float M = r_v[0];
    const int arg = r_i[0];
    double s = 0.0;
    if (M != -INFINITY)
        for (int c = tid; c < P; c += kSelThreads) {
            const float mc = part[(size_t)c * kPartStride];
            if (mc != -INFINITY) s += (double)part[(size_t)c * kPartStride + 1] * exp((double)(mc - M));
        }
    r_s[tid] = s;
    __syncthreads();
    for (int o = kSelThreads / 2; o > 0; o >>= 1) {
        if (tid < o) r_s[tid] += r_s[tid + o];
        __syncthreads();
    }
    Merged out;
    out.max = M;
    // reference argmax: index 0 when nothing beats a[0] = -inf
    out.argmax = (M == -INFINITY || arg == INT_MAX) ? 0 : arg;
    out.sum = r_s[0];
    __syncthreads();
    return out;
}

// Top-k over the per-block candidate lists (value desc, index asc); unfilled -> (-inf, 0).
__device__ void merge_topk(const float *part, int P, int k, float *out_v, int *out_i) {
    __shared__ float r_v[kSelThreads];
    __shared__ int r_i[kSelThreads];
    __shared__ int chosen[kMaxTopK];
    const int tid = threadIdx.x;
    for (int r = 0; r < k; ++r) {
        float bv = -INFINITY;
        int bi = INT_MAX;
        for (int e = tid; e < P * k; e += kSelThreads) {
            const int c = e / k, j = e % k;
            const float v = part[(size_t)c * kPartStride + 4 + j];
            const int i = __float_as_int(part[(size_t)c * kPartStride + 4 + kMaxTopK + j]);
            if (v == -INFINITY) continue;
            bool taken = false;
            for (int q = 0; q < r; ++q) taken |= chosen[q] == i;
            if (!taken && better_c(v, i, bv, bi)) {
                bv = v;
                bi = i;
            }
        }
        r_v[tid] = bv;
        r_i[tid] = bi;
        __syncthreads();
        for (int o = kSelThreads / 2; o > 0; o >>= 1) {
            if (tid < o && better_c(r_v[tid + o], r_i[tid + o], r_v[tid], r_i[tid])) {
                r_v[tid] = r_v[tid + o];
                r_i[tid] = r_i[tid + o];
            }
            __syncthreads();
        }
        if (tid == 0) {
            const bool none = r_i[0] == INT_MAX;
            out_v[r] = none ? -INFINITY : r_v[0];
            out_i[r] = none ? 0 : r_i[0];
            chosen[r] = none ? -1 : r_i[0];
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// masks of the next step (one warp)
// ---------------------------------------------------------------------------
__device__ void build_masks(const DecodeState &st, int m, const int *h, int n, bool first_ts, bool blank,
                            bool rules) {
    const int lane = threadIdx.x & 31;
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
__global__ void __launch_bounds__(kSelThreads) k_select_greedy(DecodeState st, int mode, const float *part, int P,
                                                               float *masked, int step) {
    __shared__ int s_tok;
    __shared__ double s_lp;
    pdl_trigger();
    pdl_wait();
    const int s = blockIdx.x;
    const int m = s;
    if (st.done[s]) return;
    if (mode == SEL_GREEDY) {
        const Merged mg = merge_partials(part + (size_t)m * P * kPartStride, P);
        if (threadIdx.x == 0) {
            s_tok = mg.argmax;
            // logSoftmax(last, best) with last[best] == max: (max - max) - log(sum)
            s_lp = (double)(mg.max - mg.max) - log(mg.sum);
        }
    } else {
        int tok;
        double lp;
        // the draw is keyed by (seed, stream, tokens so far): reproducible for a given seed
        sample_row(masked + (size_t)m * st.V, st.V, st.temperature, uniform01(st.seed, s, st.hist_len[0][m]), &tok,
                   &lp);
        if (threadIdx.x == 0) {
            s_tok = tok;
            s_lp = lp;
        }
    }
    __shared__ int s_len;
    if (threadIdx.x == 0) s_len = st.hist_len[0][m];
    __syncthreads();
    const int len = s_len;
    if (threadIdx.x == 0) {
        st.lp[0][m] += s_lp;
        if (s_tok == st.eot) {
            st.done[s] = 1;
            st.active[m] = 0;
        } else if (len < st.max_tokens) {
            st.hist[0][(size_t)m * st.hs + len] = s_tok;
            st.hist_len[0][m] = len + 1;
            st.tok_in[m] = s_tok;
            st.seq_pos[m] += 1;
        }
    }
    __syncthreads();
    if (threadIdx.x < 32 && s_tok != st.eot)
        build_masks(st, m, st.hist[0] + (size_t)m * st.hs, min(len + 1, st.max_tokens), false, false,
                    true);
}

// ---------------------------------------------------------------------------
// beam search: initial expansion from the prompt logits, then one step per call
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kSelThreads) k_select_beam_init(DecodeState st, const float *part, int P) {
    __shared__ float tv[kMaxTopK];
    __shared__ int ti[kMaxTopK];
    pdl_trigger();
    pdl_wait();
    const int s = blockIdx.x;
    const int B = st.beam;
    const float *pp = part + (size_t)s * P * kPartStride;
    const Merged mg = merge_partials(pp, P);
    merge_topk(pp, P, B, tv, ti);
    const float log_sum_f = (float)((double)mg.max + log(mg.sum));
    const int base = st.stream_base[s];  // prompt rows were written in the stream's first slot
    __syncthreads();
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
        build_masks(st, mb, st.hist[0] + (size_t)mb * st.hs, 1, false, false, true);
    }
}

__global__ void __launch_bounds__(kSelThreads) k_select_beam(DecodeState st, int parity, const float *part, int P) {
    constexpr int kMaxB = kMaxTopK - 1;
    __shared__ double c_score[kMaxB * (kMaxB + 1)];
    __shared__ int c_beam[kMaxB * (kMaxB + 1)], c_tok[kMaxB * (kMaxB + 1)];
    __shared__ int n_c;
    __shared__ float tv[kMaxTopK];
    __shared__ int ti[kMaxTopK];
    __shared__ int new_src[kMaxB], new_tok[kMaxB];
    __shared__ double new_score[kMaxB];
    __shared__ int fin_src[kMaxB];
    __shared__ double fin_score[kMaxB];
    __shared__ int n_fin_new, saved_s, finish;
    pdl_trigger();
    pdl_wait();
    const int s = blockIdx.x;
    if (st.done[s]) return;
    const int B = st.beam;
    const int po = parity, pn = parity ^ 1;
    const int stride = st.hs;
    if (threadIdx.x == 0) n_c = 0;
    __syncthreads();
    for (int b = 0; b < B; ++b) {
        const int mb = s * B + b;
        const int len = st.hist_len[po][mb];
        if (st.hist[po][(size_t)mb * stride + len - 1] == st.eot) continue;  // finished beam
        const float *pp = part + (size_t)mb * P * kPartStride;
        const Merged mg = merge_partials(pp, P);
        merge_topk(pp, P, B + 1, tv, ti);
        if (threadIdx.x == 0) {
            const float log_sum_f = (float)((double)mg.max + log(mg.sum));
            const double blp = st.lp[po][mb];
            for (int k = 0; k < B + 1; ++k) {
                c_score[n_c] = blp + (double)(float)(tv[k] - log_sum_f);
                c_beam[n_c] = b;
                c_tok[n_c] = ti[k];
                ++n_c;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        // stable sort by score, descending (List.sort with Double.compare)
        for (int i = 1; i < n_c; ++i) {
            const double cs = c_score[i];
            const int cb = c_beam[i], ct = c_tok[i];
            int j = i - 1;
            while (j >= 0 && dgreater(cs, c_score[j])) {
                c_score[j + 1] = c_score[j];
                c_beam[j + 1] = c_beam[j];
                c_tok[j + 1] = c_tok[j];
                --j;
            }
            c_score[j + 1] = cs;
            c_beam[j + 1] = cb;
            c_tok[j + 1] = ct;
        }
        int saved = 0, nf = 0, fin = st.fin_n[s];
        for (int i = 0; i < n_c; ++i) {
            if (c_tok[i] == st.eot) {
                fin_src[nf] = c_beam[i];
                fin_score[nf] = c_score[i];
                ++nf;
                ++fin;
                if (fin >= B) break;
                continue;
            }
            if (saved >= B) continue;
            new_src[saved] = c_beam[i];
            new_tok[saved] = c_tok[i];
            new_score[saved] = c_score[i];
            ++saved;
        }
        n_fin_new = nf;
        saved_s = saved;
        finish = (n_c == 0 || saved == 0 || fin >= B) ? 1 : 0;
    }
    __syncthreads();
    // finished sequences: copy the source beam's tokens (without the eot)
    const int fin0 = st.fin_n[s];
    for (int f = 0; f < n_fin_new; ++f) {
        const int src = s * B + fin_src[f];
        const int len = st.hist_len[po][src];
        int *dst = st.fin_tok + ((size_t)s * B + fin0 + f) * stride;
        for (int i = threadIdx.x; i < len; i += kSelThreads) dst[i] = st.hist[po][(size_t)src * stride + i];
        if (threadIdx.x == 0) {
            st.fin_len[(size_t)s * B + fin0 + f] = len;
            st.fin_lp[(size_t)s * B + fin0 + f] = fin_score[f];
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) st.fin_n[s] = fin0 + n_fin_new;
    if (finish) {
        if (threadIdx.x == 0) {
            st.done[s] = 1;
            for (int b = 0; b < B; ++b) st.active[s * B + b] = 0;  // live beams stay at parity po
        }
        return;
    }
    // rearrange: new beam b continues source beam new_src[b] (beams past `saved` copy beam 0)
    const int saved = saved_s;
    for (int b = 0; b < B; ++b) {
        const int bb = b < saved ? b : 0;
        const int src = s * B + new_src[bb];
        const int mb = s * B + b;
        const int len = st.hist_len[po][src];
        const int pos = st.seq_pos[src];  // row written this step by the source beam
        int *hd = st.hist[pn] + (size_t)mb * stride;
        const int *hs = st.hist[po] + (size_t)src * stride;
        for (int i = threadIdx.x; i < len; i += kSelThreads) hd[i] = hs[i];
        int *td = st.table[pn] + (size_t)mb * st.n_ctx;
        const int *ts = st.table[po] + (size_t)src * st.n_ctx;
        for (int i = threadIdx.x; i <= pos; i += kSelThreads) td[i] = ts[i];
        if (threadIdx.x == 0) {
            hd[len] = new_tok[bb];
            st.hist_len[pn][mb] = len + 1;
            st.lp[pn][mb] = new_score[bb];
            if (pos + 1 < st.n_ctx) td[pos + 1] = st.seq_slot[mb];
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const int pos0 = st.seq_pos[s * B];  // beams of a stream advance in lockstep
        for (int b = 0; b < B; ++b) {
            const int bb = b < saved ? b : 0;
            const int mb = s * B + b;
            st.tok_in[mb] = new_tok[bb];
            st.seq_pos[mb] = pos0 + 1;
        }
    }
    __syncthreads();
    // every beam advanced one position; positions were equal, so read them after the writes
    const int warp = threadIdx.x >> 5;
    for (int b = warp; b < B; b += kSelThreads / 32) {
        const int mb = s * B + b;
        build_masks(st, mb, st.hist[pn] + (size_t)mb * stride, st.hist_len[pn][mb], false, false, true);
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
    build_masks(st, m, st.hist[0] + (size_t)m * st.hs, 0, !beam_mode, true, !beam_mode);
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
    const Merged mg = merge_partials(part + (size_t)m * P * kPartStride, P);
    if (threadIdx.x == 0) {
        tok[m] = mg.argmax;
        lp[m] = (double)(mg.max - mg.max) - log(mg.sum);
    }
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

cudaError_t launch_select(const DecodeState &st, int mode, int parity, const float *part, int n_parts,
                          float *masked, int step, cudaStream_t s, bool pdl) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = cfg_for(dim3(st.n_streams), dim3(kSelThreads), s, pdl, attr);
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
    k_argmax_merge<<<M, kSelThreads, 0, s>>>(part, n_parts, tok, lp);
    return cudaGetLastError();
}

}  // namespace w4j
