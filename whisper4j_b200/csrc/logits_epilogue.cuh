// logits_epilogue.cuh — shared epilogue of the vocabulary-logits kernels (SIMT and tcgen05).
#pragma once
#include "w4j_internal.cuh"

namespace w4j {

constexpr int kLaneTopK = 9;   // candidates per block: beam + 1 <= 9 (beam <= 8)
constexpr int kRowRegs = 16;   // row elements per lane held in registers (blocks of <= 512 rows)
constexpr int kDynStage = 32;  // per-sequence masked ids staged in shared memory (more: read from global)
constexpr int kStatStage = 128;

// Shared-memory copy of the masks and liveness of the rows (staged before the grid wait by the
// tensor-core kernel: the select kernel of the previous step wrote them).
struct MaskStage {
    const int *active;     // [M] (null: all live)
    const int *n_ranges;   // [M]
    const int2 *ranges;    // [M][kMaxRanges]
    const int *dyn_count;  // [M]
    const int *dyn;        // [M][kDynStage]
    const int *stat;       // [min(n_static, kStatStage)]
};

__device__ __forceinline__ bool logit_better(float v1, int i1, float v2, int i2) {
    return v1 > v2 || (v1 == v2 && i1 < i2);
}

// Logit processors and block reductions over the logits of rows [lo, hi) held in shared
// memory (tile[mm][row - lo], stride ch) for sequences m0 .. m0+MT: unmasked statistics for
// the no-speech probability, the masks (suppress list, n-gram and timestamp rules), then max,
// first argmax, sum of exp and the block's top-k candidates.  One warp per sequence: warps
// w0 .. w0 + nw of the block (nw = 0: all).  The records of row m are part[m][P][..] (P = 0: one
// per block, this block's at blockIdx.x; else record `slot`).
// RR: row elements per lane held in registers (rows of up to 32 RR ids take the register path).
template <int RR = kRowRegs>
__device__ __forceinline__ void logits_rows_epilogue(const LogitsArgs &a, float *tile, int ch, int MT, int m0, int lo, int hi,
                                     bool ok, const MaskStage *ms = nullptr, int P = 0, int slot = 0, int w0 = 0,
                                     int nw = 0) {
    if (P == 0) {
        P = gridDim.x;
        slot = blockIdx.x;
    }
    if (nw == 0) nw = blockDim.x / 32;
    const int nrows = hi - lo;
    const int warp = (threadIdx.x >> 5) - w0, lane = threadIdx.x & 31;
    if (warp < 0) return;
for (int mm = warp; mm < MT; mm += nw) {
        const int m = m0 + mm;
        if (m >= a.M || !ok) continue;
        if (a.active && !(ms ? ms->active[m] : a.active[m])) continue;
        float *row = tile + (size_t)mm * ch;
        const int n = nrows;
        if (a.ns_token >= 0) {  // unmasked statistics of this row (no-speech probability)
            float mx = -INFINITY;
            for (int i = lane; i < n; i += 32) mx = fmaxf(mx, row[i]);
            mx = warp_max(mx);
            float sm = 0.f;
            for (int i = lane; i < n; i += 32) sm += (mx == -INFINITY) ? 0.f : __expf(row[i] - mx);
            sm = warp_sum(sm);
            if (lane == 0) {
                float *np = a.ns_part + ((size_t)m * P + slot) * 2;
                np[0] = mx;
                np[1] = sm;
            }
            if (a.ns_token >= lo && a.ns_token < hi && lane == 0) a.ns_value[m] = row[a.ns_token - lo];
            __syncwarp();
        }
        if (a.use_mask) {
            const MaskArgs &mk = a.mask;
            const int nrg = ms ? ms->n_ranges[m] : mk.n_ranges[m];
            for (int r = 0; r < nrg; ++r) {
                const int2 rg = ms ? ms->ranges[(size_t)m * kMaxRanges + r] : mk.ranges[(size_t)m * kMaxRanges + r];
                const int b0 = max(rg.x, lo), b1 = min(rg.y, hi);
                for (int i = b0 + lane; i < b1; i += 32) row[i - lo] = -INFINITY;
            }
            // id lists: 8 independent loads in flight per lane
            auto mask_list = [&](const int *list, int n_list) {
                for (int i0 = lane; i0 < n_list; i0 += 32 * 8) {
                    int tk[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) tk[j] = i0 + 32 * j < n_list ? list[i0 + 32 * j] : -1;
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (tk[j] >= lo && tk[j] < hi) row[tk[j] - lo] = -INFINITY;
                }
            };
            if (ms) {  // staged heads of the lists, the rest (rare) from global memory
                const int ns = min(mk.n_static, kStatStage);
                mask_list(ms->stat, ns);
                mask_list(mk.static_list + ns, mk.n_static - ns);
                const int nd = ms->dyn_count[m], nds = min(nd, kDynStage);
                mask_list(ms->dyn + (size_t)m * kDynStage, nds);
                mask_list(mk.dyn_list + (size_t)m * mk.dyn_stride + nds, nd - nds);
            } else {
                mask_list(mk.static_list, mk.n_static);
                mask_list(mk.dyn_list + (size_t)m * mk.dyn_stride, mk.dyn_count[m]);
            }
            __syncwarp();
        }
        if (a.masked_out)
            for (int i = lane; i < n; i += 32) a.masked_out[(size_t)m * a.V + lo + i] = row[i];
        const int K = a.topk;
        float *pp = a.part + ((size_t)m * P + slot) * kPartStride;
        if (n <= 32 * RR) {
            // the row in registers (lane + 32 j: ids ascending in j), then every reduction there
            float v[RR];
#pragma unroll
            for (int j = 0; j < RR; ++j) v[j] = lane + 32 * j < n ? row[lane + 32 * j] : -INFINITY;
            float bv = -INFINITY;
            int bj = -1;
#pragma unroll
            for (int j = 0; j < RR; ++j)
                if (v[j] > bv) {  // strict: the first index of the lane's maximum
                    bv = v[j];
                    bj = j;
                }
            float wv = bv;
            int wi = bj < 0 ? INT_MAX : lo + lane + 32 * bj;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, wv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, wi, o);
                if (logit_better(ov, oi, wv, wi)) {
                    wv = ov;
                    wi = oi;
                }
            }
            float sm = 0.f;
            if (wv != -INFINITY)
#pragma unroll
                for (int j = 0; j < RR; ++j) sm += __expf(v[j] - wv);  // exp(-inf) = 0
            sm = warp_sum(sm);
            if (lane == 0) {
                pp[0] = wv;
                pp[1] = sm;
                pp[2] = __int_as_float(wi == INT_MAX ? lo : wi);
            }
            // top-k of the block (value desc, index asc): k rounds of lane-best then warp-best;
            // the winning lane drops its element.  Unfilled entries: (-inf, 0).
            for (int k = 0; k < K; ++k) {
                float cv = -INFINITY;
                int cj = -1;
#pragma unroll
                for (int j = 0; j < RR; ++j)
                    if (v[j] > cv) {
                        cv = v[j];
                        cj = j;
                    }
                const int ci = cj < 0 ? INT_MAX : lo + lane + 32 * cj;
                float hv = cv;
                int hi2 = ci;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, hv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, hi2, o);
                    if (logit_better(ov, oi, hv, hi2)) {
                        hv = ov;
                        hi2 = oi;
                    }
                }
                if (lane == 0) {
                    pp[4 + k] = hi2 == INT_MAX ? -INFINITY : hv;
                    pp[4 + K + k] = __int_as_float(hi2 == INT_MAX ? 0 : hi2);
                }
                if (hi2 != INT_MAX && ci == hi2)  // ids are unique: exactly one lane owns it
#pragma unroll
                    for (int j = 0; j < RR; ++j)
                        if (j == cj) v[j] = -INFINITY;
            }
            continue;
        }
        // rows longer than the register budget: the same reductions over shared memory
        float bv = -INFINITY;
        int bi = INT_MAX;
        for (int i = lane; i < n; i += 32)
            if (logit_better(row[i], lo + i, bv, bi)) {
                bv = row[i];
                bi = lo + i;
            }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (logit_better(ov, oi, bv, bi)) {
                bv = ov;
                bi = oi;
            }
        }
        float sm = 0.f;
        if (bv != -INFINITY)
            for (int i = lane; i < n; i += 32) sm += __expf(row[i] - bv);
        sm = warp_sum(sm);
        if (lane == 0) {
            pp[0] = bv;
            pp[1] = sm;
            pp[2] = __int_as_float(bi == INT_MAX ? lo : bi);
        }
        for (int k = 0; k < K; ++k) {
            float kv = -INFINITY;
            int ki = INT_MAX;
            for (int i = lane; i < n; i += 32)
                if (row[i] != -INFINITY && logit_better(row[i], lo + i, kv, ki)) {
                    kv = row[i];
                    ki = lo + i;
                }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, kv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, ki, o);
                if (logit_better(ov, oi, kv, ki)) {
                    kv = ov;
                    ki = oi;
                }
            }
            if (lane == 0) {
                pp[4 + k] = kv;
                pp[4 + K + k] = __int_as_float(ki == INT_MAX ? 0 : ki);
            }
            if (ki != INT_MAX && ki - lo >= 0 && ki - lo < n && lane == ((ki - lo) & 31)) row[ki - lo] = -INFINITY;
            __syncwarp();
        }
    }
}

// The same processors and record for one row of at most 128 ids, run by ONE thread over a
// column-major tile (tile[i * stride + mm] = the logit of id lo + i for row m = m0 + mm): the row's
// masks, then max and first argmax in one scan and the sum of exp in a second, in id order, with no
// warp reductions.  No top-k (greedy and sampling passes).  The records are part[m][P][..] at `slot`.
__device__ __forceinline__ void logits_row_thread(const LogitsArgs &a, float *tile, int stride, int mm, int m0, int lo,
                                                  int hi, const MaskStage *ms, int P, int slot) {
    const int m = m0 + mm, n = hi - lo;
    if (m >= a.M || (a.active && !ms->active[m])) return;
    float *col = tile + mm;  // id lo + i at col[i * stride]
    if (a.ns_token >= 0) {  // unmasked statistics (no-speech probability)
        float mx = -INFINITY;
        for (int i = 0; i < n; ++i) mx = fmaxf(mx, col[i * stride]);
        float sm = 0.f;
        if (mx != -INFINITY)
            for (int i = 0; i < n; ++i) sm += __expf(col[i * stride] - mx);
        float *np = a.ns_part + ((size_t)m * P + slot) * 2;
        np[0] = mx;
        np[1] = sm;
        if (a.ns_token >= lo && a.ns_token < hi) a.ns_value[m] = col[(a.ns_token - lo) * stride];
    }
    if (a.use_mask) {
        const MaskArgs &mk = a.mask;
        const int nrg = ms->n_ranges[m];
        for (int r = 0; r < nrg; ++r) {
            const int2 rg = ms->ranges[(size_t)m * kMaxRanges + r];
            for (int i = max(rg.x, lo); i < min(rg.y, hi); ++i) col[(i - lo) * stride] = -INFINITY;
        }
        auto mask_list = [&](const int *list, int n_list) {
            for (int j = 0; j < n_list; ++j) {
                const int t = list[j];
                if (t >= lo && t < hi) col[(t - lo) * stride] = -INFINITY;
            }
        };
        const int ns = min(mk.n_static, kStatStage);
        mask_list(ms->stat, ns);
        mask_list(mk.static_list + ns, mk.n_static - ns);
        const int nd = ms->dyn_count[m], nds = min(nd, kDynStage);
        mask_list(ms->dyn + (size_t)m * kDynStage, nds);
        mask_list(mk.dyn_list + (size_t)m * mk.dyn_stride + nds, nd - nds);
    }
    if (a.masked_out)
        for (int i = 0; i < n; ++i) a.masked_out[(size_t)m * a.V + lo + i] = col[i * stride];
    float bv = -INFINITY;
    int bi = -1;
    for (int i = 0; i < n; ++i) {
        const float v = col[i * stride];
        if (v > bv) {  // strict: the first index of the maximum
            bv = v;
            bi = i;
        }
    }
    float sm = 0.f;
    if (bv != -INFINITY)
        for (int i = 0; i < n; ++i) sm += __expf(col[i * stride] - bv);  // exp(-inf) = 0
    float *pp = a.part + ((size_t)m * P + slot) * kPartStride;
    pp[0] = bv;
    pp[1] = sm;
    pp[2] = __int_as_float(bi < 0 ? lo : lo + bi);
}

}  // namespace w4j
