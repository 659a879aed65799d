// k_step.cu — one decode step of a few sequences (batch 1 - 5, beams) as one persistent launch.
//
// The step of WhisperDecoder.forward for one token per sequence (nn/WhisperDecoder.java:66-104:
// embedding, ResidualAttentionBlock.java:42-60 per layer, final LayerNorm, tied-embedding logits)
// as 8 phases per layer plus the vocabulary phase, all in one kernel with one block per SM:
//
//   QKV (LayerNorm; layer 0: token + positional embedding) -> self-attention -> attn.out + residual
//   -> cross q (LayerNorm) -> cross-attention -> cross out + residual -> mlp.0 (LayerNorm, GELU table)
//   -> mlp.2 + residual -> ... -> vocabulary logits + logit processors + per-block partial records
//
// Phases are separated by grid-wide barriers (a counter in global memory, bounded waits).  What a
// block reads from HBM is known for the whole step before it starts: its row slice of every
// projection matrix, the encoder K / V keys of its cross-attention split and its slice of the
// token embedding.  A host-side plan lists those copies per block in consumption order with
// their places in a 128 KB byte ring of shared memory; one thread keeps the ring full (bulk
// copies for weights, tensor copies with the 128-byte swizzle for encoder K / V), so while a
// block waits at a barrier its next weights are already streaming in, and after the barrier only
// the activations (a few KB from L2) stand between it and its result.  Per phase a block:
//   * GEMV phases: stages the activation rows (LayerNorm applied) in shared memory as f32, then
//     for every piece of its row slice (f16 rows in the ring) one warp per row computes the dot
//     products of all sequences with lanes along K; epilogues as the chained kernels (q store,
//     K / V rows into the self cache, GELU table, residual add).
//   * self-attention: one (sequence, head) pair, keys gathered through the beam table into a
//     swizzled tile, online softmax on warp-level tensor cores (tile_warp).
//   * cross-attention: one (stream, head, key split), its keys already in the ring; the block that
//     finishes a pair's last split combines the splits' partial results (counter per pair).
//   * vocabulary: logits of its embedding rows into a shared tile, then the shared row epilogue.
// Token selection (k_select_*) runs as the next kernel of the step graph and resets the barrier
// counter.  Every wait is bounded and reports through the device error word.
#include <algorithm>
#include <string>
#include <vector>

#include "attn_tile.cuh"
#include "k_step.cuh"
#include "logits_epilogue.cuh"
#include "tc_common.cuh"
#include "w4j_internal.cuh"

namespace w4j {

static_assert(kRowPadPw == kPwPad, "the step kernel passes its P^T blocks to tile_warp");

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(unsigned *p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Shared state of one block.
struct StepSmem {
    unsigned char *ring;
    float *act;        // [kStepMaxM][kStepSeg] f32 staged activations (attention phases: warp sums)
    __half *kt, *vt;   // self-attention key / value tile (swizzled [128][64])
    float *tile;       // vocabulary phase: [M][ch] logits (aliases kt / vt)
    uint64_t *bars;
    __half (*qh)[kHeadDim + 8];
    __half (*pw)[8][kRowPadPw];
    float (*wm)[8], (*wl)[8];
    float *acc;        // GEMV partial sums across activation segments [rows][kStepMaxM]
    int *flags;        // [0] issued, [1] released, [2] dead (a wait ran out), [3] last split, [4] landed,
                       // [5] bytes in flight, [8 + i % 16] bytes of chunk i
    float *xs;         // [64 rows][8] the block's rows b d / G .. of the residual stream x, every sequence
    int *sq;           // per sequence m: [m] token, [8 + m] position, [16 + m] cache slot, [24 + m] live;
                       // per stream s: [32 + s] cross-cache slot
    int *nph;          // the next phase's descriptor (StepPhase words)
    const StepChunk *ch;  // the block's copies
};
constexpr int kPhaseWords = (int)(sizeof(StepPhase) / 4);
static_assert(sizeof(StepPhase) % 4 == 0 && kPhaseWords <= kStepThreads, "phase descriptor words");

// Block-uniform wait for chunk i.  After any wait ran out the block is dead: it waits for nothing
// more and issues no copies (it still takes part in the grid barriers).
// One thread waits, serving the ring meanwhile (a block of threads polling the mbarrier slows the
// copies that complete it); the others meet it at the block barrier.
__device__ void step_service(const StepArgs &a, const StepSmem &sm, const CUtensorMap *kmap, const CUtensorMap *vmap);
__device__ __forceinline__ bool step_wait_chunk(const StepArgs &a, const StepSmem &sm, int i, const CUtensorMap *kmap,
                                                const CUtensorMap *vmap) {
    bool r = true;
    if (threadIdx.x == 0) {
        r = false;
        step_service(a, sm, kmap, vmap);  // refill the ring (released space) before anything else
        for (long long it = 0; !sm.flags[2] && it < (1ll << 22); ++it) {
            if (mbar_test(sm.bars + (i % kStepBars), (unsigned)((i / kStepBars) & 1))) {
                r = true;
                break;
            }
            step_service(a, sm, kmap, vmap);  // chunk i itself may still wait for the in-flight cap
            if (it > 32) __nanosleep(64);
        }
        if (!r && !sm.flags[2]) atomicExch(a.err, 2);
    }
    const bool all = __syncthreads_and(r);
    if (!all && threadIdx.x == 0) sm.flags[2] = 1;
    return all;
}

// Ring service (one thread): first count the copies that have landed, then issue every chunk whose
// ring space and mbarrier are free while fewer than a.inflight bytes are in flight.  It runs inside
// the block's waits (for a chunk, at a grid barrier) and after every release, so copies keep
// flowing while the block waits; the cap keeps the memory queues short, since a deep queue of
// weight copies would delay every other access on the step's critical path (activations, the
// barrier's atomics) by as long as the queue takes to drain.
// flags: [0] issued, [1] released, [2] dead, [4] landed, [5] bytes in flight, [8 + i % 16] bytes of chunk i
__device__ void step_service(const StepArgs &a, const StepSmem &sm, const CUtensorMap *kmap, const CUtensorMap *vmap) {
    if (sm.flags[2]) return;
    const int n = a.n_chunks[blockIdx.x];
    const StepChunk *ch = sm.ch;
    int i = sm.flags[0], landed = sm.flags[4], infl = sm.flags[5];
    while (landed < i && mbar_test(sm.bars + (landed % kStepBars), (unsigned)((landed / kStepBars) & 1))) {
        infl -= sm.flags[8 + landed % kStepBars];
        ++landed;
    }
    const int rel = sm.flags[1];
    const uint64_t pol = l2_evict_first();
    while (i < n) {
        const StepChunk c = ch[i];
        if (c.wait_rel > rel || (infl > 0 && infl + (int)c.bytes > (int)a.inflight)) break;
        uint64_t *bar = sm.bars + (i % kStepBars);
        mbar_expect_tx(bar, c.bytes);
        unsigned char *dst = sm.ring + c.off;
        if (c.kind == 0) {  // weight rows: contiguous in the row-major matrix, one bulk copy
            bulk_g2s_hint(dst, reinterpret_cast<const void *>(c.src), c.bytes, bar, pol);
        } else {
            const int y = sm.sq[32 + c.s] * a.L * a.H * a.A + (int)c.src;
            for (int t = 0; t < c.nbox; ++t) {
                tma_load_2d_hint(dst + (size_t)t * kBox, kmap, 0, y + t * kAttnKeyTile, bar, pol);
                tma_load_2d_hint(dst + (size_t)(c.nbox + t) * kBox, vmap, 0, y + t * kAttnKeyTile, bar, pol);
            }
        }
        sm.flags[8 + i % kStepBars] = (int)c.bytes;
        infl += (int)c.bytes;
        ++i;
    }
    sm.flags[0] = i;
    sm.flags[4] = landed;
    sm.flags[5] = infl;
}

// Grid-wide barrier number `k` of the step (bounded; after a time-out the block stops waiting).
// Every block adds one to the counter; the block that completes barrier k writes k into every
// block's own flag (each on its own 128-byte line), and a block waits on its flag only: no
// address is polled by all SMs at once, which would hold up one L2 slice and with it every copy.
__device__ void step_barrier(const StepArgs &a, const StepSmem &sm, unsigned k, const CUtensorMap *kmap,
                             const CUtensorMap *vmap) {
    __syncthreads();
    if (threadIdx.x == 0 && a.bar_mode == 1) {
        // every block polls the counter itself (no release stores; one more reader per address)
        red_release_add(a.gbar, 1u);  // the block's writes (ordered by the block barrier) before its arrival
        const unsigned target = k * gridDim.x;
        long long it = 0;
        while (!sm.flags[2] && ld_acquire_u32(a.gbar) < target) {
            if (++it > (1ll << 22)) {
                atomicExch(a.err, 3);
                sm.flags[2] = 1;
                break;
            }
            step_service(a, sm, kmap, vmap);
            if (it > 4) __nanosleep(64);
        }
    } else if (threadIdx.x == 0) {
        __threadfence();
        const unsigned old = atomicAdd(a.gbar, 1u);
        if (old == k * gridDim.x - 1) {  // the last to arrive releases everyone: one fence, then plain stores
            __threadfence();
            for (unsigned j = 0; j < gridDim.x; ++j)
                asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(a.gflag + 32 * j), "r"(k) : "memory");
        } else if (!sm.flags[2]) {
            const unsigned *mine = a.gflag + 32 * blockIdx.x;
            long long it = 0;
            while (ld_acquire_u32(mine) < k) {
                if (++it > (1ll << 22)) {
                    atomicExch(a.err, 3);
                    sm.flags[2] = 1;
                    break;
                }
                step_service(a, sm, kmap, vmap);
                if (it > 8) __nanosleep(32);
            }
        }
    }
    __syncthreads();
}

// Release chunk i (every thread is done with it).  The ring is refilled by the next wait (for a
// chunk or at a grid barrier), off the phase's critical path.
__device__ void step_release(const StepSmem &sm, int i) {
    fence_proxy_async();  // generic accesses to the ring precede the copies that reuse it
    __syncthreads();
    if (threadIdx.x == 0) sm.flags[1] = i + 1;
}

// Stage the activation rows of a phase (columns [k0, k0 + kn)) into sm.act, rows `ast` floats apart,
// LayerNorm applied for the LN input modes (Tensor.java:592-619: two-pass mean / variance, eps 1e-5).  Every thread first
// issues all its global loads (16-byte vectors) and only then stores, so a stage costs about one
// L2 round trip; LayerNorm then runs from shared memory, gamma / beta staged beside it (sm.kt).
__device__ void step_stage(const StepArgs &a, const StepSmem &sm, const StepPhase &ph, int k0, int kn, int ast) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, K = ph.K;
    const int q4 = kn / 4, total = a.M * q4;  // float4 of the activation rows
    constexpr int U = 4;                      // loads in flight per thread and batch
    if (ph.in_mode == SI_ACT) {
        for (int i0 = tid; i0 < total; i0 += kStepThreads * U) {
            float4 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = i0 + u * kStepThreads;
                if (i < total) v[u] = __ldcg(reinterpret_cast<const float4 *>(ph.act + (size_t)(i / q4) * K + k0) + i % q4);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int i = i0 + u * kStepThreads;
                if (i < total) *reinterpret_cast<float4 *>(sm.act + (size_t)(i / q4) * ast + 4 * (i % q4)) = v[u];
            }
        }
        return;
    }
    // LayerNorm inputs (K = d <= 1280, one segment): rows into shared memory; gamma / beta are on
    // their way there since before the phase's barrier (step_ln_prefetch)
    float *lnp = reinterpret_cast<float *>(sm.kt);  // [gamma | beta], 2 K floats
    for (int i0 = tid; i0 < total; i0 += kStepThreads * U) {
        float4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = i0 + u * kStepThreads;
            if (i < total) {
                const int m = i / q4, c = i % q4;
                if (ph.in_mode == SI_LN) {
                    v[u] = __ldcg(reinterpret_cast<const float4 *>(ph.act + (size_t)m * K) + c);
                } else {  // x = E[tok] + P[pos] (WhisperDecoder.java:66-80); the offset clamped as at :72
                    const int p = sm.sq[8 + m], pe = p > a.C - 1 ? a.C - 1 : p;
                    const uint2 e = __ldg(reinterpret_cast<const uint2 *>(a.E + (size_t)sm.sq[m] * K) + c);
                    const float4 pp = __ldg(reinterpret_cast<const float4 *>(a.pos_emb + (size_t)pe * K) + c);
                    const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&e.x));
                    const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&e.y));
                    v[u] = make_float4(lo.x + pp.x, lo.y + pp.y, hi.x + pp.z, hi.y + pp.w);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = i0 + u * kStepThreads;
            if (i < total) {
                const int m = i / q4, c = i % q4;
                *reinterpret_cast<float4 *>(sm.act + (size_t)m * ast + 4 * c) = v[u];
                // block 0 keeps the embedded rows as the residual stream
                if (ph.in_mode == SI_EMBED_LN && blockIdx.x == 0) __stcg(reinterpret_cast<float4 *>(a.x + (size_t)m * K) + c, v[u]);
            }
        }
    }
    cp_async_wait_all();
    __syncthreads();
    if (ph.in_mode == SI_EMBED_LN) {  // the block's rows of the residual stream start as the embedding
        const int x0 = (int)((long long)blockIdx.x * K / gridDim.x), x1 = (int)((long long)(blockIdx.x + 1) * K / gridDim.x);
        for (int i = tid; i < (x1 - x0) * a.M; i += kStepThreads)
            sm.xs[(i / a.M) * kStepMaxM + i % a.M] = sm.act[(size_t)(i % a.M) * ast + x0 + i / a.M];
    }
    // Every row in eight fixed column parts (part w: columns 32 w + lane + 256 i), part w summed by
    // warp w and the parts added in order: the same sums for any number of sequences.
    float *r1 = lnp + 2 * K, *r2 = r1 + kStepMaxM * kStepWarps;  // [M][8] partial sums
    for (int m = 0; m < a.M; ++m) {
        const float *row = sm.act + (size_t)m * ast;
        float s0 = 0.f;
        for (int k = warp * 32 + lane; k < K; k += kStepThreads) s0 += row[k];
        s0 = warp_sum(s0);
        if (lane == 0) r1[m * kStepWarps + warp] = s0;
    }
    __syncthreads();
    for (int m = 0; m < a.M; ++m) {
        const float *row = sm.act + (size_t)m * ast;
        float mean = 0.f;
        for (int j = 0; j < kStepWarps; ++j) mean += r1[m * kStepWarps + j];
        mean /= (float)K;
        float s2 = 0.f;
        for (int k = warp * 32 + lane; k < K; k += kStepThreads) {
            const float t = row[k] - mean;
            s2 += t * t;
        }
        s2 = warp_sum(s2);
        if (lane == 0) r2[m * kStepWarps + warp] = s2;
    }
    __syncthreads();
    for (int m = 0; m < a.M; ++m) {
        float *row = sm.act + (size_t)m * ast;
        float mean = 0.f, var = 0.f;
        for (int j = 0; j < kStepWarps; ++j) mean += r1[m * kStepWarps + j];
        for (int j = 0; j < kStepWarps; ++j) var += r2[m * kStepWarps + j];
        mean /= (float)K;
        const float inv_std = 1.0f / sqrtf(var / (float)K + 1e-5f);
        for (int k = tid; k < K; k += kStepThreads) row[k] = (row[k] - mean) * inv_std * lnp[k] + lnp[K + k];
    }
}

// Element (row rr of a piece, column k) of a weight piece in the ring: rows of K halves.
__device__ __forceinline__ const __half *step_w(const __half *w, int K, int rr, int k) { return w + (size_t)rr * K + k; }

// Dot products of W rows [r0, r1) (a piece in the ring at `w`, rows of RK halves) with the staged
// activation columns [k0, k0 + kn) (rows `ast` floats apart): one warp per row, lanes along K; sums added into
// acc[(row - rbase) * 8 + m].
__device__ void step_dots(const StepArgs &a, const StepSmem &sm, const __half *w, int RK, int r0, int r1, int rbase,
                          int k0, int kn, int ast) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, M = a.M;
    for (int r = r0 + warp; r < r1; r += kStepWarps) {
        float acc[kStepMaxM];
#pragma unroll
        for (int m = 0; m < kStepMaxM; ++m) acc[m] = 0.f;
        for (int c = lane; c < kn / 8; c += 32) {
            const uint4 wv = *reinterpret_cast<const uint4 *>(step_w(w, RK, r - r0, k0 + 8 * c));
            const __half2 *h2 = reinterpret_cast<const __half2 *>(&wv);
            float wf[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f = __half22float2(h2[j]);
                wf[2 * j] = f.x;
                wf[2 * j + 1] = f.y;
            }
#pragma unroll
            for (int m = 0; m < kStepMaxM; ++m) {
                if (m >= M) break;
                const float4 x0 = *reinterpret_cast<const float4 *>(sm.act + (size_t)m * ast + 8 * c);
                const float4 x1 = *reinterpret_cast<const float4 *>(sm.act + (size_t)m * ast + 8 * c + 4);
                float t = acc[m];
                t = fmaf(wf[0], x0.x, t);
                t = fmaf(wf[1], x0.y, t);
                t = fmaf(wf[2], x0.z, t);
                t = fmaf(wf[3], x0.w, t);
                t = fmaf(wf[4], x1.x, t);
                t = fmaf(wf[5], x1.y, t);
                t = fmaf(wf[6], x1.z, t);
                t = fmaf(wf[7], x1.w, t);
                acc[m] = t;
            }
        }
#pragma unroll
        for (int m = 0; m < kStepMaxM; ++m) {
            if (m >= M) break;
            const float v = warp_sum(acc[m]);
            if (lane == 0) sm.acc[(r - rbase) * kStepMaxM + m] += v;
        }
    }
}

// gamma / beta of a LayerNorm phase into shared memory (sm.kt), issued before the phase's barrier
__device__ __forceinline__ void step_ln_prefetch(const StepSmem &sm, const StepPhase &ph) {
    if (ph.in_mode != SI_LN && ph.in_mode != SI_EMBED_LN) return;
    float *lnp = reinterpret_cast<float *>(sm.kt);
    const int q = ph.K / 4;
    for (int i = threadIdx.x; i < 2 * q; i += kStepThreads)
        cp_async16(lnp + 4 * i, reinterpret_cast<const float4 *>(i < q ? ph.ln_g : ph.ln_b) + i % q);
    cp_async_commit();
}

// Bias values of the epilogue pairs of thread t (pairs t and t + 256: row rbase + pair / M, sequence
// pair % M), loaded before the phase's grid barrier so that they arrive while the block waits.
constexpr int kEmitU = 2;  // <= 64 rows x 8 sequences / 256 threads
__device__ __forceinline__ void step_bias_prefetch(const StepPhase &ph, int M, int rbase, int rend, float (&bv)[kEmitU]) {
#pragma unroll
    for (int u = 0; u < kEmitU; ++u) {
        const int i = threadIdx.x + u * kStepThreads;
        bv[u] = ph.kind == SK_GEMV && ph.bias && i < (rend - rbase) * M ? __ldg(ph.bias + rbase + i / M) : 0.f;
    }
}

// Epilogues of the block's output rows [rbase, rend) for every live sequence.  The residual rows
// are the block's own (sm.xs: a residual phase's rows are b d / G .. like every other one's).
__device__ void step_emit_all(const StepArgs &a, const StepSmem &sm, const StepPhase &ph, int rbase, int rend,
                              const float (&bv)[kEmitU]) {
    const int M = a.M, np = (rend - rbase) * M;
#pragma unroll
    for (int u = 0; u < kEmitU; ++u) {
        const int i = threadIdx.x + u * kStepThreads;
        if (i >= np) continue;
        const int n = rbase + i / M, m = i % M;
        if (!sm.sq[24 + m]) continue;
        const float val = sm.acc[(n - rbase) * kStepMaxM + m] + bv[u];
        switch (ph.out_mode) {
            case SO_STORE:
                __stcg(ph.y + (size_t)m * ph.N + n, val);
                break;
            case SO_GELU:  // Tensor.geluInPlace: table lookup at the f16 rounding of x
                __stcg(ph.y + (size_t)m * ph.N + n, __ldg(a.gelu_lut + __half_as_ushort(__float2half_rn(val))));
                break;
            case SO_RESIDUAL: {
                float &xr = sm.xs[(n - rbase) * kStepMaxM + m];
                xr += val;
                __stcg(ph.y + (size_t)m * ph.N + n, xr);
                break;
            }
            default: {  // SO_QKV: q rows, then K / V rows into the self cache at this step's position
                const int d = a.d, part = n / d, c = n - part * d;
                if (part == 0) {
                    __stcg(ph.y + (size_t)m * d + c, val);
                } else {
                    const int head = c / kHeadDim, dd = c % kHeadDim;
                    const size_t row = (((size_t)sm.sq[16 + m] * a.L + ph.layer) * a.H + head) * (size_t)a.n_ctx + sm.sq[8 + m];
                    (part == 1 ? a.sk : a.sv)[row * kHeadDim + dd] = __float2half_rn(val);
                }
            }
        }
    }
}

// The eight warp states of one attention item, combined in warp order: unnormalised (max, sum,
// o[64]) per query into red (= sm.act) / wm / wl.
__device__ void step_attn_warp_state(const StepSmem &sm, const float (&m)[2], const float (&l)[2],
                                     const float (&of)[4][4], int nq) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
    float *red = sm.act;  // [8 warps][8 queries][64]
    if (g == 0) {
        sm.wm[warp][2 * tq] = m[0];
        sm.wm[warp][2 * tq + 1] = m[1];
        sm.wl[warp][2 * tq] = l[0];
        sm.wl[warp][2 * tq + 1] = l[1];
    }
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
        const int q0 = 2 * tq, q1 = 2 * tq + 1, d0 = 16 * mt + g;
        if (q0 < nq) {
            red[(warp * 8 + q0) * kHeadDim + d0] = of[mt][0];
            red[(warp * 8 + q0) * kHeadDim + d0 + 8] = of[mt][2];
        }
        if (q1 < nq) {
            red[(warp * 8 + q1) * kHeadDim + d0] = of[mt][1];
            red[(warp * 8 + q1) * kHeadDim + d0 + 8] = of[mt][3];
        }
    }
    __syncthreads();
}

// Query rows of a pair as f16 (rows >= nq zero).
__device__ void step_load_q(const StepSmem &sm, const float *q, int d, int head, int nq) {
    const int t = threadIdx.x;
    if (t < 8 * kHeadDim / 4) {
        const int qi = t / (kHeadDim / 4), c = t % (kHeadDim / 4);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (qi < nq) v = __ldcg(reinterpret_cast<const float4 *>(q + (size_t)qi * d + head * kHeadDim) + c);
        const __half2 h0 = __floats2half2_rn(v.x, v.y), h1 = __floats2half2_rn(v.z, v.w);
        *reinterpret_cast<uint2 *>(&sm.qh[qi][4 * c]) =
            make_uint2(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1));
    }
}

__global__ void __launch_bounds__(kStepThreads, 1)
    k_step(StepArgs a, const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    StepSmem sm;
    sm.ring = base;
    sm.kt = reinterpret_cast<__half *>(base + kStepRing);
    sm.vt = sm.kt + kAttnKeyTile * kHeadDim;
    sm.tile = reinterpret_cast<float *>(sm.kt);
    sm.act = reinterpret_cast<float *>(base + kStepRing + 2 * kBox);
    unsigned char *misc = base + kStepRing + 2 * kBox + kStepMaxM * kStepSeg * 4;
    sm.bars = reinterpret_cast<uint64_t *>(misc);
    sm.qh = reinterpret_cast<__half(*)[kHeadDim + 8]>(misc + kStepBars * 8);
    sm.pw = reinterpret_cast<__half(*)[8][kRowPadPw]>(misc + kStepBars * 8 + 8 * (kHeadDim + 8) * 2);
    float *fl = reinterpret_cast<float *>(misc + kStepBars * 8 + 8 * (kHeadDim + 8) * 2 + kStepWarps * 8 * kRowPadPw * 2);
    sm.wm = reinterpret_cast<float(*)[8]>(fl);
    sm.wl = reinterpret_cast<float(*)[8]>(fl + 64);
    sm.acc = fl + 128;                               // [64 rows][8]
    sm.xs = sm.acc + 64 * kStepMaxM;                 // [64 rows][8]
    sm.flags = reinterpret_cast<int *>(sm.xs + 64 * kStepMaxM);  // [32]
    sm.sq = sm.flags + 32;                           // [40]
    sm.nph = sm.sq + 40;                             // [kPhaseWords]
    StepChunk *chl = reinterpret_cast<StepChunk *>(sm.nph + ((kPhaseWords + 1) & ~1));
    sm.ch = chl;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.x;
    const StepPiece *pcs = a.pieces + (size_t)b * a.max_pieces;
    const int4 *pinfo = a.pinfo + (size_t)b * (a.n_phases + 1);

    // the block's copy list and the streams' cross-cache slots (fixed for the call): shared memory,
    // so that issuing a copy reads nothing from global memory
    {
        const unsigned long long *src = reinterpret_cast<const unsigned long long *>(a.chunks + (size_t)b * a.max_chunks);
        unsigned long long *dst = reinterpret_cast<unsigned long long *>(chl);
        for (int i = tid; i < a.n_chunks[b] * 3; i += kStepThreads) dst[i] = __ldg(src + i);
        if (tid < a.S) sm.sq[32 + tid] = a.cross_stream[tid];
        if (tid < kPhaseWords) sm.nph[tid] = __ldg(reinterpret_cast<const int *>(a.phases) + tid);
    }
    __syncthreads();
    if (tid == 0) {
        for (int i = 0; i < kStepBars; ++i) mbar_init(sm.bars + i, 1);
        fence_mbar_init();
        for (int i = 0; i < 32; ++i) sm.flags[i] = 0;
        // weights and encoder K / V do not depend on the previous kernel: start streaming now
        step_service(a, sm, &kmap, &vmap);
    }
    pdl_wait();  // tokens, positions, tables and liveness come from the previous step's selection
    if (tid < a.M) {
        sm.sq[tid] = a.tok[tid];
        sm.sq[8 + tid] = a.pos[tid];
        sm.sq[16 + tid] = a.slot[tid];
        sm.sq[24 + tid] = a.active ? a.active[tid] : 1;
    }
    __syncthreads();

    bool ok = true;
    int4 pi = pinfo[0], pn = pinfo[1];
    for (int p = 0; p < a.n_phases; ++p) {
        const StepPhase ph = *reinterpret_cast<const StepPhase *>(sm.nph);  // phase p (written before a block barrier)
        const int q0 = pi.x, q1 = pn.x, rbase = pi.y, rend = pi.z;
        float bv[kEmitU];
        step_bias_prefetch(ph, a.M, rbase, rend, bv);  // in flight across the barrier
        step_ln_prefetch(sm, ph);
        if (p > 0) step_barrier(a, sm, (unsigned)p, &kmap, &vmap);
        // the next phase's descriptor, in flight during this one
        int nph_word = 0;
        int4 pnn = make_int4(0, 0, 0, 0);
        if (p + 1 < a.n_phases) {
            if (tid < kPhaseWords) nph_word = __ldg(reinterpret_cast<const int *>(a.phases + p + 1) + tid);
            pnn = pinfo[p + 2];
        }
        if (ph.kind == SK_GEMV) {
            // the whole activation rows fit in sm.act for M K <= 8 x 1280 (mlp.2 of one or two
            // sequences too): one stage; otherwise segments of 1280 columns over resident pieces
            const int K = ph.K, nseg = a.M * K <= kStepMaxM * kStepSeg ? 1 : (K + kStepSeg - 1) / kStepSeg;
            for (int i = tid; i < (rend - rbase) * kStepMaxM; i += kStepThreads) sm.acc[i] = 0.f;
            if (nseg == 1) {
                step_stage(a, sm, ph, 0, K, K);
                __syncthreads();
                for (int qi = q0; qi < q1; ++qi) {
                    const StepPiece pc = pcs[qi];
                    ok = step_wait_chunk(a, sm, pc.chunk, &kmap, &vmap) && ok;
                    if (ok) step_dots(a, sm, reinterpret_cast<const __half *>(sm.ring + sm.ch[pc.chunk].off), K, pc.r0, pc.r1,
                                      rbase, 0, K, K);
                    step_release(sm, pc.chunk);
                }
            } else {
                // every piece of the phase is resident; activations by segment
                for (int qi = q0; qi < q1; ++qi) ok = step_wait_chunk(a, sm, pcs[qi].chunk, &kmap, &vmap) && ok;
                ok = ok && !sm.flags[2];
                for (int sg = 0; sg < nseg; ++sg) {
                    const int k0 = sg * kStepSeg, kn = min(kStepSeg, K - k0);
                    __syncthreads();  // the previous segment's dot products are done with sm.act
                    step_stage(a, sm, ph, k0, kn, kStepSeg);
                    __syncthreads();
                    for (int qi = q0; qi < q1 && ok; ++qi) {
                        const StepPiece pc = pcs[qi];
                        step_dots(a, sm, reinterpret_cast<const __half *>(sm.ring + sm.ch[pc.chunk].off), K, pc.r0, pc.r1,
                                  rbase, k0, kn, kStepSeg);
                    }
                }
                for (int qi = q0; qi < q1; ++qi) step_release(sm, pcs[qi].chunk);
            }
            __syncthreads();  // acc complete
            if (ok) step_emit_all(a, sm, ph, rbase, rend, bv);
        } else if (ph.kind == SK_SELF) {
            // one (sequence, head) pair: keys gathered through the beam table, tiles of 128
            for (int qi = q0; qi < q1; ++qi) {
                const int item = pcs[qi].r0, m = item / a.H, head = item - m * a.H;
                if (!sm.sq[24 + m]) continue;  // uniform over the block
                const int len = sm.sq[8 + m] + 1;
                step_load_q(sm, a.q + (size_t)m * a.d, a.d, head, 1);
                float mm[2] = {-INFINITY, -INFINITY}, ll[2] = {0.f, 0.f}, of[4][4];
#pragma unroll
                for (int i = 0; i < 4; ++i) of[i][0] = of[i][1] = of[i][2] = of[i][3] = 0.f;
                for (int t0 = 0; t0 < len; t0 += kAttnKeyTile) {
                    const int nk = min(kAttnKeyTile, len - t0);
                    __syncthreads();  // the previous tile is consumed
                    // 128 rows x 8 chunks of K and V: 4 per thread, every load issued before the stores
                    constexpr int G4 = kAttnKeyTile * 8 / kStepThreads;
                    uint4 kv[G4], vv[G4];
#pragma unroll
                    for (int u = 0; u < G4; ++u) {
                        const int c = tid + u * kStepThreads, r = c >> 3, ch = c & 7;
                        kv[u] = make_uint4(0u, 0u, 0u, 0u);
                        vv[u] = make_uint4(0u, 0u, 0u, 0u);
                        if (r < nk) {
                            const int p = t0 + r;
                            const int sl = a.table ? a.table[(size_t)m * a.n_ctx + p] : sm.sq[16 + m];
                            const size_t off = ((((size_t)sl * a.L + ph.layer) * a.H + head) * (size_t)a.n_ctx + p) * kHeadDim + ch * 8;
                            kv[u] = __ldcg(reinterpret_cast<const uint4 *>(a.sk + off));
                            vv[u] = __ldcg(reinterpret_cast<const uint4 *>(a.sv + off));
                        }
                    }
#pragma unroll
                    for (int u = 0; u < G4; ++u) {
                        const int c = tid + u * kStepThreads, r = c >> 3, ch = c & 7;
                        const int o = r * kHeadDim + ((ch ^ (r & 7)) << 3);
                        *reinterpret_cast<uint4 *>(sm.kt + o) = kv[u];
                        *reinterpret_cast<uint4 *>(sm.vt + o) = vv[u];
                    }
                    __syncthreads();
                    tile_warp<8>(sm.kt, sm.vt, nk, sm.qh, sm.pw[warp], mm, ll, of, warp, lane);
                }
                step_attn_warp_state(sm, mm, ll, of, 1);
                for (int dd = tid; dd < kHeadDim; dd += kStepThreads) {
                    float M = -INFINITY;
                    for (int w = 0; w < kStepWarps; ++w) M = fmaxf(M, sm.wm[w][0]);
                    float num = 0.f, den = 0.f;
                    for (int w = 0; w < kStepWarps; ++w)
                        if (sm.wm[w][0] != -INFINITY) {
                            const float wt = __expf(sm.wm[w][0] - M);
                            num = fmaf(wt, sm.act[(w * 8) * kHeadDim + dd], num);
                            den = fmaf(wt, sm.wl[w][0], den);
                        }
                    __stcg(a.attn_o + (size_t)m * a.d + head * kHeadDim + dd, num / den);
                }
                __syncthreads();
            }
        } else if (ph.kind == SK_CROSS) {
            // one (stream, head, split): its keys are in the ring (two swizzled boxes of 128 at most)
            for (int qi = q0; qi < q1; ++qi) {
                const StepPiece pc = pcs[qi];
                const int pair = pc.item / a.splits, s = pair / a.H, head = pair - s * a.H;
                const int B = a.B;
                ok = step_wait_chunk(a, sm, pc.chunk, &kmap, &vmap) && ok;
                const StepChunk cc = sm.ch[pc.chunk];
                step_load_q(sm, a.q + (size_t)s * B * a.d, a.d, head, B);
                __syncthreads();
                float mm[2] = {-INFINITY, -INFINITY}, ll[2] = {0.f, 0.f}, of[4][4];
#pragma unroll
                for (int i = 0; i < 4; ++i) of[i][0] = of[i][1] = of[i][2] = of[i][3] = 0.f;
                for (int t = 0; t < cc.nbox && ok; ++t) {
                    const int nk = min(kAttnKeyTile, pc.r1 - pc.r0 - t * kAttnKeyTile);
                    __half *tk = reinterpret_cast<__half *>(sm.ring + cc.off + (size_t)t * kBox);
                    __half *tv = reinterpret_cast<__half *>(sm.ring + cc.off + (size_t)(cc.nbox + t) * kBox);
                    const int kb = 16 * warp;  // V rows past the keys meet zero probabilities: keep them finite
                    if (nk < kAttnKeyTile && kb < nk && kb + 16 > nk) {
                        for (int c = lane; c < (kb + 16 - nk) * 8; c += 32)
                            *reinterpret_cast<uint4 *>(&tv[(nk + (c >> 3)) * kHeadDim + (c & 7) * 8]) =
                                make_uint4(0u, 0u, 0u, 0u);
                        __syncwarp();
                    }
                    tile_warp<8>(tk, tv, nk, sm.qh, sm.pw[warp], mm, ll, of, warp, lane);
                }
                step_attn_warp_state(sm, mm, ll, of, B);
                // this split's unnormalised (max, sum, o) per query
                float *xp = a.xpart + (size_t)pc.item * 8 * (kHeadDim + 2);
                for (int i = tid; i < B * kHeadDim; i += kStepThreads) {
                    const int qq = i / kHeadDim, dd = i % kHeadDim;
                    float M = -INFINITY;
                    for (int w = 0; w < kStepWarps; ++w) M = fmaxf(M, sm.wm[w][qq]);
                    float num = 0.f, den = 0.f;
                    for (int w = 0; w < kStepWarps; ++w)
                        if (sm.wm[w][qq] != -INFINITY) {
                            const float wt = __expf(sm.wm[w][qq] - M);
                            num = fmaf(wt, sm.act[(w * 8 + qq) * kHeadDim + dd], num);
                            den = fmaf(wt, sm.wl[w][qq], den);
                        }
                    __stcg(xp + qq * (kHeadDim + 2) + 2 + dd, num);
                    if (dd == 0) {
                        __stcg(xp + qq * (kHeadDim + 2), M);
                        __stcg(xp + qq * (kHeadDim + 2) + 1, den);
                    }
                }
                step_release(sm, pc.chunk);
                // the block finishing a pair's last split combines the splits in split order
                __threadfence();
                __syncthreads();
                if (tid == 0) {
                    const int old = atomicAdd(a.xcnt + pair, 1);
                    sm.flags[3] = old == a.splits - 1;
                    if (sm.flags[3]) {
                        __threadfence();
                        a.xcnt[pair] = 0;
                    }
                }
                __syncthreads();
                if (sm.flags[3]) {
                    const float *xb = a.xpart + (size_t)pair * a.splits * 8 * (kHeadDim + 2);
                    for (int i = tid; i < B * kHeadDim; i += kStepThreads) {
                        const int qq = i / kHeadDim, dd = i % kHeadDim;
                        float M = -INFINITY;
                        for (int j = 0; j < a.splits; ++j) M = fmaxf(M, __ldcg(xb + ((size_t)j * 8 + qq) * (kHeadDim + 2)));
                        float num = 0.f, den = 0.f;
                        for (int j = 0; j < a.splits; ++j) {
                            const float *e = xb + ((size_t)j * 8 + qq) * (kHeadDim + 2);
                            const float mj = __ldcg(e);
                            if (mj == -INFINITY) continue;
                            const float wt = __expf(mj - M);
                            num = fmaf(wt, __ldcg(e + 2 + dd), num);
                            den = fmaf(wt, __ldcg(e + 1), den);
                        }
                        __stcg(a.attn_o + (size_t)(s * B + qq) * a.d + head * kHeadDim + dd, num / den);
                    }
                }
                __syncthreads();
            }
        } else {
            // vocabulary: logits of this block's embedding rows for every sequence, then the row epilogue
            pdl_trigger();  // the selection kernel may start its prologue
            const int lo = rbase, hi = rend, chs = hi - lo;
            step_stage(a, sm, ph, 0, ph.K, kStepSeg);
            __syncthreads();
            for (int qi = q0; qi < q1; ++qi) {
                const StepPiece pc = pcs[qi];
                ok = step_wait_chunk(a, sm, pc.chunk, &kmap, &vmap) && ok;
                const __half *w = reinterpret_cast<const __half *>(sm.ring + sm.ch[pc.chunk].off);
                for (int r = pc.r0 + warp; r < pc.r1 && ok; r += kStepWarps) {
                    float acc[kStepMaxM];
#pragma unroll
                    for (int m = 0; m < kStepMaxM; ++m) acc[m] = 0.f;
                    for (int c = lane; c < ph.K / 8; c += 32) {
                        const uint4 wv = *reinterpret_cast<const uint4 *>(step_w(w, ph.K, r - pc.r0, 8 * c));
                        const __half2 *h2 = reinterpret_cast<const __half2 *>(&wv);
                        float wf[8];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float2 f = __half22float2(h2[j]);
                            wf[2 * j] = f.x;
                            wf[2 * j + 1] = f.y;
                        }
#pragma unroll
                        for (int m = 0; m < kStepMaxM; ++m) {
                            if (m >= a.M) break;
                            const float4 x0 = *reinterpret_cast<const float4 *>(sm.act + (size_t)m * kStepSeg + 8 * c);
                            const float4 x1 = *reinterpret_cast<const float4 *>(sm.act + (size_t)m * kStepSeg + 8 * c + 4);
                            float t = acc[m];
                            t = fmaf(wf[0], x0.x, t);
                            t = fmaf(wf[1], x0.y, t);
                            t = fmaf(wf[2], x0.z, t);
                            t = fmaf(wf[3], x0.w, t);
                            t = fmaf(wf[4], x1.x, t);
                            t = fmaf(wf[5], x1.y, t);
                            t = fmaf(wf[6], x1.z, t);
                            t = fmaf(wf[7], x1.w, t);
                            acc[m] = t;
                        }
                    }
#pragma unroll
                    for (int m = 0; m < kStepMaxM; ++m) {
                        if (m >= a.M) break;
                        const float v = warp_sum(acc[m]);
                        if (lane == 0) sm.tile[(size_t)m * chs + (r - lo)] = v;
                    }
                }
                step_release(sm, pc.chunk);
            }
            __syncthreads();
            LogitsArgs la = a.lg;
            logits_rows_epilogue(la, sm.tile, chs, a.M, 0, lo, hi, ok && !sm.flags[2], nullptr);
        }
        // phase p + 1's descriptor: read at the loop's top, after this block barrier
        if (tid < kPhaseWords) sm.nph[tid] = nph_word;
        pi = pn;
        pn = pnn;
        __syncthreads();
    }
    // after a wait that ran out: the copies in flight land before the block exits
    __syncthreads();
    if (tid == 0 && (!ok || sm.flags[2])) {
        const int n = sm.flags[0];
        for (int i = sm.flags[4]; i < n; ++i)
            for (long long it = 0; it < (1ll << 20) && !mbar_test(sm.bars + (i % kStepBars), (unsigned)((i / kStepBars) & 1)); ++it) {
            }
    }
}

// ---------------------------------------------------------------------------
// host side: the plan (per block: copies in consumption order with their ring places, and the
// pieces of work of every phase)
// ---------------------------------------------------------------------------
static unsigned round1k(unsigned x) { return (x + 1023u) & ~1023u; }

bool step_plan_build(const StepPlanIn &in, StepPlanOut &out, std::string &why) {
    const int G = in.G, P = (int)in.phases.size();
    if (in.M < 1 || in.M > kStepMaxM) return why = "sequences out of range", false;
    if (in.d % 64 != 0 || in.d > kStepSeg) return why = "width", false;
    const int pairs = in.S * in.H;
    // splits of every (stream, head) pair's keys: one per block, each of at least 16 keys
    out.splits = pairs > 0 ? std::min(G / pairs, std::max(1, in.A / 16)) : 0;
    if (out.splits < 1 || (in.A + out.splits - 1) / out.splits > 2 * kAttnKeyTile) return why = "too many streams", false;
    if ((size_t)in.M * ((in.V + G - 1) / G) * 4 > 2 * kBox) return why = "vocabulary tile", false;
    out.chunks.clear();
    out.pieces.clear();
    out.box_rows.assign(P, 0);
    // weight rows per piece: a GEMV block's rows in pieces of <= 48 KB; the vocabulary rows, a stream of
    // a few hundred rows per block, in pieces of one row per warp, so that several are in flight at once
    for (int p = 0; p < P; ++p) {
        const StepPhase &ph = in.phases[p];
        if (ph.kind != SK_GEMV && ph.kind != SK_LOGITS) continue;
        if (ph.K % 64 != 0) return why = "K", false;
        const int rpb = (ph.N + G - 1) / G;
        const int np = std::max(1, (int)(((size_t)rpb * ph.K * 2 + kStepPiece - 1) / kStepPiece));
        out.box_rows[p] = ph.kind == SK_LOGITS ? std::min(rpb, kStepWarps) : (rpb + np - 1) / np;
    }
    out.n_chunks.assign(G, 0);
    out.pinfo.assign((size_t)G * (P + 1), make_int4(0, 0, 0, 0));
    std::vector<std::vector<StepChunk>> ch(G);
    std::vector<std::vector<StepPiece>> pc(G);
    for (int b = 0; b < G; ++b) {
        auto &C = ch[b];
        auto &Q = pc[b];
        std::vector<int> all_resident;  // chunk ranges that must be resident together
        for (int p = 0; p < P; ++p) {
            const StepPhase &ph = in.phases[p];
            out.pinfo[(size_t)b * (P + 1) + p].x = (int)Q.size();
            if (ph.kind == SK_GEMV || ph.kind == SK_LOGITS) {
                const int N = ph.N, K = ph.K;
                const int r0 = (int)((long long)b * N / G), r1 = (int)((long long)(b + 1) * N / G);
                if (ph.kind == SK_GEMV && r1 - r0 > 64) return why = "rows per block", false;
                out.pinfo[(size_t)b * (P + 1) + p].y = r0;
                out.pinfo[(size_t)b * (P + 1) + p].z = r1;
                const int rpp = out.box_rows[p];
                const int first = (int)C.size();
                for (int r = r0; r < r1; r += rpp) {
                    const int re = std::min(r1, r + rpp);
                    StepChunk c{};
                    c.src = (unsigned long long)(uintptr_t)(in.W[p] + (size_t)r * K);
                    c.bytes = (unsigned)(re - r) * K * 2u;  // rows [r, re): contiguous, a multiple of 128 bytes
                    c.kind = 0;
                    Q.push_back(StepPiece{(int)C.size(), r, re, 0});
                    C.push_back(c);
                }
                if (in.M * K > kStepMaxM * kStepSeg && (int)C.size() > first) {  // consumed together (by segments)
                    all_resident.push_back(first);
                    all_resident.push_back((int)C.size());
                }
            } else if (ph.kind == SK_SELF) {
                for (int it = b; it < in.M * in.H; it += G) Q.push_back(StepPiece{-1, it, it + 1, 0});
            } else {  // SK_CROSS
                for (int it = b; it < pairs * out.splits; it += G) {
                    const int pair = it / out.splits, j = it % out.splits;
                    const int j0 = (int)((long long)j * in.A / out.splits), j1 = (int)((long long)(j + 1) * in.A / out.splits);
                    StepChunk c{};
                    c.kind = 1;
                    c.s = (unsigned char)(pair / in.H);
                    c.src = ((unsigned long long)ph.layer * in.H + pair % in.H) * in.A + j0;
                    c.nbox = (unsigned char)((j1 - j0 + kAttnKeyTile - 1) / kAttnKeyTile);
                    c.bytes = 2u * c.nbox * kBox;
                    Q.push_back(StepPiece{(int)C.size(), j0, j1, it});
                    C.push_back(c);
                }
            }
        }
        out.pinfo[(size_t)b * (P + 1) + P].x = (int)Q.size();
        // ring places (sequential, wrapping) and the releases each copy waits for
        unsigned pos = 0;
        for (size_t i = 0; i < C.size(); ++i) {
            const unsigned sz = round1k(C[i].bytes);
            if (sz > kStepRing) return why = "copy larger than the ring", false;
            if (pos + sz > kStepRing) pos = 0;
            C[i].off = pos;
            pos += sz;
        }
        for (size_t j = 0; j < C.size(); ++j) {
            int w = std::max(0, (int)j - kStepBars + 1);  // its mbarrier's previous use is consumed
            const unsigned a0 = C[j].off, a1 = a0 + round1k(C[j].bytes);
            for (size_t i = 0; i < j; ++i) {
                const unsigned b0 = C[i].off, b1 = b0 + round1k(C[i].bytes);
                if (a0 < b1 && b0 < a1) w = std::max(w, (int)i + 1);
            }
            C[j].wait_rel = w;
        }
        for (size_t k = 0; k < all_resident.size(); k += 2)
            for (int j = all_resident[k]; j < all_resident[k + 1]; ++j)
                if (C[j].wait_rel > all_resident[k] || all_resident[k + 1] - all_resident[k] > kStepBars)
                    return why = "a phase's pieces do not fit the ring together", false;
        out.n_chunks[b] = (int)C.size();
        out.max_chunks = std::max(out.max_chunks, (int)C.size());
        out.max_pieces = std::max(out.max_pieces, (int)Q.size());
    }
    out.max_chunks = std::max(out.max_chunks, 1);
    if (step_smem(out.max_chunks) > (size_t)kMaxDynSmem) return why = "copy list larger than shared memory", false;
    out.max_pieces = std::max(out.max_pieces, 1);
    out.chunks.assign((size_t)G * out.max_chunks, StepChunk{});
    out.pieces.assign((size_t)G * out.max_pieces, StepPiece{});
    for (int b = 0; b < G; ++b) {
        std::copy(ch[b].begin(), ch[b].end(), out.chunks.begin() + (size_t)b * out.max_chunks);
        std::copy(pc[b].begin(), pc[b].end(), out.pieces.begin() + (size_t)b * out.max_pieces);
    }
    return true;
}

size_t step_smem(int max_chunks) {
    const size_t misc = (size_t)kStepBars * 8 + 8 * (kHeadDim + 8) * 2 + (size_t)kStepWarps * 8 * kRowPadPw * 2 +
                        (128 + 2 * 64 * kStepMaxM + 32 + 40 + ((kPhaseWords + 1) & ~1)) * 4 +
                        (size_t)max_chunks * sizeof(StepChunk);
    return (size_t)kStepRing + 2 * kBox + (size_t)kStepMaxM * kStepSeg * 4 + misc + 1024;
}

cudaError_t step_prepare() { return allow_dynamic_smem(k_step); }

cudaError_t launch_step(const StepArgs &a, int G, const void *kmap, const void *vmap, bool coop, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(kStepThreads);
    cfg.dynamicSmemBytes = step_smem(a.max_chunks);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    // every block resident at once (grid barriers): the cooperative attribute guarantees it; without
    // it one block per SM (its shared memory) and G <= SMs make it so on a device this process owns,
    // and the barriers' bounded waits turn anything else into an error
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = coop ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_step, a, *reinterpret_cast<const CUtensorMap *>(kmap),
                              *reinterpret_cast<const CUtensorMap *>(vmap));
}

}  // namespace w4j
