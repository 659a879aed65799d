// w4j_internal.cuh — shared device structures and helpers of libwhisper4j_cuda.
//
// Device data layout (all in HBM of the context's GPU):
//   matrices      f16 [N][K] row-major (GGML native, the (out, in) layout of nn.Linear) or
//                 Q8_0 split into int8 quants [N][K] followed by f16 scales [N][K/32]
//   cross K / V   f16 [stream][layer][head][n_audio_ctx][64]   (head-major, one contiguous
//                 n_audio_ctx x 128 B run per head)
//   self  K / V   f16 [seq slot][layer][head][n_text_ctx][64]
//   activations   f32 [M][d] residual stream x, q, attention output, [M][4d] MLP hidden
#pragma once
#include <vector>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace w4j {

constexpr int kHeadDim = 64;
constexpr int kMaxTopK = 16;                        // beam + 1 <= 16
constexpr int kPartStride = 4 + 2 * kMaxTopK;       // floats per logits partial
constexpr int kMaxRanges = 4;                       // masked id ranges per sequence
constexpr int kGemvThreads = 256;
constexpr int kAttnThreads = 256;
constexpr int kAttnKeyTile = 128;

enum WType : int { WT_F16 = 1, WT_Q8 = 8 };

struct DMat {
    int type = 0;   // WT_F16 / WT_Q8
    int N = 0, K = 0;
    const __half *h = nullptr;   // WT_F16: [N][K]
    const int8_t *q = nullptr;   // WT_Q8: [N][K]
    const __half *s = nullptr;   // WT_Q8: [N][K/32]
    const __half *st = nullptr;  // WT_Q8 for the tensor-core projections: scales [N/128][K/64][128][2]
};

// ---------------------------------------------------------------------------
// GEMV over M <= a few dozen rows: y[m][n] = sum_k act[m][k] * W[n][k] (+ epilogue)
// ---------------------------------------------------------------------------
enum InMode : int { IN_ACT = 0, IN_LN = 1, IN_EMBED_LN = 2 };
enum OutMode : int { OUT_STORE = 0, OUT_GELU = 1, OUT_RESIDUAL = 2, OUT_QKV = 3 };

// Bytes a later kernel of the step will read, pulled into L2 while this one runs: a weight
// matrix and, for one stream, a layer's cross K / V (stream index read on the device; the host
// writes it before the step, no kernel of the step does).
struct L2Ahead {
    const unsigned char *w = nullptr;
    size_t w_bytes = 0;
    const unsigned char *k = nullptr, *v = nullptr;  // the layer's cross K / V of stream 0
    size_t kv_bytes = 0, kv_stride = 0;              // bytes of one stream's layer, stride between streams
    const int *stream = nullptr;                     // [1] the stream whose cross K / V are read
    int n_streams = 0;
};

struct GemvArgs {
    DMat W;
    L2Ahead pf;                        // prefetched into L2 before the wait on the previous kernel
    const float *bias = nullptr;       // [N] or null
    int M = 0;
    int in_mode = IN_ACT;
    const float *act = nullptr;        // [M][K] input (IN_ACT) or residual stream x (IN_LN)
    const float *ln_g = nullptr, *ln_b = nullptr;
    // IN_EMBED_LN: x[m] = E[tok[m]] + P[pos[m]] computed in the prologue; block 0 stores x
    DMat E;
    const float *pos_emb = nullptr;    // [n_text_ctx][d]
    const int *tok = nullptr;          // [M]
    const int *pos = nullptr;          // [M] self-cache row written by OUT_QKV (the sequence position)
    // positional-embedding row of each sequence: pe_pos[m] when given, else min(pos[m], pe_rows - 1)
    // (WhisperDecoder.java:72 clamps the offset so the table is never read past n_text_ctx - 1)
    const int *pe_pos = nullptr;       // [M] or null
    int pe_rows = 0;                   // rows of the positional table (n_text_ctx)
    float *x_out = nullptr;            // [M][d]
    // outputs
    int out_mode = OUT_STORE;
    float *y = nullptr;                // [M][N] (OUT_STORE/GELU/RESIDUAL) or q [M][d] (OUT_QKV)
    const float *gelu_lut = nullptr;   // 65536 f32 entries indexed by f16 bits
    // OUT_QKV: rows [d, 2d) -> K cache, [2d, 3d) -> V cache of layer `layer`
    __half *kcache = nullptr, *vcache = nullptr;
    const int *seq_slot = nullptr;     // [M] physical self-cache slot
    int layer = 0, n_layer = 0, n_head = 0, n_ctx = 0;
    const int *active = nullptr;       // [M] nonzero: row is live (null = all live)
    int *err = nullptr;                // device error word (bounded waits that ran out)
};

// ---------------------------------------------------------------------------
// single-query attention (self: rows gathered through the beam table; cross:
// contiguous per stream), split over keys with a deterministic combine
// ---------------------------------------------------------------------------
struct AttnArgs {
    const float *q = nullptr;          // [groups*nq][d] f32 queries
    int d = 0, n_head = 0, n_layer = 0, layer = 0;
    int cross = 0;                     // 0 self, 1 cross
    const __half *kc = nullptr, *vc = nullptr;
    int n_ctx = 0;                     // self rows per slot
    int n_audio = 0;                   // cross rows per stream
    const int *seq_slot = nullptr;     // self: [groups] own slot
    const int *table = nullptr;        // self: [groups][n_ctx] slot per position (null: own slot)
    const int *pos = nullptr;          // self: [groups] position of the newest row (kv len = pos+1)
    const int *kv_len = nullptr;       // self: [groups] keys to attend (overrides pos + 1) or null
    // self: [groups] (lo, hi): keys lo <= j < hi are masked (-inf), the reference's causal mask
    // applied from key column 0 on a multi-token pass (Tensor.java:622-640); null = no mask
    const int2 *mask = nullptr;
    const int *stream_of_group = nullptr;  // cross: [groups] stream index into the cross cache
    int self_prefetch = 0;             // self rows before the newest may be staged before the wait
    int nq = 1;                        // queries per group (cross: beams of one stream)
    int groups = 0;
    int nsplit = 1;
    float *out = nullptr;              // [groups*nq][d]
    const int *active = nullptr;       // [groups]
    int *err = nullptr;                // device error word
};

// ---------------------------------------------------------------------------
// vocabulary logits with the logit processors and per-block partial results
// ---------------------------------------------------------------------------
struct MaskArgs {
    const int *static_list = nullptr;  // suppress tokens, shared
    int n_static = 0;
    const int *dyn_list = nullptr;     // [M][dyn_stride] per-sequence masked ids
    const int *dyn_count = nullptr;    // [M]
    int dyn_stride = 0;
    const int2 *ranges = nullptr;      // [M][kMaxRanges] masked [lo, hi)
    const int *n_ranges = nullptr;     // [M]
};

struct LogitsArgs {
    DMat E;                            // [V][d]
    const float *x = nullptr;          // [M][d] residual stream
    const float *ln_g = nullptr, *ln_b = nullptr;
    int M = 0, V = 0, d = 0;
    MaskArgs mask;
    int use_mask = 0;
    int topk = 0;                      // candidates kept per block (beam + 1), 0 = greedy
    float *part = nullptr;             // [M][gridDim.x][kPartStride]
    float *raw_out = nullptr;          // [M][V] pre-mask logits (forward) or null
    float *masked_out = nullptr;       // [M][V] post-mask logits (sampling) or null
    int ns_token = -1;                 // >= 0: also reduce unmasked stats and keep this id's logit
    float *ns_part = nullptr;          // [M][gridDim.x][2] unmasked (max, sum)
    float *ns_value = nullptr;         // [M]
    const int *active = nullptr;       // [M]
    int *err = nullptr;                // device error word
    int withhold = 0;                  // test hook: issue no weight copies, so the bounded waits run out
};

// ---------------------------------------------------------------------------
// decode state (device) and per-step selection
// ---------------------------------------------------------------------------
struct DecodeState {
    int n_streams = 0, beam = 1, max_tokens = 0, n_prompt = 0, n_ctx = 0, V = 0, n_parts = 0;
    int eot = 0, ts_begin = -1, ns_token = -1, n_suppress = 0;
    float temperature = 0.f;
    unsigned long long seed = 0;
    int hs = 0;                        // stride of token histories (n_text_ctx + 1)
    // per sequence (M = n_streams * beam), double-buffered by step parity where noted
    int *tok_in = nullptr;             // [M] token fed at the next step
    int *seq_slot = nullptr;           // [M]
    int *seq_pos = nullptr;            // [M]
    int *active = nullptr;             // [M]
    int *table[2] = {nullptr, nullptr};    // [M][n_ctx]
    int *hist[2] = {nullptr, nullptr};     // [M][hs]
    int *hist_len[2] = {nullptr, nullptr}; // [M]
    double *lp[2] = {nullptr, nullptr};    // [M] beam score / greedy sum of log-probs
    int *dyn_list = nullptr;           // [M][dyn_stride]
    int *dyn_count = nullptr;          // [M]
    int dyn_stride = 0;
    int2 *ranges = nullptr;            // [M][kMaxRanges]
    int *n_ranges = nullptr;           // [M]
    const int *suppress = nullptr;     // [n_suppress]
    // per stream
    int *done = nullptr;               // [S]
    const int *stream_base = nullptr;  // [S] first physical self-cache slot of the stream
    int *beam_par = nullptr;           // [S] parity of the buffers holding the live beams
    float *nsp = nullptr;              // [S] no-speech probability
    int *fin_n = nullptr;              // [S]
    int *fin_tok = nullptr;            // [S][beam][hs]
    int *fin_len = nullptr;            // [S][beam]
    double *fin_lp = nullptr;          // [S][beam]
    // outputs (finalize)
    int *out_tok = nullptr;            // [S][max_tokens]
    int *out_len = nullptr;            // [S]
    double *out_sum = nullptr;         // [S]
    int *err = nullptr;                // device error word (bounds failures), 0 = ok
    unsigned *gbar = nullptr;          // grid barrier counter of the step kernel (reset by selection)
    unsigned *gflag = nullptr;         // its per-block flags, 32 words apart (reset by selection)
    int n_gflag = 0;
};

// ---------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }


// ---- TMA bulk copies into shared memory, completed through an mbarrier ----
__device__ __forceinline__ unsigned smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *b, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
// 1-D bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16)
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *b) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(b))
                 : "memory");
}
// 16-byte asynchronous copy global -> shared (completed by cp_async_wait_*)
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
// L2 policy for data read once per step (weights, encoder K / V): evicted before anything else, so
// the small per-step working set (activations, norms, biases, caches) stays resident in L2
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void bulk_g2s_hint(void *dst, const void *src, unsigned bytes, uint64_t *b, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(b)), "l"(pol)
        : "memory");
}
// Block b of nb pulls its share of [p, p + bytes) into L2 (whole 16-byte units, 64 KB requests).
__device__ __forceinline__ void l2_prefetch_share(const unsigned char *p, size_t bytes, int b, int nb) {
    const size_t units = bytes >> 4, per = (units + nb - 1) / nb;
    const size_t u0 = (size_t)b * per, u1 = u0 + per < units ? u0 + per : units;
    for (size_t u = u0; u < u1; u += 4096) {
        const unsigned sz = (unsigned)((u1 - u < 4096 ? u1 - u : 4096) << 4);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p + (u << 4)), "r"(sz) : "memory");
    }
}
__device__ __forceinline__ void l2_ahead(const L2Ahead &f, int b, int nb) {
    if (f.w) l2_prefetch_share(f.w, f.w_bytes, b, nb);
    if (f.k && f.stream) {
        const int s = *f.stream;
        if (s < 0 || s >= f.n_streams) return;
        const size_t o = (size_t)s * f.kv_stride;
        l2_prefetch_share(f.k + o, f.kv_bytes, b, nb);
        l2_prefetch_share(f.v + o, f.kv_bytes, b, nb);
    }
}
__device__ __forceinline__ bool mbar_test(uint64_t *b, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for phase `parity` of an mbarrier; on time-out raises the error word and
// returns false (callers skip their compute, then drain with a second bounded wait).
__device__ __forceinline__ bool mbar_wait(uint64_t *b, unsigned parity, int *err) {
    for (long long it = 0; it < (1ll << 22); ++it) {
        if (mbar_test(b, parity)) return true;
        if (it > 32) __nanosleep(128);
    }
    if (err) atomicExch(err, 2);
    return false;
}


// Positional-embedding row of sequence m of a projection with the embedding prologue.
__device__ __forceinline__ int pe_row(const GemvArgs &a, int m) {
    if (a.pe_pos) return a.pe_pos[m];
    const int p = a.pos[m];
    return a.pe_rows > 0 && p > a.pe_rows - 1 ? a.pe_rows - 1 : p;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Every kernel of the decode chain asks for the largest shared-memory carveout: an SM then
// never has to drain and reconfigure its L1/shared split between two kernels of the chain,
// so a dependent kernel's blocks can become resident (and prefetch) while its predecessor's
// blocks still run.
template <typename Kern>
inline cudaError_t prefer_max_smem(Kern kern) {
    return cudaFuncSetAttribute(reinterpret_cast<const void *>(kern), cudaFuncAttributePreferredSharedMemoryCarveout,
                                (int)cudaSharedmemCarveoutMaxShared);
}

// Let `kern` use all the opt-in shared memory the device offers beside its static arrays.
template <typename Kern>
inline cudaError_t allow_dynamic_smem(Kern kern) {
    int dev = 0, optin = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, reinterpret_cast<const void *>(kern));
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(reinterpret_cast<const void *>(kern), cudaFuncAttributeMaxDynamicSharedMemorySize,
                             optin - (int)fa.sharedSizeBytes);
    return e == cudaSuccess ? prefer_max_smem(kern) : e;
}

// ---------------------------------------------------------------------------
// host launchers (defined in the kernel .cu files)
// ---------------------------------------------------------------------------
cudaError_t launch_gemv(const GemvArgs &a, cudaStream_t s, bool pdl);
cudaError_t launch_attn(const AttnArgs &a, cudaStream_t s, bool pdl);
int attn_max_splits(int nq);  // key splits of one attention launch (one thread-block cluster)
bool attn_stream_pays(const AttnArgs &a, int sms);  // the streaming kernel beats the cluster one
// cross-attention over many (group, head) pairs: one persistent block per SM; kmap / vmap are
// make_tmap_f16_rows maps of the cross K / V caches as [rows][64]
cudaError_t launch_attn_stream(const AttnArgs &a, const void *kmap, const void *vmap, int sms, cudaStream_t s, bool pdl);
// self-attention of many sequences without beam tables, masks or explicit key counts: a persistent
// warpgroup per (sequence, head) pair; kmap / vmap are make_tmap_f16_rows maps of the self K / V caches
bool attn_self_stream_pays(const AttnArgs &a, int sms);
cudaError_t launch_attn_self_stream(const AttnArgs &a, const void *kmap, const void *vmap, int sms, cudaStream_t s,
                                    bool pdl);
// the same, one warp per pair in 32-key tiles (maps with 32-row boxes)
cudaError_t launch_attn_self_warps(const AttnArgs &a, const void *kmap32, const void *vmap32, int sms, cudaStream_t s,
                                   bool pdl);
// cross-attention of many (stream, head) pairs with a warpgroup per pair (maps: the cross caches)
bool attn_pairs_pays(const AttnArgs &a, int sms);
cudaError_t launch_attn_pairs(const AttnArgs &a, const void *kmap, const void *vmap, int sms, cudaStream_t s, bool pdl);
cudaError_t launch_logits(const LogitsArgs &a, int n_parts, cudaStream_t s, bool pdl);
int logits_parts_for(int V, int sm_count);
size_t logits_smem_bytes(int M, int V, int d, int n_parts);

// select / bookkeeping kernels
enum SelectMode : int { SEL_GREEDY = 0, SEL_SAMPLE = 1, SEL_BEAM_INIT = 2, SEL_BEAM = 3 };
cudaError_t launch_select(const DecodeState &st, int mode, int parity, const float *part, int n_parts,
                          float *masked_logits, int step, cudaStream_t s, bool pdl);
// dynamic shared memory a select launch of `mode` needs (history and beam-table staging)
size_t select_smem_bytes(const DecodeState &st, int mode, int P);
cudaError_t launch_nsp(const DecodeState &st, const float *ns_part, int n_parts, const float *ns_value,
                       cudaStream_t s, bool pdl);
cudaError_t launch_init_masks(const DecodeState &st, int beam_mode, cudaStream_t s);
cudaError_t launch_finalize(const DecodeState &st, int beam_mode, int parity, cudaStream_t s);
cudaError_t launch_argmax_merge(const float *part, int n_parts, int M, int32_t *tok, double *lp, cudaStream_t s);
// after a merge: outputs of all M rows become -1 / NaN if `err` is set, and `err` is cleared
cudaError_t launch_err_apply(int M, int32_t *tok, double *lp, int *err, cudaStream_t s);
// single-block merge that also reports and clears the device error word `err`
cudaError_t launch_argmax_merge_status(const float *part, int n_parts, int M, int32_t *tok, double *lp, int *err,
                                       cudaStream_t s);

// prefill: out_k/out_v (f16 head-major) = xa . Wk^T, xa . Wv^T + bv
cudaError_t launch_cross_kv(const float *xa, int A, int d, const DMat &wk, const DMat &wv, const float *bk,
                            const float *bv, __half *kout, __half *vout, int n_head, cudaStream_t s);

cudaError_t launch_q8_repack(const void *src, int N, int K, int8_t *q, __half *scales, cudaStream_t s);
cudaError_t gemv_prepare();
cudaError_t logits_tc_prepare();
// tcgen05 vocabulary logits (f16 embedding, M <= 32); cudaErrorNotSupported outside its range
cudaError_t launch_logits_tc(const LogitsArgs &a, const void *tmap, int n_parts, cudaStream_t s, bool pdl);
// one-launch tcgen05 vocabulary pass over 33 .. kLogitsBigMaxRows rows without the beam top-k, the
// rows read as f16 LayerNorm-ed activations staged by launch_act_hilo (bmap: their hi rows, K = d, boxes
// of the chunk's NU rows): records per row of that pass (0 when it does not take the shape)
constexpr int kLogitsBigMaxRows = 256;
int logits_big_parts(int M, int V, int d, int topk);
int logits_big_box_rows(int M);
cudaError_t launch_logits_big(const LogitsArgs &a, const void *tmap, const void *bmap, int blocks, cudaStream_t s, bool pdl);
bool make_tmap_f16_rows(void *map_out, const void *base, int rows, int cols);  // 128-byte map
bool make_tmap_i8_rows(void *map_out, const void *base, int rows, int cols);   // [128 x 64] int8 boxes
// Q8_0 scales [N][K/32] -> the tile layout [N/128][K/64][128][2] of the tensor-core projections
cudaError_t launch_q8_tile_scales(const __half *s, int N, int K, __half *st, cudaStream_t stream);
cudaError_t gemm_tc_prepare();
cudaError_t xkv_tc_prepare();
// tcgen05 cross K/V projection of one stream and layer (f16 Wk / Wv, d a multiple of 128); kmap /
// vmap are make_tmap_f16_rows maps of Wk and Wv; cudaErrorNotSupported outside its range
cudaError_t launch_cross_kv_tc(const float *xa, int A, int d, const void *kmap, const void *vmap, const float *bk,
                               const float *bv, __half *kout, __half *vout, int *err, cudaStream_t s);
// tcgen05 projection (M >= 16; f16 weights, or Q8_0 with tiled scales and N a multiple of 128) with
// the GEMV's input modes and epilogues; `tmap` is make_tmap_f16_rows of a.W.h (f16) or
// make_tmap_i8_rows of a.W.q (Q8_0); cudaErrorNotSupported outside its range
// More than 128 rows (f16): `bmap` is make_tmap_f16_rows(…, rows 256) of the activations staged by
// launch_act_hilo beforehand ([act_hilo_rows(M)][K] f16), read as [act_hilo_box_rows(M) x 64] boxes.
cudaError_t launch_gemm_tc(const GemvArgs &a, const void *tmap, const void *bmap, int sms, cudaStream_t s, bool pdl);
bool gemm_tc_staged(const GemvArgs &a);  // the projection reads staged activations (launch_act_hilo first)
bool gemm_tc_supported(const GemvArgs &a, int sms);  // the tensor-core kernel takes this projection
int act_hilo_rows(int M);
int act_hilo_box_rows(int M);  // rows of one staged B tile (the tensor map box height)
cudaError_t launch_act_hilo(const GemvArgs &a, __half *out, cudaStream_t s, bool pdl);

// audio encoder (k_encoder.cu)
cudaError_t launch_enc_im2col(const float *src, int in_ch, int in_len, bool time_major, int stride, int out_len, int kp,
                              float *out, cudaStream_t s);
cudaError_t launch_enc_add(float *x, const float *p, long long n, cudaStream_t s);
cudaError_t launch_enc_ln(const float *x, int rows, int n, const float *g, const float *b, float *y, cudaStream_t s);
cudaError_t launch_enc_qkv_f16(const float *qkv, int T, int H, __half *out, cudaStream_t s);
cudaError_t launch_enc_attn(const __half *qkvh, int T, int H, float *out, cudaStream_t s);
// log-mel front end (k_logmel.cu)
void logmel_tables(int n_fft, std::vector<float> &tabs);
int logmel_frames(int n_samples, int n_fft, int hop);
cudaError_t launch_logmel(const float *audio, int n_valid, int n_total, int n, int hop, const float *tabs,
                          const float *filt, int n_mels, int n_bins, int out_frames, float *spec, float *fmx, float *fmn,
                          float *out, cudaStream_t s);// tensor map of a row-major f16 matrix read in [box_rows x 64 cols] boxes, 128-byte swizzle
bool make_tmap_f16_box(void *map_out, const void *base, int rows, int cols, int box_rows);
cudaError_t select_prepare();
cudaError_t attn_prepare();
cudaError_t launch_f32_to_f16(const float *src, __half *dst, size_t n, cudaStream_t s);

}  // namespace w4j
