// runtime.cu — host runtime and C ABI of libwhisper4j_cuda.so.
//
// The decoder context replaces the reference's WhisperDecoder object
// (nn/WhisperDecoder.java:36-56) and its per-call kvCache maps: weights live on one GPU in
// their GGML storage type, the KV caches are preallocated device arrays, and a decode call
// runs the whole token loop on the device.  The prompt steps are launched directly; every
// later step is one CUDA-graph replay (kernels chained with programmatic dependent launch),
// and only token ids, log-prob sums and the no-speech probability come back to the host.
#include <zlib.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "../../include/whisper4j_cuda.h"
#include "k_step.cuh"
#include "w4j_internal.cuh"

using namespace w4j;

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------
static thread_local std::string g_err;

static int set_err(int code, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

// A failed call leaves its error as the thread's last CUDA error (cudaGetLastError); it is consumed
// here, so a later launch check does not report an earlier, already handled failure (a refused
// allocation, for instance).
#define CUDA_TRY(expr)                                                                             \
    do {                                                                                           \
        cudaError_t e_ = (expr);                                                                   \
        if (e_ != cudaSuccess) {                                                                   \
            cudaGetLastError();                                                                    \
            return set_err(e_ == cudaErrorMemoryAllocation ? W4J_ERR_OOM : W4J_ERR_CUDA, "%s: %s (%s:%d)", \
                           #expr, cudaGetErrorString(e_), __FILE__, __LINE__);                     \
        }                                                                                          \
    } while (0)

#define TRY(expr)            \
    do {                     \
        int r_ = (expr);     \
        if (r_ < 0) return r_; \
    } while (0)

// ---------------------------------------------------------------------------
// context
// ---------------------------------------------------------------------------
struct LayerDev {
    DMat qkv, o, xq, xk, xv, xo, m0, m2;
    float *bqkv = nullptr, *bo = nullptr, *bxq = nullptr, *bxk = nullptr, *bxv = nullptr, *bxo = nullptr;
    float *bm0 = nullptr, *bm2 = nullptr;
    float *ln1g = nullptr, *ln1b = nullptr, *ln2g = nullptr, *ln2b = nullptr, *ln3g = nullptr, *ln3b = nullptr;
    int qkv_type = 0;
    // TMA maps of the f16 projections for the tensor-core kernels (M >= 16; cross K / V prefill), by PROJ_*
    alignas(64) unsigned char tmap[8][128] = {};
    bool tmap_ok[8] = {};
};
enum Proj : int { PROJ_QKV = 0, PROJ_O = 1, PROJ_XQ = 2, PROJ_XO = 3, PROJ_M0 = 4, PROJ_M2 = 5, PROJ_XK = 6, PROJ_XV = 7 };

// The audio encoder on the same device as the decoder (WhisperEncoder.java:27-39): its weights come
// through w4j_upload_tensor ("encoder.*", raw GGML payloads like the decoder's), its work buffers
// are allocated at the first w4j_encoder_forward.
struct EncLayer {
    DMat qkv, o, m0, m2;  // q, k, v fused into [3 d][d] (the key has no bias: zeros)
    float *bqkv = nullptr, *bo = nullptr, *bm0 = nullptr, *bm2 = nullptr;
    float *ln1g = nullptr, *ln1b = nullptr, *ln2g = nullptr, *ln2b = nullptr;
    alignas(64) unsigned char tmap[4][128] = {};  // qkv, o, m0, m2
};
struct EncDev {
    DMat c1, c2;  // conv weights as [d][in * 3] f16 (Conv1d's weightMatrix); conv1's columns padded to k1
    float *b1 = nullptr, *b2 = nullptr, *pos = nullptr, *lng = nullptr, *lnb = nullptr;
    std::vector<EncLayer> layers;
    alignas(64) unsigned char c1map[128] = {}, c2map[128] = {};
    int k1 = 0;
    bool maps_ok = false, q8_skipped = false;
    std::set<std::string> uploaded;
    float *mel = nullptr, *col = nullptr, *y1 = nullptr, *x = nullptr, *qkv = nullptr, *att = nullptr, *hid = nullptr,
          *xa = nullptr;
    __half *qkvh = nullptr, *hilo = nullptr;
    // log-mel front end: the model's filters, the transform tables, the audio and its spectrogram
    float *filt = nullptr, *tabs = nullptr, *audio = nullptr, *spec = nullptr, *fmx = nullptr, *fmn = nullptr;
    int filt_bins = 0;
    size_t audio_cap = 0, frames_cap = 0;
};

struct GraphKey {
    int mode, S, B, eot, ts_begin, n_sup, max_tokens, ns, n_prompt, time_class;
    float temperature;
    unsigned long long seed;
    bool operator<(const GraphKey &o) const { return memcmp(this, &o, sizeof *this) < 0; }
};

struct w4j_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::mutex mu;
    int V = 0, C = 0, A = 0, d = 0, H = 0, L = 0;
    w4j_dims dims{};
    EncDev enc;
    int max_streams = 0, max_beam = 0, n_slots = 0, M_max = 0;
    int cap = 0;   // self-cache rows per slot: n_text_ctx, grown on demand (the reference's cache is unbounded)
    int Mbuf = 0;  // activation rows: max(M_max, n_text_ctx) (a multi-token forward is one pass of its tokens)
    int sm_count = 148;
    std::vector<LayerDev> layers;
    DMat E;
    float *pos_emb = nullptr, *lng = nullptr, *lnb = nullptr, *gelu_lut = nullptr;
    std::set<std::string> uploaded;
    std::vector<void *> allocs;
    // caches
    __half *ck = nullptr, *cv = nullptr, *sk = nullptr, *sv = nullptr;
    std::vector<int> cache_len;
    std::vector<char> has_xa;
    // activations / scratch
    float *x = nullptr, *q = nullptr, *attn = nullptr, *h = nullptr, *xa_stage = nullptr;
    int n_parts = 0;
    float *logit_part = nullptr, *ns_part = nullptr, *ns_value = nullptr;
    float *masked = nullptr;  // M_max x V (sampling)
    float *raw = nullptr;     // n_text_ctx x V (forward)
    int *op_err = nullptr;    // error word of the op-level vocabulary pass (w4j_op_logits_argmax)
    __half *op_st = nullptr;  // tiled Q8_0 scales of the op-level linear (w4j_op_linear)
    size_t op_st_n = 0;
    // activations of the staged projections (f16, 16 rows and more) as f16 hi / lo B-operand rows
    // ([act_hilo_rows(Mbuf)][K] for K = d and 4d); their tensor maps are made per launch
    __half *hilo = nullptr;
    bool hilo_ok = false;
    __half *op_hilo = nullptr;  // the same for w4j_op_linear, grown on demand
    size_t op_hilo_n = 0;
    // decode state
    DecodeState st;
    int *d_int_area = nullptr;     // per-call small int arrays (see layout in prepare_call)
    int *h_int_area = nullptr;     // pinned mirror
    size_t int_area_n = 0;
    int *d_done_snapshot = nullptr;
    int *h_done = nullptr;
    // graphs
    std::map<GraphKey, cudaGraphExec_t> graphs;
    std::map<GraphKey, long long> graph_launches;  // kernels in each cached step graph
    std::atomic<int> cancel{0};
    double last_ms = 0;
    int last_steps = 0;
    long long last_launches = 0;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    // host encoder outputs: two staging buffers, copied on their own stream, so that one stream's
    // upload overlaps the previous stream's cross K/V projection
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t xa_copied[2] = {nullptr, nullptr}, xa_used[2] = {nullptr, nullptr};
    float *xa_stage2 = nullptr;
    int xa_flip = 0;
    alignas(64) unsigned char e_tmap[128] = {};  // TMA map of the f16 token embedding
    alignas(64) unsigned char xk_tmap[128] = {}, xv_tmap[128] = {};  // cross K / V caches as [rows][64]
    alignas(64) unsigned char sk_tmap[128] = {}, sv_tmap[128] = {};  // self K / V caches as [rows][64]
    alignas(64) unsigned char sk_tmap32[128] = {}, sv_tmap32[128] = {};  // the same, 32-row boxes
    bool self_warps = true;  // W4J_SELF_PAIRS=1: many-sequence self-attention on k_attn_pairs instead
    bool big_logits = true;  // W4J_LOGITS_CHUNKED=1: 33 .. 256 rows in 32-row launches instead of one
    int l2_ahead = 0;        // W4J_L2_AHEAD=n: a GEMV projection pulls the weights n projections on into L2 (0: off)
    bool s_tmap_ok = false;
    bool x_tmap_ok = false;
    bool e_tmap_ok = false;
    bool tc_logits = true;
    bool tc_gemm = true;  // tcgen05 projections once M >= 16
    // the persistent step kernel (k_step) for up to 8 sequences: plans per (streams, beams)
    struct StepPlanDev {
        bool ok = false;
        StepArgs base;  // plan pointers and model fields; per-call fields are set at capture
    };
    bool use_step = false;  // W4J_STEP_KERNEL=1: one persistent kernel per step of <= 8 sequences
    bool step_coop = true;  // launch it with the cooperative attribute (dropped if capture refuses it)
    bool verbose = false;   // W4J_VERBOSE=1: say on stderr why a faster path was not taken
    unsigned step_inflight = 128u << 10;  // W4J_STEP_INFLIGHT_KB: copy bytes in flight per block of the step kernel
    int step_bar_mode = 0;               // W4J_STEP_BAR: the step kernel's grid barrier (0 flags, 1 counter)
    bool attn_pairs = true;  // W4J_NO_ATTN_PAIRS=1: cross-attention of many streams on k_attn_stream
    std::map<std::pair<int, int>, StepPlanDev> step_plans;
    unsigned *gbar = nullptr;  // grid barrier counter of the step kernel
    unsigned *gflag = nullptr; // its per-block release flags (32 words apart)
    int *xcnt = nullptr;       // finished cross-attention splits per (stream, head)
    float *xpart = nullptr;    // cross-attention partial results of the step kernel
    // in-chain kernel timing (w4j_set_kernel_timing): step graphs captured with external event
    // records around every launch of one kernel class; read back after each step
    int time_class = 0;
    bool timing_capture = false;
    int tev_used = 0, tev_pairs = 0;
    std::vector<cudaEvent_t> tev;
    double class_ms = 0;
    long long class_launches = 0;
};

// Kernel classes of w4j_set_kernel_timing.
enum KClass : int { KC_PROJ = 1, KC_SELF_ATTN = 2, KC_CROSS_ATTN = 3, KC_LOGITS = 4, KC_SELECT = 5, KC_STEP = 6 };

// Around one launch of class `cls` while a timed step graph is being captured: an external event
// record before (begin) and after (!begin) it.
static cudaError_t tmark(w4j_ctx *c, int cls, bool begin) {
    if (!c->timing_capture || c->time_class != cls) return cudaSuccess;
    if ((size_t)c->tev_used >= c->tev.size()) {
        cudaEvent_t e;
        const cudaError_t r = cudaEventCreate(&e);
        if (r != cudaSuccess) return r;
        c->tev.push_back(e);
    }
    const cudaError_t r = cudaEventRecordWithFlags(c->tev[c->tev_used], c->stream, cudaEventRecordExternal);
    ++c->tev_used;
    if (!begin) c->tev_pairs = c->tev_used / 2;
    return r;
}

template <typename T>
static int dalloc(w4j_ctx *c, T **p, size_t n) {
    void *v = nullptr;
    if (n == 0) n = 1;
    CUDA_TRY(cudaMalloc(&v, n * sizeof(T)));
    CUDA_TRY(cudaMemset(v, 0, n * sizeof(T)));
    c->allocs.push_back(v);
    *p = reinterpret_cast<T *>(v);
    return 0;
}

static void dfree(w4j_ctx *c, void *p) {
    if (!p) return;
    auto it = std::find(c->allocs.begin(), c->allocs.end(), p);
    if (it != c->allocs.end()) c->allocs.erase(it);
    cudaFree(p);
}

static void free_all(w4j_ctx *c) {
    for (auto &kv : c->graphs) cudaGraphExecDestroy(kv.second);
    c->graphs.clear();
    for (cudaEvent_t e : c->tev) cudaEventDestroy(e);
    c->tev.clear();
    for (void *p : c->allocs) cudaFree(p);
    c->allocs.clear();
    if (c->h_int_area) cudaFreeHost(c->h_int_area);
    if (c->h_done) cudaFreeHost(c->h_done);
    if (c->ev0) cudaEventDestroy(c->ev0);
    if (c->ev1) cudaEventDestroy(c->ev1);
    for (int i = 0; i < 2; ++i) {
        if (c->xa_copied[i]) cudaEventDestroy(c->xa_copied[i]);
        if (c->xa_used[i]) cudaEventDestroy(c->xa_used[i]);
    }
    if (c->copy_stream) cudaStreamDestroy(c->copy_stream);
    if (c->stream) cudaStreamDestroy(c->stream);
}

// Tensor.java:493-501: GELU table over every f16 bit pattern (tanh form, evaluated as the
// reference does: float arithmetic with the tanh in double).
static void build_gelu_lut(std::vector<float> &t) {
    t.resize(65536);
    const float s = (float)std::sqrt(2.0 / M_PI);
    for (int i = 0; i < 65536; ++i) {
        __half_raw hr;
        hr.x = (unsigned short)i;
        const float x = __half2float(__half(hr));
        t[i] = 0.5f * x * (1.0f + (float)std::tanh((double)(s * (x + 0.044715f * x * x * x))));
    }
}

// Key splits of an attention launch: enough blocks to cover the SMs twice, at least one
// full 128-key tile per split, and no more partials than the combine can stage.
// Key splits of one attention launch: one 128-key tile per split block (every tile then
// streams in before the block's wait), bounded by the combine's staging capacity.  Self-
// attention blocks past ceil(len / 128) exit at once, so the grid can be sized for the
// longest context.
static int choose_split(int len, int nq) {
    return std::max(1, std::min((len + kAttnKeyTile - 1) / kAttnKeyTile, attn_max_splits(nq)));
}

// The self-cache capacity (rows per slot) and everything sized by it: the self K / V caches
// (keep_rows: the rows of the old caches are copied into the new ones), the beam tables, the
// token histories and mask lists, the finished lists and the output tokens.  The reference's
// cache grows without bound once a sequence passes n_text_ctx (WhisperDecoder.java:72 clamps only
// the positional offset); here it grows on demand up to kMaxSelfRows.  Graphs captured with the
// old arrays are dropped.
constexpr int kMaxSelfRows = 4096;

static int size_self(w4j_ctx *c, int cap, bool keep_rows) {
    DecodeState &st = c->st;
    const size_t M = c->M_max, S = c->max_streams, L = c->L, d = c->d;
    const int hs = cap + 1, dyn_stride = 2 * (cap + 1) + 8;
    __half *sk = nullptr, *sv = nullptr;
    int *t0 = nullptr, *t1 = nullptr, *h0 = nullptr, *h1 = nullptr, *dl = nullptr, *ft = nullptr, *ot = nullptr;
    auto undo = [&](int rc) {
        for (void *p : {(void *)sk, (void *)sv, (void *)t0, (void *)t1, (void *)h0, (void *)h1, (void *)dl, (void *)ft,
                        (void *)ot})
            dfree(c, p);
        return rc;
    };
    int rc;
    if ((rc = dalloc(c, &sk, (size_t)c->n_slots * L * cap * d)) || (rc = dalloc(c, &sv, (size_t)c->n_slots * L * cap * d)) ||
        (rc = dalloc(c, &t0, M * cap)) || (rc = dalloc(c, &t1, M * cap)) || (rc = dalloc(c, &h0, M * hs)) ||
        (rc = dalloc(c, &h1, M * hs)) || (rc = dalloc(c, &dl, M * dyn_stride)) || (rc = dalloc(c, &ft, M * hs)) ||
        (rc = dalloc(c, &ot, S * hs)))
        return undo(rc);
    if (keep_rows && c->sk) {
        // [slot][layer][head][rows][64]: one run of old-capacity rows per (slot, layer, head)
        const size_t runs = (size_t)c->n_slots * L * c->H, old_b = (size_t)c->cap * kHeadDim * 2,
                     new_b = (size_t)cap * kHeadDim * 2;
        cudaError_t e = cudaMemcpy2DAsync(sk, new_b, c->sk, old_b, old_b, runs, cudaMemcpyDeviceToDevice, c->stream);
        if (e == cudaSuccess)
            e = cudaMemcpy2DAsync(sv, new_b, c->sv, old_b, old_b, runs, cudaMemcpyDeviceToDevice, c->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
        if (e != cudaSuccess) return undo(set_err(W4J_ERR_CUDA, "self-cache growth: %s", cudaGetErrorString(e)));
    }
    for (auto &kv : c->graphs) cudaGraphExecDestroy(kv.second);
    c->graphs.clear();
    c->graph_launches.clear();
    for (void *p : {(void *)c->sk, (void *)c->sv, (void *)st.table[0], (void *)st.table[1], (void *)st.hist[0],
                    (void *)st.hist[1], (void *)st.dyn_list, (void *)st.fin_tok, (void *)st.out_tok})
        dfree(c, p);
    c->sk = sk;
    c->sv = sv;
    st.table[0] = t0;
    st.table[1] = t1;
    st.hist[0] = h0;
    st.hist[1] = h1;
    st.dyn_list = dl;
    st.fin_tok = ft;
    st.out_tok = ot;
    st.n_ctx = cap;
    st.hs = hs;
    st.dyn_stride = dyn_stride;
    c->cap = cap;
    const size_t srows = (size_t)c->n_slots * L * c->H * cap;
    c->s_tmap_ok = srows < (size_t)INT32_MAX && make_tmap_f16_rows(c->sk_tmap, c->sk, (int)srows, kHeadDim) &&
                   make_tmap_f16_rows(c->sv_tmap, c->sv, (int)srows, kHeadDim) &&
                   make_tmap_f16_box(c->sk_tmap32, c->sk, (int)srows, kHeadDim, 32) &&
                   make_tmap_f16_box(c->sv_tmap32, c->sv, (int)srows, kHeadDim, 32);
    return 0;
}

// Make room for `rows` self-cache rows per slot (keeping the cached rows).
static int grow_self(w4j_ctx *c, int rows) {
    if (rows <= c->cap) return 0;
    if (rows > kMaxSelfRows)
        return set_err(W4J_ERR_ARG, "%d self-attention positions exceed this library's limit of %d", rows, kMaxSelfRows);
    int cap = std::max(rows, c->cap + c->cap / 2);
    cap = std::min(kMaxSelfRows, (cap + 63) / 64 * 64);
    return size_self(c, cap, true);
}

extern "C" const char *w4j_last_error(void) { return g_err.c_str(); }
extern "C" const char *w4j_version(void) { return "whisper4j-b200 0.1 (sm_100a)"; }

extern "C" int w4j_ctx_create(const w4j_dims *dims, int device, int max_streams, int max_beam, w4j_ctx **out) {
    if (!dims || !out) return set_err(W4J_ERR_ARG, "w4j_ctx_create: null argument");
    *out = nullptr;
    const int d = dims->n_text_state, H = dims->n_text_head;
    if (d <= 0 || H <= 0 || d != H * kHeadDim)
        return set_err(W4J_ERR_ARG, "n_text_state must equal n_text_head * 64 (got %d, %d)", d, H);
    if (d % 64 != 0 || d > 4096) return set_err(W4J_ERR_ARG, "n_text_state %d unsupported", d);
    if (dims->n_vocab <= 0 || dims->n_text_ctx <= 0 || dims->n_audio_ctx <= 0 || dims->n_text_layer <= 0)
        return set_err(W4J_ERR_ARG, "invalid model dimensions");
    if (max_streams < 1 || max_beam < 1 || max_beam > 8)
        return set_err(W4J_ERR_ARG, "max_streams >= 1 and 1 <= max_beam <= 8 required");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
        return set_err(W4J_ERR_CUDA, "no CUDA device available");
    if (device < 0 || device >= ndev) return set_err(W4J_ERR_ARG, "device %d out of range", device);
    CUDA_TRY(cudaSetDevice(device));
    cudaDeviceProp prop;
    CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) return set_err(W4J_ERR_STATE, "libwhisper4j_cuda is built for sm_100a (B200); device is sm_%d%d",
                                         prop.major, prop.minor);
    w4j_ctx *c = new w4j_ctx();
    c->device = device;
    c->dims = *dims;
    c->V = dims->n_vocab;
    c->C = dims->n_text_ctx;
    c->A = dims->n_audio_ctx;
    c->d = d;
    c->H = H;
    c->L = dims->n_text_layer;
    c->max_streams = max_streams;
    c->max_beam = max_beam;
    c->n_slots = max_streams * max_beam + 1;  // + one private slot for forward without a cache
    c->M_max = max_streams * max_beam;
    c->cap = dims->n_text_ctx;
    c->Mbuf = std::max(c->M_max, dims->n_text_ctx);
    c->sm_count = prop.multiProcessorCount;
    if (const char *ev = getenv("W4J_NO_TC_LOGITS")) c->tc_logits = ev[0] == '0';
    if (const char *ev = getenv("W4J_NO_TC_GEMM")) c->tc_gemm = ev[0] == '0';
    if (const char *ev = getenv("W4J_STEP_KERNEL")) c->use_step = ev[0] == '1';
    if (const char *ev = getenv("W4J_NO_ATTN_PAIRS")) c->attn_pairs = ev[0] == '0';
    if (const char *ev = getenv("W4J_STEP_BAR")) c->step_bar_mode = ev[0] == '1';
    if (const char *ev = getenv("W4J_SELF_PAIRS")) c->self_warps = ev[0] != '1';
    if (const char *ev = getenv("W4J_LOGITS_CHUNKED")) c->big_logits = ev[0] != '1';
    if (const char *ev = getenv("W4J_L2_AHEAD")) c->l2_ahead = (int)strtol(ev, nullptr, 10);
    if (const char *ev = getenv("W4J_STEP_INFLIGHT_KB")) {
        const long kb = strtol(ev, nullptr, 10);
        if (kb >= 16 && kb <= 128) c->step_inflight = (unsigned)kb << 10;
    }
    if (const char *ev = getenv("W4J_VERBOSE")) c->verbose = ev[0] == '1';
    c->layers.resize(c->L);
    c->cache_len.assign(max_streams, 0);
    c->has_xa.assign(max_streams, 0);
    int rc = 0;
    auto fail = [&](int r) {
        free_all(c);
        delete c;
        return r;
    };
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) return fail(set_err(W4J_ERR_CUDA, "stream"));
    cudaEventCreate(&c->ev0);
    cudaEventCreate(&c->ev1);
    if (cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking) != cudaSuccess)
        return fail(set_err(W4J_ERR_CUDA, "copy stream"));
    for (int i = 0; i < 2; ++i)
        if (cudaEventCreateWithFlags(&c->xa_copied[i], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&c->xa_used[i], cudaEventDisableTiming) != cudaSuccess)
            return fail(set_err(W4J_ERR_CUDA, "events"));
    if ((rc = (int)gemv_prepare()) != 0 || (rc = (int)select_prepare()) != 0 || (rc = (int)logits_tc_prepare()) != 0 ||
        (rc = (int)attn_prepare()) != 0 || (rc = (int)gemm_tc_prepare()) != 0 || (rc = (int)xkv_tc_prepare()) != 0 ||
        (rc = (int)step_prepare()) != 0)
        return fail(set_err(W4J_ERR_CUDA, "kernel attributes: %s", cudaGetErrorString((cudaError_t)rc)));
    const size_t V = c->V, C = c->C, A = c->A, L = c->L;
    const size_t M = c->M_max, MB = c->Mbuf;
    // caches
    const size_t cross = (size_t)max_streams * L * A * d;
    if ((rc = dalloc(c, &c->ck, cross)) || (rc = dalloc(c, &c->cv, cross))) return fail(rc);
    c->x_tmap_ok = cross / kHeadDim < (size_t)INT32_MAX &&
                   make_tmap_f16_rows(c->xk_tmap, c->ck, (int)(cross / kHeadDim), kHeadDim) &&
                   make_tmap_f16_rows(c->xv_tmap, c->cv, (int)(cross / kHeadDim), kHeadDim);
    // activations
    if ((rc = dalloc(c, &c->x, MB * d)) || (rc = dalloc(c, &c->q, MB * d)) || (rc = dalloc(c, &c->attn, MB * d)) ||
        (rc = dalloc(c, &c->h, MB * 4 * d)) || (rc = dalloc(c, &c->xa_stage, A * d)) ||
        (rc = dalloc(c, &c->xa_stage2, A * d)))
        return fail(rc);
    {
        const int rows = act_hilo_rows(c->Mbuf);
        if ((rc = dalloc(c, &c->hilo, (size_t)rows * 4 * d))) return fail(rc);
        c->hilo_ok = c->hilo != nullptr;  // its tensor maps are made per launch (box height by row count)
    }
    c->n_parts = logits_parts_for(c->V, c->sm_count);
    // records per row: one per block, or one per 128-row embedding tile (the one-launch pass)
    const size_t parts_max = std::max(c->n_parts, (c->V + 127) / 128);
    if ((rc = dalloc(c, &c->logit_part, MB * parts_max * kPartStride)) ||
        (rc = dalloc(c, &c->ns_part, MB * parts_max * 2)) || (rc = dalloc(c, &c->ns_value, MB)) ||
        (rc = dalloc(c, &c->masked, M * V)) || (rc = dalloc(c, &c->raw, C * V)) || (rc = dalloc(c, &c->op_err, 1)))
        return fail(rc);
    // GELU table
    {
        std::vector<float> lut;
        build_gelu_lut(lut);
        if ((rc = dalloc(c, &c->gelu_lut, 65536))) return fail(rc);
        if (cudaMemcpy(c->gelu_lut, lut.data(), 65536 * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return fail(set_err(W4J_ERR_CUDA, "gelu table upload"));
    }
    // decode state (the arrays sized by the self-cache capacity are allocated by size_self)
    DecodeState &st = c->st;
    st.V = (int)V;
    if ((rc = dalloc(c, &st.tok_in, M)) || (rc = dalloc(c, &st.seq_slot, M)) || (rc = dalloc(c, &st.seq_pos, M)) ||
        (rc = dalloc(c, &st.active, M)) || (rc = dalloc(c, &st.hist_len[0], M)) || (rc = dalloc(c, &st.hist_len[1], M)) ||
        (rc = dalloc(c, &st.lp[0], M)) || (rc = dalloc(c, &st.lp[1], M)) || (rc = dalloc(c, &st.dyn_count, M)) ||
        (rc = dalloc(c, &st.ranges, M * kMaxRanges)) || (rc = dalloc(c, &st.n_ranges, M)) ||
        (rc = dalloc(c, &st.done, (size_t)max_streams)) || (rc = dalloc(c, &st.beam_par, (size_t)max_streams)) ||
        (rc = dalloc(c, &st.nsp, (size_t)max_streams)) || (rc = dalloc(c, &st.fin_n, (size_t)max_streams)) ||
        (rc = dalloc(c, &st.fin_len, M)) || (rc = dalloc(c, &st.fin_lp, M)) ||
        (rc = dalloc(c, &st.out_len, (size_t)max_streams)) || (rc = dalloc(c, &st.out_sum, (size_t)max_streams)) ||
        (rc = dalloc(c, &st.err, 1)) || (rc = dalloc(c, &c->gbar, 1)) ||
        (rc = dalloc(c, &c->gflag, (size_t)32 * c->sm_count)) ||
        (rc = dalloc(c, &c->xcnt, (size_t)max_streams * H)) ||
        (rc = dalloc(c, &c->xpart, (size_t)c->sm_count * 8 * (kHeadDim + 2))))
        return fail(rc);
    st.gbar = c->gbar;
    st.gflag = c->gflag;
    st.n_gflag = c->sm_count;
    if ((rc = size_self(c, c->cap, false))) return fail(rc);
    // per-call int arrays: a decode call's prompt tokens [C][S], prompt positions [C][S], stream
    // base [S], cross stream [S] and suppress list [V]; or a forward call's nine per-token
    // arrays [9][C] (forward_layout)
    c->int_area_n = std::max(2 * C * (size_t)max_streams + 2 * (size_t)max_streams + V, 9 * C) + 16;
    if ((rc = dalloc(c, &c->d_int_area, c->int_area_n)) || (rc = dalloc(c, &c->d_done_snapshot, (size_t)max_streams)))
        return fail(rc);
    if (cudaMallocHost(&c->h_int_area, c->int_area_n * sizeof(int)) != cudaSuccess ||
        cudaMallocHost(&c->h_done, (size_t)max_streams * sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        return fail(set_err(W4J_ERR_OOM, "pinned host buffers"));
    }
    // fused self-attention bias (key bias defaults to zero)
    for (int l = 0; l < c->L; ++l) {
        LayerDev &ly = c->layers[l];
        if ((rc = dalloc(c, &ly.bqkv, 3 * (size_t)d))) return fail(rc);
    }
    *out = c;
    return W4J_OK;
}

extern "C" int w4j_ctx_destroy(w4j_ctx *c) {
    if (!c) return W4J_OK;
    {
        std::lock_guard<std::mutex> g(c->mu);
        cudaSetDevice(c->device);
        cudaStreamSynchronize(c->stream);
        free_all(c);
    }
    delete c;
    return W4J_OK;
}

// ---------------------------------------------------------------------------
// weight upload (raw GGML payloads)
// ---------------------------------------------------------------------------
static float half_bits_to_float(uint16_t b) {
    __half_raw hr;
    hr.x = b;
    return __half2float(__half(hr));
}

// Host dequantisation of small tensors (biases, LayerNorm, positional table).
static int host_f32(const void *data, size_t nbytes, int type, size_t n, std::vector<float> &out) {
    out.resize(n);
    if (type == W4J_GGML_F32) {
        if (nbytes != n * 4) return set_err(W4J_ERR_ARG, "payload size %zu != %zu", nbytes, n * 4);
        memcpy(out.data(), data, n * 4);
    } else if (type == W4J_GGML_F16) {
        if (nbytes != n * 2) return set_err(W4J_ERR_ARG, "payload size %zu != %zu", nbytes, n * 2);
        const uint16_t *p = reinterpret_cast<const uint16_t *>(data);
        for (size_t i = 0; i < n; ++i) out[i] = half_bits_to_float(p[i]);
    } else if (type == W4J_GGML_Q8_0) {
        if (n % 32 || nbytes != n / 32 * 34) return set_err(W4J_ERR_ARG, "Q8_0 payload size mismatch");
        const uint8_t *p = reinterpret_cast<const uint8_t *>(data);
        for (size_t b = 0; b < n / 32; ++b) {
            const float sc = half_bits_to_float((uint16_t)(p[b * 34] | (p[b * 34 + 1] << 8)));
            for (int i = 0; i < 32; ++i) out[b * 32 + i] = (float)(int8_t)p[b * 34 + 2 + i] * sc;
        }
    } else {
        return set_err(W4J_ERR_ARG, "unsupported GGML type %d", type);
    }
    return 0;
}

static int upload_vec(w4j_ctx *c, float **dst, size_t n, const void *data, size_t nbytes, int type, size_t offset = 0) {
    std::vector<float> v;
    TRY(host_f32(data, nbytes, type, n, v));
    if (!*dst) TRY(dalloc(c, dst, n));
    CUDA_TRY(cudaMemcpy(*dst + offset, v.data(), n * 4, cudaMemcpyHostToDevice));
    return 0;
}

// Matrix (N x K) into DMat `m` rows [row0, row0 + N) of a buffer holding `rows_total` rows.
static int upload_mat(w4j_ctx *c, DMat &m, int rows_total, int row0, int N, int K, const void *data, size_t nbytes,
                      int type, int *type_slot = nullptr) {
    const int want = type == W4J_GGML_Q8_0 ? WT_Q8 : WT_F16;
    if (type != W4J_GGML_F16 && type != W4J_GGML_F32 && type != W4J_GGML_Q8_0)
        return set_err(W4J_ERR_ARG, "unsupported GGML type %d for a matrix (F32, F16, Q8_0 accepted)", type);
    if (type == W4J_GGML_Q8_0 && K % 32) return set_err(W4J_ERR_ARG, "Q8_0 rows must be a multiple of 32");
    const size_t n = (size_t)N * K;
    const size_t expect = type == W4J_GGML_F32 ? n * 4 : type == W4J_GGML_F16 ? n * 2 : n / 32 * 34;
    if (nbytes != expect) return set_err(W4J_ERR_ARG, "payload size %zu, expected %zu", nbytes, expect);
    if (m.type == 0) {
        m.type = want;
        m.N = rows_total;
        m.K = K;
        if (want == WT_F16) {
            __half *p = nullptr;
            TRY(dalloc(c, &p, (size_t)rows_total * K));
            m.h = p;
        } else {
            int8_t *q = nullptr;
            __half *s = nullptr;
            TRY(dalloc(c, &q, (size_t)rows_total * K));
            TRY(dalloc(c, &s, (size_t)rows_total * (K / 32)));
            m.q = q;
            m.s = s;
        }
    } else if (m.type != want) {
        return set_err(W4J_ERR_ARG, "attn.query/key/value of one layer must share a storage type (F16/F32 vs Q8_0)");
    }
    if (type_slot) *type_slot = want;
    void *stage = nullptr;
    CUDA_TRY(cudaMalloc(&stage, nbytes));
    cudaError_t e = cudaMemcpy(stage, data, nbytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) {
        if (type == W4J_GGML_F16) {
            e = cudaMemcpy(const_cast<__half *>(m.h) + (size_t)row0 * K, stage, nbytes, cudaMemcpyDeviceToDevice);
        } else if (type == W4J_GGML_F32) {
            e = launch_f32_to_f16(reinterpret_cast<const float *>(stage), const_cast<__half *>(m.h) + (size_t)row0 * K, n, 0);
        } else {
            e = launch_q8_repack(stage, N, K, const_cast<int8_t *>(m.q) + (size_t)row0 * K,
                                 const_cast<__half *>(m.s) + (size_t)row0 * (K / 32), 0);
        }
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaFree(stage);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_err(W4J_ERR_CUDA, "matrix upload: %s", cudaGetErrorString(e));
    }
    return 0;
}

// An "encoder.*" tensor (WhisperEncoder.java:27-39, :86-105): matrices stored f16 ([N][K] rows, the
// convolutions as Conv1d's (out, in * 3) weightMatrix), vectors f32.  Q8_0 encoder matrices are
// skipped (return 1): the encoder's row counts (1500 and 3000) run on the tensor cores with f16 weights.
static int upload_encoder_tensor(w4j_ctx *c, const std::string &nm, int type, int64_t nel, const void *data,
                                 size_t nbytes) {
    const w4j_dims &dm = c->dims;
    const int d = dm.n_audio_state, T = dm.n_audio_ctx, nmel = dm.n_mels;
    if (d <= 0 || d % 64 || dm.n_audio_head <= 0 || d != dm.n_audio_head * kHeadDim || dm.n_audio_layer <= 0 ||
        nmel <= 0 || T <= 0)
        return set_err(W4J_ERR_ARG, "encoder dims: n_audio_state must be 64 x n_audio_head");
    EncDev &e = c->enc;
    if (e.layers.empty()) {
        e.layers.resize(dm.n_audio_layer);
        for (EncLayer &ly : e.layers) TRY(dalloc(c, &ly.bqkv, 3 * (size_t)d));
        e.k1 = (nmel * 3 + 63) / 64 * 64;
    }
    if (type == W4J_GGML_Q8_0 && nel > d) {  // skipped (the decoder still loads); w4j_encoder_forward says why
        e.q8_skipped = true;
        return 1;
    }
    const std::string s = nm.substr(8);
    auto vec = [&](float **dst, int64_t n, size_t off = 0) -> int {
        if (nel != n) return set_err(W4J_ERR_ARG, "%s: expected %lld elements", nm.c_str(), (long long)n);
        return upload_vec(c, dst, (size_t)n, data, nbytes, type, off);
    };
    if (s == "conv1.weight") {  // (d, n_mels, 3): rows of n_mels * 3, padded with zeros to k1 columns
        if (nel != (int64_t)d * nmel * 3) return set_err(W4J_ERR_ARG, "%s: expected (%d, %d, 3)", nm.c_str(), d, nmel);
        std::vector<float> f;
        TRY(host_f32(data, nbytes, type, (size_t)nel, f));
        std::vector<__half> h((size_t)d * e.k1, __float2half(0.f));
        for (int o = 0; o < d; ++o)
            for (int r = 0; r < nmel * 3; ++r) h[(size_t)o * e.k1 + r] = __float2half_rn(f[(size_t)o * nmel * 3 + r]);
        TRY(upload_mat(c, e.c1, d, 0, d, e.k1, h.data(), h.size() * 2, W4J_GGML_F16));
    } else if (s == "conv2.weight") {
        if (nel != (int64_t)d * d * 3) return set_err(W4J_ERR_ARG, "%s: expected (%d, %d, 3)", nm.c_str(), d, d);
        TRY(upload_mat(c, e.c2, d, 0, d, 3 * d, data, nbytes, type));
    } else if (s == "conv1.bias") {
        TRY(vec(&e.b1, d));
    } else if (s == "conv2.bias") {
        TRY(vec(&e.b2, d));
    } else if (s == "positional_embedding") {
        TRY(vec(&e.pos, (int64_t)T * d));
    } else if (s == "ln_post.weight") {
        TRY(vec(&e.lng, d));
    } else if (s == "ln_post.bias") {
        TRY(vec(&e.lnb, d));
    } else {
        int li = -1, off = 0;
        if (sscanf(s.c_str(), "blocks.%d.%n", &li, &off) != 1 || li < 0 || li >= dm.n_audio_layer)
            return set_err(W4J_ERR_ARG, "unknown encoder tensor %s", nm.c_str());
        EncLayer &ly = e.layers[li];
        const std::string t = s.substr(off);
        struct MatRole { const char *nm; DMat *m; int rows_total, row0, N, K; };
        const MatRole mats[] = {
            {"attn.query.weight", &ly.qkv, 3 * d, 0, d, d}, {"attn.key.weight", &ly.qkv, 3 * d, d, d, d},
            {"attn.value.weight", &ly.qkv, 3 * d, 2 * d, d, d}, {"attn.out.weight", &ly.o, d, 0, d, d},
            {"mlp.0.weight", &ly.m0, 4 * d, 0, 4 * d, d}, {"mlp.2.weight", &ly.m2, d, 0, d, 4 * d},
        };
        bool found = false;
        for (const MatRole &r : mats) {
            if (t != r.nm) continue;
            if (nel != (int64_t)r.N * r.K) return set_err(W4J_ERR_ARG, "%s: expected (%d, %d)", nm.c_str(), r.N, r.K);
            TRY(upload_mat(c, *r.m, r.rows_total, r.row0, r.N, r.K, data, nbytes, type));
            found = true;
        }
        struct VecRole { const char *nm; float **dst; int n; size_t off; };
        const VecRole vecs[] = {
            {"attn.query.bias", &ly.bqkv, d, 0},      {"attn.key.bias", &ly.bqkv, d, (size_t)d},
            {"attn.value.bias", &ly.bqkv, d, 2 * (size_t)d}, {"attn.out.bias", &ly.bo, d, 0},
            {"mlp.0.bias", &ly.bm0, 4 * d, 0},        {"mlp.2.bias", &ly.bm2, d, 0},
            {"attn_ln.weight", &ly.ln1g, d, 0},       {"attn_ln.bias", &ly.ln1b, d, 0},
            {"mlp_ln.weight", &ly.ln2g, d, 0},        {"mlp_ln.bias", &ly.ln2b, d, 0},
        };
        for (const VecRole &r : vecs) {
            if (found || t != r.nm) continue;
            TRY(vec(r.dst, r.n, r.off));
            found = true;
        }
        if (!found) return set_err(W4J_ERR_ARG, "unknown encoder tensor %s", nm.c_str());
    }
    e.uploaded.insert(nm);
    e.maps_ok = false;
    return W4J_OK;
}

extern "C" int w4j_upload_tensor(w4j_ctx *c, const char *name, int type, const int64_t *ne, int n_dims,
                                 const void *data, size_t nbytes) {
    if (!c || !name || !ne || !data) return set_err(W4J_ERR_ARG, "w4j_upload_tensor: null argument");
    std::lock_guard<std::mutex> g(c->mu);
    CUDA_TRY(cudaSetDevice(c->device));
    const std::string nm(name);
    const bool enc = nm.rfind("encoder.", 0) == 0;
    if (!enc && nm.rfind("decoder.", 0) != 0) return 1;  // neither encoder nor decoder: not on this path
    if (n_dims < 1 || n_dims > 4) return set_err(W4J_ERR_ARG, "%s: n_dims %d", name, n_dims);
    int64_t nel = 1;
    for (int i = 0; i < n_dims; ++i) {
        if (ne[i] <= 0) return set_err(W4J_ERR_ARG, "%s: bad shape", name);
        nel *= ne[i];
    }
    if (enc) return upload_encoder_tensor(c, nm, type, nel, data, nbytes);
    const int d = c->d;
    auto shape_is = [&](int64_t in, int64_t out) { return ne[0] == in && nel == in * out; };
    std::string s = nm.substr(8);
    if (s == "token_embedding.weight") {
        if (!shape_is(d, c->V)) return set_err(W4J_ERR_ARG, "%s: expected (%d, %d)", name, c->V, d);
        TRY(upload_mat(c, c->E, c->V, 0, c->V, d, data, nbytes, type));
        c->e_tmap_ok = c->tc_logits && c->E.type == WT_F16 && make_tmap_f16_rows(c->e_tmap, c->E.h, c->V, d);
    } else if (s == "positional_embedding") {
        if (!shape_is(d, c->C)) return set_err(W4J_ERR_ARG, "%s: expected (%d, %d)", name, c->C, d);
        TRY(upload_vec(c, &c->pos_emb, (size_t)c->C * d, data, nbytes, type));
    } else if (s == "ln.weight" || s == "ln.bias") {
        if (nel != d) return set_err(W4J_ERR_ARG, "%s: expected %d elements", name, d);
        TRY(upload_vec(c, s == "ln.weight" ? &c->lng : &c->lnb, d, data, nbytes, type));
    } else {
        int li = -1, off = 0;
        if (sscanf(s.c_str(), "blocks.%d.%n", &li, &off) != 1 || li < 0 || li >= c->L)
            return set_err(W4J_ERR_ARG, "unknown decoder tensor %s", name);
        LayerDev &ly = c->layers[li];
        const std::string t = s.substr(off);
        struct MatRole { const char *nm; DMat *m; int rows_total, row0, N, K; };
        const MatRole mats[] = {
            {"attn.query.weight", &ly.qkv, 3 * d, 0, d, d},         {"attn.key.weight", &ly.qkv, 3 * d, d, d, d},
            {"attn.value.weight", &ly.qkv, 3 * d, 2 * d, d, d},     {"attn.out.weight", &ly.o, d, 0, d, d},
            {"cross_attn.query.weight", &ly.xq, d, 0, d, d},        {"cross_attn.key.weight", &ly.xk, d, 0, d, d},
            {"cross_attn.value.weight", &ly.xv, d, 0, d, d},        {"cross_attn.out.weight", &ly.xo, d, 0, d, d},
            {"mlp.0.weight", &ly.m0, 4 * d, 0, 4 * d, d},           {"mlp.2.weight", &ly.m2, d, 0, d, 4 * d},
        };
        for (const MatRole &r : mats) {
            if (t != r.nm) continue;
            if (!shape_is(r.K, r.N)) return set_err(W4J_ERR_ARG, "%s: expected (%d, %d)", name, r.N, r.K);
            TRY(upload_mat(c, *r.m, r.rows_total, r.row0, r.N, r.K, data, nbytes, type));
            c->uploaded.insert(nm);
            return W4J_OK;
        }
        struct VecRole { const char *nm; float **dst; int n; size_t off; };
        const VecRole vecs[] = {
            {"attn.query.bias", &ly.bqkv, d, 0},          {"attn.key.bias", &ly.bqkv, d, (size_t)d},
            {"attn.value.bias", &ly.bqkv, d, 2 * (size_t)d}, {"attn.out.bias", &ly.bo, d, 0},
            {"cross_attn.query.bias", &ly.bxq, d, 0},     {"cross_attn.key.bias", &ly.bxk, d, 0},
            {"cross_attn.value.bias", &ly.bxv, d, 0},     {"cross_attn.out.bias", &ly.bxo, d, 0},
            {"mlp.0.bias", &ly.bm0, 4 * d, 0},            {"mlp.2.bias", &ly.bm2, d, 0},
            {"attn_ln.weight", &ly.ln1g, d, 0},           {"attn_ln.bias", &ly.ln1b, d, 0},
            {"cross_attn_ln.weight", &ly.ln2g, d, 0},     {"cross_attn_ln.bias", &ly.ln2b, d, 0},
            {"mlp_ln.weight", &ly.ln3g, d, 0},            {"mlp_ln.bias", &ly.ln3b, d, 0},
        };
        bool found = false;
        for (const VecRole &r : vecs) {
            if (t != r.nm) continue;
            if (nel != r.n) return set_err(W4J_ERR_ARG, "%s: expected %d elements", name, r.n);
            TRY(upload_vec(c, r.dst, r.n, data, nbytes, type, r.off));
            found = true;
            break;
        }
        if (!found) return set_err(W4J_ERR_ARG, "unknown decoder tensor %s", name);
    }
    c->uploaded.insert(nm);
    return W4J_OK;
}

static std::vector<std::string> required_names(int L) {
    std::vector<std::string> r = {"decoder.token_embedding.weight", "decoder.positional_embedding",
                                  "decoder.ln.weight", "decoder.ln.bias"};
    const char *per[] = {"attn.query.weight", "attn.query.bias", "attn.key.weight", "attn.value.weight",
                         "attn.value.bias", "attn.out.weight", "attn.out.bias", "attn_ln.weight", "attn_ln.bias",
                         "cross_attn.query.weight", "cross_attn.query.bias", "cross_attn.key.weight",
                         "cross_attn.value.weight", "cross_attn.value.bias", "cross_attn.out.weight",
                         "cross_attn.out.bias", "cross_attn_ln.weight", "cross_attn_ln.bias", "mlp.0.weight",
                         "mlp.0.bias", "mlp.2.weight", "mlp.2.bias", "mlp_ln.weight", "mlp_ln.bias"};
    for (int l = 0; l < L; ++l)
        for (const char *p : per) r.push_back("decoder.blocks." + std::to_string(l) + "." + p);
    return r;
}

static int check_ready(w4j_ctx *c) {
    for (const std::string &n : required_names(c->L))
        if (!c->uploaded.count(n)) return set_err(W4J_ERR_STATE, "weight not found: %s", n.c_str());
    return 0;
}

extern "C" int w4j_finalize(w4j_ctx *c) {
    if (!c) return set_err(W4J_ERR_ARG, "null context");
    std::lock_guard<std::mutex> g(c->mu);
    TRY(check_ready(c));
    CUDA_TRY(cudaSetDevice(c->device));
    for (LayerDev &ly : c->layers) {
        DMat *m[8] = {&ly.qkv, &ly.o, &ly.xq, &ly.xo, &ly.m0, &ly.m2, &ly.xk, &ly.xv};
        for (int i = 0; i < 8; ++i) {
            ly.tmap_ok[i] = false;
            if (!c->tc_gemm) continue;
            if (m[i]->type == WT_F16) {
                ly.tmap_ok[i] = make_tmap_f16_rows(ly.tmap[i], m[i]->h, m[i]->N, m[i]->K);
            } else if (m[i]->type == WT_Q8 && m[i]->N % 128 == 0 && m[i]->K % 64 == 0 && i < 6) {
                // the tensor-core projections read Q8_0 scales per (128-row tile, 64-wide k-block)
                if (!m[i]->st) {
                    __half *st = nullptr;
                    TRY(dalloc(c, &st, (size_t)m[i]->N * (m[i]->K / 32)));
                    CUDA_TRY(launch_q8_tile_scales(m[i]->s, m[i]->N, m[i]->K, st, 0));
                    m[i]->st = st;
                }
                ly.tmap_ok[i] = make_tmap_i8_rows(ly.tmap[i], m[i]->q, m[i]->N, m[i]->K);
            }
        }
    }
    CUDA_TRY(cudaDeviceSynchronize());
    return W4J_OK;
}

// ---------------------------------------------------------------------------
// cross K/V prefill
// ---------------------------------------------------------------------------
static int prefill(w4j_ctx *c, int slot, const float *xa_dev, bool sync = true) {
    for (int l = 0; l < c->L; ++l) {
        LayerDev &ly = c->layers[l];
        const size_t off = ((size_t)slot * c->L + l) * (size_t)c->H * c->A * kHeadDim;
        // tensor cores for f16 weights, else the SIMT GEMM
        cudaError_t e = cudaErrorNotSupported;
        if (ly.tmap_ok[PROJ_XK] && ly.tmap_ok[PROJ_XV] && ly.xk.type == WT_F16 && ly.xv.type == WT_F16)
            e = launch_cross_kv_tc(xa_dev, c->A, c->d, ly.tmap[PROJ_XK], ly.tmap[PROJ_XV], ly.bxk, ly.bxv,
                                   c->ck + off, c->cv + off, c->st.err, c->stream);
        if (e == cudaErrorNotSupported)
            e = launch_cross_kv(xa_dev, c->A, c->d, ly.xk, ly.xv, ly.bxk, ly.bxv, c->ck + off, c->cv + off, c->H,
                                c->stream);
        CUDA_TRY(e);
    }
    if (sync) CUDA_TRY(cudaStreamSynchronize(c->stream));
    c->has_xa[slot] = 1;
    c->cache_len[slot] = 0;
    return 0;
}

extern "C" int w4j_set_encoder_output(w4j_ctx *c, int slot, const float *xa, int n_audio_ctx) {
    if (!c || !xa) return set_err(W4J_ERR_ARG, "w4j_set_encoder_output: null argument");
    std::lock_guard<std::mutex> g(c->mu);
    CUDA_TRY(cudaSetDevice(c->device));
    TRY(check_ready(c));
    if (slot < 0 || slot >= c->max_streams) return set_err(W4J_ERR_ARG, "slot %d out of range", slot);
    if (n_audio_ctx != c->A) return set_err(W4J_ERR_ARG, "encoder output has %d frames, model expects %d", n_audio_ctx, c->A);
    // the copy into the staging buffer the call before last used (its projection has read it: the
    // copy stream waits for that), the host buffer free again when this call returns; the
    // projection itself runs behind the next call's copy (the decode after it is ordered on the
    // same stream)
    const int b = c->xa_flip;
    c->xa_flip ^= 1;
    float *stage = b ? c->xa_stage2 : c->xa_stage;
    CUDA_TRY(cudaStreamWaitEvent(c->copy_stream, c->xa_used[b], 0));
    CUDA_TRY(cudaMemcpyAsync(stage, xa, (size_t)c->A * c->d * 4, cudaMemcpyHostToDevice, c->copy_stream));
    CUDA_TRY(cudaEventRecord(c->xa_copied[b], c->copy_stream));
    CUDA_TRY(cudaEventSynchronize(c->xa_copied[b]));
    CUDA_TRY(cudaStreamWaitEvent(c->stream, c->xa_copied[b], 0));
    TRY(prefill(c, slot, stage, false));
    CUDA_TRY(cudaEventRecord(c->xa_used[b], c->stream));
    return W4J_OK;
}

extern "C" int w4j_set_encoder_output_device(w4j_ctx *c, int slot, const float *xa, int n_audio_ctx) {
    if (!c || !xa) return set_err(W4J_ERR_ARG, "w4j_set_encoder_output_device: null argument");
    std::lock_guard<std::mutex> g(c->mu);
    CUDA_TRY(cudaSetDevice(c->device));
    TRY(check_ready(c));
    if (slot < 0 || slot >= c->max_streams) return set_err(W4J_ERR_ARG, "slot %d out of range", slot);
    if (n_audio_ctx != c->A) return set_err(W4J_ERR_ARG, "encoder output has %d frames, model expects %d", n_audio_ctx, c->A);
    return prefill(c, slot, xa);
}

// ---------------------------------------------------------------------------
// audio encoder (WhisperEncoder.forward, WhisperEncoder.java:42-76)
// ---------------------------------------------------------------------------
static std::vector<std::string> encoder_names(int L) {
    std::vector<std::string> r = {"encoder.conv1.weight", "encoder.conv1.bias", "encoder.conv2.weight",
                                  "encoder.conv2.bias", "encoder.positional_embedding", "encoder.ln_post.weight",
                                  "encoder.ln_post.bias"};
    const char *per[] = {"attn.query.weight", "attn.query.bias", "attn.key.weight", "attn.value.weight",
                         "attn.value.bias", "attn.out.weight", "attn.out.bias", "attn_ln.weight", "attn_ln.bias",
                         "mlp.0.weight", "mlp.0.bias", "mlp.2.weight", "mlp.2.bias", "mlp_ln.weight", "mlp_ln.bias"};
    for (int l = 0; l < L; ++l)
        for (const char *q : per) r.push_back("encoder.blocks." + std::to_string(l) + "." + q);
    return r;
}

// y = act . W^T + bias (+ epilogue) on the tcgen05 GEMM; above 128 rows (every real model: 1500 and
// 3000) the activations are first staged as f16 hi / lo rows (LayerNorm applied when ln_g is given).
static int enc_gemm(w4j_ctx *c, const DMat &W, const void *wmap, int M, const float *act, const float *bias,
                    const float *ln_g, const float *ln_b, int out_mode, float *y) {
    GemvArgs g;
    g.W = W;
    g.bias = bias;
    g.M = M;
    g.in_mode = ln_g ? IN_LN : IN_ACT;
    g.act = act;
    g.ln_g = ln_g;
    g.ln_b = ln_b;
    g.out_mode = out_mode;
    g.y = y;
    g.gelu_lut = c->gelu_lut;
    if (!gemm_tc_supported(g, c->sm_count))
        return set_err(W4J_ERR_ARG, "encoder projection %d x %d x %d outside the tensor-core GEMM", M, W.N, W.K);
    if (!gemm_tc_staged(g)) {  // up to 128 rows (short test models): the B operand built in shared memory
        CUDA_TRY(launch_gemm_tc(g, wmap, nullptr, c->sm_count, c->stream, false));
        return 0;
    }
    alignas(64) unsigned char bmap[128];
    if (!make_tmap_f16_box(bmap, c->enc.hilo, act_hilo_rows(M), W.K, act_hilo_box_rows(M)))
        return set_err(W4J_ERR_CUDA, "encoder: activation tensor map");
    CUDA_TRY(launch_act_hilo(g, c->enc.hilo, c->stream, false));
    CUDA_TRY(launch_gemm_tc(g, wmap, bmap, c->sm_count, c->stream, false));
    return 0;
}

static int enc_prepare(w4j_ctx *c) {
    EncDev &e = c->enc;
    const w4j_dims &dm = c->dims;
    for (const std::string &n : encoder_names(dm.n_audio_layer))
        if (!e.uploaded.count(n))
            return set_err(W4J_ERR_STATE, "encoder weight not uploaded: %s%s", n.c_str(),
                           e.q8_skipped ? " (Q8_0 encoder matrices are not taken by the device encoder)" : "");
    const int d = dm.n_audio_state, T = dm.n_audio_ctx;
    if (!e.maps_ok) {
        bool ok = make_tmap_f16_rows(e.c1map, e.c1.h, d, e.k1) && make_tmap_f16_rows(e.c2map, e.c2.h, d, 3 * d);
        for (EncLayer &ly : e.layers)
            ok = ok && make_tmap_f16_rows(ly.tmap[0], ly.qkv.h, 3 * d, d) && make_tmap_f16_rows(ly.tmap[1], ly.o.h, d, d) &&
                 make_tmap_f16_rows(ly.tmap[2], ly.m0.h, 4 * d, d) && make_tmap_f16_rows(ly.tmap[3], ly.m2.h, d, 4 * d);
        if (!ok) return set_err(W4J_ERR_CUDA, "encoder: weight tensor maps");
        e.maps_ok = true;
    }
    if (!e.mel) TRY(dalloc(c, &e.mel, (size_t)dm.n_mels * 2 * T));
    if (!e.col) {
        const size_t T1 = 2 * (size_t)T;
        TRY(dalloc(c, &e.col, std::max(T1 * e.k1, (size_t)T * 3 * d)));
        TRY(dalloc(c, &e.y1, T1 * d));
        TRY(dalloc(c, &e.x, (size_t)T * d));
        TRY(dalloc(c, &e.qkv, (size_t)T * 3 * d));
        TRY(dalloc(c, &e.att, (size_t)T * d));
        TRY(dalloc(c, &e.hid, (size_t)T * 4 * d));
        TRY(dalloc(c, &e.xa, (size_t)T * d));
        TRY(dalloc(c, &e.qkvh, (size_t)T * 3 * d));
        TRY(dalloc(c, &e.hilo, (size_t)act_hilo_rows((int)T1) * std::max(e.k1, 4 * d)));
    }
    return 0;
}

// The encoder over one mel spectrogram (n_mels x 2 n_audio_ctx, device), output in c->enc.xa.
static int enc_run(w4j_ctx *c) {
    EncDev &e = c->enc;
    const w4j_dims &dm = c->dims;
    const int d = dm.n_audio_state, T = dm.n_audio_ctx, T1 = 2 * T, H = dm.n_audio_head;
    cudaStream_t st = c->stream;
    // conv1 + GELU (:46-47), conv2 + GELU (:50-51), + positional embedding (:56-58)
    CUDA_TRY(launch_enc_im2col(e.mel, dm.n_mels, T1, false, 1, T1, e.k1, e.col, st));
    TRY(enc_gemm(c, e.c1, e.c1map, T1, e.col, e.b1, nullptr, nullptr, OUT_GELU, e.y1));
    CUDA_TRY(launch_enc_im2col(e.y1, d, T1, true, 2, T, 3 * d, e.col, st));
    TRY(enc_gemm(c, e.c2, e.c2map, T, e.col, e.b2, nullptr, nullptr, OUT_GELU, e.x));
    CUDA_TRY(launch_enc_add(e.x, e.pos, (long long)T * d, st));
    // blocks (:60-70): x += attn(attn_ln(x)); x += mlp(mlp_ln(x))
    for (EncLayer &ly : e.layers) {
        TRY(enc_gemm(c, ly.qkv, ly.tmap[0], T, e.x, ly.bqkv, ly.ln1g, ly.ln1b, OUT_STORE, e.qkv));
        CUDA_TRY(launch_enc_qkv_f16(e.qkv, T, H, e.qkvh, st));
        CUDA_TRY(launch_enc_attn(e.qkvh, T, H, e.att, st));
        TRY(enc_gemm(c, ly.o, ly.tmap[1], T, e.att, ly.bo, nullptr, nullptr, OUT_RESIDUAL, e.x));
        TRY(enc_gemm(c, ly.m0, ly.tmap[2], T, e.x, ly.bm0, ly.ln2g, ly.ln2b, OUT_GELU, e.hid));
        TRY(enc_gemm(c, ly.m2, ly.tmap[3], T, e.hid, ly.bm2, nullptr, nullptr, OUT_RESIDUAL, e.x));
    }
    CUDA_TRY(launch_enc_ln(e.x, T, d, e.lng, e.lnb, e.xa, st));  // ln_post (:72)
    return 0;
}

// room for n samples of device audio (c->enc.audio)
static int audio_reserve(w4j_ctx *c, int n) {
    EncDev &e = c->enc;
    if ((size_t)std::max(n, 1) <= e.audio_cap) return 0;
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    dfree(c, e.audio);
    e.audio = nullptr;
    e.audio_cap = 0;
    TRY(dalloc(c, &e.audio, (size_t)std::max(n, 1)));
    e.audio_cap = (size_t)std::max(n, 1);
    return 0;
}

// log-mel of n_total samples (the first n_valid from device audio, the rest zero) into c->enc.mel
// (n_mels x 2 n_audio_ctx): FeatureExtractor.extract + padOrTrim
static int logmel_device(w4j_ctx *c, const float *dev_audio, int n_valid, int n_total) {
    EncDev &e = c->enc;
    const w4j_dims &dm = c->dims;
    if (!e.filt) return set_err(W4J_ERR_STATE, "mel filters not uploaded (w4j_upload_mel_filters)");
    const int n_fft = 2 * (e.filt_bins - 1), hop = 160;
    const int frames = logmel_frames(n_total, n_fft, hop);
    if (!e.mel) TRY(dalloc(c, &e.mel, (size_t)dm.n_mels * 2 * dm.n_audio_ctx));
    if ((size_t)frames > e.frames_cap) {
        CUDA_TRY(cudaStreamSynchronize(c->stream));
        dfree(c, e.spec);
        dfree(c, e.fmx);
        dfree(c, e.fmn);
        e.spec = e.fmx = e.fmn = nullptr;
        e.frames_cap = 0;
        TRY(dalloc(c, &e.spec, (size_t)dm.n_mels * frames));
        TRY(dalloc(c, &e.fmx, (size_t)frames));
        TRY(dalloc(c, &e.fmn, (size_t)frames));
        e.frames_cap = (size_t)frames;
    }
    CUDA_TRY(launch_logmel(dev_audio, n_valid, n_total, n_fft, hop, e.tabs, e.filt, dm.n_mels, e.filt_bins,
                           2 * dm.n_audio_ctx, e.spec, e.fmx, e.fmn, e.mel, c->stream));
    return 0;
}

// log-mel of host audio into c->enc.mel
static int logmel_run(w4j_ctx *c, const float *audio, int n_samples) {
    EncDev &e = c->enc;
    if (!e.filt) return set_err(W4J_ERR_STATE, "mel filters not uploaded (w4j_upload_mel_filters)");
    if (n_samples < 0) return set_err(W4J_ERR_ARG, "n_samples %d", n_samples);
    TRY(audio_reserve(c, n_samples));
    if (n_samples > 0)
        CUDA_TRY(cudaMemcpyAsync(e.audio, audio, (size_t)n_samples * 4, cudaMemcpyHostToDevice, c->stream));
    return logmel_device(c, e.audio, n_samples, n_samples);
}

extern "C" int w4j_upload_mel_filters(w4j_ctx *c, const float *filters, int n_mels, int n_bins) {
    if (!c || !filters) return set_err(W4J_ERR_ARG, "w4j_upload_mel_filters: null argument");
    std::lock_guard<std::mutex> g(c->mu);
    CUDA_TRY(cudaSetDevice(c->device));
    if (n_mels != c->dims.n_mels) return set_err(W4J_ERR_ARG, "%d mel filters, the model has %d", n_mels, c->dims.n_mels);
    if (n_bins < 2 || 2 * (n_bins - 1) > 512) return set_err(W4J_ERR_ARG, "n_bins %d (n_fft = 2 (n_bins - 1) <= 512)", n_bins);
    EncDev &e = c->enc;
    if (e.filt && e.filt_bins != n_bins) return set_err(W4J_ERR_STATE, "mel filters already uploaded with %d bins", e.filt_bins);
    std::vector<float> tabs;
    logmel_tables(2 * (n_bins - 1), tabs);
    if (!e.filt) {
        TRY(dalloc(c, &e.filt, (size_t)n_mels * n_bins));
        TRY(dalloc(c, &e.tabs, tabs.size()));
    }
    e.filt_bins = n_bins;
    CUDA_TRY(cudaMemcpy(e.filt, filters, (size_t)n_mels * n_bins * 4, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(e.tabs, tabs.data(), tabs.size() * 4, cudaMemcpyHostToDevice));
    return W4J_OK;
}

extern "C" int w4j_log_mel(w4j_ctx *c, const float *audio, int n_samples, float *mel_out) {
    if (!c || (!audio && n_samples > 0)) return set_err(W4J_ERR_ARG, "w4j_log_mel: null argument");
    std::lock_guard<std::mutex> g(c->mu);
    CUDA_TRY(cudaSetDevice(c->device));
    TRY(logmel_run(c, audio, n_samples));
    const w4j_dims &dm = c->dims;
    if (mel_out)
        CUDA_TRY(cudaMemcpyAsync(mel_out, c->enc.mel, (size_t)dm.n_mels * 2 * dm.n_audio_ctx * 4, cudaMemcpyDeviceToHost,
                                 c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    return W4J_OK;
}

// encoder over c->enc.mel, then the output to the host and / or a decode slot
static int enc_finish(w4j_ctx *c, float *xa_out, int slot) {
    const w4j_dims &dm = c->dims;
    TRY(enc_run(c));
    if (xa_out)
        CUDA_TRY(cudaMemcpyAsync(xa_out, c->enc.xa, (size_t)dm.n_audio_ctx * dm.n_audio_state * 4, cudaMemcpyDeviceToHost,
                                 c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    if (slot >= 0) TRY(prefill(c, slot, c->enc.xa));
    return W4J_OK;
}

static int enc_check_slot(w4j_ctx *c, int slot) {
    if (slot < 0) return 0;
    TRY(check_ready(c));
    if (slot >= c->max_streams) return set_err(W4J_ERR_ARG, "slot %d out of range", slot);
    if (c->dims.n_audio_state != c->d) return set_err(W4J_ERR_ARG, "n_audio_state differs from n_text_state");
    return 0;
}

extern "C" int w4j_encode_audio(w4j_ctx *c, const float *audio, int n_samples, float *xa_out, int slot) {
    if (!c || (!audio && n_samples > 0)) return set_err(W4J_ERR_ARG, "w4j_encode_audio: null argument");
    std::lock_guard<std::mutex> g(c->mu);
    CUDA_TRY(cudaSetDevice(c->device));
    TRY(enc_check_slot(c, slot));
    TRY(enc_prepare(c));
    TRY(logmel_run(c, audio, n_samples));
    return enc_finish(c, xa_out, slot);
}

extern "C" int w4j_encoder_forward(w4j_ctx *c, const float *mel, int n_frames, float *xa_out, int slot) {
    if (!c || !mel) return set_err(W4J_ERR_ARG, "w4j_encoder_forward: null argument");
    std::lock_guard<std::mutex> g(c->mu);
    CUDA_TRY(cudaSetDevice(c->device));
    const w4j_dims &dm = c->dims;
    if (n_frames != 2 * dm.n_audio_ctx)
        return set_err(W4J_ERR_ARG, "mel has %d frames, the encoder takes %d", n_frames, 2 * dm.n_audio_ctx);
    TRY(enc_check_slot(c, slot));
    TRY(enc_prepare(c));
    const size_t mel_bytes = (size_t)dm.n_mels * n_frames * 4;
    CUDA_TRY(cudaMemcpyAsync(c->enc.mel, mel, mel_bytes, cudaMemcpyHostToDevice, c->stream));
    return enc_finish(c, xa_out, slot);
}

// ---------------------------------------------------------------------------
// one decoder pass over M rows (all layers)
// ---------------------------------------------------------------------------
struct PassArgs {
    int M;                 // rows (sequences)
    const int *tok, *pos;  // [M]
    const int *seq_slot;   // [M] self-cache slots
    const int *table;      // [M][C] or null
    const int *active;     // [M] or null
    // cross attention grouping
    int groups, nq;
    const int *cross_stream;  // [groups]
    const int *group_active;  // [groups] or null
    int self_prefetch;        // older self-cache rows were written by an earlier graph launch
    const int *pe_pos;        // [M] positional-embedding rows, or null: min(pos, n_text_ctx - 1)
    const int *kv_len;        // [M] self-attention keys, or null: pos + 1
    const int2 *mask;         // [M] masked self-attention keys [lo, hi), or null
};

// One projection: the tcgen05 kernel from 16 rows on (past 128 rows of f16 weights after staging the
// activations as f16 hi / lo rows), else the GEMV.
static cudaError_t run_proj(w4j_ctx *c, const GemvArgs &g, const LayerDev &ly, Proj p, bool pdl, long long &launches) {
    cudaError_t e = tmark(c, KC_PROJ, true);
    if (e != cudaSuccess) return e;
    e = cudaErrorNotSupported;
    if (ly.tmap_ok[p] && g.M >= 16 && gemm_tc_supported(g, c->sm_count)) {
        const void *bmap = nullptr;
        if (gemm_tc_staged(g)) {
            alignas(64) unsigned char bm[128];
            if (c->hilo_ok && (g.W.K == c->d || g.W.K == 4 * c->d) &&
                make_tmap_f16_box(bm, c->hilo, act_hilo_rows(c->Mbuf), g.W.K, act_hilo_box_rows(g.M))) {
                e = launch_act_hilo(g, c->hilo, c->stream, pdl);
                if (e != cudaSuccess) return e;
                ++launches;
                bmap = bm;
                e = launch_gemm_tc(g, ly.tmap[p], bmap, c->sm_count, c->stream, pdl);
            }
        } else {
            e = launch_gemm_tc(g, ly.tmap[p], nullptr, c->sm_count, c->stream, pdl);
        }
    }
    if (e == cudaErrorNotSupported) e = launch_gemv(g, c->stream, pdl);
    ++launches;
    return e != cudaSuccess ? e : tmark(c, KC_PROJ, false);
}

static const DMat &proj_mat(const LayerDev &ly, int p) {
    switch (p) {
        case PROJ_QKV: return ly.qkv;
        case PROJ_O: return ly.o;
        case PROJ_XQ: return ly.xq;
        case PROJ_XO: return ly.xo;
        case PROJ_M0: return ly.m0;
        default: return ly.m2;
    }
}

// What projection p of layer l pulls into L2 for later kernels of the step: the weights of the
// projection c->l2_ahead places further along the chain (wrapping to the next step's first
// layer), and with the cross query's weights, for a pass over one stream, that layer's cross K / V.
static L2Ahead l2_ahead_for(const w4j_ctx *c, const PassArgs &pa, int l, int p) {
    L2Ahead f;
    if (c->l2_ahead <= 0 || pa.M >= 16) return f;
    const int n = 6 * c->L, t = (6 * l + p + c->l2_ahead) % n;
    const int tl = t / 6, tp = t % 6;
    const DMat &m = proj_mat(c->layers[tl], tp);
    f.w = m.type == WT_F16 ? reinterpret_cast<const unsigned char *>(m.h) : reinterpret_cast<const unsigned char *>(m.q);
    f.w_bytes = (size_t)m.N * m.K * (m.type == WT_F16 ? 2 : 1);
    if (tp == PROJ_XQ && pa.groups == 1 && c->ck && c->cv) {
        const size_t layer_elems = (size_t)c->H * c->A * kHeadDim;
        f.k = reinterpret_cast<const unsigned char *>(c->ck + (size_t)tl * layer_elems);
        f.v = reinterpret_cast<const unsigned char *>(c->cv + (size_t)tl * layer_elems);
        f.kv_bytes = layer_elems * 2;
        f.kv_stride = (size_t)c->L * layer_elems * 2;
        f.stream = pa.cross_stream;
        f.n_streams = c->max_streams;
    }
    return f;
}

static int run_layers(w4j_ctx *c, const PassArgs &pa, long long &launches) {
    const bool pdl = true;
    const int d = c->d;
    const int self_split = choose_split(c->cap, 1);
    const int cross_split = choose_split(c->A, pa.nq);
    for (int l = 0; l < c->L; ++l) {
        LayerDev &ly = c->layers[l];
        GemvArgs g;
        g.W = ly.qkv;
        g.bias = ly.bqkv;
        g.M = pa.M;
        g.in_mode = l == 0 ? IN_EMBED_LN : IN_LN;
        g.act = c->x;
        g.ln_g = ly.ln1g;
        g.ln_b = ly.ln1b;
        g.E = c->E;
        g.pos_emb = c->pos_emb;
        g.tok = pa.tok;
        g.pos = pa.pos;
        g.pe_pos = pa.pe_pos;
        g.pe_rows = c->C;
        g.x_out = c->x;
        g.out_mode = OUT_QKV;
        g.y = c->q;
        g.kcache = c->sk;
        g.vcache = c->sv;
        g.seq_slot = pa.seq_slot;
        g.layer = l;
        g.n_layer = c->L;
        g.n_head = c->H;
        g.n_ctx = c->cap;
        g.active = pa.active;
        g.err = c->st.err;
        g.pf = l2_ahead_for(c, pa, l, PROJ_QKV);
        CUDA_TRY(run_proj(c, g, ly, PROJ_QKV, pdl, launches));

        AttnArgs sa;
        sa.q = c->q;
        sa.d = d;
        sa.n_head = c->H;
        sa.n_layer = c->L;
        sa.layer = l;
        sa.cross = 0;
        sa.kc = c->sk;
        sa.vc = c->sv;
        sa.n_ctx = c->cap;
        sa.seq_slot = pa.seq_slot;
        sa.table = pa.table;
        sa.pos = pa.pos;
        sa.kv_len = pa.kv_len;
        sa.mask = pa.mask;
        sa.nq = 1;
        sa.groups = pa.M;
        sa.nsplit = self_split;
        sa.out = c->attn;
        sa.active = pa.active;
        sa.err = c->st.err;
        sa.self_prefetch = pa.self_prefetch;
        CUDA_TRY(tmark(c, KC_SELF_ATTN, true));
        if (c->s_tmap_ok && attn_self_stream_pays(sa, c->sm_count))
            CUDA_TRY(c->self_warps ? launch_attn_self_warps(sa, c->sk_tmap32, c->sv_tmap32, c->sm_count, c->stream, pdl)
                                   : launch_attn_self_stream(sa, c->sk_tmap, c->sv_tmap, c->sm_count, c->stream, pdl));
        else CUDA_TRY(launch_attn(sa, c->stream, pdl));
        CUDA_TRY(tmark(c, KC_SELF_ATTN, false));

        GemvArgs go;
        go.W = ly.o;
        go.bias = ly.bo;
        go.M = pa.M;
        go.in_mode = IN_ACT;
        go.act = c->attn;
        go.out_mode = OUT_RESIDUAL;
        go.y = c->x;
        go.active = pa.active;
        go.err = c->st.err;
        go.pf = l2_ahead_for(c, pa, l, PROJ_O);
        CUDA_TRY(run_proj(c, go, ly, PROJ_O, pdl, launches));

        GemvArgs gq;
        gq.W = ly.xq;
        gq.bias = ly.bxq;
        gq.M = pa.M;
        gq.in_mode = IN_LN;
        gq.act = c->x;
        gq.ln_g = ly.ln2g;
        gq.ln_b = ly.ln2b;
        gq.out_mode = OUT_STORE;
        gq.y = c->q;
        gq.err = c->st.err;
        gq.pf = l2_ahead_for(c, pa, l, PROJ_XQ);
        CUDA_TRY(run_proj(c, gq, ly, PROJ_XQ, pdl, launches));

        AttnArgs ca;
        ca.q = c->q;
        ca.d = d;
        ca.n_head = c->H;
        ca.n_layer = c->L;
        ca.layer = l;
        ca.cross = 1;
        ca.kc = c->ck;
        ca.vc = c->cv;
        ca.n_audio = c->A;
        ca.stream_of_group = pa.cross_stream;
        ca.nq = pa.nq;
        ca.groups = pa.groups;
        ca.nsplit = cross_split;
        ca.out = c->attn;
        ca.active = pa.group_active;
        ca.err = c->st.err;
        CUDA_TRY(tmark(c, KC_CROSS_ATTN, true));
        if (c->x_tmap_ok && c->attn_pairs && attn_pairs_pays(ca, c->sm_count))
            CUDA_TRY(launch_attn_pairs(ca, c->xk_tmap, c->xv_tmap, c->sm_count, c->stream, pdl));
        else if (c->x_tmap_ok && attn_stream_pays(ca, c->sm_count))
            CUDA_TRY(launch_attn_stream(ca, c->xk_tmap, c->xv_tmap, c->sm_count, c->stream, pdl));
        else CUDA_TRY(launch_attn(ca, c->stream, pdl));
        CUDA_TRY(tmark(c, KC_CROSS_ATTN, false));

        GemvArgs gxo;
        gxo.W = ly.xo;
        gxo.bias = ly.bxo;
        gxo.M = pa.M;
        gxo.in_mode = IN_ACT;
        gxo.act = c->attn;
        gxo.out_mode = OUT_RESIDUAL;
        gxo.y = c->x;
        gxo.active = pa.active;
        gxo.err = c->st.err;
        gxo.pf = l2_ahead_for(c, pa, l, PROJ_XO);
        CUDA_TRY(run_proj(c, gxo, ly, PROJ_XO, pdl, launches));

        GemvArgs g1;
        g1.W = ly.m0;
        g1.bias = ly.bm0;
        g1.M = pa.M;
        g1.in_mode = IN_LN;
        g1.act = c->x;
        g1.ln_g = ly.ln3g;
        g1.ln_b = ly.ln3b;
        g1.out_mode = OUT_GELU;
        g1.y = c->h;
        g1.gelu_lut = c->gelu_lut;
        g1.err = c->st.err;
        g1.pf = l2_ahead_for(c, pa, l, PROJ_M0);
        CUDA_TRY(run_proj(c, g1, ly, PROJ_M0, pdl, launches));

        GemvArgs g2;
        g2.W = ly.m2;
        g2.bias = ly.bm2;
        g2.M = pa.M;
        g2.in_mode = IN_ACT;
        g2.act = c->h;
        g2.out_mode = OUT_RESIDUAL;
        g2.y = c->x;
        g2.active = pa.active;
        g2.err = c->st.err;
        g2.pf = l2_ahead_for(c, pa, l, PROJ_M2);
        CUDA_TRY(run_proj(c, g2, ly, PROJ_M2, pdl, launches));
        launches += 2;  // the two attentions
    }
    return 0;
}

static LogitsArgs logits_args(w4j_ctx *c, int M, const int *active) {
    LogitsArgs la;
    la.E = c->E;
    la.x = c->x;
    la.ln_g = c->lng;
    la.ln_b = c->lnb;
    la.M = M;
    la.V = c->V;
    la.d = c->d;
    la.part = c->logit_part;
    la.active = active;
    la.err = c->st.err;
    return la;
}

// Rows [m0, m0 + n) of a vocabulary pass: every per-row pointer advanced by m0 rows.
static LogitsArgs logits_rows(const LogitsArgs &la, int m0, int n, int n_parts) {
    LogitsArgs r = la;
    r.M = n;
    r.x = la.x + (size_t)m0 * la.d;
    r.part = la.part + (size_t)m0 * n_parts * kPartStride;
    if (la.raw_out) r.raw_out = la.raw_out + (size_t)m0 * la.V;
    if (la.masked_out) r.masked_out = la.masked_out + (size_t)m0 * la.V;
    if (la.ns_part) r.ns_part = la.ns_part + (size_t)m0 * n_parts * 2;
    if (la.ns_value) r.ns_value = la.ns_value + m0;
    if (la.active) r.active = la.active + m0;
    if (la.use_mask) {
        r.mask.dyn_list = la.mask.dyn_list + (size_t)m0 * la.mask.dyn_stride;
        r.mask.dyn_count = la.mask.dyn_count + m0;
        r.mask.ranges = la.mask.ranges + (size_t)m0 * kMaxRanges;
        r.mask.n_ranges = la.mask.n_ranges + m0;
    }
    return r;
}

// The vocabulary pass over la.M rows takes the one-launch tcgen05 kernel (33 .. 256 rows, no beam
// top-k, the rows staged as f16 through the activation buffer) when the embedding is f16.
static bool logits_big(const w4j_ctx *c, const LogitsArgs &la) {
    return c->e_tmap_ok && c->hilo_ok && c->big_logits && la.M <= c->Mbuf &&
           logits_big_parts(la.M, la.V, la.d, la.topk) > 0;
}

// Records per row that the vocabulary pass for la writes (what the select kernels merge).
static int logit_parts(const w4j_ctx *c, const LogitsArgs &la) {
    return logits_big(c, la) ? logits_big_parts(la.M, la.V, la.d, la.topk) : c->n_parts;
}

// The vocabulary pass: the one-launch tcgen05 kernel for 33 .. 256 rows (after staging the rows), the
// 32-row tcgen05 kernel (one launch per 32 rows) otherwise when the embedding is f16, else the SIMT
// one.  Returns the launches enqueued in `launches`.
static cudaError_t run_logits_untimed(w4j_ctx *c, const LogitsArgs &la, bool pdl, long long &launches);
static cudaError_t run_logits(w4j_ctx *c, const LogitsArgs &la, bool pdl, long long &launches) {
    cudaError_t e = tmark(c, KC_LOGITS, true);
    if (e == cudaSuccess) e = run_logits_untimed(c, la, pdl, launches);
    return e != cudaSuccess ? e : tmark(c, KC_LOGITS, false);
}
static cudaError_t run_logits_untimed(w4j_ctx *c, const LogitsArgs &la, bool pdl, long long &launches) {
    if (logits_big(c, la)) {
        // the final LayerNorm of the rows, as f16 hi (and lo) rows of the staged buffer
        GemvArgs g;
        g.W.type = WT_F16;
        g.W.N = la.V;
        g.W.K = la.d;
        g.M = la.M;
        g.in_mode = IN_LN;
        g.act = la.x;
        g.ln_g = la.ln_g;
        g.ln_b = la.ln_b;
        alignas(64) unsigned char bm[128];
        if (!make_tmap_f16_box(bm, c->hilo, act_hilo_rows(c->Mbuf), la.d, logits_big_box_rows(la.M)))
            return cudaErrorInvalidValue;
        cudaError_t e = launch_act_hilo(g, c->hilo, c->stream, pdl);
        if (e != cudaSuccess) return e;
        e = launch_logits_big(la, c->e_tmap, bm, c->n_parts, c->stream, pdl);
        launches += 2;
        return e;
    }
    if (c->e_tmap_ok) {
        const int chunks = (la.M + 31) / 32;
        cudaError_t e = cudaSuccess;
        int done = 0;
        for (int i = 0; i < chunks && e == cudaSuccess; ++i) {
            const int m0 = (i * la.M) / chunks, m1 = ((i + 1) * la.M) / chunks;
            e = launch_logits_tc(logits_rows(la, m0, m1 - m0, c->n_parts), c->e_tmap, c->n_parts, c->stream, pdl);
            if (e == cudaSuccess) ++done;
        }
        launches += done;
        // unsupported shapes are refused by the first chunk; a refusal after a launch is an error
        if (e != cudaErrorNotSupported || done > 0) return e;
    }
    ++launches;
    return launch_logits(la, c->n_parts, c->stream, pdl);
}

// ---------------------------------------------------------------------------
// forward (WhisperDecoder.forward)
// ---------------------------------------------------------------------------
extern "C" int w4j_forward(w4j_ctx *c, int slot, const int32_t *tokens, int n, int use_cache, float *out_logits) {
    if (!c || !tokens || !out_logits) return set_err(W4J_ERR_ARG, "w4j_forward: null argument");
    std::lock_guard<std::mutex> g(c->mu);
    CUDA_TRY(cudaSetDevice(c->device));
    TRY(check_ready(c));
    if (slot < 0 || slot >= c->max_streams) return set_err(W4J_ERR_ARG, "slot %d out of range", slot);
    if (!c->has_xa[slot]) return set_err(W4J_ERR_STATE, "no encoder output set for slot %d", slot);
    if (n <= 0) return set_err(W4J_ERR_ARG, "empty token list");
    // WhisperDecoder.java:72: offset = min(cache length, n_ctx - seqLen); a sequence longer than
    // the positional table has no valid offset (the reference fails reading the table)
    if (n > c->C) return set_err(W4J_ERR_ARG, "%d tokens exceed n_text_ctx %d", n, c->C);
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= c->V) return set_err(W4J_ERR_ARG, "token id %d out of range", tokens[i]);
    const int start = use_cache ? c->cache_len[slot] : 0;
    const int offset = std::min(start, c->C - n);
    TRY(grow_self(c, start + n));  // the cache keeps growing past n_text_ctx, as the reference's does
    const int phys = use_cache ? slot * c->max_beam : c->n_slots - 1;
    // one pass over the n tokens as n rows (forward_layout: [9][C] ints): every layer appends all
    // their K / V rows before its attention, which for n > 1 applies the reference's causal mask
    // from key column 0 (MultiHeadAttention.java:84-88, Tensor.java:622-640): query t attends keys
    // [0, t] and [n_ctx, kv_len); with an empty cache that is the usual causal mask
    const int C = c->C, kv = start + n;
    int *hi = c->h_int_area;
    int *di = c->d_int_area;
    for (int t = 0; t < n; ++t) {
        hi[t] = tokens[t];
        hi[C + t] = start + t;
        hi[2 * C + t] = offset + t;
        hi[3 * C + t] = phys;
        hi[4 * C + t] = slot;
        hi[5 * C + t] = kv;
        hi[6 * C + 2 * t] = n > 1 ? t + 1 : 0;
        hi[6 * C + 2 * t + 1] = n > 1 ? std::min(kv, C) : 0;
    }
    CUDA_TRY(cudaMemcpyAsync(di, hi, 8 * (size_t)C * 4, cudaMemcpyHostToDevice, c->stream));
    long long launches = 0;
    PassArgs pa{};
    pa.M = n;
    pa.tok = di;
    pa.pos = di + C;
    pa.pe_pos = di + 2 * C;
    pa.seq_slot = di + 3 * C;
    pa.cross_stream = di + 4 * C;
    pa.kv_len = di + 5 * C;
    pa.mask = reinterpret_cast<const int2 *>(di + 6 * C);
    pa.groups = n;
    pa.nq = 1;
    TRY(run_layers(c, pa, launches));
    LogitsArgs la = logits_args(c, n, nullptr);
    la.raw_out = c->raw;
    CUDA_TRY(run_logits(c, la, true, launches));
    CUDA_TRY(cudaMemcpyAsync(out_logits, c->raw, (size_t)n * c->V * 4, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    int errw = 0;
    CUDA_TRY(cudaMemcpy(&errw, c->st.err, 4, cudaMemcpyDeviceToHost));
    if (errw) {
        cudaMemset(c->st.err, 0, 4);
        return set_err(W4J_ERR_CUDA, "a bounded device wait ran out (copy never completed)");
    }
    if (use_cache) c->cache_len[slot] = start + n;
    return W4J_OK;
}

extern "C" int w4j_reset_cache(w4j_ctx *c, int slot) {
    if (!c) return set_err(W4J_ERR_ARG, "null context");
    std::lock_guard<std::mutex> g(c->mu);
    if (slot < 0 || slot >= c->max_streams) return set_err(W4J_ERR_ARG, "slot %d out of range", slot);
    c->cache_len[slot] = 0;
    return W4J_OK;
}

// ---------------------------------------------------------------------------
// decode loops
// ---------------------------------------------------------------------------
enum { MODE_GREEDY = 0, MODE_SAMPLE = 1, MODE_BEAM = 2 };

struct CallArgs {
    const int32_t *slots;
    int S;
    const int32_t *prompts;
    int n_prompt;
    int eot, max_tokens;
    const int32_t *suppress;
    int n_sup;
    int ns;
    float temperature;
    int ts_begin;
    unsigned long long seed;
    int beam;
};

// Device int area layout for a decode call (offsets in ints).
struct CallLayout {
    size_t ptok, ppos, base, cross, sup, total;
};

static CallLayout call_layout(w4j_ctx *c, int S, int n_prompt, int n_sup) {
    CallLayout L;
    L.ptok = 0;
    L.ppos = L.ptok + (size_t)n_prompt * S;
    L.base = L.ppos + (size_t)n_prompt * S;
    L.cross = L.base + S;
    L.sup = L.cross + S;
    L.total = L.sup + std::max(1, n_sup);
    (void)c;
    return L;
}

static int validate_call(w4j_ctx *c, const CallArgs &a) {
    if (!a.slots || !a.prompts) return set_err(W4J_ERR_ARG, "null argument");
    if (a.S < 1 || a.S > c->max_streams) return set_err(W4J_ERR_ARG, "n_streams %d out of [1, %d]", a.S, c->max_streams);
    if (a.beam < 1 || a.beam > c->max_beam)
        return set_err(W4J_ERR_ARG, "beam %d out of [1, %d] (context max_beam)", a.beam, c->max_beam);
    if (a.n_prompt < 1 || a.n_prompt > c->C) return set_err(W4J_ERR_ARG, "prompt length %d", a.n_prompt);
    if (a.eot < 0 || a.eot >= c->V) return set_err(W4J_ERR_ARG, "eot token %d out of range", a.eot);
    if (a.max_tokens < 0) return set_err(W4J_ERR_ARG, "max_tokens must be >= 0");
    if (a.beam > 1 && a.max_tokens < 1) return set_err(W4J_ERR_ARG, "beam search needs max_tokens >= 1");
    // positions past n_text_ctx reuse its last positional row (WhisperDecoder.java:72) while the
    // self cache keeps growing; the capacity is made at the start of the call (grow_self)
    if ((long long)a.n_prompt + std::max(a.max_tokens, 1) - 1 > kMaxSelfRows)
        return set_err(W4J_ERR_ARG, "prompt (%d) + max_tokens (%d) exceeds this library's limit of %d positions",
                       a.n_prompt, a.max_tokens, kMaxSelfRows);
    if (a.n_sup < 0 || (a.n_sup > 0 && !a.suppress)) return set_err(W4J_ERR_ARG, "suppress list");
    if (a.n_sup > c->V) return set_err(W4J_ERR_ARG, "suppress list longer than the vocabulary");
    if (a.temperature < 0.f || !(a.temperature == a.temperature)) return set_err(W4J_ERR_ARG, "temperature");
    std::set<int> seen;
    for (int s = 0; s < a.S; ++s) {
        const int sl = a.slots[s];
        if (sl < 0 || sl >= c->max_streams) return set_err(W4J_ERR_ARG, "slot %d out of range", sl);
        if (!seen.insert(sl).second) return set_err(W4J_ERR_ARG, "slot %d listed twice", sl);
        if (!c->has_xa[sl]) return set_err(W4J_ERR_STATE, "no encoder output set for slot %d", sl);
    }
    for (int i = 0; i < a.S * a.n_prompt; ++i)
        if (a.prompts[i] < 0 || a.prompts[i] >= c->V) return set_err(W4J_ERR_ARG, "prompt token %d out of range", a.prompts[i]);
    return 0;
}

// Upload per-call inputs and reset the decode state.
static int prepare_call(w4j_ctx *c, const CallArgs &a, const CallLayout &Ly) {
    if (Ly.total > c->int_area_n) return set_err(W4J_ERR_ARG, "call too large for the context");
    int *hi = c->h_int_area;
    for (int s = 0; s < a.S; ++s)
        for (int i = 0; i < a.n_prompt; ++i) {
            hi[Ly.ptok + (size_t)i * a.S + s] = a.prompts[(size_t)s * a.n_prompt + i];
            hi[Ly.ppos + (size_t)i * a.S + s] = i;
        }
    for (int s = 0; s < a.S; ++s) {
        hi[Ly.base + s] = a.slots[s] * c->max_beam;
        hi[Ly.cross + s] = a.slots[s];
    }
    for (int i = 0; i < a.n_sup; ++i) hi[Ly.sup + i] = a.suppress[i];
    CUDA_TRY(cudaMemcpyAsync(c->d_int_area, hi, Ly.total * 4, cudaMemcpyHostToDevice, c->stream));
    // per-sequence state
    const int B = a.beam, M = a.S * B;
    std::vector<int> slot(M), pos(M, a.n_prompt - 1), ones(M, 1);
    for (int s = 0; s < a.S; ++s)
        for (int b = 0; b < B; ++b) slot[s * B + b] = a.slots[s] * c->max_beam + b;
    DecodeState &st = c->st;
    CUDA_TRY(cudaMemcpyAsync(st.seq_slot, slot.data(), M * 4, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(cudaMemcpyAsync(st.seq_pos, pos.data(), M * 4, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(cudaMemcpyAsync(st.active, ones.data(), M * 4, cudaMemcpyHostToDevice, c->stream));
    CUDA_TRY(cudaMemsetAsync(st.hist_len[0], 0, M * 4, c->stream));
    CUDA_TRY(cudaMemsetAsync(st.hist_len[1], 0, M * 4, c->stream));
    CUDA_TRY(cudaMemsetAsync(st.lp[0], 0, M * 8, c->stream));
    CUDA_TRY(cudaMemsetAsync(st.lp[1], 0, M * 8, c->stream));
    CUDA_TRY(cudaMemsetAsync(st.dyn_count, 0, M * 4, c->stream));
    CUDA_TRY(cudaMemsetAsync(st.n_ranges, 0, M * 4, c->stream));
    CUDA_TRY(cudaMemsetAsync(st.done, 0, a.S * 4, c->stream));
    CUDA_TRY(cudaMemsetAsync(st.beam_par, 0, a.S * 4, c->stream));
    CUDA_TRY(cudaMemsetAsync(st.fin_n, 0, a.S * 4, c->stream));
    CUDA_TRY(cudaMemsetAsync(st.nsp, 0, a.S * 4, c->stream));
    CUDA_TRY(cudaMemsetAsync(st.err, 0, 4, c->stream));
    CUDA_TRY(cudaMemsetAsync(c->xcnt, 0, (size_t)c->max_streams * c->H * 4, c->stream));
    CUDA_TRY(cudaMemsetAsync(c->gbar, 0, 4, c->stream));
    CUDA_TRY(cudaMemsetAsync(c->gflag, 0, (size_t)32 * c->sm_count * 4, c->stream));
    st.n_streams = a.S;
    st.beam = B;
    st.max_tokens = a.max_tokens;
    st.n_prompt = a.n_prompt;
    st.eot = a.eot;
    st.ts_begin = a.ts_begin;
    st.ns_token = (a.ns >= 0 && a.ns < c->V) ? a.ns : -1;
    st.n_suppress = a.n_sup;
    st.temperature = a.temperature;
    st.seed = a.seed;
    st.n_parts = c->n_parts;
    st.suppress = c->d_int_area + Ly.sup;
    st.stream_base = c->d_int_area + Ly.base;
    return 0;
}

static MaskArgs mask_args(w4j_ctx *c) {
    MaskArgs mk;
    mk.static_list = c->st.suppress;
    mk.n_static = c->st.n_suppress;
    mk.dyn_list = c->st.dyn_list;
    mk.dyn_count = c->st.dyn_count;
    mk.dyn_stride = c->st.dyn_stride;
    mk.ranges = c->st.ranges;
    mk.n_ranges = c->st.n_ranges;
    return mk;
}

// The prompt: one pass per prompt token over all streams (beam 0 slots), then the first decision.
static int run_prompt(w4j_ctx *c, const CallArgs &a, const CallLayout &Ly, int mode, long long &launches) {
    DecodeState &st = c->st;
    const int S = a.S;
    const int *di = c->d_int_area;
    for (int i = 0; i < a.n_prompt; ++i) {
        PassArgs pa{};
        pa.M = S;
        pa.tok = di + Ly.ptok + (size_t)i * S;
        pa.pos = di + Ly.ppos + (size_t)i * S;
        pa.seq_slot = st.stream_base;
        pa.groups = S;
        pa.nq = 1;
        pa.cross_stream = di + Ly.cross;
        TRY(run_layers(c, pa, launches));
        const bool last = i == a.n_prompt - 1;
        const bool ns_here = i == 0 && st.ns_token >= 0;
        if (!last && !ns_here) continue;
        if (last) {
            CUDA_TRY(launch_init_masks(st, mode == MODE_BEAM, c->stream));
            ++launches;
        }
        LogitsArgs la = logits_args(c, S, nullptr);
        if (last) {
            la.use_mask = 1;
            la.mask = mask_args(c);
            la.topk = mode == MODE_BEAM ? a.beam : 0;
            if (mode == MODE_SAMPLE) la.masked_out = c->masked;
        }
        if (ns_here) {
            la.ns_token = st.ns_token;
            la.ns_part = c->ns_part;
            la.ns_value = c->ns_value;
        }
        CUDA_TRY(run_logits(c, la, !last, launches));
        const int P = logit_parts(c, la);
        if (ns_here) {
            CUDA_TRY(launch_nsp(st, c->ns_part, P, c->ns_value, c->stream, true));
            ++launches;
        }
        if (last) {
            const int sel = mode == MODE_BEAM ? SEL_BEAM_INIT : mode == MODE_SAMPLE ? SEL_SAMPLE : SEL_GREEDY;
            CUDA_TRY(launch_select(st, sel, 0, c->logit_part, P, c->masked, 0, c->stream, true));
            ++launches;
        }
    }
    return 0;
}

// The step kernel's plan for S streams of B beams (built once per shape; ok = false when the
// shape or the weights do not fit it, and the chained kernels run instead).
static const w4j_ctx::StepPlanDev *get_step_plan(w4j_ctx *c, int S, int B) {
    auto key = std::make_pair(S, B);
    auto it = c->step_plans.find(key);
    if (it != c->step_plans.end()) return &it->second;
    w4j_ctx::StepPlanDev &pd = c->step_plans[key];
    const int M = S * B, d = c->d, G = c->n_parts;
    if (!c->use_step || M > 8 || !c->x_tmap_ok || c->E.type != WT_F16 || G > c->sm_count) return &pd;
    StepPlanIn in;
    in.G = G;
    in.M = M;
    in.S = S;
    in.B = B;
    in.H = c->H;
    in.A = c->A;
    in.V = c->V;
    in.d = d;
    auto gemv = [&](int in_mode, int out_mode, int l, int K, int N, const float *bias, const float *g, const float *bb,
                    const float *act, float *y, const DMat &W) {
        StepPhase ph{};
        ph.kind = SK_GEMV;
        ph.in_mode = in_mode;
        ph.out_mode = out_mode;
        ph.layer = l;
        ph.K = K;
        ph.N = N;
        ph.bias = bias;
        ph.ln_g = g;
        ph.ln_b = bb;
        ph.act = act;
        ph.y = y;
        in.phases.push_back(ph);
        in.W.push_back(W.h);
        return W.type == WT_F16;
    };
    auto attn = [&](int kind, int l) {
        StepPhase ph{};
        ph.kind = kind;
        ph.layer = l;
        in.phases.push_back(ph);
        in.W.push_back(nullptr);
    };
    bool f16 = true;
    for (int l = 0; l < c->L; ++l) {
        const LayerDev &ly = c->layers[l];
        f16 &= gemv(l == 0 ? SI_EMBED_LN : SI_LN, SO_QKV, l, d, 3 * d, ly.bqkv, ly.ln1g, ly.ln1b, c->x, c->q, ly.qkv);
        attn(SK_SELF, l);
        f16 &= gemv(SI_ACT, SO_RESIDUAL, l, d, d, ly.bo, nullptr, nullptr, c->attn, c->x, ly.o);
        f16 &= gemv(SI_LN, SO_STORE, l, d, d, ly.bxq, ly.ln2g, ly.ln2b, c->x, c->q, ly.xq);
        attn(SK_CROSS, l);
        f16 &= gemv(SI_ACT, SO_RESIDUAL, l, d, d, ly.bxo, nullptr, nullptr, c->attn, c->x, ly.xo);
        f16 &= gemv(SI_LN, SO_GELU, l, d, 4 * d, ly.bm0, ly.ln3g, ly.ln3b, c->x, c->h, ly.m0);
        f16 &= gemv(SI_ACT, SO_RESIDUAL, l, 4 * d, d, ly.bm2, nullptr, nullptr, c->h, c->x, ly.m2);
    }
    {
        StepPhase ph{};
        ph.kind = SK_LOGITS;
        ph.in_mode = SI_LN;
        ph.K = d;
        ph.N = c->V;
        ph.ln_g = c->lng;
        ph.ln_b = c->lnb;
        ph.act = c->x;
        in.phases.push_back(ph);
        in.W.push_back(c->E.h);
    }
    if (!f16) return &pd;
    StepPlanOut out;
    std::string why;
    if (!step_plan_build(in, out, why)) {
        if (c->verbose) fprintf(stderr, "w4j: step kernel plan refused for %d x %d: %s\n", S, B, why.c_str());
        return &pd;
    }
    for (size_t p = 0; p < in.phases.size(); ++p) {
        in.phases[p].box_rows = out.box_rows[p];
        in.phases[p].w = in.W[p];
    }
    StepPhase *dph = nullptr;
    StepChunk *dch = nullptr;
    StepPiece *dpc = nullptr;
    int *dnc = nullptr;
    int4 *dpp = nullptr;
    if (dalloc(c, &dph, in.phases.size()) || dalloc(c, &dch, out.chunks.size()) || dalloc(c, &dpc, out.pieces.size()) ||
        dalloc(c, &dnc, out.n_chunks.size()) || dalloc(c, &dpp, out.pinfo.size()))
        return &pd;
    if (cudaMemcpy(dph, in.phases.data(), in.phases.size() * sizeof(StepPhase), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dch, out.chunks.data(), out.chunks.size() * sizeof(StepChunk), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dpc, out.pieces.data(), out.pieces.size() * sizeof(StepPiece), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dnc, out.n_chunks.data(), out.n_chunks.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dpp, out.pinfo.data(), out.pinfo.size() * sizeof(int4), cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaGetLastError();
        return &pd;
    }
    StepArgs &a = pd.base;
    a = StepArgs{};
    a.phases = dph;
    a.n_phases = (int)in.phases.size();
    a.chunks = dch;
    a.n_chunks = dnc;
    a.pieces = dpc;
    a.pinfo = dpp;
    a.max_chunks = out.max_chunks;
    a.max_pieces = out.max_pieces;
    a.d = d;
    a.H = c->H;
    a.L = c->L;
    a.V = c->V;
    a.C = c->C;
    a.A = c->A;
    a.splits = out.splits;
    a.E = c->E.h;
    a.pos_emb = c->pos_emb;
    a.lng = c->lng;
    a.lnb = c->lnb;
    a.gelu_lut = c->gelu_lut;
    a.M = M;
    a.S = S;
    a.B = B;
    a.x = c->x;
    a.q = c->q;
    a.attn_o = c->attn;
    a.xpart = c->xpart;
    a.xcnt = c->xcnt;
    a.gbar = c->gbar;
    a.gflag = c->gflag;
    a.inflight = c->step_inflight;
    a.bar_mode = c->step_bar_mode;
    pd.ok = true;
    return &pd;
}

// One decode step after the prompt (captured into a graph).
static int enqueue_step(w4j_ctx *c, const CallArgs &a, const CallLayout &Ly, int mode, int parity, long long &launches) {
    DecodeState &st = c->st;
    const int S = a.S, B = a.beam, M = S * B;
    PassArgs pa{};
    pa.M = M;
    pa.tok = st.tok_in;
    pa.pos = st.seq_pos;
    pa.seq_slot = st.seq_slot;
    pa.table = mode == MODE_BEAM ? st.table[parity] : nullptr;
    pa.active = st.active;
    pa.groups = S;
    pa.nq = B;
    pa.cross_stream = c->d_int_area + Ly.cross;
    pa.group_active = B == 1 ? st.active : nullptr;
    pa.self_prefetch = 1;  // each step is its own graph launch: older rows are complete
    LogitsArgs la = logits_args(c, M, st.active);
    la.use_mask = 1;
    la.mask = mask_args(c);
    la.topk = mode == MODE_BEAM ? B + 1 : 0;
    if (mode == MODE_SAMPLE) la.masked_out = c->masked;
    const w4j_ctx::StepPlanDev *sp = c->use_step ? get_step_plan(c, S, B) : nullptr;
    if (sp && sp->ok) {
        // the whole step in one persistent launch (k_step.cu), then the selection
        StepArgs sa = sp->base;
        sa.n_ctx = c->cap;
        sa.sk = c->sk;
        sa.sv = c->sv;
        sa.tok = st.tok_in;
        sa.pos = st.seq_pos;
        sa.slot = st.seq_slot;
        sa.table = pa.table;
        sa.active = st.active;
        sa.cross_stream = pa.cross_stream;
        sa.lg = la;
        sa.err = st.err;
        CUDA_TRY(tmark(c, KC_STEP, true));
        CUDA_TRY(launch_step(sa, c->n_parts, c->xk_tmap, c->xv_tmap, c->step_coop, c->stream));
        CUDA_TRY(tmark(c, KC_STEP, false));
        ++launches;
    } else {
        TRY(run_layers(c, pa, launches));
        CUDA_TRY(run_logits(c, la, true, launches));
    }
    const int sel = mode == MODE_BEAM ? SEL_BEAM : mode == MODE_SAMPLE ? SEL_SAMPLE : SEL_GREEDY;
    CUDA_TRY(tmark(c, KC_SELECT, true));
    CUDA_TRY(launch_select(st, sel, parity, c->logit_part, sp && sp->ok ? c->n_parts : logit_parts(c, la), c->masked, 0,
                           c->stream, true));
    CUDA_TRY(tmark(c, KC_SELECT, false));
    launches += 1;
    return 0;
}

static int get_step_graph(w4j_ctx *c, const CallArgs &a, const CallLayout &Ly, int mode, int parity,
                          cudaGraphExec_t *out, long long &per_step) {
    GraphKey k;
    memset(&k, 0, sizeof k);
    k.mode = mode * 2 + parity;
    k.S = a.S;
    k.B = a.beam;
    k.eot = a.eot;
    k.ts_begin = a.ts_begin;
    k.n_sup = a.n_sup;
    k.max_tokens = a.max_tokens;
    k.ns = c->st.ns_token;
    k.n_prompt = a.n_prompt;
    k.temperature = a.temperature;
    k.seed = a.seed;
    k.time_class = c->time_class;
    long long launches = 0;
    auto it = c->graphs.find(k);
    if (it != c->graphs.end()) {
        *out = it->second;
        per_step = c->graph_launches[k];
        return 0;
    }
    if (c->graphs.size() >= 16) {
        for (auto &kv : c->graphs) cudaGraphExecDestroy(kv.second);
        c->graphs.clear();
        c->graph_launches.clear();
    }
    cudaGraph_t graph = nullptr;
    // the step kernel's plan allocates and uploads: build it before the capture begins
    if (c->use_step && a.S * a.beam <= 8) get_step_plan(c, a.S, a.beam);
    CUDA_TRY(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    c->timing_capture = c->time_class != 0;
    c->tev_used = 0;
    int rc = enqueue_step(c, a, Ly, mode, parity, launches);
    c->timing_capture = false;
    cudaError_t e = cudaStreamEndCapture(c->stream, &graph);
    cudaGraphExec_t exec = nullptr;
    if (rc >= 0 && e == cudaSuccess) {
        e = cudaGraphInstantiate(&exec, graph, 0);
        if (e != cudaSuccess) exec = nullptr;
    }
    if (graph) cudaGraphDestroy(graph);
    if ((rc < 0 || e != cudaSuccess) && c->use_step) {
        // a capture that refuses the step kernel: without the cooperative attribute, then the
        // chained kernels
        cudaGetLastError();
        if (c->verbose)
            fprintf(stderr, "w4j: step graph capture failed (%s; %s), %s\n", cudaGetErrorString(e), g_err.c_str(),
                    c->step_coop ? "retrying without the cooperative attribute" : "using the chained kernels");
        if (c->step_coop) c->step_coop = false;
        else c->use_step = false;
        return get_step_graph(c, a, Ly, mode, parity, out, per_step);
    }
    if (rc < 0) return rc;
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_err(W4J_ERR_CUDA, "graph capture: %s", cudaGetErrorString(e));
    }
    c->graphs[k] = exec;
    c->graph_launches[k] = launches;
    *out = exec;
    per_step = launches;
    return 0;
}

static int read_results(w4j_ctx *c, const CallArgs &a, w4j_result *r) {
    DecodeState &st = c->st;
    const int S = a.S;
    std::vector<int> toks((size_t)S * std::max(a.max_tokens, 1)), lens(S), errw(1);
    std::vector<double> sums(S);
    std::vector<float> nsp(S);
    if (a.max_tokens > 0)
        CUDA_TRY(cudaMemcpyAsync(toks.data(), st.out_tok, (size_t)S * a.max_tokens * 4, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaMemcpyAsync(lens.data(), st.out_len, S * 4, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaMemcpyAsync(sums.data(), st.out_sum, S * 8, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaMemcpyAsync(nsp.data(), st.nsp, S * 4, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaMemcpyAsync(errw.data(), st.err, 4, cudaMemcpyDeviceToHost, c->stream));
    CUDA_TRY(cudaStreamSynchronize(c->stream));
    if (errw[0] == 2) return set_err(W4J_ERR_CUDA, "a bounded device wait ran out (copy never completed)");
    if (errw[0]) return set_err(W4J_ERR_STATE, "device bookkeeping overflow (mask list)");
    for (int s = 0; s < S; ++s) {
        const int n = std::min(lens[s], a.max_tokens);
        if (r->tokens)
            for (int i = 0; i < n; ++i) r->tokens[(size_t)s * a.max_tokens + i] = toks[(size_t)s * a.max_tokens + i];
        if (r->lens) r->lens[s] = n;
        if (r->sum_logprob) r->sum_logprob[s] = sums[s];
        if (r->avg_logprob) r->avg_logprob[s] = n > 0 ? (float)(sums[s] / n) : 0.f;
        if (r->no_speech_prob) r->no_speech_prob[s] = nsp[s];
        if (r->compression) r->compression[s] = w4j_compression_ratio(toks.data() + (size_t)s * a.max_tokens, n);
    }
    return 0;
}

static int decode_impl(w4j_ctx *c, const CallArgs &a, w4j_result *r) {
    CUDA_TRY(cudaSetDevice(c->device));
    TRY(check_ready(c));
    TRY(validate_call(c, a));
    const int mode = a.beam > 1 ? MODE_BEAM : a.temperature > 0.f ? MODE_SAMPLE : MODE_GREEDY;
    c->cancel.store(0);
    c->last_ms = 0;
    c->last_steps = 0;
    c->last_launches = 0;
    c->class_ms = 0;
    c->class_launches = 0;
    if (a.max_tokens == 0) {  // the reference's loop body never runs: empty result
        for (int s = 0; s < a.S; ++s) {
            if (r->lens) r->lens[s] = 0;
            if (r->sum_logprob) r->sum_logprob[s] = 0;
            if (r->avg_logprob) r->avg_logprob[s] = 0;
            if (r->compression) r->compression[s] = 0;
            if (r->no_speech_prob) r->no_speech_prob[s] = 0;
        }
        return W4J_OK;
    }
    TRY(grow_self(c, a.n_prompt + a.max_tokens - 1));
    {
        // the select kernels stage each sequence's history and beam table in shared memory
        DecodeState probe = c->st;
        probe.beam = a.beam;
        const int sel = mode == MODE_BEAM ? SEL_BEAM : SEL_GREEDY;
        if (select_smem_bytes(probe, sel, c->n_parts) > 227 * 1024)
            return set_err(W4J_ERR_ARG, "beam %d with %d positions needs more shared memory than a block has",
                           a.beam, a.n_prompt + a.max_tokens - 1);
    }
    const CallLayout Ly = call_layout(c, a.S, a.n_prompt, a.n_sup);
    TRY(prepare_call(c, a, Ly));
    long long launches = 0;
    CUDA_TRY(cudaEventRecord(c->ev0, c->stream));
    TRY(run_prompt(c, a, Ly, mode, launches));
    // steps 1 .. max_tokens-1 (both loops produce max_tokens decisions in total)
    int steps = 0;
    bool cancelled = false;
    bool snapshot_pending = false;
    for (int step = 1; step < a.max_tokens; ++step) {
        if (c->cancel.load()) {
            cancelled = true;
            break;
        }
        const int parity = mode == MODE_BEAM ? (step - 1) & 1 : 0;
        cudaGraphExec_t g = nullptr;
        long long per = 0;
        TRY(get_step_graph(c, a, Ly, mode, parity, &g, per));
        CUDA_TRY(cudaGraphLaunch(g, c->stream));
        launches += per;
        ++steps;
        if (c->time_class) {  // in-chain durations of this step's launches of the timed class
            CUDA_TRY(cudaStreamSynchronize(c->stream));
            for (int i = 0; i < c->tev_pairs; ++i) {
                float ms = 0.f;
                CUDA_TRY(cudaEventElapsedTime(&ms, c->tev[2 * i], c->tev[2 * i + 1]));
                c->class_ms += ms;
            }
            c->class_launches += c->tev_pairs;
        }
        // every 16 steps look at a done-flag snapshot taken 16 steps earlier (no stall)
        if ((step & 15) == 0) {
            if (snapshot_pending && cudaEventQuery(c->ev1) == cudaSuccess) {
                bool all = true;
                for (int s = 0; s < a.S; ++s) all &= c->h_done[s] != 0;
                if (all) break;
            }
            CUDA_TRY(cudaMemcpyAsync(c->h_done, c->st.done, a.S * 4, cudaMemcpyDeviceToHost, c->stream));
            CUDA_TRY(cudaEventRecord(c->ev1, c->stream));
            snapshot_pending = true;
        }
    }
    CUDA_TRY(launch_finalize(c->st, mode == MODE_BEAM, 0, c->stream));
    ++launches;
    cudaEvent_t stop;
    CUDA_TRY(cudaEventCreate(&stop));
    CUDA_TRY(cudaEventRecord(stop, c->stream));
    CUDA_TRY(cudaEventSynchronize(stop));
    float ms = 0.f;
    cudaEventElapsedTime(&ms, c->ev0, stop);
    cudaEventDestroy(stop);
    TRY(read_results(c, a, r));
    c->last_ms = ms;
    c->last_steps = steps;
    c->last_launches = launches;
    if (cancelled) return set_err(W4J_ERR_CANCELLED, "decode cancelled");
    return W4J_OK;
}

extern "C" int w4j_decode(w4j_ctx *c, const int32_t *slots, int S, const int32_t *prompts, int n_prompt, int32_t eot,
                          int max_tokens, const int32_t *suppress, int n_sup, int32_t ns, float temperature,
                          int32_t ts_begin, uint64_t seed, w4j_result *out) {
    if (!c || !out) return set_err(W4J_ERR_ARG, "w4j_decode: null argument");
    std::lock_guard<std::mutex> g(c->mu);
    CallArgs a{slots, S, prompts, n_prompt, eot, max_tokens, suppress, n_sup, ns, temperature, ts_begin, seed, 1};
    return decode_impl(c, a, out);
}

extern "C" int w4j_decode_beam(w4j_ctx *c, const int32_t *slots, int S, const int32_t *prompts, int n_prompt,
                               int32_t eot, int max_tokens, const int32_t *suppress, int n_sup, int32_t ns,
                               int32_t ts_begin, int beam, w4j_result *out) {
    if (!c || !out) return set_err(W4J_ERR_ARG, "w4j_decode_beam: null argument");
    if (beam < 1) return set_err(W4J_ERR_ARG, "beam size must be >= 1");
    std::lock_guard<std::mutex> g(c->mu);
    CallArgs a{slots, S, prompts, n_prompt, eot, max_tokens, suppress, n_sup, ns, 0.f, ts_begin, 0, beam};
    return decode_impl(c, a, out);
}

// WhisperDecoder.java:435-440
extern "C" int w4j_needs_fallback(float cr, float avg, float nsp) {
    if (cr > 2.4f) return !(nsp > 0.6f && avg < -1.0f);
    return avg < -1.0f && !(nsp > 0.6f);
}

// WhisperDecoder.java:628-647: tokens as little-endian 16-bit pairs, zlib (Deflater default level)
extern "C" float w4j_compression_ratio(const int32_t *tokens, int n) {
    if (!tokens || n <= 0) return 0.f;
    std::vector<unsigned char> bytes((size_t)n * 2);
    for (int i = 0; i < n; ++i) {
        bytes[2 * i] = (unsigned char)(tokens[i] & 0xff);
        bytes[2 * i + 1] = (unsigned char)((tokens[i] >> 8) & 0xff);
    }
    uLongf cap = compressBound((uLong)bytes.size());
    std::vector<unsigned char> outb(cap);
    if (compress2(outb.data(), &cap, bytes.data(), (uLong)bytes.size(), Z_DEFAULT_COMPRESSION) != Z_OK) return 0.f;
    return (float)bytes.size() / (float)std::max<uLongf>(1, cap);
}

extern "C" int w4j_decode_with_fallback(w4j_ctx *c, const int32_t *slots, int S, const int32_t *prompts, int n_prompt,
                                        int32_t eot, int max_tokens, const int32_t *suppress, int n_sup, int32_t ns,
                                        int32_t ts_begin, int beam, uint64_t seed, w4j_result *out, float *out_temp) {
    if (!c || !out || !slots || !prompts) return set_err(W4J_ERR_ARG, "w4j_decode_with_fallback: null argument");
    if (S < 1) return set_err(W4J_ERR_ARG, "n_streams must be >= 1");
    const float temps[] = {0.0f, 0.2f, 0.4f, 0.6f, 0.8f, 1.0f};
    const int mt = std::max(max_tokens, 1);
    std::vector<int> pending(S), best_set(S, 0), finished(S, 0);
    for (int s = 0; s < S; ++s) pending[s] = s;
    std::vector<int32_t> btok((size_t)S * mt), blen(S);
    std::vector<double> bsum(S);
    std::vector<float> bavg(S), bcr(S), bnsp(S), btemp(S);
    for (float temp : temps) {
        const int P = (int)pending.size();
        if (P == 0) break;
        std::vector<int32_t> sl(P), pr((size_t)P * n_prompt), tok((size_t)P * mt), len(P);
        std::vector<double> sum(P);
        std::vector<float> avg(P), cr(P), nsp(P);
        for (int i = 0; i < P; ++i) {
            sl[i] = slots[pending[i]];
            memcpy(&pr[(size_t)i * n_prompt], prompts + (size_t)pending[i] * n_prompt, n_prompt * 4);
        }
        w4j_result r{tok.data(), len.data(), sum.data(), avg.data(), cr.data(), nsp.data()};
        int rc = (beam > 1 && temp == 0.0f)
                     ? w4j_decode_beam(c, sl.data(), P, pr.data(), n_prompt, eot, max_tokens, suppress, n_sup, ns,
                                       ts_begin, beam, &r)
                     : w4j_decode(c, sl.data(), P, pr.data(), n_prompt, eot, max_tokens, suppress, n_sup, ns, temp,
                                  ts_begin, seed, &r);
        if (rc < 0) return rc;
        std::vector<int> next;
        for (int i = 0; i < P; ++i) {
            const int s = pending[i];
            auto take = [&]() {
                best_set[s] = 1;
                memcpy(&btok[(size_t)s * mt], &tok[(size_t)i * mt], mt * 4);
                blen[s] = len[i];
                bsum[s] = sum[i];
                bavg[s] = avg[i];
                bcr[s] = cr[i];
                bnsp[s] = nsp[i];
                btemp[s] = temp;
            };
            if (!w4j_needs_fallback(cr[i], avg[i], nsp[i])) {
                take();
                continue;
            }
            if (!best_set[s] || avg[i] > bavg[s]) take();
            if (temp == 0.0f && cr[i] <= 2.4f) continue;
            if (temp > 0.0f && avg[i] < bavg[s] - 1.0f) continue;
            next.push_back(s);
        }
        pending.swap(next);
    }
    for (int s = 0; s < S; ++s) {
        if (out->tokens) memcpy(out->tokens + (size_t)s * max_tokens, &btok[(size_t)s * mt], std::max(0, blen[s]) * 4);
        if (out->lens) out->lens[s] = blen[s];
        if (out->sum_logprob) out->sum_logprob[s] = bsum[s];
        if (out->avg_logprob) out->avg_logprob[s] = bavg[s];
        if (out->compression) out->compression[s] = bcr[s];
        if (out->no_speech_prob) out->no_speech_prob[s] = bnsp[s];
        if (out_temp) out_temp[s] = btemp[s];
    }
    return W4J_OK;
}

extern "C" int w4j_cancel(w4j_ctx *c) {
    if (!c) return set_err(W4J_ERR_ARG, "null context");
    c->cancel.store(1);
    return W4J_OK;
}

extern "C" int w4j_set_kernel_timing(w4j_ctx *c, int kernel_class) {
    if (!c) return set_err(W4J_ERR_ARG, "null context");
    if (kernel_class < 0 || kernel_class > KC_STEP) return set_err(W4J_ERR_ARG, "kernel class %d", kernel_class);
    std::lock_guard<std::mutex> g(c->mu);
    c->time_class = kernel_class;
    return W4J_OK;
}

extern "C" int w4j_kernel_timing(w4j_ctx *c, double *ms, long long *launches) {
    if (!c) return set_err(W4J_ERR_ARG, "null context");
    if (ms) *ms = c->class_ms;
    if (launches) *launches = c->class_launches;
    return W4J_OK;
}

extern "C" int w4j_last_timing(w4j_ctx *c, double *ms, int *steps, long long *launches) {
    if (!c) return set_err(W4J_ERR_ARG, "null context");
    if (ms) *ms = c->last_ms;
    if (steps) *steps = c->last_steps;
    if (launches) *launches = c->last_launches;
    return W4J_OK;
}

// ---------------------------------------------------------------------------
// op-level entry points
// ---------------------------------------------------------------------------
extern "C" int w4j_op_linear(w4j_ctx *c, const float *x, int M, int K, const void *W, int w_type, int N,
                             const float *bias, const float *ln_g, const float *ln_b, int epilogue, float *y,
                             void *stream) {
    if (!c || !x || !W || !y) return set_err(W4J_ERR_ARG, "w4j_op_linear: null argument");
    if (M < 1 || K < 8 || N < 1 || K % 8) return set_err(W4J_ERR_ARG, "w4j_op_linear: bad shape");
    if (w_type == W4J_GGML_Q8_0 && K % 32) return set_err(W4J_ERR_ARG, "Q8_0 needs K % 32 == 0");
    if ((ln_g == nullptr) != (ln_b == nullptr)) return set_err(W4J_ERR_ARG, "LayerNorm needs both gamma and beta");
    if (epilogue < 0 || epilogue > 2) return set_err(W4J_ERR_ARG, "epilogue must be 0, 1 or 2");
    // one weight row, one activation row and the LayerNorm parameters must fit a block's shared
    // memory (larger M runs in passes)
    if ((size_t)K * (2 + 3 * 4) > 200 * 1024) return set_err(W4J_ERR_ARG, "K too large");
    std::lock_guard<std::mutex> lk(c->mu);  // the op scratch belongs to the context
    CUDA_TRY(cudaSetDevice(c->device));
    GemvArgs g;
    g.W.N = N;
    g.W.K = K;
    if (w_type == W4J_GGML_F16) {
        g.W.type = WT_F16;
        g.W.h = reinterpret_cast<const __half *>(W);
    } else if (w_type == W4J_GGML_Q8_0) {
        g.W.type = WT_Q8;
        g.W.q = reinterpret_cast<const int8_t *>(W);
        g.W.s = reinterpret_cast<const __half *>(g.W.q + (size_t)N * K);
    } else {
        return set_err(W4J_ERR_ARG, "w_type must be F16 (1) or Q8_0 (8)");
    }
    g.bias = bias;
    g.M = M;
    g.in_mode = ln_g ? IN_LN : IN_ACT;
    g.act = x;
    g.ln_g = ln_g;
    g.ln_b = ln_b;
    g.out_mode = epilogue == 0 ? OUT_STORE : epilogue == 1 ? OUT_GELU : OUT_RESIDUAL;
    g.y = y;
    g.gelu_lut = c->gelu_lut;
    cudaStream_t s = stream ? reinterpret_cast<cudaStream_t>(stream) : 0;
    cudaError_t e = cudaErrorNotSupported;
    alignas(64) unsigned char map[128];
    if (c->tc_gemm && M >= 16) {
        if (g.W.type == WT_F16 && gemm_tc_supported(g, c->sm_count) && make_tmap_f16_rows(map, W, N, K)) {
            if (gemm_tc_staged(g)) {
                // the staged activations in the context's op scratch (grown on demand)
                const size_t need = (size_t)act_hilo_rows(M) * K;
                if (need > c->op_hilo_n) {
                    CUDA_TRY(cudaStreamSynchronize(s));
                    dfree(c, c->op_hilo);
                    c->op_hilo = nullptr;
                    c->op_hilo_n = 0;
                    TRY(dalloc(c, &c->op_hilo, need));
                    c->op_hilo_n = need;
                }
                alignas(64) unsigned char bmap[128];
                if (make_tmap_f16_box(bmap, c->op_hilo, act_hilo_rows(M), K, act_hilo_box_rows(M))) {
                    e = launch_act_hilo(g, c->op_hilo, s, false);
                    if (e == cudaSuccess) e = launch_gemm_tc(g, map, bmap, c->sm_count, s, false);
                }
            } else {
                e = launch_gemm_tc(g, map, nullptr, c->sm_count, s, false);
            }
        } else if (g.W.type == WT_Q8 && N % 128 == 0 && K % 64 == 0 && make_tmap_i8_rows(map, W, N, K)) {
            // tiled scales in the context's op scratch (grown on demand, stream-ordered reuse)
            const size_t need = (size_t)N * (K / 32);
            if (need > c->op_st_n) {
                CUDA_TRY(cudaStreamSynchronize(s));
                dfree(c, c->op_st);
                c->op_st = nullptr;
                c->op_st_n = 0;
                TRY(dalloc(c, &c->op_st, need));
                c->op_st_n = need;
            }
            g.W.st = c->op_st;
            if (gemm_tc_supported(g, c->sm_count)) {
                CUDA_TRY(launch_q8_tile_scales(g.W.s, N, K, c->op_st, s));
                e = launch_gemm_tc(g, map, nullptr, c->sm_count, s, false);
            }
        }
    }
    if (e == cudaErrorNotSupported) e = launch_gemv(g, s, false);
    CUDA_TRY(e);
    return W4J_OK;
}

extern "C" int w4j_q8_0_repack(const void *src, int N, int K, void *dst, void *stream) {
    if (!src || !dst || N < 1 || K < 32 || K % 32) return set_err(W4J_ERR_ARG, "w4j_q8_0_repack: bad argument");
    int8_t *q = reinterpret_cast<int8_t *>(dst);
    __half *sc = reinterpret_cast<__half *>(q + (size_t)N * K);
    CUDA_TRY(launch_q8_repack(src, N, K, q, sc, reinterpret_cast<cudaStream_t>(stream)));
    return W4J_OK;
}

// Test hook (w4j_test_withhold_logits_copies): op-level vocabulary passes that still withhold.
static std::atomic<int> g_withhold_logits{0};

static int take_withhold() {
    int n = g_withhold_logits.load();
    while (n > 0 && !g_withhold_logits.compare_exchange_weak(n, n - 1)) {
    }
    return n > 0;
}

extern "C" int w4j_test_withhold_logits_copies(int n_launches) {
    if (n_launches < 0) return set_err(W4J_ERR_ARG, "n_launches must be >= 0");
    g_withhold_logits.store(n_launches);
    return W4J_OK;
}

extern "C" int w4j_op_logits_argmax(w4j_ctx *c, const float *x, int M, const void *E, int V, const float *ln_g,
                                    const float *ln_b, int32_t *out_token, double *out_logprob, void *stream) {
    if (!c || !x || !E || !ln_g || !ln_b || !out_token || !out_logprob)
        return set_err(W4J_ERR_ARG, "w4j_op_logits_argmax: null argument");
    if (M < 1 || M > c->Mbuf) return set_err(W4J_ERR_ARG, "M %d out of [1, %d]", M, c->Mbuf);
    if (V < 1 || V > c->V) return set_err(W4J_ERR_ARG, "V %d out of [1, %d]", V, c->V);
    CUDA_TRY(cudaSetDevice(c->device));
    std::lock_guard<std::mutex> g(c->mu);
    LogitsArgs la;
    la.E.type = WT_F16;
    la.E.N = V;
    la.E.K = c->d;
    la.E.h = reinterpret_cast<const __half *>(E);
    la.x = x;
    la.ln_g = ln_g;
    la.ln_b = ln_b;
    la.M = M;
    la.V = V;
    la.d = c->d;
    la.part = c->logit_part;
    la.err = c->op_err;
    la.withhold = take_withhold();
    const int P = logits_parts_for(V, c->sm_count);
    cudaStream_t s = stream ? reinterpret_cast<cudaStream_t>(stream) : 0;
    alignas(64) unsigned char map[128];
    cudaError_t e = cudaErrorNotSupported;
    if (c->tc_logits && make_tmap_f16_rows(map, E, V, c->d)) {
        // one tcgen05 launch per chunk of at most 32 rows, as in the decode step
        const int chunks = (M + 31) / 32;
        int done = 0;
        e = cudaSuccess;
        for (int i = 0; i < chunks && e == cudaSuccess; ++i) {
            const int m0 = (i * M) / chunks, m1 = ((i + 1) * M) / chunks;
            e = launch_logits_tc(logits_rows(la, m0, m1 - m0, P), map, P, s, false);
            if (e == cudaSuccess) ++done;
        }
        if (e == cudaErrorNotSupported && done > 0) CUDA_TRY(e);
    }
    if (e == cudaErrorNotSupported) e = launch_logits(la, P, s, false);
    CUDA_TRY(e);
    CUDA_TRY(launch_argmax_merge(c->logit_part, P, M, out_token, out_logprob, s));
    CUDA_TRY(launch_err_apply(M, out_token, out_logprob, c->op_err, s));
    return W4J_OK;
}

// ---------------------------------------------------------------------------
// w4j_op_logits_argmax_noalloc: the same vocabulary pass with no context and no allocation.
// The per-block partials and the device error word live in file-scope device arrays, one copy
// per device, whose addresses are looked up once per device.
// ---------------------------------------------------------------------------
static __device__ __align__(256) float g_noalloc_part[W4J_NOALLOC_MAX_ROWS * W4J_NOALLOC_MAX_PARTS * kPartStride];
static __device__ __align__(256) int g_noalloc_err;  // zero at load; cleared by every call's merge

namespace {
constexpr int kNoAllocMaxDevices = 64;
struct NoAllocDevice {
    std::once_flag once;
    int rc = W4J_OK;
    std::string msg;
    float *part = nullptr;
    int *err = nullptr;
    int sms = 0;
    bool tc = true;  // tcgen05 vocabulary pass (off with W4J_NO_TC_LOGITS=1, as for a context)
};
NoAllocDevice g_noalloc_dev[kNoAllocMaxDevices];

// Called once per device: kernel attributes, the SM count and the two symbol addresses.
void noalloc_setup(int device, NoAllocDevice &nd) {
    auto fail = [&](cudaError_t e, const char *what) {
        nd.rc = W4J_ERR_CUDA;
        nd.msg = std::string("w4j_op_logits_argmax_noalloc set-up on device ") + std::to_string(device) + ": " +
                 what + ": " + cudaGetErrorString(e);
    };
    cudaError_t e;
    if (const char *ev = getenv("W4J_NO_TC_LOGITS")) nd.tc = ev[0] == '0';
    if ((e = gemv_prepare()) != cudaSuccess) return fail(e, "kernel attributes");
    if ((e = logits_tc_prepare()) != cudaSuccess) return fail(e, "kernel attributes");
    if ((e = cudaDeviceGetAttribute(&nd.sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess)
        return fail(e, "cudaDeviceGetAttribute");
    if ((e = cudaGetSymbolAddress(reinterpret_cast<void **>(&nd.part), g_noalloc_part)) != cudaSuccess)
        return fail(e, "cudaGetSymbolAddress(partials)");
    if ((e = cudaGetSymbolAddress(reinterpret_cast<void **>(&nd.err), g_noalloc_err)) != cudaSuccess)
        return fail(e, "cudaGetSymbolAddress(error word)");
}
}  // namespace

extern "C" int w4j_op_logits_argmax_noalloc(int device, const float *x, int M, int d, const void *E, int V,
                                            const float *ln_g, const float *ln_b, int32_t *out_token,
                                            double *out_logprob, void *stream) {
    if (!x || !E || !ln_g || !ln_b || !out_token || !out_logprob)
        return set_err(W4J_ERR_ARG, "w4j_op_logits_argmax_noalloc: null argument");
    if (M < 1 || M > W4J_NOALLOC_MAX_ROWS)
        return set_err(W4J_ERR_ARG,
                       "w4j_op_logits_argmax_noalloc: M = %d rows is outside [1, %d], the size of its static "
                       "scratch; use w4j_op_logits_argmax with a context for more rows",
                       M, W4J_NOALLOC_MAX_ROWS);
    if (d < 64 || d > 1280 || d % 64 != 0)
        return set_err(W4J_ERR_ARG, "w4j_op_logits_argmax_noalloc: d = %d must be a multiple of 64 in [64, 1280]", d);
    if (V < 1) return set_err(W4J_ERR_ARG, "w4j_op_logits_argmax_noalloc: V = %d must be positive", V);
    const uintptr_t align = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(E) |
                            reinterpret_cast<uintptr_t>(ln_g) | reinterpret_cast<uintptr_t>(ln_b);
    if (align & 15) return set_err(W4J_ERR_ARG, "w4j_op_logits_argmax_noalloc: x, E, ln_g and ln_b must be 16-byte aligned");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
        return set_err(W4J_ERR_CUDA, "w4j_op_logits_argmax_noalloc: no CUDA device available");
    if (device < 0 || device >= ndev || device >= kNoAllocMaxDevices)
        return set_err(W4J_ERR_ARG, "w4j_op_logits_argmax_noalloc: device %d out of range", device);
    CUDA_TRY(cudaSetDevice(device));
    NoAllocDevice &nd = g_noalloc_dev[device];
    std::call_once(nd.once, noalloc_setup, device, std::ref(nd));
    if (nd.rc != W4J_OK) return set_err(nd.rc, "%s", nd.msg.c_str());
    const int P = logits_parts_for(V, nd.sms);
    if (P > W4J_NOALLOC_MAX_PARTS)
        return set_err(W4J_ERR_ARG, "w4j_op_logits_argmax_noalloc: %d vocabulary blocks exceed the static scratch (%d)", P,
                       W4J_NOALLOC_MAX_PARTS);
    LogitsArgs la;
    la.E.type = WT_F16;
    la.E.N = V;
    la.E.K = d;
    la.E.h = reinterpret_cast<const __half *>(E);
    la.x = x;
    la.ln_g = ln_g;
    la.ln_b = ln_b;
    la.M = M;
    la.V = V;
    la.d = d;
    la.part = nd.part;
    la.err = nd.err;
    la.withhold = take_withhold();
    cudaStream_t s = stream ? reinterpret_cast<cudaStream_t>(stream) : 0;
    alignas(64) unsigned char map[128];
    cudaError_t e = cudaErrorNotSupported;
    if (nd.tc && make_tmap_f16_rows(map, E, V, d)) e = launch_logits_tc(la, map, P, s, false);
    if (e == cudaErrorNotSupported) e = launch_logits(la, P, s, false);
    CUDA_TRY(e);
    CUDA_TRY(launch_argmax_merge_status(nd.part, P, M, out_token, out_logprob, nd.err, s));
    return W4J_OK;
}

// ---------------------------------------------------------------------------
// chunked transcription (WhisperModel.transcribeChunked, WhisperModel.java:334-427)
// ---------------------------------------------------------------------------
namespace {
struct TsOut {
    w4j_transcript *t;
    int add(float start, float end, const std::vector<int32_t> &toks) {
        if (t->n_segments >= t->segments_cap || t->n_tokens + (int)toks.size() > t->tokens_cap)
            return set_err(W4J_ERR_ARG, "transcript buffers too small (%d segments, %d tokens)", t->segments_cap,
                           t->tokens_cap);
        w4j_segment &s = t->segments[t->n_segments++];
        s.start = start;
        s.end = end;
        s.token_begin = t->n_tokens;
        s.n_tokens = (int32_t)toks.size();
        for (int32_t v : toks) t->tokens[t->n_tokens++] = v;
        return 0;
    }
};

std::vector<int32_t> text_tokens(const int32_t *tok, int n, int ts_begin) {  // filterTextTokens (:503-505)
    std::vector<int32_t> r;
    for (int i = 0; i < n; ++i)
        if (tok[i] < ts_begin) r.push_back(tok[i]);
    return r;
}

// parseTimestampSegments (:430-490)
int timestamp_segments(const int32_t *tok, int n, int ts_begin, float offset, float precision, TsOut &out) {
    std::vector<int> ts;
    for (int i = 0; i < n; ++i)
        if (tok[i] >= ts_begin) ts.push_back(i);
    if (ts.size() < 2) {
        const std::vector<int32_t> text = text_tokens(tok, n, ts_begin);
        if (!text.empty()) {
            const float end = ts.empty() ? offset + 30.0f : offset + (float)(tok[ts[0]] - ts_begin) * precision;
            TRY(out.add(offset, end, text));
        }
        return 0;
    }
    int last = 0;
    for (size_t i = 0; i + 1 < ts.size(); ++i) {
        if (ts[i + 1] != ts[i] + 1) continue;
        const int slice_end = ts[i + 1];
        float start = offset, end = offset + 30.0f;
        for (int j = last; j < slice_end; ++j)
            if (tok[j] >= ts_begin) {
                start = offset + (float)(tok[j] - ts_begin) * precision;
                break;
            }
        for (int j = slice_end - 1; j >= last; --j)
            if (tok[j] >= ts_begin) {
                end = offset + (float)(tok[j] - ts_begin) * precision;
                break;
            }
        const std::vector<int32_t> text = text_tokens(tok + last, slice_end - last, ts_begin);
        if (!text.empty()) TRY(out.add(start, end, text));
        last = slice_end;
    }
    return 0;
}
}  // namespace

extern "C" int w4j_transcribe(w4j_ctx *c, const float *audio, int n_samples, const w4j_transcribe_opts *o,
                              w4j_transcript *out) {
    if (!c || !o || !out || (!audio && n_samples > 0) || !o->sot || o->n_sot < 1 || !out->tokens || !out->segments)
        return set_err(W4J_ERR_ARG, "w4j_transcribe: null argument");
    if (n_samples < 0) return set_err(W4J_ERR_ARG, "n_samples %d", n_samples);
    out->n_tokens = out->n_segments = out->n_windows = 0;
    const w4j_dims &dm = c->dims;
    const int n_frames = 2 * dm.n_audio_ctx, stride = n_frames / dm.n_audio_ctx, hop = 160;
    const int chunk = n_frames * hop;
    const float precision = (float)stride * 160.0f / 16000.0f;
    const int total_frames = (int)((float)n_samples / 160.0f);
    const float duration = (float)n_samples / 16000.0f;
    const bool with_ts = o->ts_begin > 0;
    {  // the recording on the device once
        std::lock_guard<std::mutex> g(c->mu);
        CUDA_TRY(cudaSetDevice(c->device));
        TRY(check_ready(c));
        if (dm.n_audio_state != c->d) return set_err(W4J_ERR_ARG, "n_audio_state differs from n_text_state");
        TRY(enc_prepare(c));
        TRY(audio_reserve(c, n_samples));
        if (n_samples > 0)
            CUDA_TRY(cudaMemcpyAsync(c->enc.audio, audio, (size_t)n_samples * 4, cudaMemcpyHostToDevice, c->stream));
    }
    std::vector<int32_t> base(o->sot, o->sot + o->n_sot);  // buildPrompt (:573-582)
    if (!with_ts) base.push_back(o->no_timestamps);
    std::vector<int32_t> prev;
    const int max_tok_full = dm.n_text_ctx / 2;
    std::vector<int32_t> tok((size_t)max_tok_full);
    TsOut so{out};
    int seek = 0;
    c->cancel.store(0);
    while (seek < total_frames) {
        if (c->cancel.load()) break;
        const float offset = (float)seek * 160.0f / 16000.0f;
        const int seg_size = std::min(n_frames, total_frames - seek);
        const int a0 = seek * hop, n_valid = std::min(n_samples - a0, chunk);
        {  // log-mel of the zero-filled 30 s window, encoder, cross K/V of stream 0 (:352-366)
            std::lock_guard<std::mutex> g(c->mu);
            CUDA_TRY(cudaSetDevice(c->device));
            TRY(logmel_device(c, c->enc.audio + a0, std::max(n_valid, 0), chunk));
            TRY(enc_finish(c, nullptr, 0));
        }
        ++out->n_windows;
        // buildPromptWithContext (:507-530)
        std::vector<int32_t> prompt = base;
        if (o->condition_on_previous && !prev.empty()) {
            const int max_prev = (dm.n_text_ctx / 2 - 1) - (int)base.size() - 1;
            if (max_prev > 0) {
                const int n = std::min((int)prev.size(), max_prev);
                prompt.assign(1, o->sot_prev);
                prompt.insert(prompt.end(), prev.end() - n, prev.end());
                prompt.insert(prompt.end(), base.begin(), base.end());
            }
        }
        int max_tokens = max_tok_full;
        if (seg_size < n_frames) max_tokens = std::max(8, max_tokens * seg_size / n_frames);
        int32_t len = 0;
        double sum = 0;
        float avg = 0, cr = 0, nsp = 0, temp = 0;
        auto run = [&](const std::vector<int32_t> &p) -> int {
            const int32_t slot = 0;
            w4j_result r{tok.data(), &len, &sum, &avg, &cr, &nsp};
            return w4j_decode_with_fallback(c, &slot, 1, p.data(), (int)p.size(), o->eot, max_tokens, o->suppress,
                                            o->n_suppress, o->no_speech, o->ts_begin, std::max(1, o->beam_size), o->seed,
                                            &r, &temp);
        };
        TRY(run(prompt));
        if (o->condition_on_previous && !prev.empty() && avg < -1.0f) {  // :383-391
            TRY(run(base));
            prev.clear();
        }
        if (nsp > 0.6f && avg < -1.0f) {  // no speech (:396-399)
            seek += seg_size;
            continue;
        }
        if (with_ts) {  // :402-413
            TRY(timestamp_segments(tok.data(), len, o->ts_begin, offset, precision, so));
            int last_ts = -1;
            for (int i = len - 1; i >= 0; --i)
                if (tok[i] >= o->ts_begin) {
                    last_ts = tok[i] - o->ts_begin;
                    break;
                }
            seek += last_ts > 0 ? std::max(last_ts * stride, stride) : seg_size;
        } else {  // one segment per window (:414-421)
            if (len > 0) TRY(so.add(offset, std::min(offset + (float)seg_size * 160.0f / 16000.0f, duration),
                                    std::vector<int32_t>(tok.begin(), tok.begin() + len)));
            seek += seg_size;
        }
        if (o->condition_on_previous) prev.assign(tok.begin(), tok.begin() + len);  // :424-426
    }
    return c->cancel.load() ? set_err(W4J_ERR_CANCELLED, "cancelled") : W4J_OK;
}
