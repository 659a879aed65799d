// k_step.cuh — the persistent decode-step kernel (k_step.cu): plan structures and host entry points.
#pragma once
#include <string>
#include <vector>

#include <cuda.h>

#include "w4j_internal.cuh"

namespace w4j {

constexpr int kStepThreads = 256, kStepWarps = kStepThreads / 32;
constexpr int kStepMaxM = 8;                 // sequences (streams x beams) of a step
constexpr unsigned kStepRing = 128 * 1024;   // byte ring for the step's copies
constexpr int kStepBars = 16;                // ring mbarriers (chunk i uses i % 16)
constexpr int kStepSeg = 1280;               // activation columns staged at a time
constexpr unsigned kStepPiece = 48 * 1024;   // bytes of one weight piece (at most)
constexpr unsigned kBox = kAttnKeyTile * kHeadDim * 2;  // one [128 x 64] f16 key tile: 16 KB
constexpr int kRowPadPw = 24;  // halves per row of a warp's P^T block (kPwPad of attn_tile.cuh)
constexpr int kMaxDynSmem = 227 * 1024;  // opt-in shared memory of one block on sm_100

enum StepKind : int { SK_GEMV = 0, SK_SELF = 1, SK_CROSS = 2, SK_LOGITS = 3 };
enum StepIn : int { SI_ACT = 0, SI_LN = 1, SI_EMBED_LN = 2 };
enum StepOut : int { SO_QKV = 0, SO_STORE = 1, SO_GELU = 2, SO_RESIDUAL = 3 };

// consumption-ordered copies of one block (the kernel keeps its block's list in shared memory)
struct StepChunk {
    unsigned long long src;  // kind 0: global address of the weight rows (one bulk copy); kind 1: key row of
                             // the first box without the stream term, (layer * H + head) * A + first key
    unsigned bytes;          // bytes the chunk's mbarrier expects
    int wait_rel;            // chunks consumed before this one may be issued
    unsigned off;            // ring offset (1024-aligned)
    unsigned char kind;      // 0 weight rows, 1 encoder K / V boxes
    unsigned char s;         // kind 1: stream index
    unsigned char nbox;      // kind 1: boxes per K and per V
    unsigned char pad;
};
static_assert(sizeof(StepChunk) == 24, "StepChunk is copied to shared memory as three 8-byte words");

struct StepPiece {
    int chunk;  // ring chunk (-1: none)
    int r0, r1; // GEMV / logits: matrix rows; cross: keys [r0, r1); self: item (sequence * H + head)
    int item;   // cross: pair * splits + split
};

struct StepPhase {
    int kind, in_mode, out_mode, layer, K, N;
    int box_rows;      // GEMV / vocabulary: weight rows per piece (a piece is [rows x K] f16, row-major)
    const __half *w;   // GEMV / vocabulary: the weight matrix, f16 [N][K]
    const float *bias, *ln_g, *ln_b;
    const float *act;  // input rows (SI_ACT, SI_LN)
    float *y;          // output rows
};

struct StepArgs {
    // plan (device)
    const StepPhase *phases;
    int n_phases;
    const StepChunk *chunks;      // [G][max_chunks]
    const int *n_chunks;          // [G]
    const StepPiece *pieces;      // [G][max_pieces]
    const int4 *pinfo;            // [G][n_phases + 1]: first piece, first and end row of the block's slice
    int max_chunks, max_pieces;
    // model
    int d, H, L, V, C, A, n_ctx, splits;
    const __half *E;
    const float *pos_emb, *lng, *lnb, *gelu_lut;
    __half *sk, *sv;              // self K / V caches [slot][layer][head][n_ctx][64]
    // sequences: M = S * B, sequence m belongs to stream m / B
    int M, S, B;
    const int *tok, *pos, *slot, *table, *active, *cross_stream;
    float *x, *q, *attn_o, *xpart;
    int *xcnt;                    // [S * H] finished splits per pair (the last one resets it)
    unsigned *gbar;               // grid barrier counter (reset by the select kernel)
    unsigned *gflag;              // per block, 128 bytes apart: the last barrier it may pass (reset likewise)
    LogitsArgs lg;                // vocabulary phase (x, part, masks, top-k; E, V, d)
    unsigned inflight;            // bytes of copies a block keeps in flight (at least one copy)
    int bar_mode;                 // grid barrier: 0 last arriver releases per-block flags, 1 all poll the counter
    int *err;
};

// Input of the host planner: phases in execution order and, per phase, its weight matrix (f16
// [N][K] rows; GEMV and vocabulary phases).
struct StepPlanIn {
    int G = 0, M = 0, S = 0, B = 0, H = 0, A = 0, V = 0, d = 0;
    std::vector<StepPhase> phases;
    std::vector<const __half *> W;
};

struct StepPlanOut {
    int splits = 0, max_chunks = 0, max_pieces = 0;
    std::vector<int> box_rows;       // per phase (weight phases)
    std::vector<StepChunk> chunks;   // [G][max_chunks]
    std::vector<StepPiece> pieces;   // [G][max_pieces]
    std::vector<int> n_chunks;       // [G]
    std::vector<int4> pinfo;         // [G][phases + 1]
};

// false (with the reason) when the step does not fit the kernel (too many streams, rows, ...)
bool step_plan_build(const StepPlanIn &in, StepPlanOut &out, std::string &why);
size_t step_smem(int max_chunks);
cudaError_t step_prepare();
// G blocks (one per SM, all resident); kmap / vmap: make_tmap_f16_rows maps of the cross K / V caches
cudaError_t launch_step(const StepArgs &a, int G, const void *kmap, const void *vmap, bool coop, cudaStream_t s);

}  // namespace w4j
