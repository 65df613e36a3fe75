// Host-side declarations shared by the eva_b200 CUDA translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/eva_moe.h"

namespace eva {

constexpr int RUN_ROWS = 8;          // slots of one expert per run (MMA N dimension)
constexpr int PARTA_ITEMS = 4096;    // split-k partial buffers of the gate/up stage
constexpr int ROUTER_KSLICE = 512;   // k elements per router GEMV warp
constexpr int ROUTER_TC_MIN_ROWS = 33;   // tensor-core router GEMM from this many tokens (bf16 inputs)

// Byte offsets of the workspace regions for calls of up to max_rows tokens.
struct WsLayout {
    int max_rows, S, R, imax, nchA, nchH, ks_router;
    size_t status, counters, n_counters, runs, run_expert, estart, slot_act, tok_expect;
    size_t logits, wsplit, idx, w, xrot, act, dpart, partA, xsum, asum, total;
    size_t tstart, pxg, pxu, pap;   // prefill: tile prefix, sorted rotated inputs, sorted down inputs
    size_t pscan;                   // multi-CTA permutation: per-chunk expert counts and prefixes
    size_t tmaps;                   // decode kernel: per-CTA tensor maps of the items in flight
    int max_split;   // largest gate/up k-split the partial buffer allows (1 = none)
    int hpad, ipad;  // row widths (halves) of the fragment-layout input buffers (one stage of slack)
};

// allow_split = false leaves out the split-k partial buffer (gate/up items are then never split);
// routing = false leaves out the router's regions (weight split planes, slice partial logits), which
// come last, so every other offset is the same either way. tensor_core = false leaves out the
// tensor-core path's sorted input copies (pxg, pxu, pap) for calls that always take the decode kernel.
WsLayout ws_layout(const EvaMoeShape& s, int max_rows, bool allow_split = true, bool routing = true,
                   bool tensor_core = true);

// Counter block layout inside `counters` (int32 indices).
struct CtrLayout {
    int work, ctr0, ctrA, ctrAk, ctrB, n;
};
CtrLayout ctr_layout(const WsLayout& L);

// Router logits into `part` ([ks][M][E] slice partials, *ks_used slices). wsplit: 3 E H bf16 of
// workspace for the tensor-core path (may be null: SIMT path); status: the workspace status word.
cudaError_t launch_router_logits(const void* x, int x_bf16, int M, int H, int E, const float* W, float* part,
                                 void* wsplit, int* status, int* ks_used, cudaStream_t stream);
// Tensor-core router GEMM: k slices for M tokens (0: shape not handled; kper_out: k per slice),
// partial-logit rows a workspace for up to max_rows tokens holds, and the launch.
int router_tc_split(int M, int H, int E, int* kper_out);
size_t router_part_rows(int max_rows, int H, int E);
bool router_tc_usable(const void* x, int x_bf16, int M, int H, int E, const void* wsplit);
cudaError_t launch_router_tc(const void* x, int M, int H, int E, const float* W, void* wsplit, float* part, int* status,
                             int* ks_used, cudaStream_t stream);
cudaError_t launch_topk(const EvaMoeShape& s, const float* part, int ks, int M, const float* bias,
                        float* logits_out, int32_t* idx, float* w, cudaStream_t stream);

struct PermuteArgs {
    const void* sel;
    int sel64;
    const float* rw;
    int M, topk, n_local, capacity, has_shared, H;
    int sh0, shn;               // the shared expert applies to tokens sh0 .. sh0 + shn - 1
    const int64_t* tables[9];   // may be null: no pointer validation
    int32_t* runs;
    int32_t* run_expert;        // may be null
    int32_t* estart;            // may be null
    int32_t* tstart;            // may be null: [E + 2] prefix of PF_TILE_ROWS-row tiles per expert (+ shared)
    int32_t* slot_act;          // may be null
    int32_t* tok_expect;        // may be null
    int32_t* counters;          // zeroed when non-null
    int n_counters;
    int32_t* status;            // may be null
    float* out_f32;             // rows with no arrivals are zeroed (may be null)
    void* out_bf16;
    int32_t* scratch;           // may be null: permute_scratch_ints(M, E) ints for the multi-CTA form
};
cudaError_t launch_permute(const PermuteArgs& a, cudaStream_t stream);
// Tokens per CTA of the multi-CTA permutation and the scratch it needs for M tokens, E experts.
constexpr int PERM_TOK_CHUNK = 128;
inline size_t permute_scratch_ints(int M, int E)
{
    return static_cast<size_t>((M + PERM_TOK_CHUNK - 1) / PERM_TOK_CHUNK) * E + 2 * (static_cast<size_t>(E) + 1) + 4;
}

struct ExpertsArgs {
    const EvaMoeShape* shape;
    const void* x;
    int x_bf16, M;
    const void* sel;
    int sel64;
    const float* rw;
    const int64_t* tables[9];
    int64_t shared[9];
    void* ws;
    WsLayout L;
    float* out_f32;
    void* out_bf16;
    int sh0, shn;               // shared-expert token window
};
cudaError_t launch_experts(const ExpertsArgs& a, cudaStream_t stream);
cudaError_t launch_prefill(const ExpertsArgs& a, cudaStream_t stream);

constexpr int DEC_MAX_CTAS = 256;       // decode kernel grid cap (tensor-map slots per CTA in the workspace)
constexpr int DEC_MAP_SETS = 6;         // tensor-map sets per CTA: one per item, reused after (ring stages + 1) items
constexpr int PREFILL_MIN_ROWS = 129;   // eva_moe_experts takes the tensor-core path from this many rows
constexpr int PF_TILE_ROWS = 256;       // rows of one expert per tensor-core CTA (two 128-row MMA halves)

// Argument checks of the fused expert entry points (pointers, alignment, shared-expert tables):
// EVA_OK or EVA_ERR_INVALID; no device work.
int experts_validate(const EvaMoeShape* shape, const void* x, int32_t M, const void* sel, const float* rw,
                     const int64_t* const* tables, const int64_t* shared, const float* out_f32, const void* out_bf16);

// Permutation + fused experts on a caller-provided workspace laid out by
// ws_layout(shape, M, allow_split, false, path != 1): path 1 (decode kernel only) needs no
// tensor-core buffers.
int experts_impl(const EvaMoeShape* shape, const void* x, int32_t x_is_bf16, int32_t M, const void* sel,
                 int32_t sel_is_i64, const float* rw, const int64_t* const* tables, const int64_t* shared,
                 void* workspace, size_t workspace_bytes, float* out_f32, void* out_bf16, cudaStream_t st,
                 bool allow_split = true, int path = 0,     // path: 0 by size, 1 decode kernel, 2 tensor-core
                 int shared_row0 = 0, int shared_rows = -1); // shared expert on rows row0 .. row0 + rows - 1 (-1: all)

cudaError_t launch_dequant(const void* trellis, int in, int out, int K, uint16_t* w, cudaStream_t stream);

int num_sms();

// Pair-MMA layout self-test (prefill.cu), M = 256 or 128: out[2][128][256] u32.
cudaError_t pf_pair_selftest_launch(int M, uint32_t* out, int* status, cudaStream_t stream);

}  // namespace eva
