/*
 * eva_moe.h - C ABI of the B200 (sm_100a) DeepSeek MoE hot path.
 *
 * Plain pointers and sizes only. Device pointers are CUDA device addresses; `stream` is a
 * cudaStream_t passed as void*. Every entry point is asynchronous on `stream`, performs no
 * host<->device synchronisation and no allocation, and returns an EVA_* status for argument and
 * launch errors. Device-side problems (expert id outside the tables, an unbound pointer, a bounded
 * wait that gave up) are OR-ed into a status word inside the workspace; read it with
 * eva_moe_read_status() after the stream has reached that point.
 *
 * Reference interfaces replaced (paths within the Findddx/eva project):
 *   eva_moe_experts     runtime/ds41/csrc/moe_coop2048/binding.cu:73-145 `run(x, sel, rw, tables[9],
 *                       scratch[8], k, limit, check_bounds)` (also moe_coop512/binding.cu:71-146 and
 *                       moe_coop3072/moe_coop3072.cu:42-176): routed EXL3 experts + combine
 *                       (+ the shared expert, which the reference runs separately through
 *                       exllamav3 LinearEXL3, runtime/ds41/model.py:441-452).
 *   eva_moe_permute     runtime/ds41/csrc/moe_coop2048/binding.cu:149-174 `prepare_routes(sel, rw, runs,
 *                       capacity, n_local)`: the int32 run table [n_runs, 0, run_start[S+1], order[S]].
 *   eva_moe_route       runtime/ds41/model.py:404-416 `Block.route(x)` (FP32 logits, scoring, biased top-k,
 *                       normalised weights).
 *   eva_moe_topk        the scoring/top-k half of Block.route, from given FP32 logits.
 *   eva_moe_forward     runtime/ds41/model.py:454-499 `Block.experts(x)` (route + experts + shared).
 *   eva_exl3_dequant    the vendored ExLlamaV3 dq_dispatch<K, mul1> decode
 *                       (runtime/ds41/csrc/moe_coop2048/vendor/quant/exl3_dq.cuh:287-330), as a
 *                       standalone projection dequantiser.
 */
#ifndef EVA_MOE_H
#define EVA_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* return codes */
#define EVA_OK 0
#define EVA_ERR_INVALID 1      /* bad argument: shape, null pointer, unsupported K, alignment */
#define EVA_ERR_CUDA 2         /* a CUDA launch or runtime call failed */
#define EVA_ERR_WORKSPACE 3    /* workspace smaller than eva_moe_workspace_bytes() */

/* device status bits (eva_moe_read_status) */
#define EVA_STATUS_BAD_EXPERT 1   /* a selected expert id is outside [0, n_local) or has a zero pointer */
#define EVA_STATUS_TIMEOUT 2      /* a bounded device wait gave up (results of that call are invalid) */
#define EVA_STATUS_CAPACITY 4     /* more rows than the workspace was sized for */

/* router kinds */
#define EVA_ROUTER_SOFTMAX 0       /* DeepSeek-V2-Lite greedy top-k over softmax probabilities */
#define EVA_ROUTER_SIGMOID 1       /* DeepSeek-V3: sigmoid + bias, group-limited top-k */
#define EVA_ROUTER_SQRTSOFTPLUS 2  /* eva DS4.1: sqrt(softplus) + bias top-k (model.py:404-416) */

/* activation modes of the gated MLP */
#define EVA_ACT_CLAMP_AFTER 0     /* silu(g) then clamp (MoE coop act_gate, exl3_moe_coop_kernel.cuh:115-129) */
#define EVA_ACT_CLAMP_BEFORE 1    /* clamp then silu(g) * u (torch swiglu, kernels.py:213-217) */

typedef struct EvaMoeShape {
    int32_t hidden;        /* H, multiple of 256 */
    int32_t inter;         /* routed expert intermediate width I, multiple of 128 */
    int32_t n_experts;     /* routed experts in the pointer tables (n_local) */
    int32_t topk;          /* selected experts per token, 1..32 */
    int32_t bits;          /* EXL3 K of the routed experts: 2, 3 or 4 */
    int32_t shared_inter;  /* shared expert intermediate width, 0 = no shared expert */
    int32_t shared_bits;   /* EXL3 K of the shared expert */
    int32_t router;        /* EVA_ROUTER_* */
    int32_t n_group;       /* group-limited routing: number of groups (1 = off) */
    int32_t topk_group;    /* groups kept per token */
    int32_t norm_topk;     /* renormalise the selected weights (sum + 1e-20) */
    int32_t act_routed;    /* EVA_ACT_* for routed experts */
    int32_t act_shared;    /* EVA_ACT_* for the shared expert */
    float route_scale;     /* routed_scaling_factor / route_scale */
    float swiglu_limit;    /* 0 = no clamp */
} EvaMoeShape;

/* Bytes of device workspace needed for calls of up to `max_rows` tokens. */
size_t eva_moe_workspace_bytes(const EvaMoeShape* shape, int32_t max_rows);

/* Clears the workspace's status word (asynchronous). */
int eva_moe_clear_status(void* workspace, void* stream);

/* Copies the status word to *status_host (synchronises `stream`). */
int eva_moe_read_status(const void* workspace, int32_t* status_host, void* stream);

/* Router: logits_out (may be NULL) float [M][E]; idx_out int32 [M][topk]; w_out float [M][topk].
 * x is bf16 (x_is_bf16 = 1) or fp16 [M][H]; router_w float [E][H]; router_b float [E] (NULL = 0). */
int eva_moe_route(const EvaMoeShape* shape, const void* x, int32_t x_is_bf16, int32_t M,
                  const float* router_w, const float* router_b, float* logits_out,
                  int32_t* idx_out, float* w_out, void* workspace, size_t workspace_bytes, void* stream);

/* Scoring + top-k from FP32 logits [M][E] (router_b may be NULL). */
int eva_moe_topk(const EvaMoeShape* shape, const float* logits, int32_t M, const float* router_b,
                 int32_t* idx_out, float* w_out, void* stream);

/* Permutation. sel: [M][topk] int32 (sel_is_i64 = 0) or int64; rw: float [M][topk] (0 = inactive).
 * runs: int32 [2 + 2 * capacity * topk + 1] in the reference layout
 *       [n_runs, 0, run_start[S + 1], order[S]], S = capacity * topk, unused entries zero.
 * expert_start (may be NULL): int32 [n_local + 1], exclusive prefix of active slots per expert. */
int eva_moe_permute(const EvaMoeShape* shape, const void* sel, int32_t sel_is_i64, const float* rw,
                    int32_t M, int32_t capacity, int32_t* runs, int32_t* expert_start, void* stream);

/* The same table with a caller workspace (eva_moe_workspace_bytes for >= M rows): for batches above
 * 256 tokens it is built by a multi-CTA form (per-chunk counts, one scan, per-chunk scatter) instead
 * of one CTA. Same result, bit for bit. No counterpart in the reference (its prepare_routes is
 * eva_moe_permute). */
int eva_moe_permute_ws(const EvaMoeShape* shape, const void* sel, int32_t sel_is_i64, const float* rw,
                       int32_t M, int32_t capacity, int32_t* runs, int32_t* expert_start, void* workspace,
                       size_t workspace_bytes, void* stream);

/* Fused experts: permutation + rotation + gate/up + activation + down + routed combine + shared
 * expert, one persistent launch after the permutation.
 *   x:        [M][H] bf16 or fp16 (x_is_bf16)
 *   sel, rw:  as eva_moe_permute
 *   tables:   host array of 9 device pointers, each an int64 [n_experts] table of device addresses in
 *             the reference row order [g.trellis, g.suh, g.svh, u.trellis, u.suh, u.svh, d.trellis,
 *             d.suh, d.svh] (runtime/ds41/cache.py:1864-1887); 0 = unbound
 *   shared:   host array of 9 device addresses of the shared expert (NULL when shape->shared_inter == 0)
 *   out_f32:  float [M][H] or NULL; out_bf16: bf16 [M][H] or NULL (at least one)
 */
int eva_moe_experts(const EvaMoeShape* shape, const void* x, int32_t x_is_bf16, int32_t M,
                    const void* sel, int32_t sel_is_i64, const float* rw,
                    const int64_t* const* tables, const int64_t* shared,
                    void* workspace, size_t workspace_bytes, float* out_f32, void* out_bf16, void* stream);

/* eva_moe_experts forced onto one of its two implementations (eva_moe_experts picks by row count:
 * the tensor-core path from 129 rows on). Same arguments and results.
 *   _decode:  the persistent register-decode GEMV kernel (mma.sync), best for decode batches
 *   _prefill: expert-sorted tcgen05 grouped GEMMs with TMEM accumulators (prefill) */
int eva_moe_experts_decode(const EvaMoeShape* shape, const void* x, int32_t x_is_bf16, int32_t M,
                           const void* sel, int32_t sel_is_i64, const float* rw,
                           const int64_t* const* tables, const int64_t* shared,
                           void* workspace, size_t workspace_bytes, float* out_f32, void* out_bf16, void* stream);
int eva_moe_experts_prefill(const EvaMoeShape* shape, const void* x, int32_t x_is_bf16, int32_t M,
                            const void* sel, int32_t sel_is_i64, const float* rw,
                            const int64_t* const* tables, const int64_t* shared,
                            void* workspace, size_t workspace_bytes, float* out_f32, void* out_bf16, void* stream);

/* eva_moe_experts with the shared expert applied to rows shared_row0 .. shared_row0 + shared_rows - 1
 * only (other rows get their routed experts alone; rows with neither are zero). An expert-parallel
 * rank uses it to run its own tokens' shared expert in the same launch as the rows other ranks sent
 * it (its own tokens are one contiguous segment of the received rows). */
int eva_moe_experts_window(const EvaMoeShape* shape, const void* x, int32_t x_is_bf16, int32_t M,
                           const void* sel, int32_t sel_is_i64, const float* rw,
                           const int64_t* const* tables, const int64_t* shared,
                           int32_t shared_row0, int32_t shared_rows, void* workspace, size_t workspace_bytes,
                           float* out_f32, void* out_bf16, void* stream);

/* Whole layer: eva_moe_route + eva_moe_experts. idx_out / w_out / logits_out may be NULL.
 * eva_moe_route, eva_moe_experts(_decode/_prefill/_window) and eva_moe_forward only queue work on
 * `stream` (no host synchronisation, no allocation), so they can be captured in a CUDA graph and the
 * graph replayed with new data at the captured addresses; calls that share a workspace must not run
 * concurrently, captured or not. (The reference's binding refuses capture,
 * runtime/ds41/csrc/moe_coop2048/binding.cu:83-85.) */
int eva_moe_forward(const EvaMoeShape* shape, const void* x, int32_t x_is_bf16, int32_t M,
                    const float* router_w, const float* router_b,
                    const int64_t* const* tables, const int64_t* shared,
                    void* workspace, size_t workspace_bytes, float* out_f32, void* out_bf16,
                    float* logits_out, int32_t* idx_out, float* w_out, void* stream);

/* Dequantise one EXL3 projection: trellis int16 [in/16][out/16][16K] -> fp16 bits [in][out]. */
int eva_exl3_dequant(const void* trellis, int32_t in_features, int32_t out_features, int32_t bits,
                     uint16_t* w_out, void* stream);

/* Size of the fixed device scratch behind eva_moe_experts_noalloc: 16 MiB, reserved on every GPU that
 * loads this library until the process exits. */
#define EVA_NOALLOC_SCRATCH_BYTES (16u << 20)

/* eva_moe_experts without a workspace: it allocates nothing. No counterpart in the reference.
 *
 * For callers that cannot allocate device memory: a serving runtime that has already reserved the
 * GPU's memory in its own pool (a cudaMalloc would fail or fragment it), a plugin host that hands
 * over input and output buffers but no allocator, or a latency-critical loop that must not call
 * cudaMalloc because it can synchronise the device. The caller passes inputs and outputs exactly as
 * for eva_moe_experts; the scratch is a file-scope device array of EVA_NOALLOC_SCRATCH_BYTES.
 *   - Calls whose scratch would exceed that size are rejected with EVA_ERR_WORKSPACE (for the
 *     DeepSeek-V3 shape this allows up to 27 tokens per call, DeepSeek-V2-Lite 90, eva's own
 *     H5120 / 384-expert shape 47). Every call takes the decode kernel, whatever its row count.
 *   - Argument errors (EVA_ERR_INVALID) and the size check (EVA_ERR_WORKSPACE) are reported before
 *     any device call.
 *   - The first call on each device looks up the array's device address (cudaGetSymbolAddress)
 *     with that device current; make that first call before any stream capture.
 *   - All calls share the one array, which keeps the previous call's contents. Each call clears
 *     what must start at zero on its own stream. Calls that overlap on the GPU race on the array:
 *     issue them in order on one stream.
 *   - status_out (device int32, may be NULL) receives the call's EVA_STATUS_* bits; a call with M = 0
 *     returns EVA_OK without touching the device and leaves *status_out as it was.
 * No cudaMalloc, cudaFree or other allocating routine is called. */
int eva_moe_experts_noalloc(const EvaMoeShape* shape, const void* x, int32_t x_is_bf16, int32_t M,
                            const void* sel, int32_t sel_is_i64, const float* rw,
                            const int64_t* const* tables, const int64_t* shared,
                            float* out_f32, void* out_bf16, int32_t* status_out, void* stream);

/* ---- expert parallelism (one process per GPU; rows move by this library's peer-memory stores over
 * NVLink (eva_ep_dispatch_peers / eva_ep_combine_peers) or, with the plan and pack below, by NCCL
 * send/recv and all-to-all issued by the host) ----------------------------------------------------
 * No counterpart in the reference, which has no expert parallelism: these replace the kernel-side
 * local-expert filter slot_info (runtime/ds41/csrc/moe_coop2048/vendor/exl3_moe_coop_kernel.cuh:208-223)
 * and the empty-row path write_empty_row_chunk (:573-610) with an explicit dispatch and combine.
 *
 * eva_ep_dispatch: plan and pack the rows this rank sends. Token m goes to rank r once when at least
 * one of its slots with a non-zero weight has an expert owned by r.
 *   x:            [M][H] rows of x_elem_bytes (2: bf16/fp16, 4: fp32) elements, 16-byte aligned
 *   idx, w:       int32 / float [M][topk] global expert ids and routing weights (eva_moe_route)
 *   owner:        int32 [n_experts] rank holding each global expert; local_id: int32 [n_experts] the
 *                 expert's column in that rank's pointer tables
 *   segment_rows: 0 = rows for rank r packed after rank r-1's (exact splits: read counts on the host);
 *                 > 0 = rank r's rows start at r * segment_rows, padding rows zeroed (fixed splits,
 *                 no host synchronisation; needs segment_rows >= rows sent to any rank)
 *   capacity:     rows in send_x / send_sel / send_rw (>= world * segment_rows in fixed mode;
 *                 M * min(topk, world) always suffices in packed mode)
 *   counts:       int32 [world] rows for each rank; pos: int32 [world][M] send row of (rank, token), -1 if none
 *   send_sel/rw:  int32 / float [capacity][topk]: destination-local expert ids, and the weights with 0 for
 *                 the slots whose expert is on another rank (inactive in eva_moe_experts)
 *   status:       device int32 (may be NULL): EVA_STATUS_BAD_EXPERT for ids outside [0, n_experts) or
 *                 owners outside [0, world); EVA_STATUS_CAPACITY when rows did not fit (they are dropped) */
int eva_ep_dispatch(int32_t H, int32_t topk, int32_t n_experts, const void* x, int32_t x_elem_bytes, int32_t M,
                    const int32_t* idx, const float* w, int32_t world, const int32_t* owner, const int32_t* local_id,
                    int32_t capacity, int32_t segment_rows, int32_t* counts, int32_t* pos, void* send_x,
                    int32_t* send_sel, float* send_rw, int32_t* status, void* stream);

/* eva_ep_combine: out[m] = base[m] + sum over r = 0 .. world-1 (in that order) of back[pos[r][m]],
 * skipping pos < 0. back: float [rows][H], the routed partial sums returned in send order;
 * base: float [M][H] (the shared expert's output) or NULL; out_f32 / out_bf16 (at least one). */
int eva_ep_combine(int32_t H, int32_t M, int32_t world, const float* back, const int32_t* pos,
                   const float* base, float* out_f32, void* out_bf16, void* stream);

/* ---- expert parallelism over NVLink peer memory (no collective library in the data path) -------
 * Every rank owns one arena in its GPU memory, mapped into every other rank's process (CUDA IPC):
 *   flags     epoch (this rank's step count), a block counter, the "partials ready" flag, and one
 *             "rows ready" flag per source rank
 *   recv_x    [world][segment_rows][H]   rows sent to this rank, source-major
 *   recv_sel  int32 [world][segment_rows][topk], recv_rw float [same]: destination-local expert ids
 *             and weights (0 for the slots of other ranks' experts and for padding rows)
 *   part      float [world][segment_rows][H]: this rank's routed partial sums of the received rows
 * A step: eva_ep_dispatch_peers (plan; each row stored straight into its destination's recv_*; the
 * last block releases every destination's "rows ready" flag for this source) -> eva_ep_wait_rows
 * -> eva_moe_experts on the recv_* rows into part -> eva_ep_combine_peers (publishes this rank's
 * "partials ready" flag, waits for every rank's, then reads the partial rows of this rank's tokens
 * from the peers' arenas; eva_ep_signal_partials publishes the flag earlier, on its own). Flags hold step numbers, so no reset is needed between steps, and a
 * rank cannot overwrite a peer's rows before the peer has finished the previous step (its combine
 * waited for that peer's partials). Every wait is bounded (2 s) and sets EVA_STATUS_TIMEOUT. */
#define EVA_EP_MAX_WORLD 32

typedef struct EvaEpPeers {
    int32_t world, rank;              /* ranks, this rank */
    int32_t H, topk, n_experts;       /* hidden size, slots per token, routed experts (global) */
    int32_t segment_rows;             /* rows each source may send to each destination per step */
    int32_t x_elem_bytes;             /* 2 (bf16 / fp16 rows) */
    int32_t reserved;
    uint64_t off_x, off_sel, off_rw, off_part, bytes;   /* arena layout: eva_ep_arena_layout fills these */
    void* arena[EVA_EP_MAX_WORLD];    /* every rank's arena as mapped in this process (own included) */
    const int32_t* owner;             /* device int32 [n_experts]: rank holding each expert */
    const int32_t* local_id;          /* device int32 [n_experts]: its column in that rank's tables */
} EvaEpPeers;

/* Fill the off_* / bytes fields of *p from world, H, topk, segment_rows and x_elem_bytes. */
int eva_ep_arena_layout(EvaEpPeers* p);

/* Arena memory: allocate (zeroed) and export a 64-byte CUDA IPC handle; map a peer's handle; unmap;
 * free. Setup-time calls (they allocate and synchronise), unlike every other entry point. */
int eva_peer_alloc(size_t bytes, void** ptr, void* handle_out);
int eva_peer_open(const void* handle, void** ptr);
int eva_peer_close(void* ptr);
int eva_peer_free(void* ptr);

/* Plan + pack: token rows (x [M][H], routes idx/w [M][topk]) stored into the destinations' arenas.
 * all_to_self != 0: every token also goes to this rank (its own segment then holds all M tokens in
 * order, for eva_moe_experts_window's shared expert). pos: int32 [world][M], the token's row within its
 * segment at rank r (-1: not sent); counts: int32 [world]. EVA_STATUS_CAPACITY when a destination would
 * get more than segment_rows rows (dropped). */
int eva_ep_dispatch_peers(const EvaEpPeers* p, const void* x, int32_t M, const int32_t* idx, const float* w,
                          int32_t all_to_self, int32_t* counts, int32_t* pos, int32_t* status, void* stream);
/* Wait until every source's rows of this step are in this rank's arena. */
int eva_ep_wait_rows(const EvaEpPeers* p, int32_t* status, void* stream);
/* Publish this rank's partial sums of this step (after the experts launch that wrote part); optional,
 * eva_ep_combine_peers publishes them too. */
int eva_ep_signal_partials(const EvaEpPeers* p, void* stream);
/* out[m] = base[m] + sum over r (rank order) of rank r's partial row for token m; publishes this
 * rank's partials (stream order after the experts launch that wrote part) and waits for every rank's
 * first. base: float [M][H] or NULL; out_f32 / out_bf16 at least one. */
int eva_ep_combine_peers(const EvaEpPeers* p, int32_t M, const int32_t* pos, const float* base, float* out_f32,
                         void* out_bf16, int32_t* status, void* stream);

/* ---- layer stack ----------------------------------------------------------------------------
 * Residual add + RMSNorm between MoE layers (runtime/ds41/model.py:968-970 `rms`, mean square in FP32,
 * model.py:168-176): resid[m] += add[m] (add may be NULL), then
 * h_out[m] = bf16((weight * resid[m]) * rsqrt(mean(resid[m]^2) + eps)).
 *   resid: float [M][H] residual stream (in/out), 16-byte aligned; add: float [M][H] or NULL
 *   weight: [H] bf16 (weight_is_bf16 = 1) or fp16; h_out: bf16 [M][H] */
int eva_rmsnorm_residual(int32_t H, int32_t M, float* resid, const float* add, const void* weight,
                         int32_t weight_is_bf16, float eps, void* h_out, void* stream);

/* Library identification: sm arch the kernels were built for (100 for sm_100a). */
int32_t eva_moe_arch(void);

/* ---- device-side expert cache (rows of the reference's ExpertCache: cache.py:1852-2080) --------
 * A pool of device record slots shared by every layer on the GPU. Replaces _install_if_absent /
 * _blit / _bind / _unbind / _flush and prefetch_gpu (runtime/ds41/cache.py:1852-1996, 2064-2080) and
 * the host sync on the routes that decides what to install (cache.py:2315): the needed set, the slot
 * choice (CLOCK, free slots first, slots in use by the running or the planned layer protected) and
 * the pointer-table updates run on the device; copies read the pinned host records by their unified
 * addresses. Nothing synchronises the host.
 *
 * EvaExpertPool (device arrays): slots n_slots * record_bytes; owner [n_slots] (layer << 16 | expert,
 *   -1 free); stamp int64 [n_slots]; state int32 [8] = {hand, 0, status bits, 0, bytes copied (int64),
 *   plan counter (int64)}, zero-initialised with owner = -1. Stamps and the counter are 64-bit so that
 *   they never wrap (one exact plan per layer per step).
 * EvaPoolLayer (one per layer, an array of them in device memory): layer's n_local (<= 1024) experts;
 *   host_records: pinned host memory, n_local records of record_bytes; row_off: byte offsets of the 9
 *   tensors inside a record (handle row order); slot_of [n_local] (-1 = not resident); last_needed:
 *   bitmap of the last exact plan (what a prefetch predicts); table: the layer's int64 [9][n_local]
 *   pointer-table handle, kept bound to the resident copies (0 = not resident).
 *
 * eva_pool_plan: exact (prefetch = 0): the experts selected by rows x topk routes (rw != 0) of layer
 *   `layer` become resident (misses get slots; their copy jobs go to jobs = {n, (expert, slot) x n});
 *   prefetch (prefetch = 1): the same for the layer's last exact needed set, issued while another
 *   layer runs (that layer's slots are protected; best effort: it stops when no slot is free). Status
 *   bit EVA_STATUS_CAPACITY in state[2] when the pool cannot hold a layer's needed set; the routes of
 *   the experts left without a slot then get weight 0 (in rw itself when rw_hit is NULL), so that no
 *   launch reads an unbound expert. rw_hit / rw_miss (optional, device float [rows x topk], exact
 *   plans only): rw split into the routes of experts already resident and of those being copied, so
 *   that one experts launch over rw_hit can overlap the copies and a second one over rw_miss follows
 *   them. jobs: device int32 [1 + 2 n_local].
 * eva_pool_copy: copies the jobs of the last plan of `layer` (stream order after the plan). */
typedef struct {
    int32_t n_slots;
    int32_t reserved;
    int64_t record_bytes;
    void* slots;
    int32_t* owner;
    int64_t* stamp;
    int32_t* state;
} EvaExpertPool;

typedef struct {
    int32_t layer, n_local;
    const void* host_records;
    int64_t row_off[9];
    int32_t* slot_of;
    uint32_t* last_needed;
    int64_t* table;
} EvaPoolLayer;

int eva_pool_plan(const EvaExpertPool* pool, const EvaPoolLayer* layers, int32_t layer, const void* sel,
                  int32_t sel_is_i64, float* rw, int32_t rows, int32_t topk, int32_t prefetch, int32_t* jobs,
                  float* rw_hit, float* rw_miss, void* stream);
int eva_pool_copy(const EvaExpertPool* pool, const EvaPoolLayer* layers, int32_t layer, const int32_t* jobs,
                  void* stream);

/* 1 when p is pinned host memory that kernels can read at the same address (unified addressing), else 0.
 * Callers of eva_pool_copy check their host records with it. */
int eva_host_mapped(const void* p);

/* ---- measurement and self-test entry points (no counterpart in the reference) ----------------
 *
 * eva_decode_microbench: the EXL3 decode loop alone, on trellis tiles resident in shared memory (no
 * HBM traffic), one CTA per SM. variant 0: the mma.sync decode of the fused decode kernel; 1 / 2:
 * decode into tensor memory (mul1 products for kind::i8 / raw codebook fp16 for kind::f16), no MMA;
 * 3 / 4: the same with tcgen05.mma reading A from tensor memory through a slot ring; 5: variant 1
 * without splitting the window extraction between the ALU and FMA pipes; 6..10: the two-word decode
 * with mma.sync (pair packing by IMAD or PRMT, 0 / 2 / 4 windows extracted on the FMA pipe); 11:
 * variant 8 with a fused-kernel stage's bookkeeping around each pass; 12 / 13: variant 8 fed by
 * the fused kernel's bulk-copy ring from a 1 GB (HBM) / 32 MB (L2) source, allocated by the call;
 * 14: 5 ring stages; 15: decoders not waiting for the data; 16: one contiguous copy per stage;
 * 17: one 2-D tensor copy per stage; 18: cp.async 16-byte copies by the producer warp; 19: variant 8
 * with the byte sum left to 8-bit MMAs (m16n8k32, the mul1 products as u8 A, two activation digits).
 * bits: EXL3 K (2..4).
 * out[5] = {decoded weights per SM clock, SM clocks of the launch (max over CTAs), weights decoded,
 * device status bits, event time of the launch in ms}. Synchronises the stream.
 *
 * eva_tc_selftest: one CTA checks a tensor-memory layout. what 0: out[128][16] u32 = TMEM read back
 * (32x32b) after 16x256b.x2 stores of tags (half << 12 | lane << 4 | register) at lanes 32 w + 16 half;
 * what 1: out[128][16] s32 = A x B^T with A u8 [128][32] stored in TMEM, B s8 [16][32] in shared
 * memory (tcgen05.mma.kind::i8); what 2: out[128][16] f32 = A x B^T with A f16 [128][16] in TMEM and
 * B f16 [16][16] (kind::f16); what 3 / 4: a cluster of two CTAs runs one tcgen05.mma.cta_group::2.kind::f16
 * of M = 256 / 128 rows and N = 256 whose D[i][n] = (i + 1) + 256 (n + 1), each CTA dumps its 128 TMEM
 * lanes x 256 columns (0xffffffff where the MMA wrote nothing): out[2][128][256] u32. a, b: device
 * arrays of those shapes (what 1, 2); status: device int32. */
int eva_decode_microbench(int32_t variant, int32_t bits, int32_t iters, double* out, void* stream);
int eva_tc_selftest(int32_t what, const uint32_t* a, const uint32_t* b, uint32_t* out, int32_t* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* EVA_MOE_H */
