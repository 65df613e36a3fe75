// extern "C" entry points of libeva_moe.so (declared in include/eva_moe.h).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "internal.h"

namespace eva {

static size_t up256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

WsLayout ws_layout(const EvaMoeShape& s, int max_rows, bool allow_split, bool routing, bool tensor_core)
{
    WsLayout L{};
    L.max_rows = max_rows;
    L.S = max_rows * s.topk;
    L.R = L.S + (max_rows + RUN_ROWS - 1) / RUN_ROWS;
    L.imax = std::max(s.inter, s.shared_inter);
    L.nchA = L.imax / 128;
    L.nchH = s.hidden / 128;
    L.ks_router = (s.hidden + ROUTER_KSLICE - 1) / ROUTER_KSLICE;
    const size_t S = L.S, R = L.R, M = max_rows, H = s.hidden, E = s.n_experts;
    const size_t St = S + M;
    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t at = o;
        o += up256(bytes);
        return at;
    };
    L.status = take(256);
    const CtrLayout C = ctr_layout(L);
    L.n_counters = C.n;
    L.counters = take(C.n * 4);
    L.runs = take((2 + 2 * S + 1) * 4);
    L.run_expert = take(S * 4);
    L.estart = take((E + 1) * 4);
    L.slot_act = take(S * 4);
    L.tok_expect = take(M * 4);
    L.idx = take(M * s.topk * 4);
    L.w = take(M * s.topk * 4);
    // fragment-layout copies of the GEMV inputs: rows padded by one stage (32 k-tile rows = 512
    // elements) so the last stage's reads past the end of a row stay inside the buffer
    L.hpad = (s.hidden + 511) / 512 * 512 + 512;
    L.ipad = (L.imax + 511) / 512 * 512 + 512;
    L.xrot = take(2 * St * static_cast<size_t>(L.hpad) * 2);
    L.act = take(St * static_cast<size_t>(L.ipad) * 2);
    L.dpart = take(St * H * 4);
    L.xsum = take(2 * St * L.nchH * 4);
    L.asum = take(St * L.nchA * 4);
    L.tstart = take((E + 2) * 4);
    L.pscan = take(permute_scratch_ints(max_rows, static_cast<int>(E)) * 4);
    // tensor maps: decode kernel per-CTA item sets, or the tensor-core path's per-expert trellis maps
    L.tmaps = take(std::max(static_cast<size_t>(DEC_MAX_CTAS) * DEC_MAP_SETS * 2, (E + 1) * 3) * 128);
    L.pxg = take(tensor_core ? St * H * 2 : 0);
    L.pxu = take(tensor_core ? St * H * 2 : 0);
    L.pap = take(tensor_core ? St * L.imax * 2 : 0);
    const size_t pa = allow_split ? std::min<size_t>(PARTA_ITEMS, R * L.nchA * 4) : 0;
    L.partA = take(pa * 2 * RUN_ROWS * 128 * 4);
    L.max_split = allow_split ? 4 : 1;
    // router regions last, so that every other offset is the same with and without them
    if (routing) {
        L.logits = take(router_part_rows(max_rows, s.hidden, s.n_experts) * E * 4);
        L.wsplit = take(max_rows >= ROUTER_TC_MIN_ROWS ? 3 * E * H * 2 : 0);
    }
    L.total = o;
    return L;
}

CtrLayout ctr_layout(const WsLayout& L)
{
    CtrLayout C{};
    C.work = 0;
    C.ctr0 = 32;
    C.ctrA = C.ctr0 + L.R;
    C.ctrAk = C.ctrA + L.R;
    C.ctrB = C.ctrAk + L.R * L.nchA;
    C.n = C.ctrB + L.max_rows * L.nchH;
    return C;
}

int num_sms()
{
    static int cached[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!cached[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cached[dev] = n > 0 ? n : 1;
    }
    return cached[dev];
}

// Shape of an experts / permutation call: the slots per row (topk) may exceed the experts in the tables
// (an expert-parallel shard holds n_experts / world of them; the other slots are inactive).
static bool shape_ok(const EvaMoeShape* s)
{
    if (!s) return false;
    if (s->hidden <= 0 || s->hidden % 256) return false;
    if (s->inter <= 0 || s->inter % 128) return false;
    if (s->n_experts < 1 || s->n_experts > 1024) return false;
    if (s->topk < 1 || s->topk > 32) return false;
    if (s->bits < 2 || s->bits > 4) return false;
    if (s->shared_inter < 0 || s->shared_inter % 128) return false;
    if (s->shared_inter && (s->shared_bits < 2 || s->shared_bits > 4)) return false;
    if (s->act_routed < 0 || s->act_routed > 1 || s->act_shared < 0 || s->act_shared > 1) return false;
    return true;
}

// Shape of a routing call: top-k over all n_experts, group limits consistent.
static bool route_ok(const EvaMoeShape* s)
{
    if (!shape_ok(s) || s->topk > s->n_experts) return false;
    if (s->router < 0 || s->router > 2) return false;
    if (s->n_group < 1 || s->n_group > 32 || s->n_experts % s->n_group) return false;
    if (s->topk_group < 1 || s->topk_group > s->n_group) return false;
    if (s->n_group > 1 && s->topk > s->topk_group * (s->n_experts / s->n_group)) return false;
    return true;
}

static bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

static int cuda_status(cudaError_t e) { return e == cudaSuccess ? EVA_OK : EVA_ERR_CUDA; }

static void fill_permute(PermuteArgs& pa, const EvaMoeShape& s, const void* sel, int sel64, const float* rw, int M,
                         int capacity)
{
    std::memset(&pa, 0, sizeof(pa));
    pa.sel = sel;
    pa.sel64 = sel64;
    pa.rw = rw;
    pa.M = M;
    pa.topk = s.topk;
    pa.n_local = s.n_experts;
    pa.capacity = capacity;
    pa.has_shared = s.shared_inter > 0;
    pa.H = s.hidden;
    pa.sh0 = 0;
    pa.shn = pa.has_shared ? M : 0;
}

}  // namespace eva

using namespace eva;

extern "C" {

size_t eva_moe_workspace_bytes(const EvaMoeShape* shape, int32_t max_rows)
{
    if (!shape_ok(shape) || max_rows < 1) return 0;
    return ws_layout(*shape, max_rows).total;
}

int eva_moe_clear_status(void* workspace, void* stream)
{
    if (!workspace) return EVA_ERR_INVALID;
    return cuda_status(cudaMemsetAsync(workspace, 0, 4, static_cast<cudaStream_t>(stream)));
}

int eva_moe_read_status(const void* workspace, int32_t* status_host, void* stream)
{
    if (!workspace || !status_host) return EVA_ERR_INVALID;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(status_host, workspace, 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    return cuda_status(e);
}

int eva_moe_topk(const EvaMoeShape* shape, const float* logits, int32_t M, const float* router_b,
                 int32_t* idx_out, float* w_out, void* stream)
{
    if (!route_ok(shape) || M < 0 || !logits || !idx_out || !w_out) return EVA_ERR_INVALID;
    if (M == 0) return EVA_OK;
    return cuda_status(launch_topk(*shape, logits, 1, M, router_b, nullptr, idx_out, w_out, static_cast<cudaStream_t>(stream)));
}

int eva_moe_route(const EvaMoeShape* shape, const void* x, int32_t x_is_bf16, int32_t M, const float* router_w,
                  const float* router_b, float* logits_out, int32_t* idx_out, float* w_out, void* workspace,
                  size_t workspace_bytes, void* stream)
{
    if (!route_ok(shape) || M < 0 || !x || !router_w || !idx_out || !w_out || !workspace) return EVA_ERR_INVALID;
    if (!aligned(x, 8) || !aligned(router_w, 16)) return EVA_ERR_INVALID;
    if (M == 0) return EVA_OK;
    const WsLayout L = ws_layout(*shape, M);
    if (workspace_bytes < L.total) return EVA_ERR_WORKSPACE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* part = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + L.logits);
    int ks = 1;
    void* wsplit = M >= ROUTER_TC_MIN_ROWS ? static_cast<uint8_t*>(workspace) + L.wsplit : nullptr;
    int* status = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + L.status);
    cudaError_t e = launch_router_logits(x, x_is_bf16 ? 1 : 0, M, shape->hidden, shape->n_experts, router_w, part, wsplit,
                                         status, &ks, st);
    if (e != cudaSuccess) return EVA_ERR_CUDA;
    return cuda_status(launch_topk(*shape, part, ks, M, router_b, logits_out, idx_out, w_out, st));
}

int eva_moe_permute(const EvaMoeShape* shape, const void* sel, int32_t sel_is_i64, const float* rw, int32_t M,
                    int32_t capacity, int32_t* runs, int32_t* expert_start, void* stream)
{
    if (!shape_ok(shape) || M < 0 || !sel || !rw || !runs || capacity < M || capacity < 1) return EVA_ERR_INVALID;
    if (static_cast<long long>(capacity) * shape->topk > 65535 * 16) return EVA_ERR_INVALID;
    PermuteArgs pa;
    fill_permute(pa, *shape, sel, sel_is_i64 ? 1 : 0, rw, M, capacity);
    pa.runs = runs;
    pa.estart = expert_start;
    return cuda_status(launch_permute(pa, static_cast<cudaStream_t>(stream)));
}

int eva_moe_permute_ws(const EvaMoeShape* shape, const void* sel, int32_t sel_is_i64, const float* rw, int32_t M,
                       int32_t capacity, int32_t* runs, int32_t* expert_start, void* workspace, size_t workspace_bytes,
                       void* stream)
{
    if (!shape_ok(shape) || M < 0 || !sel || !rw || !runs || capacity < M || capacity < 1 || !workspace)
        return EVA_ERR_INVALID;
    if (static_cast<long long>(capacity) * shape->topk > 65535 * 16) return EVA_ERR_INVALID;
    if (M == 0) return eva_moe_permute(shape, sel, sel_is_i64, rw, M, capacity, runs, expert_start, stream);
    const WsLayout L = ws_layout(*shape, M, true, /*routing=*/false);
    if (workspace_bytes < L.total) return EVA_ERR_WORKSPACE;
    PermuteArgs pa;
    fill_permute(pa, *shape, sel, sel_is_i64 ? 1 : 0, rw, M, capacity);
    pa.runs = runs;
    pa.estart = expert_start;
    pa.scratch = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + L.pscan);
    return cuda_status(launch_permute(pa, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"

namespace eva {

int experts_validate(const EvaMoeShape* shape, const void* x, int32_t M, const void* sel, const float* rw,
                     const int64_t* const* tables, const int64_t* shared, const float* out_f32, const void* out_bf16)
{
    if (!shape_ok(shape) || M < 0 || !x || !sel || !rw || !tables) return EVA_ERR_INVALID;
    if (!out_f32 && !out_bf16) return EVA_ERR_INVALID;
    if (shape->shared_inter && !shared) return EVA_ERR_INVALID;
    if (!aligned(x, 8) || !aligned(out_f32, 16) || !aligned(out_bf16, 8)) return EVA_ERR_INVALID;
    for (int i = 0; i < 9; ++i)
        if (!tables[i] || !aligned(tables[i], 8)) return EVA_ERR_INVALID;
    if (shape->shared_inter)
        for (int i = 0; i < 9; ++i)
            if (shared[i] == 0 || (shared[i] & 15)) return EVA_ERR_INVALID;   // bulk copies need 16 B
    return EVA_OK;
}

int experts_impl(const EvaMoeShape* shape, const void* x, int32_t x_is_bf16, int32_t M, const void* sel,
                 int32_t sel_is_i64, const float* rw, const int64_t* const* tables, const int64_t* shared,
                 void* workspace, size_t workspace_bytes, float* out_f32, void* out_bf16, cudaStream_t st,
                 bool allow_split, int path, int shared_row0, int shared_rows)
{
    if (shared_rows < 0) {
        shared_row0 = 0;
        shared_rows = M;
    }
    if (shared_row0 < 0 || shared_row0 + shared_rows > M) return EVA_ERR_INVALID;
    if (!workspace) return EVA_ERR_INVALID;
    const int v = experts_validate(shape, x, M, sel, rw, tables, shared, out_f32, out_bf16);
    if (v != EVA_OK) return v;
    if (M == 0) return EVA_OK;
    const WsLayout L = ws_layout(*shape, M, allow_split, /*routing=*/false, /*tensor_core=*/path != 1);
    if (workspace_bytes < L.total) return EVA_ERR_WORKSPACE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    PermuteArgs pa;
    const bool tensor = path == 2 || (path == 0 && M >= PREFILL_MIN_ROWS);
    fill_permute(pa, *shape, sel, sel_is_i64 ? 1 : 0, rw, M, M);
    for (int i = 0; i < 9; ++i) pa.tables[i] = tables[i];
    pa.runs = reinterpret_cast<int32_t*>(ws + L.runs);
    pa.estart = reinterpret_cast<int32_t*>(ws + L.estart);
    pa.tstart = reinterpret_cast<int32_t*>(ws + L.tstart);
    pa.slot_act = reinterpret_cast<int32_t*>(ws + L.slot_act);
    pa.scratch = reinterpret_cast<int32_t*>(ws + L.pscan);
    if (!tensor) {
        // the fused decode kernel's run owners, arrival counts and work counters; the tensor-core
        // path writes every output row in its combine and needs none of them
        pa.run_expert = reinterpret_cast<int32_t*>(ws + L.run_expert);
        pa.tok_expect = reinterpret_cast<int32_t*>(ws + L.tok_expect);
        pa.counters = reinterpret_cast<int32_t*>(ws + L.counters);
        pa.n_counters = static_cast<int>(L.n_counters);
    }
    pa.status = reinterpret_cast<int32_t*>(ws + L.status);
    pa.out_f32 = out_f32;
    pa.out_bf16 = out_bf16;
    pa.sh0 = shared_row0;
    pa.shn = shape->shared_inter ? shared_rows : 0;
    cudaError_t e = launch_permute(pa, st);
    if (e != cudaSuccess) return EVA_ERR_CUDA;
    ExpertsArgs ea;
    std::memset(&ea, 0, sizeof(ea));
    ea.shape = shape;
    ea.x = x;
    ea.x_bf16 = x_is_bf16 ? 1 : 0;
    ea.M = M;
    ea.sel = sel;
    ea.sel64 = sel_is_i64 ? 1 : 0;
    ea.rw = rw;
    for (int i = 0; i < 9; ++i) {
        ea.tables[i] = tables[i];
        ea.shared[i] = shape->shared_inter ? shared[i] : 0;
    }
    ea.ws = workspace;
    ea.L = L;
    ea.out_f32 = out_f32;
    ea.out_bf16 = out_bf16;
    ea.sh0 = shared_row0;
    ea.shn = shape->shared_inter ? shared_rows : 0;
    return cuda_status(tensor ? launch_prefill(ea, st) : launch_experts(ea, st));
}

}  // namespace eva

extern "C" {

int eva_moe_experts(const EvaMoeShape* shape, const void* x, int32_t x_is_bf16, int32_t M, const void* sel,
                    int32_t sel_is_i64, const float* rw, const int64_t* const* tables, const int64_t* shared,
                    void* workspace, size_t workspace_bytes, float* out_f32, void* out_bf16, void* stream)
{
    return experts_impl(shape, x, x_is_bf16, M, sel, sel_is_i64, rw, tables, shared, workspace, workspace_bytes,
                        out_f32, out_bf16, static_cast<cudaStream_t>(stream));
}

int eva_moe_experts_prefill(const EvaMoeShape* shape, const void* x, int32_t x_is_bf16, int32_t M, const void* sel,
                            int32_t sel_is_i64, const float* rw, const int64_t* const* tables, const int64_t* shared,
                            void* workspace, size_t workspace_bytes, float* out_f32, void* out_bf16, void* stream)
{
    return experts_impl(shape, x, x_is_bf16, M, sel, sel_is_i64, rw, tables, shared, workspace, workspace_bytes,
                        out_f32, out_bf16, static_cast<cudaStream_t>(stream), true, 2);
}

int eva_moe_experts_window(const EvaMoeShape* shape, const void* x, int32_t x_is_bf16, int32_t M, const void* sel,
                           int32_t sel_is_i64, const float* rw, const int64_t* const* tables, const int64_t* shared,
                           int32_t shared_row0, int32_t shared_rows, void* workspace, size_t workspace_bytes,
                           float* out_f32, void* out_bf16, void* stream)
{
    if (shared_rows < 0) return EVA_ERR_INVALID;
    return experts_impl(shape, x, x_is_bf16, M, sel, sel_is_i64, rw, tables, shared, workspace, workspace_bytes,
                        out_f32, out_bf16, static_cast<cudaStream_t>(stream), true, 0, shared_row0, shared_rows);
}

int eva_moe_experts_decode(const EvaMoeShape* shape, const void* x, int32_t x_is_bf16, int32_t M, const void* sel,
                           int32_t sel_is_i64, const float* rw, const int64_t* const* tables, const int64_t* shared,
                           void* workspace, size_t workspace_bytes, float* out_f32, void* out_bf16, void* stream)
{
    return experts_impl(shape, x, x_is_bf16, M, sel, sel_is_i64, rw, tables, shared, workspace, workspace_bytes,
                        out_f32, out_bf16, static_cast<cudaStream_t>(stream), true, 1);
}

int eva_moe_forward(const EvaMoeShape* shape, const void* x, int32_t x_is_bf16, int32_t M, const float* router_w,
                    const float* router_b, const int64_t* const* tables, const int64_t* shared, void* workspace,
                    size_t workspace_bytes, float* out_f32, void* out_bf16, float* logits_out, int32_t* idx_out,
                    float* w_out, void* stream)
{
    if (!route_ok(shape) || M < 0 || !workspace) return EVA_ERR_INVALID;
    if (M == 0) return EVA_OK;
    const WsLayout L = ws_layout(*shape, M);
    if (workspace_bytes < L.total) return EVA_ERR_WORKSPACE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    int32_t* idx = idx_out ? idx_out : reinterpret_cast<int32_t*>(ws + L.idx);
    float* w = w_out ? w_out : reinterpret_cast<float*>(ws + L.w);
    int rc = eva_moe_route(shape, x, x_is_bf16, M, router_w, router_b, logits_out, idx, w, workspace, workspace_bytes, stream);
    if (rc != EVA_OK) return rc;
    return experts_impl(shape, x, x_is_bf16, M, idx, 0, w, tables, shared, workspace, workspace_bytes, out_f32, out_bf16,
                        static_cast<cudaStream_t>(stream));
}

int eva_exl3_dequant(const void* trellis, int32_t in_features, int32_t out_features, int32_t bits, uint16_t* w_out,
                     void* stream)
{
    if (!trellis || !w_out || in_features <= 0 || out_features <= 0 || in_features % 16 || out_features % 16) return EVA_ERR_INVALID;
    if (bits < 2 || bits > 4 || !aligned(trellis, 4)) return EVA_ERR_INVALID;
    return cuda_status(launch_dequant(trellis, in_features, out_features, bits, w_out, static_cast<cudaStream_t>(stream)));
}

int32_t eva_moe_arch(void) { return 100; }

}  // extern "C"
