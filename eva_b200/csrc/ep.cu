// Expert parallelism: dispatch plan + pack of token rows per destination rank, and the rank-ordered
// combine of the returned partial sums.
//
// The reference has no expert parallelism. Its kernel only anticipates it: slot_info
// (runtime/ds41/csrc/moe_coop2048/vendor/exl3_moe_coop_kernel.cuh:208-223) drops slots whose expert
// is outside [min_expert, max_expert], and write_empty_row_chunk (:573-610) gives tokens with no
// local expert a shared-only or zero row. Here the filtering happens before the exchange instead:
// every rank sends each of its tokens once to every rank that owns at least one of the token's
// experts, with the slots of other ranks' experts given weight 0 (inactive in eva_moe_experts).
//
// Layout of the exchange (world ranks, M tokens on this rank, topk slots):
//   pos[r][m]   row of token m in the send buffer for rank r (-1: not sent). Rows for rank r are
//               contiguous and in token order; with segment_rows > 0 rank r's rows start at
//               r * segment_rows (fixed splits, no host synchronisation), else they are packed.
//   send_x      [rows][H] copies of x rows
//   send_sel    int32 [rows][topk] expert ids local to the destination (0 for inactive slots)
//   send_rw     float [rows][topk] routing weights (0 for inactive slots and padding rows)
#include <cuda_runtime.h>

#include <cstring>

#include "common.cuh"

namespace eva {

constexpr int EP_PLAN_THREADS = 1024;
constexpr int EP_MAX_WORLD = 32;

struct EpDispatchArgs {
    int H, topk, n_experts, M, world, capacity, segment, elem_bytes;
    int within;              // 1: pos = index within the destination's segment (peer-memory exchange)
    const uint8_t* x;
    const int32_t* idx;
    const float* w;
    const int32_t* owner;
    const int32_t* local_id;
    int32_t* counts;
    int32_t* pos;
    uint8_t* send_x;
    int32_t* send_sel;
    float* send_rw;
    int32_t* status;
    uint32_t* epoch;         // peer-memory exchange: this rank's step counter, advanced by the plan
    int force_self;          // >= 0: every token also goes to this rank
};

__device__ __forceinline__ int slot_dest(const EpDispatchArgs& a, int m, int j, bool flag)
{
    const int s = m * a.topk + j;
    if (a.w[s] == 0.0f) return -1;
    const int e = a.idx[s];
    if (e < 0 || e >= a.n_experts) {
        if (flag && a.status) atomicOr(a.status, ST_BAD_EXPERT);
        return -1;
    }
    const int r = a.owner[e];
    if (r < 0 || r >= a.world) {
        if (flag && a.status) atomicOr(a.status, ST_BAD_EXPERT);
        return -1;
    }
    return r;
}

// One CTA: per destination a block-wide exclusive scan of "token m goes to rank r", 1024 tokens at a time.
__global__ void __launch_bounds__(EP_PLAN_THREADS) ep_plan_kernel(EpDispatchArgs a)
{
    __shared__ int run[EP_MAX_WORLD];
    __shared__ int off[EP_MAX_WORLD + 1];
    __shared__ int wtot[EP_PLAN_THREADS / 32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid < a.world) run[tid] = 0;
    if (tid == 0 && a.epoch) *a.epoch += 1;
    __syncthreads();
    for (int c0 = 0; c0 < a.M; c0 += EP_PLAN_THREADS) {
        const int m = c0 + tid;
        uint32_t mask = 0;
        if (m < a.M) {
            for (int j = 0; j < a.topk; ++j) {
                const int r = slot_dest(a, m, j, true);
                if (r >= 0) mask |= 1u << r;
            }
            if (a.force_self >= 0) mask |= 1u << a.force_self;
        }
        for (int r = 0; r < a.world; ++r) {
            const bool bit = (mask >> r) & 1u;
            const uint32_t b = __ballot_sync(0xffffffffu, bit);
            if (lane == 0) wtot[warp] = __popc(b);
            __syncthreads();
            if (warp == 0) {
                const int v = wtot[lane];
                int inc = v;
#pragma unroll
                for (int d = 1; d < 32; d <<= 1) {
                    const int t = __shfl_up_sync(0xffffffffu, inc, d);
                    if (lane >= d) inc += t;
                }
                wtot[lane] = inc - v;   // exclusive
                if (lane == 31) off[EP_MAX_WORLD] = inc;
            }
            __syncthreads();
            if (m < a.M)
                a.pos[static_cast<size_t>(r) * a.M + m] =
                    bit ? run[r] + wtot[warp] + __popc(b & ((1u << lane) - 1u)) : -1;
            __syncthreads();
            if (tid == 0) run[r] += off[EP_MAX_WORLD];
            __syncthreads();
        }
    }
    if (tid == 0) {
        int o = 0;
        bool over = false;
        for (int r = 0; r < a.world; ++r) {
            off[r] = a.within ? 0 : a.segment > 0 ? r * a.segment : o;
            over = over || (a.segment > 0 && run[r] > a.segment);
            o += run[r];
            a.counts[r] = run[r];
        }
        over = over || (a.segment == 0 && o > a.capacity);
        if (over && a.status) atomicOr(a.status, EVA_STATUS_CAPACITY);
    }
    __syncthreads();
    for (int i = tid; i < a.world * a.M; i += EP_PLAN_THREADS) {
        const int p = a.pos[i];
        if (p >= 0) {
            const int r = i / a.M;
            const int q = off[r] + p;
            const bool fits = a.segment > 0 ? p < a.segment : q < a.capacity;
            a.pos[i] = fits ? q : -1;
        }
    }
}

// One warp copies a row, 4 loads in flight per lane.
__device__ __forceinline__ void copy_row_warp(const uint4* src, uint4* dst, size_t n16, int lane)
{
    for (size_t i = lane; i < n16; i += 4 * 32) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (i + u * 32 < n16) v[u] = __ldcs(src + i + u * 32);
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (i + u * 32 < n16) dst[i + u * 32] = v[u];
    }
}

// Warp per (token, destination): copy the x row and write the destination-local slot metadata.
// With fixed segments, warps past the tokens zero the padding rows' metadata.
__global__ void __launch_bounds__(256) ep_pack_kernel(EpDispatchArgs a)
{
    const int lane = threadIdx.x & 31;
    const long long gw = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const long long n_pairs = static_cast<long long>(a.M) * a.world;
    const size_t row_bytes = static_cast<size_t>(a.H) * a.elem_bytes;
    if (gw < n_pairs) {
        const int m = static_cast<int>(gw / a.world), r = static_cast<int>(gw % a.world);
        const int p = a.pos[static_cast<size_t>(r) * a.M + m];
        if (p < 0) return;
        const uint4* src = reinterpret_cast<const uint4*>(a.x + static_cast<size_t>(m) * row_bytes);
        uint4* dst = reinterpret_cast<uint4*>(a.send_x + static_cast<size_t>(p) * row_bytes);
        copy_row_warp(src, dst, row_bytes / 16, lane);
        for (int j = lane; j < a.topk; j += 32) {
            const int d = slot_dest(a, m, j, false);
            const bool on = d == r;
            const int s = m * a.topk + j;
            a.send_sel[static_cast<size_t>(p) * a.topk + j] = on ? a.local_id[a.idx[s]] : 0;
            a.send_rw[static_cast<size_t>(p) * a.topk + j] = on ? a.w[s] : 0.0f;
        }
        return;
    }
    if (a.segment <= 0) return;
    // padding rows: row q of the fixed buffer is padding when q - r * segment >= counts[r]
    const long long q = gw - n_pairs;
    if (q >= static_cast<long long>(a.world) * a.segment) return;
    const int r = static_cast<int>(q / a.segment), i = static_cast<int>(q % a.segment);
    if (i < a.counts[r]) return;
    for (int j = lane; j < a.topk; j += 32) {
        a.send_sel[static_cast<size_t>(q) * a.topk + j] = 0;
        a.send_rw[static_cast<size_t>(q) * a.topk + j] = 0.0f;
    }
    uint4* dst = reinterpret_cast<uint4*>(a.send_x + static_cast<size_t>(q) * row_bytes);
    for (size_t k = lane; k < row_bytes / 16; k += 32) dst[k] = make_uint4(0, 0, 0, 0);
}

// Thread per (token, 4 columns): out = base + sum over ranks (in rank order) of the returned rows.
__global__ void __launch_bounds__(256) ep_combine_kernel(int H, int M, int world, const float* __restrict__ back,
                                                         const int32_t* __restrict__ pos, const float* __restrict__ base,
                                                         float* out_f32, __nv_bfloat16* out_bf16)
{
    const long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int q = H / 4;
    if (t >= static_cast<long long>(M) * q) return;
    const int m = static_cast<int>(t / q), c = static_cast<int>(t % q) * 4;
    float4 acc = base ? *reinterpret_cast<const float4*>(base + static_cast<size_t>(m) * H + c)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < world; ++r) {
        const int p = pos[static_cast<size_t>(r) * M + m];
        if (p < 0) continue;
        const float4 v = __ldcs(reinterpret_cast<const float4*>(back + static_cast<size_t>(p) * H + c));
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    if (out_f32) *reinterpret_cast<float4*>(out_f32 + static_cast<size_t>(m) * H + c) = acc;
    if (out_bf16) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
        uint2 v;
        v.x = *reinterpret_cast<uint32_t*>(&lo);
        v.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(out_bf16 + static_cast<size_t>(m) * H + c) = v;
    }
}

}  // namespace eva

using namespace eva;

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

extern "C" int eva_ep_dispatch(int32_t H, int32_t topk, int32_t n_experts, const void* x, int32_t x_elem_bytes,
                               int32_t M, const int32_t* idx, const float* w, int32_t world, const int32_t* owner,
                               const int32_t* local_id, int32_t capacity, int32_t segment_rows, int32_t* counts,
                               int32_t* pos, void* send_x, int32_t* send_sel, float* send_rw, int32_t* status,
                               void* stream)
{
    if (H <= 0 || H % 8 || topk < 1 || topk > 32 || n_experts < 1 || M < 0 || world < 1 || world > EP_MAX_WORLD)
        return EVA_ERR_INVALID;
    if (x_elem_bytes != 2 && x_elem_bytes != 4) return EVA_ERR_INVALID;
    if (segment_rows < 0 || capacity < 0) return EVA_ERR_INVALID;
    if (segment_rows > 0 && capacity < static_cast<long long>(segment_rows) * world) return EVA_ERR_INVALID;
    if (!counts || (M > 0 && (!x || !idx || !w || !owner || !local_id || !pos || !send_x || !send_sel || !send_rw)))
        return EVA_ERR_INVALID;
    if (!al16(x) || !al16(send_x)) return EVA_ERR_INVALID;
    EpDispatchArgs a{H, topk, n_experts, M, world, capacity, segment_rows, x_elem_bytes, 0,
                     static_cast<const uint8_t*>(x), idx, w, owner, local_id, counts, pos,
                     static_cast<uint8_t*>(send_x), send_sel, send_rw, status, nullptr, -1};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    ep_plan_kernel<<<1, EP_PLAN_THREADS, 0, s>>>(a);
    const long long warps = static_cast<long long>(M) * world + (segment_rows > 0 ? static_cast<long long>(world) * segment_rows : 0);
    if (warps > 0) {
        const long long blocks = (warps * 32 + 255) / 256;
        if (blocks > 0x7fffffffLL) return EVA_ERR_INVALID;
        ep_pack_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(a);
    }
    return cudaGetLastError() == cudaSuccess ? EVA_OK : EVA_ERR_CUDA;
}

extern "C" int eva_ep_combine(int32_t H, int32_t M, int32_t world, const float* back, const int32_t* pos,
                              const float* base, float* out_f32, void* out_bf16, void* stream)
{
    if (H <= 0 || H % 4 || M < 0 || world < 1 || world > EP_MAX_WORLD) return EVA_ERR_INVALID;
    if (!out_f32 && !out_bf16) return EVA_ERR_INVALID;
    if (M == 0) return EVA_OK;
    if (!pos || (!back && world > 0)) return EVA_ERR_INVALID;
    if (!al16(back) || !al16(base) || !al16(out_f32) || (reinterpret_cast<uintptr_t>(out_bf16) & 7)) return EVA_ERR_INVALID;
    const long long n = static_cast<long long>(M) * (H / 4);
    const long long blocks = (n + 255) / 256;
    if (blocks > 0x7fffffffLL) return EVA_ERR_INVALID;
    ep_combine_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        H, M, world, back, pos, base, out_f32, static_cast<__nv_bfloat16*>(out_bf16));
    return cudaGetLastError() == cudaSuccess ? EVA_OK : EVA_ERR_CUDA;
}

// ---------------------------------------------------------------------------------------------
// Exchange over NVLink peer memory (arena layout and protocol: include/eva_moe.h, EvaEpPeers)

namespace eva {

constexpr size_t ARENA_FLAGS = 4096;
constexpr size_t FLAG_EPOCH = 0, FLAG_CTR = 64, FLAG_PART = 128, FLAG_ROWS = 256;

__device__ __forceinline__ uint8_t* arena_of(const EvaEpPeers& P, int r) { return static_cast<uint8_t*>(P.arena[r]); }

__device__ __forceinline__ uint32_t* flag_at(const EvaEpPeers& P, int r, size_t off)
{
    return reinterpret_cast<uint32_t*>(arena_of(P, r) + off);
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p)
{
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Block per (token, destination) row (its threads copy the row with 4 loads in flight each), then
// blocks of 8 padding rows (warp per row); the last block to finish releases the "rows ready" flag of
// this source at every destination.
constexpr int PACK_THREADS = 256;
constexpr int PACK_PAD_ROWS = PACK_THREADS / 32;

__global__ void __launch_bounds__(PACK_THREADS) ep_pack_peers_kernel(EpDispatchArgs a, EvaEpPeers P)
{
    const int lane = threadIdx.x & 31;
    const long long n_pairs = static_cast<long long>(a.M) * a.world;
    const size_t row_bytes = static_cast<size_t>(a.H) * a.elem_bytes;
    const int seg = a.segment, k = a.topk;
    if (blockIdx.x < n_pairs) {
        const int m = static_cast<int>(blockIdx.x / a.world), r = static_cast<int>(blockIdx.x % a.world);
        const int p = a.pos[static_cast<size_t>(r) * a.M + m];
        if (p >= 0) {
            const size_t row = static_cast<size_t>(P.rank) * seg + p;
            uint8_t* dst = arena_of(P, r);
            const uint4* src = reinterpret_cast<const uint4*>(a.x + static_cast<size_t>(m) * row_bytes);
            uint4* dx = reinterpret_cast<uint4*>(dst + P.off_x + row * row_bytes);
            const size_t n16 = row_bytes / 16;
            for (size_t i = threadIdx.x; i < n16; i += 4 * PACK_THREADS) {
                uint4 v[4];
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (i + u * PACK_THREADS < n16) v[u] = __ldcs(src + i + u * PACK_THREADS);
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (i + u * PACK_THREADS < n16) dx[i + u * PACK_THREADS] = v[u];
            }
            if (threadIdx.x < 32) {
                int32_t* ds = reinterpret_cast<int32_t*>(dst + P.off_sel) + row * k;
                float* dw = reinterpret_cast<float*>(dst + P.off_rw) + row * k;
                for (int j = lane; j < k; j += 32) {
                    const int d = slot_dest(a, m, j, false);
                    const int s = m * k + j;
                    ds[j] = d == r ? a.local_id[a.idx[s]] : 0;
                    dw[j] = d == r ? a.w[s] : 0.0f;
                }
            }
        }
    } else {
        const long long q = (blockIdx.x - n_pairs) * PACK_PAD_ROWS + (threadIdx.x >> 5);
        if (q < static_cast<long long>(a.world) * seg) {
            const int r = static_cast<int>(q / seg), i = static_cast<int>(q % seg);
            if (i >= a.counts[r]) {
                uint8_t* dst = arena_of(P, r);
                const size_t row = static_cast<size_t>(P.rank) * seg + i;
                for (int j = lane; j < k; j += 32) {
                    reinterpret_cast<int32_t*>(dst + P.off_sel)[row * k + j] = 0;
                    reinterpret_cast<float*>(dst + P.off_rw)[row * k + j] = 0.0f;
                }
            }
        }
    }
    // the block's stores are ordered before thread 0's system-scope fence by the barrier (one fence
    // per block instead of one per thread), and the fence before its counter increment
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        uint32_t* ctr = flag_at(P, P.rank, FLAG_CTR);
        const uint32_t prev = atomicAdd(ctr, 1u);
        if (prev == gridDim.x - 1) {
            __threadfence_system();
            const uint32_t ep = *reinterpret_cast<volatile uint32_t*>(flag_at(P, P.rank, FLAG_EPOCH));
            for (int r = 0; r < a.world; ++r) st_release_sys(flag_at(P, r, FLAG_ROWS + 4 * P.rank), ep);
            *ctr = 0;
        }
    }
}

// One warp: lane r waits until flag(r) >= this rank's epoch (bounded).
// PUBLISH (the partials wait): thread 0 first publishes this rank's partial sums, as ep_signal_kernel
// does (the experts launch that wrote them has completed before this launch), so that a step needs no
// launch of its own for the signal.
template <bool ROWS, bool PUBLISH = false>
__global__ void __launch_bounds__(32) ep_wait_kernel(EvaEpPeers P, int32_t* status)
{
    const int r = threadIdx.x;
    const uint32_t ep = *reinterpret_cast<volatile uint32_t*>(flag_at(P, P.rank, FLAG_EPOCH));
    if (PUBLISH && r == 0) {
        __threadfence_system();
        st_release_sys(flag_at(P, P.rank, FLAG_PART), ep);
    }
    if (r >= P.world) return;
    const uint32_t* f = ROWS ? flag_at(P, P.rank, FLAG_ROWS + 4 * r) : flag_at(P, r, FLAG_PART);
    if (ld_acquire_sys(f) >= ep) return;
    const uint64_t t0 = globaltimer();
    while (ld_acquire_sys(f) < ep) {
        __nanosleep(100);
        if (globaltimer() - t0 > WAIT_LIMIT_NS) {
            if (status) atomicOr(status, ST_TIMEOUT);
            return;
        }
    }
}

__global__ void ep_signal_kernel(EvaEpPeers P)
{
    __threadfence_system();
    const uint32_t ep = *reinterpret_cast<volatile uint32_t*>(flag_at(P, P.rank, FLAG_EPOCH));
    st_release_sys(flag_at(P, P.rank, FLAG_PART), ep);
}

// Thread per (token, 4 columns): base + the token's partial rows read from every rank's arena.
__global__ void __launch_bounds__(256) ep_combine_peers_kernel(EvaEpPeers P, int M, const int32_t* __restrict__ pos,
                                                               const float* __restrict__ base, float* out_f32,
                                                               __nv_bfloat16* out_bf16)
{
    const int H = P.H;
    const long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int q = H / 4;
    if (t >= static_cast<long long>(M) * q) return;
    const int m = static_cast<int>(t / q), c = static_cast<int>(t % q) * 4;
    float4 acc = base ? *reinterpret_cast<const float4*>(base + static_cast<size_t>(m) * H + c)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < P.world; ++r) {
        const int p = pos[static_cast<size_t>(r) * M + m];
        if (p < 0) continue;
        const float* part = reinterpret_cast<const float*>(arena_of(P, r) + P.off_part);
        const float4 v = __ldcv(reinterpret_cast<const float4*>(
            part + (static_cast<size_t>(P.rank) * P.segment_rows + p) * H + c));
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    if (out_f32) *reinterpret_cast<float4*>(out_f32 + static_cast<size_t>(m) * H + c) = acc;
    if (out_bf16) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
        uint2 v;
        v.x = *reinterpret_cast<uint32_t*>(&lo);
        v.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(out_bf16 + static_cast<size_t>(m) * H + c) = v;
    }
}

static size_t up256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

static bool peers_ok(const EvaEpPeers* p)
{
    if (!p || p->world < 1 || p->world > EVA_EP_MAX_WORLD || p->rank < 0 || p->rank >= p->world) return false;
    if (p->H <= 0 || p->H % 256 || p->topk < 1 || p->topk > 32 || p->n_experts < 1 || p->segment_rows < 1) return false;
    if (p->x_elem_bytes != 2) return false;
    for (int r = 0; r < p->world; ++r)
        if (!p->arena[r] || (reinterpret_cast<uintptr_t>(p->arena[r]) & 255)) return false;
    return true;
}

}  // namespace eva

extern "C" int eva_ep_arena_layout(EvaEpPeers* p)
{
    if (!p || p->world < 1 || p->world > EVA_EP_MAX_WORLD || p->H <= 0 || p->topk < 1 || p->segment_rows < 1 ||
        (p->x_elem_bytes != 2 && p->x_elem_bytes != 4))
        return EVA_ERR_INVALID;
    const size_t rows = static_cast<size_t>(p->world) * p->segment_rows;
    size_t o = eva::ARENA_FLAGS;
    p->off_x = o;
    o += eva::up256(rows * p->H * p->x_elem_bytes);
    p->off_sel = o;
    o += eva::up256(rows * p->topk * 4);
    p->off_rw = o;
    o += eva::up256(rows * p->topk * 4);
    p->off_part = o;
    o += eva::up256(rows * p->H * 4);
    p->bytes = o;
    return EVA_OK;
}

extern "C" int eva_peer_alloc(size_t bytes, void** ptr, void* handle_out)
{
    if (!ptr || !handle_out || bytes == 0) return EVA_ERR_INVALID;
    void* d = nullptr;
    if (cudaMalloc(&d, bytes) != cudaSuccess) return EVA_ERR_CUDA;
    cudaIpcMemHandle_t h;
    if (cudaMemset(d, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, d) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(d);
        return EVA_ERR_CUDA;
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    memcpy(handle_out, &h, 64);
    *ptr = d;
    return EVA_OK;
}

extern "C" int eva_peer_open(const void* handle, void** ptr)
{
    if (!handle || !ptr) return EVA_ERR_INVALID;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, 64);
    return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? EVA_OK : EVA_ERR_CUDA;
}

extern "C" int eva_peer_close(void* ptr)
{
    if (!ptr) return EVA_ERR_INVALID;
    return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? EVA_OK : EVA_ERR_CUDA;
}

extern "C" int eva_peer_free(void* ptr)
{
    if (!ptr) return EVA_ERR_INVALID;
    return cudaFree(ptr) == cudaSuccess ? EVA_OK : EVA_ERR_CUDA;
}

extern "C" int eva_ep_dispatch_peers(const EvaEpPeers* p, const void* x, int32_t M, const int32_t* idx,
                                     const float* w, int32_t all_to_self, int32_t* counts, int32_t* pos,
                                     int32_t* status, void* stream)
{
    if (!peers_ok(p) || M < 0 || !counts || (M > 0 && (!x || !idx || !w || !pos)) || !p->owner || !p->local_id)
        return EVA_ERR_INVALID;
    if (!al16(x)) return EVA_ERR_INVALID;
    EpDispatchArgs a{p->H, p->topk, p->n_experts, M, p->world, p->world * p->segment_rows, p->segment_rows,
                     p->x_elem_bytes, 1, static_cast<const uint8_t*>(x), idx, w, p->owner, p->local_id, counts, pos,
                     nullptr, nullptr, nullptr, status,
                     reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(p->arena[p->rank]) + FLAG_EPOCH),
                     all_to_self ? p->rank : -1};
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    ep_plan_kernel<<<1, EP_PLAN_THREADS, 0, s>>>(a);
    const long long pad_rows = static_cast<long long>(p->world) * p->segment_rows;
    const long long blocks = static_cast<long long>(M) * p->world + (pad_rows + PACK_PAD_ROWS - 1) / PACK_PAD_ROWS;
    if (blocks > 0x7fffffffLL) return EVA_ERR_INVALID;
    ep_pack_peers_kernel<<<static_cast<unsigned>(blocks), PACK_THREADS, 0, s>>>(a, *p);
    return cudaGetLastError() == cudaSuccess ? EVA_OK : EVA_ERR_CUDA;
}

extern "C" int eva_ep_wait_rows(const EvaEpPeers* p, int32_t* status, void* stream)
{
    if (!peers_ok(p)) return EVA_ERR_INVALID;
    ep_wait_kernel<true><<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(*p, status);
    return cudaGetLastError() == cudaSuccess ? EVA_OK : EVA_ERR_CUDA;
}

extern "C" int eva_ep_signal_partials(const EvaEpPeers* p, void* stream)
{
    if (!peers_ok(p)) return EVA_ERR_INVALID;
    ep_signal_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(*p);
    return cudaGetLastError() == cudaSuccess ? EVA_OK : EVA_ERR_CUDA;
}

extern "C" int eva_ep_combine_peers(const EvaEpPeers* p, int32_t M, const int32_t* pos, const float* base,
                                    float* out_f32, void* out_bf16, int32_t* status, void* stream)
{
    if (!peers_ok(p) || M < 0 || (!out_f32 && !out_bf16) || (M > 0 && !pos)) return EVA_ERR_INVALID;
    if (!al16(base) || !al16(out_f32) || (reinterpret_cast<uintptr_t>(out_bf16) & 7)) return EVA_ERR_INVALID;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    ep_wait_kernel<false, true><<<1, 32, 0, s>>>(*p, status);
    if (M > 0) {
        const long long n = static_cast<long long>(M) * (p->H / 4);
        const long long blocks = (n + 255) / 256;
        if (blocks > 0x7fffffffLL) return EVA_ERR_INVALID;
        ep_combine_peers_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(*p, M, pos, base, out_f32,
                                                                             static_cast<__nv_bfloat16*>(out_bf16));
    }
    return cudaGetLastError() == cudaSuccess ? EVA_OK : EVA_ERR_CUDA;
}
