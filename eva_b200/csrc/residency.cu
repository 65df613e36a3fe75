// Device-side expert cache: a pool of device record slots shared by all layers of a GPU, filled from
// pinned host memory without any host synchronisation.
//
// The reference keeps a layer's experts in host memory / NVMe and copies misses into device slots
// (runtime/ds41/cache.py:1852-1996: _blit, _bind, _unbind, _flush, _install_if_absent; prefetch on a
// side stream, :2064-2080 prefetch_gpu). It learns which experts a step needs with a host sync on the
// routes (cache.py:2315, indices.tolist()) and publishes pointers through a host table copied to the
// device (_flush). Here the needed set, the slot choice and the pointer-table updates happen on the
// device (eva_pool_plan, one CTA), and the copies are done by a kernel that reads the pinned host
// records through their unified addresses (eva_pool_copy), so a layer's staging is two launches in
// stream order and a prefetch of the next layer's predicted experts can run on a side stream under
// the current layer's compute.
//
// Policy: CLOCK over the pool's slots (a hand that skips slots stamped at or after `protect`, i.e.
// in use by the layer running now or needed by the layer being planned), free slots first. The pool
// holds at least as many slots as one layer has local experts, so a layer's needed set always fits.
#include <cuda_runtime.h>

#include "common.cuh"
#include "internal.h"

namespace eva {
namespace {

constexpr int POOL_MAX_LOCAL = 1024;
constexpr int PLAN_THREADS = 1024;
constexpr int COPY_CHUNK = 64 * 1024;   // bytes per copy work unit
constexpr int COPY_CTAS = 32;

__device__ __forceinline__ bool need_bit(const uint32_t* need, int e) { return (need[e >> 5] >> (e & 31)) & 1u; }

// Exclusive prefix sum of a 0/1 flag over the block; *total receives the block's sum. Every thread
// of the block calls it (it synchronises).
__device__ __forceinline__ int block_scan01(int flag, int* warp_sums, int* total)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const unsigned bal = __ballot_sync(0xffffffffu, flag);
    const int in_warp = __popc(bal & ((1u << lane) - 1u));
    __syncthreads();                                   // warp_sums free from the previous call
    if (lane == 0) warp_sums[warp] = __popc(bal);
    __syncthreads();
    int before = 0, sum = 0;
    for (int w = 0; w < nwarps; ++w) {
        const int v = warp_sums[w];
        before += w < warp ? v : 0;
        sum += v;
    }
    *total = sum;
    return before + in_warp;
}

// state (int32 words): [0] hand, [1] unused, [2] status, [3] unused; [4..5] int64 bytes copied;
// [6..7] int64 plan counter. Stamps and the counter are 64-bit: one exact plan per layer per step
// would take a 32-bit counter past 2^31 within hours of serving a 58-layer model, after which
// "stamped before `protect`" would no longer mean "older".
//
// The plan is the sequential CLOCK walk (misses in expert order, each taking the next slot from the
// hand that is free or stamped before `protect`) computed in parallel: a slot taken by one miss
// becomes ineligible and the hand moves past it, so the k-th miss takes the k-th eligible slot in
// circular order from the hand, and the hand ends one past the last slot taken.
__global__ void __launch_bounds__(PLAN_THREADS) pool_plan_kernel(EvaExpertPool pool, const EvaPoolLayer* layers,
                                                                 int32_t li, const void* sel, int32_t sel64,
                                                                 float* rw, int32_t rows, int32_t topk,
                                                                 int32_t prefetch, int32_t* jobs, float* rw_hit,
                                                                 float* rw_miss)
{
    __shared__ uint32_t need[POOL_MAX_LOCAL / 32];
    __shared__ uint32_t missbits[POOL_MAX_LOCAL / 32];   // misses given a slot by this plan
    __shared__ uint32_t lostbits[POOL_MAX_LOCAL / 32];   // misses left without one
    __shared__ int16_t miss[POOL_MAX_LOCAL];
    __shared__ int take[POOL_MAX_LOCAL];
    __shared__ int take_pos[POOL_MAX_LOCAL];
    __shared__ int warp_sums[PLAN_THREADS / 32];
    const EvaPoolLayer L = layers[li];
    if (L.n_local < 1 || L.n_local > POOL_MAX_LOCAL) {
        if (threadIdx.x == 0) {
            atomicOr(&pool.state[2], ST_CAPACITY);
            jobs[0] = 0;
        }
        return;
    }
    const int t = threadIdx.x;
    const int nw = (L.n_local + 31) / 32;
    for (int i = t; i < nw; i += blockDim.x) {
        need[i] = prefetch ? L.last_needed[i] : 0u;
        missbits[i] = 0u;
        lostbits[i] = 0u;
    }
    __syncthreads();
    if (!prefetch) {
        for (int i = t; i < rows * topk; i += blockDim.x) {
            if (rw[i] == 0.0f) continue;
            const long long e = sel64 ? static_cast<const long long*>(sel)[i] : static_cast<const int32_t*>(sel)[i];
            if (e >= 0 && e < L.n_local) atomicOr(&need[e >> 5], 1u << (e & 31));
        }
        __syncthreads();
        for (int i = t; i < nw; i += blockDim.x) L.last_needed[i] = need[i];
    }
    int* st = pool.state;
    // exact plan: a new stamp, protecting what it stamps now; prefetch (issued after the plan of the
    // layer that runs meanwhile): the next stamp, protecting that layer's slots too
    long long* counter = reinterpret_cast<long long*>(st + 6);
    const long long cur = *counter;
    const long long stamp = cur + 1;
    const long long protect = prefetch ? cur : stamp;
    const int hand = st[0];
    const int n = pool.n_slots;
    // hits stamped first, so that every needed resident slot is protected before any eviction; the
    // misses listed in expert order (n_local <= blockDim.x)
    int is_miss = 0;
    if (t < L.n_local && need_bit(need, t)) {
        const int s = L.slot_of[t];
        if (s >= 0) pool.stamp[s] = stamp;
        else is_miss = 1;
    }
    int n_miss;
    const int mi = block_scan01(is_miss, warp_sums, &n_miss);
    if (is_miss) miss[mi] = static_cast<int16_t>(t);
    // the k-th eligible slot in circular order from the hand, k < n_miss (the stamps written above
    // are visible to the block after the scan's barriers)
    int n_take = 0;
    for (int base = 0; base < n && n_take < n_miss; base += blockDim.x) {
        const int p = base + t;
        int c = -1, elig = 0;
        if (p < n) {
            c = hand + p < n ? hand + p : hand + p - n;
            elig = pool.owner[c] < 0 || pool.stamp[c] < protect;
        }
        int cnt;
        const int r = n_take + block_scan01(elig, warp_sums, &cnt);
        if (elig && r < n_miss) {
            take[r] = c;
            take_pos[r] = p;
        }
        n_take += cnt;
    }
    n_take = min(n_take, n_miss);
    __syncthreads();
    // bind: every miss with a slot, its slot's previous owner unbound from its layer's table
    for (int k = t; k < n_take; k += blockDim.x) {
        const int e = miss[k], s = take[k];
        const int old = pool.owner[s];
        if (old >= 0) {
            const EvaPoolLayer O = layers[old >> 16];
            const int oe = old & 0xffff;
            O.slot_of[oe] = -1;
            for (int r = 0; r < 9; ++r) O.table[static_cast<size_t>(r) * O.n_local + oe] = 0;
        }
        pool.owner[s] = (li << 16) | e;
        pool.stamp[s] = stamp;
        L.slot_of[e] = s;
        const int64_t b = reinterpret_cast<int64_t>(pool.slots) + static_cast<int64_t>(s) * pool.record_bytes;
        for (int r = 0; r < 9; ++r) L.table[static_cast<size_t>(r) * L.n_local + e] = b + L.row_off[r];
        jobs[1 + 2 * k] = e;
        jobs[2 + 2 * k] = s;
    }
    if (!prefetch) {
        if (t < n_miss) atomicOr(t < n_take ? &missbits[miss[t] >> 5] : &lostbits[miss[t] >> 5], 1u << (miss[t] & 31));
        __syncthreads();
        if (rw_hit != nullptr || n_take < n_miss) {
            for (int i = t; i < rows * topk; i += blockDim.x) {
                const long long e = sel64 ? static_cast<const long long*>(sel)[i] : static_cast<const int32_t*>(sel)[i];
                const bool ok = e >= 0 && e < L.n_local;
                const bool lost = ok && need_bit(lostbits, static_cast<int>(e));
                const float w = lost ? 0.0f : rw[i];
                if (rw_hit != nullptr) {
                    const bool copied = ok && need_bit(missbits, static_cast<int>(e));
                    rw_hit[i] = copied ? 0.0f : w;
                    rw_miss[i] = copied ? w : 0.0f;
                } else if (lost) {
                    rw[i] = 0.0f;
                }
            }
        }
    }
    if (t == 0) {
        if (!prefetch) *counter = stamp;
        if (n_take < n_miss && !prefetch) atomicOr(&st[2], ST_CAPACITY);   // the pool is smaller than a layer
        if (n_take > 0) st[0] = take_pos[n_take - 1] + 1 + hand >= n ? take_pos[n_take - 1] + 1 + hand - n
                                                                     : take_pos[n_take - 1] + 1 + hand;
        jobs[0] = n_take;
        *reinterpret_cast<long long*>(st + 4) += static_cast<long long>(n_take) * pool.record_bytes;
    }
}

// Copy the planned records: work unit = (job, 64 KB chunk), 16-byte loads from the pinned host
// record (unified address) and 16-byte stores into the device slot.
__global__ void __launch_bounds__(512) pool_copy_kernel(EvaExpertPool pool, const EvaPoolLayer* layers, int32_t li,
                                                        const int32_t* jobs)
{
    const EvaPoolLayer L = layers[li];
    const int njobs = jobs[0];
    const long long chunks = (pool.record_bytes + COPY_CHUNK - 1) / COPY_CHUNK;
    const long long units = static_cast<long long>(njobs) * chunks;
    for (long long u = blockIdx.x; u < units; u += gridDim.x) {
        const int j = static_cast<int>(u / chunks);
        const long long c = u % chunks;
        const int e = jobs[1 + 2 * j], s = jobs[2 + 2 * j];
        const long long off = c * COPY_CHUNK;
        const long long n = min(static_cast<long long>(COPY_CHUNK), pool.record_bytes - off) / 16;
        const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(L.host_records) +
                                                          static_cast<long long>(e) * pool.record_bytes + off);
        uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(pool.slots) + static_cast<long long>(s) * pool.record_bytes + off);
        long long i = threadIdx.x;
        for (; i + 3 * blockDim.x < n; i += 4 * blockDim.x) {      // 4 host reads in flight per thread
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = src[i + u * blockDim.x];
#pragma unroll
            for (int u = 0; u < 4; ++u) dst[i + u * blockDim.x] = v[u];
        }
        for (; i < n; i += blockDim.x) dst[i] = src[i];
    }
}

}  // namespace
}  // namespace eva

using namespace eva;

extern "C" int eva_pool_plan(const EvaExpertPool* pool, const EvaPoolLayer* layers, int32_t layer, const void* sel,
                             int32_t sel_is_i64, float* rw, int32_t rows, int32_t topk, int32_t prefetch,
                             int32_t* jobs, float* rw_hit, float* rw_miss, void* stream)
{
    if (!pool || !layers || !jobs || layer < 0 || layer > 0x7fff || rows < 0 || topk < 1) return EVA_ERR_INVALID;
    if (!prefetch && rows > 0 && (!sel || !rw)) return EVA_ERR_INVALID;
    if ((rw_hit == nullptr) != (rw_miss == nullptr) || (prefetch && rw_hit)) return EVA_ERR_INVALID;
    if (pool->n_slots < 1 || pool->record_bytes <= 0 || pool->record_bytes % 16 || !pool->slots || !pool->owner ||
        !pool->stamp || !pool->state)
        return EVA_ERR_INVALID;
    pool_plan_kernel<<<1, PLAN_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(*pool, layers, layer, sel, sel_is_i64 ? 1 : 0,
                                                                                rw, rows, topk, prefetch ? 1 : 0, jobs,
                                                                                rw_hit, rw_miss);
    return cudaGetLastError() == cudaSuccess ? EVA_OK : EVA_ERR_CUDA;
}

extern "C" int eva_pool_copy(const EvaExpertPool* pool, const EvaPoolLayer* layers, int32_t layer, const int32_t* jobs,
                             void* stream)
{
    if (!pool || !layers || !jobs || layer < 0) return EVA_ERR_INVALID;
    // 32 CTAs already read host memory at the link's rate; more would only take issue slots from the
    // experts kernel that a prefetch runs beside
    pool_copy_kernel<<<COPY_CTAS, 512, 0, static_cast<cudaStream_t>(stream)>>>(*pool, layers, layer, jobs);
    return cudaGetLastError() == cudaSuccess ? EVA_OK : EVA_ERR_CUDA;
}

extern "C" int eva_host_mapped(const void* p)
{
    cudaPointerAttributes a;
    if (!p || cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return a.type == cudaMemoryTypeHost && a.devicePointer == p ? 1 : 0;
}
