// eva_moe_experts_noalloc: the fused expert path with its scratch in a fixed, file-scope device
// array instead of a caller-provided workspace, for callers that cannot allocate device memory.
//
// The scratch (counters, run table, rotated inputs, activations, per-slot partial outputs, status
// word) lives in g_noalloc_scratch below: EVA_NOALLOC_SCRATCH_BYTES per GPU, reserved on every
// device that loads this library for as long as the process lives. Every call shares it and it
// keeps the previous call's contents; everything that must start at zero (the status word, the
// completion counters, the work counter) is cleared by each call on its stream before use. Two
// calls whose work overlaps on the GPU (different streams, or different host threads without
// ordering) race on this memory and corrupt each other's results; order them on one stream.
#include <cuda_runtime.h>

#include <mutex>

#include "internal.h"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[EVA_NOALLOC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_setup_mutex;
void* g_scratch_addr[MAX_DEVICES] = {};

// Device address of the array for the current device. In host code the array's name is only a
// host-side stand-in, so the real address is looked up once per device with that device current.
cudaError_t scratch_address(void** out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= MAX_DEVICES) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return cudaSuccess;
}

}  // namespace

using namespace eva;

extern "C" int eva_moe_experts_noalloc(const EvaMoeShape* shape, const void* x, int32_t x_is_bf16, int32_t M,
                                       const void* sel, int32_t sel_is_i64, const float* rw,
                                       const int64_t* const* tables, const int64_t* shared, float* out_f32,
                                       void* out_bf16, int32_t* status_out, void* stream)
{
    if (!shape || M < 0) return EVA_ERR_INVALID;
    if (eva_moe_workspace_bytes(shape, 1) == 0) return EVA_ERR_INVALID;
    if (M == 0) return EVA_OK;
    // every call takes the decode kernel (path 1), so the layout holds no tensor-core buffers
    const WsLayout L = ws_layout(*shape, M, /*allow_split=*/false, /*routing=*/false, /*tensor_core=*/false);
    if (L.total > EVA_NOALLOC_SCRATCH_BYTES) return EVA_ERR_WORKSPACE;   // too many rows for the fixed scratch
    // all argument checks before any device call (symbol lookup, memset, launches)
    const int v = experts_validate(shape, x, M, sel, rw, tables, shared, out_f32, out_bf16);
    if (v != EVA_OK) return v;
    void* base = nullptr;
    if (scratch_address(&base) != cudaSuccess) return EVA_ERR_CUDA;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the status word is the only state read before it is written; counters are zeroed by the
    // permutation kernel of this call
    if (cudaMemsetAsync(static_cast<unsigned char*>(base) + L.status, 0, 4, st) != cudaSuccess) return EVA_ERR_CUDA;
    const int rc = experts_impl(shape, x, x_is_bf16, M, sel, sel_is_i64, rw, tables, shared, base, L.total, out_f32,
                                out_bf16, st, /*allow_split=*/false, /*path=*/1);
    if (rc != EVA_OK) return rc;
    if (status_out &&
        cudaMemcpyAsync(status_out, static_cast<unsigned char*>(base) + L.status, 4, cudaMemcpyDeviceToDevice, st) !=
            cudaSuccess)
        return EVA_ERR_CUDA;
    return EVA_OK;
}
