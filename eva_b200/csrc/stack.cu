// Layer-stack glue between MoE layers: residual add + RMSNorm, one kernel per layer boundary.
//
// Reference: runtime/ds41/model.py:968-970 `rms(x, weight, eps)` = (weight * x.float() *
// rsqrt(mean_square(x) + eps)).to(x.dtype), mean_square over the last dimension in FP32
// (model.py:168-176). Here the residual stream is kept in FP32 ([M][H]); the kernel first adds the
// previous layer's output to it, then writes the normalised BF16 input of the next layer.
#include <cuda_runtime.h>

#include "common.cuh"

namespace eva {

constexpr int RMS_THREADS = 256;

// CTA per row. resid[m] += add[m] (if add); h[m] = bf16((w * resid[m]) * rsqrt(mean(resid[m]^2) + eps)).
__global__ void __launch_bounds__(RMS_THREADS) rmsnorm_residual_kernel(int H, float* __restrict__ resid,
                                                                       const float* __restrict__ add,
                                                                       const void* __restrict__ weight, int w_bf16,
                                                                       float eps, __nv_bfloat16* __restrict__ h)
{
    __shared__ float red[RMS_THREADS / 32];
    const int m = blockIdx.x;
    float* r = resid + static_cast<size_t>(m) * H;
    const float* a = add ? add + static_cast<size_t>(m) * H : nullptr;
    float ss = 0.0f;
    for (int c = threadIdx.x * 4; c < H; c += RMS_THREADS * 4) {
        float4 v = *reinterpret_cast<const float4*>(r + c);
        if (a) {
            const float4 d = *reinterpret_cast<const float4*>(a + c);
            v.x += d.x;
            v.y += d.y;
            v.z += d.z;
            v.w += d.w;
            *reinterpret_cast<float4*>(r + c) = v;
        }
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < RMS_THREADS / 32; ++i) tot += red[i];
    const float inv = rsqrtf(tot / static_cast<float>(H) + eps);
    __nv_bfloat16* hr = h + static_cast<size_t>(m) * H;
    for (int c = threadIdx.x * 4; c < H; c += RMS_THREADS * 4) {
        const float4 v = *reinterpret_cast<const float4*>(r + c);
        float w[4];
        load4_x(weight, c, w_bf16, w);
        const __nv_bfloat162 lo = __floats2bfloat162_rn((w[0] * v.x) * inv, (w[1] * v.y) * inv);
        const __nv_bfloat162 hi = __floats2bfloat162_rn((w[2] * v.z) * inv, (w[3] * v.w) * inv);
        uint2 u;
        u.x = *reinterpret_cast<const uint32_t*>(&lo);
        u.y = *reinterpret_cast<const uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(hr + c) = u;
    }
}

}  // namespace eva

using namespace eva;

extern "C" int eva_rmsnorm_residual(int32_t H, int32_t M, float* resid, const float* add, const void* weight,
                                    int32_t weight_is_bf16, float eps, void* h_out, void* stream)
{
    if (H <= 0 || H % 4 || M < 0 || !(eps >= 0.0f)) return EVA_ERR_INVALID;
    if (M == 0) return EVA_OK;
    if (!resid || !weight || !h_out) return EVA_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(resid) & 15) || (reinterpret_cast<uintptr_t>(add) & 15) ||
        (reinterpret_cast<uintptr_t>(h_out) & 7) || (reinterpret_cast<uintptr_t>(weight) & 7))
        return EVA_ERR_INVALID;
    rmsnorm_residual_kernel<<<M, RMS_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
        H, resid, add, weight, weight_is_bf16 ? 1 : 0, eps, static_cast<__nv_bfloat16*>(h_out));
    return cudaGetLastError() == cudaSuccess ? EVA_OK : EVA_ERR_CUDA;
}
