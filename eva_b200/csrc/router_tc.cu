// Router logits for prefill-sized batches on the tensor cores, at FP32 accuracy.
//
// The reference computes the logits as an FP32 product of the activations and the FP32 router
// weight (runtime/ds41/model.py:404-406, F.linear(x.float(), W)). Here the activations are bf16
// (exact in bf16) and each FP32 weight is split into three bf16 parts w = hi + mid + lo (8 + 8 + 8
// significand bits: exact for every normal weight), so x * w = x * hi + x * mid + x * lo with each
// bf16 x bf16 product exact in the FP32 accumulator. Two TMEM accumulators keep the hi products apart
// from the two smaller ones and are summed in the epilogue.
//
// One CTA: 128 tokens x 128 experts over one k slice, 3-stage TMA ring (x tile + the three weight
// parts, 64 KB per 64-wide k step), one thread issuing tcgen05.mma (M = 128, N = 128, K = 16), four
// epilogue warps reading TMEM. The k range is split so that (token tiles x expert tiles x k slices)
// fills the SMs; the slices' partial logits [ks][M][E] are summed in slice order by the top-k kernel.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "tc.cuh"

namespace eva {

constexpr int RT_BM = 128, RT_BN = 128, RT_BK = 64, RT_STAGES = 3;
constexpr int RT_TILE = RT_BM * RT_BK * 2;             // 16 KB: one 128-row x 64-k bf16 tile
constexpr int RT_STAGE = 4 * RT_TILE;                   // x, w_hi, w_mid, w_lo
constexpr int RT_SMEM = RT_STAGES * RT_STAGE + 1024;    // + alignment slack of the swizzled ring
constexpr int RT_THREADS = 192;                         // warps 0-3 epilogue, 4 producer, 5 MMA
constexpr int RT_TARGET_CTAS = 148;                     // B200 SMs: the k split fills one wave
constexpr int RT_MIN_KSLICE = 512;

static_assert(RT_BM == 128 && RT_BN % 16 == 0 && RT_BN <= 256, "tcgen05 M = 128 shape");

// w (fp32, n elements) -> hi, mid, lo planes of n bf16 each
__global__ void __launch_bounds__(256) router_split_kernel(const float* __restrict__ w, size_t n,
                                                           __nv_bfloat16* __restrict__ out)
{
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const float v = w[i];
        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
        const float r1 = v - __bfloat162float(hi);
        const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
        const float r2 = r1 - __bfloat162float(mid);
        out[i] = hi;
        out[n + i] = mid;
        out[2 * n + i] = __float2bfloat16_rn(r2);
    }
}

struct RtBars {
    uint64_t full[RT_STAGES], empty[RT_STAGES], done;
    uint32_t tmem;
};

__global__ void __launch_bounds__(RT_THREADS, 1)
    router_tc_kernel(const __grid_constant__ CUtensorMap mx, const __grid_constant__ CUtensorMap mw, int M, int H, int E,
                     int kper, float* __restrict__ part, int* status)
{
    extern __shared__ uint8_t smem_raw[];
    __shared__ RtBars B;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * RT_BM, n0 = blockIdx.y * RT_BN, ks = blockIdx.z;
    const int k0 = ks * kper, k1 = min(H, k0 + kper);
    const int nk = (k1 - k0 + RT_BK - 1) / RT_BK;
    uint8_t* ring = align1024(smem_raw);
    if (threadIdx.x == 0) {
        for (int i = 0; i < RT_STAGES; ++i) {
            mbar_init(&B.full[i], 1);
            mbar_init(&B.empty[i], 1);
        }
        mbar_init(&B.done, 1);
        fence_barrier_init();
    }
    if (warp == 5) tmem_alloc(&B.tmem, 2 * RT_BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = B.tmem;

    if (warp == 4) {
        if (lane == 0) {
            for (int it = 0; it < nk; ++it) {
                const int st = it % RT_STAGES;
                mbar_wait(&B.empty[st], ((it / RT_STAGES) & 1) ^ 1, status);
                uint8_t* stage = ring + st * RT_STAGE;
                const int k = k0 + it * RT_BK;
                mbar_arrive_expect_tx(&B.full[st], RT_STAGE);
                tma_load_2d(stage, &mx, k, m0, &B.full[st]);
#pragma unroll
                for (int p = 0; p < 3; ++p) tma_load_3d(stage + (1 + p) * RT_TILE, &mw, k, n0, p, &B.full[st]);
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_bf16(RT_BM, RT_BN);
            for (int it = 0; it < nk; ++it) {
                const int st = it % RT_STAGES;
                mbar_wait(&B.full[st], (it / RT_STAGES) & 1, status);
                tc_fence_after();
                const uint32_t sa = smem_u32(ring + st * RT_STAGE);
#pragma unroll
                for (int kk = 0; kk < RT_BK / 16; ++kk) {
                    const uint64_t da = umma_desc_sw128(sa + kk * 32);
                    const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
                    umma_f16(tmem, da, umma_desc_sw128(sa + RT_TILE + kk * 32), idesc, acc);
                    umma_f16(tmem + RT_BN, da, umma_desc_sw128(sa + 2 * RT_TILE + kk * 32), idesc, acc);
                    umma_f16(tmem + RT_BN, da, umma_desc_sw128(sa + 3 * RT_TILE + kk * 32), idesc, 1u);
                }
                umma_commit(&B.empty[st]);
            }
            umma_commit(&B.done);
        }
    } else {
        // epilogue: warp w owns TMEM lanes (token rows) 32 w .. 32 w + 31
        mbar_wait(&B.done, 0, status);
        tc_fence_after();
        const int row = m0 + warp * 32 + lane;
        const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
        float* orow = part + (static_cast<size_t>(ks) * M + row) * E;
        for (int c = 0; c < RT_BN / 32; ++c) {
            const int n = n0 + c * 32;
            if (n >= E) break;   // warp-uniform
            float hi[32], lo[32];
            tmem_ld32(tmem + lane_base + c * 32, hi);
            tmem_ld32(tmem + lane_base + RT_BN + c * 32, lo);
            if (row < M) {
                if ((E & 3) == 0 && n + 32 <= E) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<float4*>(orow + n + j) =
                            make_float4(hi[j] + lo[j], hi[j + 1] + lo[j + 1], hi[j + 2] + lo[j + 2], hi[j + 3] + lo[j + 3]);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (n + j < E) orow[n + j] = hi[j] + lo[j];
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, 2 * RT_BN);
    }
}

int router_tc_split(int M, int H, int E, int* kper_out)
{
    if (M < ROUTER_TC_MIN_ROWS || H % RT_BK != 0 || E < 1) return 0;
    const long long tiles = static_cast<long long>((M + RT_BM - 1) / RT_BM) * ((E + RT_BN - 1) / RT_BN);
    const int max_ks = std::max(1, H / RT_MIN_KSLICE);
    const int want = static_cast<int>(std::max<long long>(1, std::min<long long>(max_ks, RT_TARGET_CTAS / tiles)));
    const int steps = H / RT_BK;
    const int kper = (steps + want - 1) / want * RT_BK;
    if (kper_out) *kper_out = kper;
    return (H + kper - 1) / kper;
}

size_t router_part_rows(int max_rows, int H, int E)
{
    size_t rows = std::max<size_t>(max_rows, static_cast<size_t>((H + ROUTER_KSLICE - 1) / ROUTER_KSLICE) *
                                                 std::min(max_rows, ROUTER_TC_MIN_ROWS - 1));
    // ks(M) depends on M only through ceil(M / 128): within each such block the largest M needs the
    // most rows
    for (int t = 1; (t - 1) * RT_BM < max_rows; ++t) {
        const int m = std::min(t * RT_BM, max_rows);
        rows = std::max(rows, static_cast<size_t>(router_tc_split(m, H, E, nullptr)) * m);
    }
    return rows;
}

// bf16 [rows][cols] row-major (2-D) or [planes][rows][cols] (3-D), box 64 x 128 (x 1), 128B swizzle
static bool make_bf16_map(CUtensorMap* m, const void* base, uint64_t planes, uint64_t rows, uint64_t cols)
{
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[3] = {cols, rows, planes};
    const cuuint64_t strides[2] = {cols * 2, rows * cols * 2};
    const cuuint32_t box[3] = {RT_BK, RT_BM, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const cuuint32_t rank = planes > 1 ? 3 : 2;
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool router_tc_usable(const void* x, int x_bf16, int M, int H, int E, const void* wsplit)
{
    return x_bf16 && wsplit && router_tc_split(M, H, E, nullptr) > 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
           (reinterpret_cast<uintptr_t>(wsplit) & 15) == 0 && encode_fn() != nullptr;
}

cudaError_t launch_router_tc(const void* x, int M, int H, int E, const float* W, void* wsplit, float* part, int* status,
                             int* ks_used, cudaStream_t stream)
{
    int kper = 0;
    const int ks = router_tc_split(M, H, E, &kper);
    if (ks < 1) return cudaErrorInvalidValue;
    CUtensorMap mx, mw;
    if (!make_bf16_map(&mx, x, 1, M, H) || !make_bf16_map(&mw, wsplit, 3, E, H)) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(router_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, RT_SMEM);
    if (e != cudaSuccess) return e;
    const size_t n = static_cast<size_t>(E) * H;
    router_split_kernel<<<static_cast<unsigned>(std::min<size_t>((n + 255) / 256, 148 * 8)), 256, 0, stream>>>(
        W, n, static_cast<__nv_bfloat16*>(wsplit));
    dim3 grid((M + RT_BM - 1) / RT_BM, (E + RT_BN - 1) / RT_BN, ks);
    router_tc_kernel<<<grid, RT_THREADS, RT_SMEM, stream>>>(mx, mw, M, H, E, kper, part, status);
    *ks_used = ks;
    return cudaGetLastError();
}

}  // namespace eva
