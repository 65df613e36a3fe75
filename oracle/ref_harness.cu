// GPU golden from the reference itself — TEST INFRASTRUCTURE ONLY.
//
// Compiled by oracle/build_ref.py straight from the reference checkout (the headers are included
// in place with -I, never copied into this repository) into oracle/_ref/libref_coop.so. It exposes
// the reference's own EXL3 decoder and MoE coop kernels through a small C ABI so the GPU tests can
// compare the eva_b200 kernels with them on the same device and inputs.
//
// What runs is the reference's code (paths within Findddx/eva):
//   runtime/ds41/csrc/moe_coop2048/vendor/quant/exl3_dq.cuh:287-330    dq_dispatch<K, mul1>
//   runtime/ds41/csrc/moe_coop2048/prepare_runs.cuh:8-66               ds41_prepare_runs2048
//   runtime/ds41/csrc/moe_coop2048/vendor/quant/exl3_moe_coop_kernel.cuh rot / A / B kernels
// This file is only the launcher: it restates binding.cu:42-71 (launch<K>) and :125-141 (the
// parameter block) for any H / I / top-k instead of the hard-coded 5120 / 2304 / 6, and adds a
// per-tile decode kernel around dq_dispatch.
#define EXL3_MOE_COOP_DEFINE_ROT
#define DS41_EXTERNAL_RUN_PREPARE
#include "vendor/quant/exl3_moe_coop_kernel.cuh"
#include "prepare_runs.cuh"

#include <cuda_runtime.h>

namespace {

template <int K>
__global__ void ref_dequant_kernel(const uint32_t* tr, int in, int out, half* w)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntn = out / 16;
    const long long tile = (long long) blockIdx.x * 8 + warp;
    if (tile >= (long long) (in / 16) * ntn) return;
    const int kt = (int) (tile / ntn), nt = (int) (tile % ntn);
    FragB f0, f1;
    dq_dispatch<K, 2>(tr + tile * 8 * K, lane << 3, f0, f1);
    // positions 8 lane + j, j = 0..7 -> B fragment of mma.m16n8k16: f0 feeds output columns 0-7 of
    // the tile, f1 columns 8-15; element e of a fragment is k = 2 (lane % 4) + (e % 2) + 8 (e / 2)
    const half v[8] = {__low2half(f0[0]), __high2half(f0[0]), __low2half(f0[1]), __high2half(f0[1]),
                       __low2half(f1[0]), __high2half(f1[0]), __low2half(f1[1]), __high2half(f1[1])};
    for (int j = 0; j < 8; ++j) {
        const int e = j & 3;
        const int n = (lane >> 2) + 8 * (j >> 2);
        const int k = 2 * (lane & 3) + (e & 1) + 8 * (e >> 1);
        w[(size_t) (kt * 16 + k) * out + nt * 16 + n] = v[j];
    }
}

template <int K>
void launch(MoeCoopParams p, cudaStream_t stream)
{
    using namespace ds41_moe_coop2048_ns;
    p.a_global = p.bsz > 1;
    p.ksplit_a = p.ksplit_b = 1;
    p.dbg = 0;
    constexpr int CB_MUL1 = 2;
    void* ka = (void*) exl3_moe_coop_a_kernel<K, CB_MUL1, false>;
    void* kb = (void*) exl3_moe_coop_b_kernel<K, CB_MUL1, false>;
    const int smem_a = smem_a_bytes<K>(p.Hi);
    const int smem_b = smem_b_bytes<K>();
    cudaFuncSetAttribute(ka, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_a);
    cudaFuncSetAttribute(kb, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_b);
    const int slots = p.bsz * p.topk;
    ds41_prepare_runs2048<<<1, 512, 0, stream>>>(p);
    if (p.a_global) {
        const int items = slots * (p.Hi / 128) * 2;
        const int grid = (items + MOE_COOP_THREADS / 32 - 1) / (MOE_COOP_THREADS / 32);
        exl3_moe_coop_rot_kernel<<<grid, MOE_COOP_THREADS, 0, stream>>>(p);
    }
    void* arguments[] = {(void*) &p};
    cudaLaunchKernel(ka, dim3(slots * 2 * (p.I / MOE_COOP_COLS)), dim3(MOE_COOP_THREADS), arguments, smem_a, stream);
    cudaLaunchKernel(kb, dim3(slots * (p.Ho / MOE_COOP_COLS)), dim3(MOE_COOP_THREADS), arguments, smem_b, stream);
}

}  // namespace

extern "C" {

int ref_dequant(const void* trellis, int in, int out, int K, void* w, void* stream)
{
    const long long tiles = (long long) (in / 16) * (out / 16);
    const unsigned grid = (unsigned) ((tiles + 7) / 8);
    cudaStream_t st = (cudaStream_t) stream;
    const uint32_t* tr = (const uint32_t*) trellis;
    half* wo = (half*) w;
    if (K == 2) ref_dequant_kernel<2><<<grid, 256, 0, st>>>(tr, in, out, wo);
    else if (K == 3) ref_dequant_kernel<3><<<grid, 256, 0, st>>>(tr, in, out, wo);
    else if (K == 4) ref_dequant_kernel<4><<<grid, 256, 0, st>>>(tr, in, out, wo);
    else return 1;
    return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

// Int32 scratch needed by the coop kernels (completion counters + run table).
long long ref_coop_ctr_len(int capacity, int topk, int inter, int hidden)
{
    return exl3_moe_coop_ctr_len((long long) capacity * topk, capacity, inter, hidden);
}

// One call of the reference's routed MoE kernels (no shared expert), as binding.cu run():
//   x Half [bsz, H]; sel int64 [bsz, topk]; rw Half [bsz, topk]; tables: 9 device int64 [n_local]
//   scratch: had_g, had_u Half [slots, H]; gu_g, gu_u, act_out Half [slots, I]; d_out Float [slots, H];
//   ctr int32 [ref_coop_ctr_len]; out Float [capacity, H]; slots = capacity * topk.
int ref_coop_run(const void* x, const void* sel, const void* rw, int bsz, int topk, int H, int I,
                 const int64_t* const* tables, int n_local, void* had_g, void* had_u, void* gu_g, void* gu_u,
                 void* act_out, void* d_out, void* ctr, int capacity, void* out, int K, float limit, void* stream)
{
    if (bsz < 1 || bsz > capacity || capacity * topk > 2048 || H % 128 || I % 128) return 1;
    cudaStream_t st = (cudaStream_t) stream;
    MoeCoopParams p = {};
    const int slots = capacity * topk;
    p.x = (const half*) x;
    p.x_stride = H;
    p.sel = (const int64_t*) sel;
    p.rw = (const half*) rw;
    p.bsz = bsz;
    p.topk = topk;
    p.H = p.Hi = p.Ho = p.H_out = H;
    p.I = I;
    p.min_expert = -1;
    p.max_expert = 0;
    p.n_local = n_local;
    p.g_trellis = tables[0]; p.g_suh = tables[1]; p.g_svh = tables[2];
    p.u_trellis = tables[3]; p.u_suh = tables[4]; p.u_svh = tables[5];
    p.d_trellis = tables[6]; p.d_suh = tables[7]; p.d_svh = tables[8];
    p.gated = true;
    p.act = MOE_COOP_ACT_SILU;
    p.act_limit = limit;
    p.gu_f32 = false;
    p.had_g = (half*) had_g;
    p.had_u = (half*) had_u;
    p.gu_g = gu_g;
    p.gu_u = gu_u;
    p.act_out = (half*) act_out;
    p.d_out = (float*) d_out;
    p.slots_max = slots;
    p.rows_max = capacity;
    p.ctr_a_len = slots * (I / 128);
    p.ctr_b_len = capacity * (H / 128);
    p.ctr_a = (int*) ctr;
    p.ctr_b = p.ctr_a + p.ctr_a_len;
    p.runs = p.ctr_b + p.ctr_b_len;
    p.out = (float*) out;
    p.out_stride = H;
    cudaMemsetAsync(p.ctr_a, 0, ref_coop_ctr_len(capacity, topk, I, H) * sizeof(int), st);
    if (K == 2) launch<2>(p, st);
    else if (K == 3) launch<3>(p, st);
    else if (K == 4) launch<4>(p, st);
    else return 1;
    return cudaGetLastError() == cudaSuccess ? 0 : 2;
}

}  // extern "C"
