// Prefill-shaped MoE experts on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Tokens are grouped by expert (the permutation's sorted order), so each expert is a dense
// [rows x H] x [H x I] problem. A cluster of two CTAs on neighbouring SMs computes one 256-row x
// 256-column output tile with tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16): CTA r holds
// rows 128 r .. 128 r + 127 of the activations and decodes weight columns 128 r .. 128 r + 127,
// the tensor cores of both SMs read both halves, and each CTA's TMEM receives its 128 rows x 256
// columns. Per SM this reads half the shared-memory bytes per MAC of a one-SM 128 x 128 tile,
// which is what bounds a tcgen05 kernel whose weights are written to shared memory by warps.
// A tile of at most 128 rows (an expert's last, or a small expert's only tile) runs as M = 128
// pair MMAs instead: each CTA holds 64 rows, the tensor work on padding rows halves, the decode is
// unchanged (its accumulators lie folded in TMEM: pf_tmem_to_smem_half).
//   warp 0      activation producer: 2-D TMA loads of the CTA's activation rows (completion counted
//               on the leader CTA's barrier) into the activation/weight ring (PfCfg: stages, depth)
//   last warp   trellis producer: one 2-D tensor copy per stage (per-expert maps from pf_maps) of
//               the CTA's trellis rows into a ring of their own, whose slots the decoders release as soon as they have read their words
//   warps 2..   decoders: EXL3 decode of the stage's weight tiles into raw codebook values
//               h = 1024 + bytesum (exact fp16) straight into the UMMA K-major 128B-swizzled layout;
//               they arrive on the leader's barrier (the peer CTA's from across the cluster). The
//               codebook's affine map w = c0 h + c1 is applied in the epilogues: x . w = c0 (x . h)
//               + c1 sum(x), with sum(x) over the row's stored fp16 inputs (pf_rotate and the gate/up
//               epilogue write per-chunk partial sums)
//   warp 1      leader CTA: one thread issues the pair MMAs and commits each stage to both CTAs
//   all warps   epilogue: tcgen05.ld of the CTA's accumulators, Hadamard / scales / activation in
//               registers, fp16 or fp32 stores.
// Kernels:
//   pf_rotate    x -> fp16(H128(x * suh)) for gate and up, rows in expert-sorted order
//   pf_gateup    gate and up accumulators (TMEM columns 0-255 / 256-511), epilogue = the MoE
//                coop A epilogue (exl3_moe_coop_kernel.cuh:758-808): H128, svh, SiLU*mul, suh_down,
//                H128 -> fp16 down input
//   pf_down      down projection, epilogue H128 * svh * routing weight -> per-slot fp32 rows
//   pf_combine   per token: slots in slot order, then the shared expert (as the coop B kernel,
//                exl3_moe_coop_kernel.cuh:906-949) -> bf16 / fp32 output
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "decode_tc.cuh"
#include "internal.h"
#include "tc.cuh"

namespace eva {

constexpr int PF_BM = 128;                               // rows per CTA: one half of the pair's M = 256
constexpr int PF_BN = 128;                               // weight columns decoded per CTA: half of N = 256
constexpr int PF_BK = 64;
constexpr int PF_PAIR_N = 2 * PF_BN;
constexpr int NT_PF = 8;                                 // 16-column tiles per 128-column chunk
constexpr int PF_A_BYTES = PF_BM * PF_BK * 2;            // 16 KB
constexpr int PF_B_BYTES = PF_BN * PF_BK * 2;            // 16 KB
constexpr int PF_T_BYTES = 4 * 8 * 32 * 4;               // 4 k-tile rows x 8 tiles x 32K bytes (K <= 4)
constexpr int PF_TSLOTS_MAX = 8;
constexpr int PF_EPI_LD = 129;                           // padded row (floats) of the epilogue tiles
static_assert(PF_TILE_ROWS == 2 * PF_BM, "a CTA pair covers one expert tile");

// Per-kernel shape of the CTA: decoder warps, ring stages, CTAs per SM, 64-deep k blocks per stage.
// Each decoder warp takes 4 weight tiles per stage: with fewer, the per-stage waits and barrier
// arrivals cost a larger share of its time and its decode has less independent work in flight.
//   gate/up: one CTA per SM (its 512 TMEM columns fill the SM), 16 decoders, 3 stages of 128-deep
//            k blocks (two 64-deep halves each)
//   down:    its main loop is short (K = I), so two CTAs share an SM (256 TMEM columns, 8 decoders,
//            3 stages of 64-deep k blocks each) and one's epilogue overlaps the other's main loop
template <int NDEC, int NSTAGE, int MINB, int KSUB, int TSLOTS>
struct PfCfg {
    static constexpr int dec = NDEC, stages = NSTAGE, min_blocks = MINB, ksub = KSUB, tslots = TSLOTS;
    static constexpr int threads = (3 + NDEC) * 32;       // activation producer, MMA, decoders, trellis producer
    static constexpr int tiles_per_dec = 32 * KSUB / NDEC;  // of the 32 KSUB weight tiles of a stage
    static constexpr int a_bytes = KSUB * PF_A_BYTES;     // KSUB 64-deep activation sub-tiles
    static constexpr int b_bytes = KSUB * PF_B_BYTES;     // KSUB 64-deep weight sub-tiles
    static constexpr int stage = a_bytes + b_bytes;
    static constexpr int tslot = KSUB * PF_T_BYTES;       // trellis of one stage, in its own ring
    static constexpr size_t ring_bytes = static_cast<size_t>(NSTAGE) * stage;
    static constexpr size_t smem = 1024 + ring_bytes + static_cast<size_t>(TSLOTS) * tslot + 256;
    static_assert(TSLOTS <= PF_TSLOTS_MAX, "trellis ring barriers");
    static_assert((32 * KSUB) % NDEC == 0 && 8 % (32 * KSUB / NDEC) == 0, "a decoder's tiles lie in one k-tile row");
    static_assert(smem * MINB <= 228 * 1024, "shared memory per SM");
};
using PfGateCfg = PfCfg<16, 3, 1, 2, 4>;
using PfDownCfg = PfCfg<8, 3, 2, 1, 3>;
static_assert(2 * PF_BM * PF_EPI_LD * 4 <= PfGateCfg::stages * PfGateCfg::stage, "epilogue tiles reuse the ring");
static_assert(PF_BM * PF_EPI_LD * 4 <= PfDownCfg::stages * PfDownCfg::stage, "epilogue tile reuses the ring");

struct PfParams {
    int M, H, I, I_sh, topk, S_cap, n_local, K, K_sh, has_shared, imax, act_routed, act_shared;
    int sh0, shn;           // the shared expert's tokens: sh0 .. sh0 + shn - 1
    float limit;
    const void* x;
    int x_bf16;
    const float* rw;
    const int64_t* tables[9];
    int64_t sh[9];
    const int* runs;        // reference-layout run table (order[] = slots in expert order)
    const int* estart;      // [E + 1] first sorted row of each expert
    const int* tstart;      // [E + 2] first 128-row tile of each expert; [E + 1] = total incl. shared
    const void* sel;
    int sel64;
    __half* xg;             // [S_cap + M][H] rotated gate inputs, sorted rows (shared rows at S_cap)
    __half* xu;             // [S_cap + M][H] rotated up inputs
    __half* ap;             // [S_cap + M][imax] down inputs
    float* dpart;           // [S_cap + M][H] per-slot weighted down outputs
    float* xsum;            // [2][S_cap + M][H / 128] sums of the stored fp16 gate / up inputs per 128 chunk
    float* asum;            // [S_cap + M][imax / 128] sums of the stored fp16 down inputs per 128 chunk
    const int* slot_act;
    float* out_f32;
    __nv_bfloat16* out_bf16;
    int* status;
    const CUtensorMap* tmaps;   // [E + 1][3] trellis maps (gate, up, down) per expert, the shared expert last
};

// ---------------------------------------------------------------------------------------------
// CTA-pair tcgen05 / TMA helpers

// 2-D TMA load of this CTA's rows whose completion is counted on the pair leader's barrier
// (bar: shared::cluster address). Plain per-CTA load, no cross-CTA delivery of data.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void umma_f16_pair(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc)
{
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(acc));
}

// Arrive on the mbarrier at shared::cluster address bar when the pair MMAs issued so far complete.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ uint32_t cluster_ctarank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_rank(const void* p, uint32_t rank)
{
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
}


__device__ __forceinline__ uint8_t* pf_ring_align(uint8_t* raw)
{
    const uint32_t a = smem_u32(raw);
    return raw + ((1024 - (a & 1023)) & 1023);
}

// Store an mma.m16n8k16 A fragment (the lane's 4 registers: rows g / g + 8 x k 2t.. / 2t + 8..) as
// its four 8 x 8 matrices; addr: this lane's row address (see the decoders).
__device__ __forceinline__ void stsm_x4(uint32_t addr, const uint32_t (&r)[4])
{
    asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(r[0]), "r"(r[1]),
                 "r"(r[2]), "r"(r[3])
                 : "memory");
}

// Byte offset of element (row, k) (k < 64, fp16) in a K-major 128B-swizzled 128 x 64 tile.
__device__ __forceinline__ uint32_t sw128_off(int row, int k)
{
    const int kb = k * 2;
    return row * 128 + ((((kb >> 4) ^ (row & 7)) << 4) | (kb & 15));
}

// ---------------------------------------------------------------------------------------------
// Layout self-test of the pair MMA (eva_tc_selftest what 3 / 4): one cluster of two CTAs, one
// tcgen05.mma.cta_group::2.kind::f16 of M = 256 or 128 rows (CTA r holds rows M/2 r .. M/2 r + M/2 - 1
// of A), N = 256 (CTA r holds B rows 128 r .. 128 r + 127), K = 16, with A[i][0] = i + 1,
// A[i][1] = 256, B[n][0] = 1, B[n][1] = n + 1 and zeros elsewhere, so D[i][n] = (i + 1) + 256 (n + 1)
// names its own row and column. Each CTA fills its 256 TMEM columns with 0xffffffff first, then
// writes every lane and column it holds after the MMA: out[rank][lane 0..127][col 0..255].
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(128)
    pf_pair_selftest(int M, uint32_t* out, int* status)
{
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t accb;
    __shared__ uint32_t tmem_slot;
    uint8_t* sm = pf_ring_align(smem_raw);
    const uint32_t rank = cluster_ctarank();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* A = sm;
    uint8_t* B = sm + PF_A_BYTES;
    for (int i = threadIdx.x; i < (PF_A_BYTES + PF_B_BYTES) / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(sm)[i] = 0;
    __syncthreads();
    {
        const int i = threadIdx.x;   // local row of A and of B
        const int grow = static_cast<int>(rank) * (M / 2) + i;
        if (i < M / 2) {
            *reinterpret_cast<__half*>(A + sw128_off(i, 0)) = __float2half(static_cast<float>(grow + 1));
            *reinterpret_cast<__half*>(A + sw128_off(i, 1)) = __float2half(256.0f);
        }
        const int n = static_cast<int>(rank) * 128 + i;
        *reinterpret_cast<__half*>(B + sw128_off(i, 0)) = __float2half(1.0f);
        *reinterpret_cast<__half*>(B + sw128_off(i, 1)) = __float2half(static_cast<float>(n + 1));
    }
    fence_proxy_async_smem();
    if (threadIdx.x == 0) {
        mbar_init(&accb, 1);
        fence_barrier_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)), "r"(256));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    {
        uint32_t r[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) r[i] = 0xffffffffu;
        for (int c = 0; c < 256; c += 8) tmem_st32x32_x8(tmem + (static_cast<uint32_t>(warp * 32) << 16) + c, r);
        tmem_wait_st();
    }
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    if (rank == 0 && threadIdx.x == 0) {
        umma_f16_pair(tmem, umma_desc_sw128(smem_u32(A)), umma_desc_sw128(smem_u32(B)),
                      M == 128 ? umma_idesc_f16(128, 256) : umma_idesc_f16(256, 256), 0u);
        umma_commit_pair(mapa_rank(&accb, 0));
        umma_commit_pair(mapa_rank(&accb, 1));
    }
    mbar_wait(&accb, 0, status);
    tc_fence_after();
    for (int c = 0; c < 256; c += 32) {
        float v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + c, v);
#pragma unroll
        for (int j = 0; j < 32; ++j)
            out[(static_cast<size_t>(rank) * 128 + warp * 32 + lane) * 256 + c + j] = __float_as_uint(v[j]);
    }
    tc_fence_before();
    cluster_sync_all();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256));
    }
}

cudaError_t pf_pair_selftest_launch(int M, uint32_t* out, int* status, cudaStream_t stream)
{
    const int smem = 1024 + PF_A_BYTES + PF_B_BYTES;
    cudaError_t e = cudaFuncSetAttribute(pf_pair_selftest, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    pf_pair_selftest<<<2, 128, smem, stream>>>(M, out, status);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// Tile -> expert. Experts 0..E-1 routed, E = shared.

struct PfTile {
    int e;         // expert, n_local = shared
    int row0;      // first sorted row of the tile
    int rows;      // valid rows (<= PF_TILE_ROWS)
    bool shared;
};

__device__ __forceinline__ bool pf_tile(const PfParams& p, int mt, PfTile& t)
{
    const int E = p.n_local;
    if (mt >= p.tstart[E + 1]) return false;
    if (mt >= p.tstart[E]) {
        t.e = E;
        t.shared = true;
        const int j = mt - p.tstart[E];
        t.row0 = p.S_cap + p.sh0 + j * PF_TILE_ROWS;
        t.rows = min(PF_TILE_ROWS, p.shn - j * PF_TILE_ROWS);
        return true;
    }
    int lo = 0, hi = E - 1;   // last e with tstart[e] <= mt
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (p.tstart[mid] <= mt) lo = mid;
        else hi = mid - 1;
    }
    t.e = lo;
    t.shared = false;
    const int j = mt - p.tstart[lo];
    t.row0 = p.estart[lo] + j * PF_TILE_ROWS;
    t.rows = min(PF_TILE_ROWS, p.estart[lo + 1] - t.row0);
    return true;
}

__device__ __forceinline__ int64_t pf_ptr(const PfParams& p, const PfTile& t, int row)
{
    return t.shared ? p.sh[row] : p.tables[row][t.e];
}

__device__ __forceinline__ int pf_row_slot(const PfParams& p, int pos)
{
    return pos >= p.S_cap ? pos : p.runs[2 + p.S_cap + 1 + pos];
}

// ---------------------------------------------------------------------------------------------
// pf_rotate: four lanes per (projection, sorted row, 128-column chunk), eight chunks per warp.
//
// Lane r of a chunk's four holds elements n = 32 j + 8 r + e (j, e = 0..3, 0..7): its 16-byte loads
// and stores are contiguous 64-byte runs per chunk. The 128-point Hadamard transform takes its
// butterflies in the order of the index bits, 0 to 6, as had128_warp does (bits 0-2 and 5-6 in
// registers, bits 3-4 by two shuffles): the same operations, so the same fp32 results, with 2
// shuffle stages per 32 values instead of 5 per 4. The lane's values are held as packed pairs
// (elements 2k, 2k + 1): every butterfly level but bit 0's, the input scaling and the output
// scaling take one two-wide instruction per pair.

// 8 consecutive activations (bf16 or fp16) as floats; al16: the address is 16-byte aligned
__device__ __forceinline__ void load8_x(const void* x, size_t off, int is_bf16, bool al16, float (&v)[8])
{
    uint32_t w[4];
    if (al16) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + off));
        w[0] = u.x, w[1] = u.y, w[2] = u.z, w[3] = u.w;
    } else {
        const uint2 u0 = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(x) + off));
        const uint2 u1 = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(x) + off + 4));
        w[0] = u0.x, w[1] = u0.y, w[2] = u1.x, w[3] = u1.y;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if (is_bf16) {
            v[2 * i] = __uint_as_float(w[i] << 16);
            v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        } else {
            const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
            v[2 * i] = __low2float(h);
            v[2 * i + 1] = __high2float(h);
        }
    }
}

__global__ void __launch_bounds__(256) pf_rotate(const PfParams p)
{
    const int lane = threadIdx.x & 31, q = lane >> 2, r = lane & 3;
    const int n_act = p.runs[2 + p.runs[0]];
    const int n_rows = n_act + (p.has_shared ? p.shn : 0);
    const unsigned nch = static_cast<unsigned>(p.H / 128);
    // rows x chunks of one projection stay below 2^32: each (row, chunk) owns 512 bytes of rotated
    // activations in the workspace, so 2^32 of them would be 2 TB
    const long long per_proj = static_cast<long long>(n_rows) * nch;
    const long long n_units = 2 * per_proj;   // (projection, row, chunk), chunk fastest
    const bool al16 = (reinterpret_cast<uintptr_t>(p.x) & 15) == 0;
    const long long warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
    for (long long u0 = ((static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5) * 8; u0 < n_units;
         u0 += warps * 8) {
        const long long u = u0 + q;
        const bool valid = u < n_units;   // the lanes of a past-the-end chunk still take part in the shuffles
        // v[k] holds elements 2k, 2k + 1 of the lane's 32 (index i = 8 j + e): packed pairs
        float2 v[16];
        int pj = 0, pos = 0, c = 0;
        if (valid) {
            pj = u >= per_proj;
            const unsigned rem = static_cast<unsigned>(u - pj * per_proj);
            const unsigned row = rem / nch;
            c = static_cast<int>(rem - row * nch);
            pos = static_cast<int>(row) < n_act ? static_cast<int>(row) : p.S_cap + p.sh0 + (static_cast<int>(row) - n_act);
            int tok;
            const __half* suh;
            if (pos >= p.S_cap) {
                tok = pos - p.S_cap;
                suh = reinterpret_cast<const __half*>(p.sh[pj ? 4 : 1]);
            } else {
                const int slot = p.runs[2 + p.S_cap + 1 + pos];
                tok = slot / p.topk;
                const long long e = p.sel64 ? static_cast<const long long*>(p.sel)[slot] : static_cast<const int*>(p.sel)[slot];
                suh = reinterpret_cast<const __half*>(p.tables[pj ? 4 : 1][e]);
            }
            const size_t xoff = static_cast<size_t>(tok) * p.H + c * 128 + r * 8;
            const __half* sp = suh + c * 128 + r * 8;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float xv[8];
                load8_x(p.x, xoff + j * 32, p.x_bf16, al16, xv);
                const uint4 su = __ldg(reinterpret_cast<const uint4*>(sp + j * 32));
                const uint32_t sw[4] = {su.x, su.y, su.z, su.w};
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    v[j * 4 + i] = mul2(make_float2(xv[2 * i], xv[2 * i + 1]),
                                        __half22float2(*reinterpret_cast<const __half2*>(&sw[i])));
            }
        } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) v[k] = make_float2(0.0f, 0.0f);
        }
        // index bit 0: inside the pairs
#pragma unroll
        for (int k = 0; k < 16; ++k) v[k] = make_float2(v[k].x + v[k].y, v[k].x - v[k].y);
        // index bits 1-2 (the rest of e): between pairs k and k + h
#pragma unroll
        for (int h = 1; h < 4; h <<= 1)
#pragma unroll
            for (int k = 0; k < 16; ++k)
                if ((k & h) == 0) {
                    const float2 a = v[k], b = v[k + h];
                    v[k] = add2(a, b);
                    v[k + h] = sub2(a, b);
                }
        // index bits 3-4: r (lane bits 0-1)
#pragma unroll
        for (int m = 1; m < 4; m <<= 1) {
            const float s1 = (r & m) ? -1.0f : 1.0f;   // upper lane o - v, lower v + o, as one fma
            const float2 sg = make_float2(s1, s1);
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const float2 o =
                    make_float2(__shfl_xor_sync(0xffffffffu, v[k].x, m), __shfl_xor_sync(0xffffffffu, v[k].y, m));
                v[k] = fma2(v[k], sg, o);
            }
        }
        // index bits 5-6: j
#pragma unroll
        for (int h = 4; h < 16; h <<= 1)
#pragma unroll
            for (int k = 0; k < 16; ++k)
                if ((k & h) == 0) {
                    const float2 a = v[k], b = v[k + h];
                    v[k] = add2(a, b);
                    v[k + h] = sub2(a, b);
                }
        // sums of the values as stored (fp16), for the raw-codebook correction: even and odd
        // elements accumulated as a pair, then added
        float2 sm2 = make_float2(0.0f, 0.0f);
        if (valid) {
            const float2 sc = make_float2(0.08838834764831845f, 0.08838834764831845f);   // 1/sqrt(128)
            __half* dst = (pj ? p.xu : p.xg) + static_cast<size_t>(pos) * p.H + c * 128 + r * 8;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t w[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const __half2 h = __float22half2_rn(mul2(v[j * 4 + i], sc));
                    w[i] = *reinterpret_cast<const uint32_t*>(&h);
                    sm2 = add2(sm2, __half22float2(h));
                }
                *reinterpret_cast<uint4*>(dst + j * 32) = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
        float sm = sm2.x + sm2.y;
        sm += __shfl_xor_sync(0xffffffffu, sm, 1);
        sm += __shfl_xor_sync(0xffffffffu, sm, 2);
        if (valid && r == 0) p.xsum[(static_cast<size_t>(pj) * (p.S_cap + p.M) + pos) * nch + c] = sm;
    }
}


// ---------------------------------------------------------------------------------------------
// Shared main loop of the two GEMM kernels (one CTA of the pair).
//   nproj   projections accumulated (gate+up: 2, down: 1); projection j accumulates into TMEM
//           columns 256 j .. 256 j + 255
//   nkb     stages (k blocks of 64 ksub) per projection
//   amap    tensor maps of the activation rows per projection; trellis bases per projection
//   chunk   the 128-column weight chunk this CTA decodes (dec_valid = 0: past the end, not decoded)

struct PfLoop {
    const CUtensorMap* amap[2];
    const CUtensorMap* tmap[2];   // the trellis maps of the projections
    int chunk, dec_valid;
    int nproj, nkb, row0;    // row0: this CTA's first activation row
    uint32_t rank;           // 0 = leader (issues the MMAs)
    int half;                // tile of <= 128 rows: M = 128 pair MMAs, 64 rows per CTA
};

template <int NS>
struct PfBars {
    uint64_t afull[NS], bfull[NS], empty[NS], accb;
    uint64_t tfull[PF_TSLOTS_MAX], tempty[PF_TSLOTS_MAX];   // the trellis ring
};

template <int K, class CFG>
__device__ __forceinline__ void pf_mainloop(const PfLoop& L, uint8_t* ring, PfBars<CFG::stages>& B, uint32_t tmem,
                                            int warp, int lane, int* status)
{
    constexpr int PF_STAGES = CFG::stages, TPW = CFG::tiles_per_dec, KSUB = CFG::ksub, TS = CFG::tslots;
    constexpr int PF_STAGE = CFG::stage, A_BYTES = CFG::a_bytes;
    const int total = L.nproj * L.nkb;
    constexpr uint32_t TROW = NT_PF * 32 * K;   // bytes of one k-tile row's 8 tiles
    if (warp == 0) {
        // activation producer: own activation rows (counted on the leader's afull). The MMA commits
        // each stage to the leader's empty barrier only; the leader's producer, once it sees a stage
        // released, forwards the release to the peer CTA's barrier.
        for (int s = 0; s < total; ++s) {
            const int st = s % PF_STAGES;
            mbar_wait(&B.empty[st], ((s / PF_STAGES) & 1) ^ 1, status);
            if (lane == 0) {
                if (L.rank == 0 && s >= PF_STAGES) mbar_arrive_remote(mapa_rank(&B.empty[st], 1));
                const int pj = s / L.nkb, kb = s % L.nkb;
                uint8_t* stage = ring + st * PF_STAGE;
                if (L.rank == 0) mbar_arrive_expect_tx(&B.afull[st], 2 * A_BYTES);
#pragma unroll
                for (int j = 0; j < KSUB; ++j)
                    tma_load_2d_pair(stage + j * PF_A_BYTES, pj ? L.amap[1] : L.amap[0], (kb * KSUB + j) * PF_BK, L.row0,
                                     mapa_rank(&B.afull[st], 0));
            }
            __syncwarp();
        }
    } else if (warp == CFG::dec + 2) {
        // trellis producer: the stage's 4 KSUB k-tile rows of this CTA's 128 columns as one 2-D
        // tensor copy (per-row bulk copies throttle the copy engine), into the trellis ring, whose
        // slots the decoders release as soon as they have read them (so the copies run TSLOTS - 1
        // decode stages ahead, independent of the MMA)
        uint8_t* tring = ring + CFG::ring_bytes;
        if (lane == 0 && L.dec_valid)
            for (int j = 0; j < (L.nproj > 1 ? 2 : 1); ++j) tmap_acquire(L.tmap[j]);
        for (int s = 0; s < total; ++s) {
            const int ts = s % TS;
            mbar_wait(&B.tempty[ts], ((s / TS) & 1) ^ 1, status);
            const int pj = s / L.nkb, kb = s % L.nkb;
            if (lane == 0) {
                if (L.dec_valid) {
                    mbar_arrive_expect_tx(&B.tfull[ts], 4 * KSUB * TROW);
                    tma_load_2d(tring + ts * CFG::tslot, pj ? L.tmap[1] : L.tmap[0], L.chunk * NT_PF * 4 * K,
                                kb * 4 * KSUB, &B.tfull[ts]);
                } else {
                    mbar_arrive(&B.tfull[ts]);
                }
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        if (L.rank != 0 || lane != 0) return;
        // leader, one thread: pair MMAs (M = 256 over both CTAs' rows, N = 256 over both CTAs'
        // decoded columns), one commit per stage
        const uint32_t idesc = L.half ? umma_idesc_f16(PF_BM, PF_PAIR_N) : umma_idesc_f16(2 * PF_BM, PF_PAIR_N);
        int st = 0, pj = 0, kb = 0;
        uint32_t ph = 0;
        for (int s = 0; s < total; ++s) {
            mbar_wait(&B.afull[st], ph, status);
            mbar_wait(&B.bfull[st], ph, status);
            tc_fence_after();
            const uint32_t sa = smem_u32(ring + st * PF_STAGE);
            const uint32_t sb = sa + A_BYTES;
#pragma unroll
            for (int j = 0; j < KSUB; ++j)
#pragma unroll
                for (int k = 0; k < PF_BK / 16; ++k)
                    umma_f16_pair(tmem + pj * PF_PAIR_N, umma_desc_sw128(sa + j * PF_A_BYTES + k * 32),
                                  umma_desc_sw128(sb + j * PF_B_BYTES + k * 32), idesc, (kb > 0 || j > 0 || k > 0) ? 1u : 0u);
            umma_commit_pair(smem_u32(&B.empty[st]));
            if (++kb == L.nkb) {
                kb = 0;
                ++pj;
            }
            if (++st == PF_STAGES) {
                st = 0;
                ph ^= 1u;
            }
        }
        umma_commit_pair(mapa_rank(&B.accb, 0));
        umma_commit_pair(mapa_rank(&B.accb, 1));
    } else {
        // decoders: warp d takes tiles TPW d .. TPW d + TPW - 1 of the stage's 32 KSUB (k-tile row
        // q / 8, 16-column tile q % 8); k-tile row ktl lies in 64-deep weight sub-tile ktl / 4
        const int d = warp - 2;
        const int ktl = (d * TPW) >> 3, nt0 = (d * TPW) & 7;
        const LaneW lw = lane_w<K>(lane);
        const uint32_t ring_s = smem_u32(ring);
        // swizzled offsets of the lane's 4 words in each of its tiles (fixed for the whole loop)
        // A tile's four 8 x 8 fragments (rows n / n + 8 x k / k + 8) go out in one stmatrix.x4: lane
        // i gives the address of row i % 8 of fragment i / 8, a 16-byte run of the swizzled layout
        uint32_t so[TPW];
#pragma unroll
        for (int t = 0; t < TPW; ++t) {
            const int mi = lane >> 3;
            const int n = (nt0 + t) * 16 + (mi & 1) * 8 + (lane & 7);   // output column within the chunk (B row)
            const int k = (ktl & 3) * 16 + (mi >> 1) * 8;              // k within the 64-deep sub-tile
            so[t] = (ktl >> 2) * PF_B_BYTES + sw128_off(n, k);
        }
        const uint32_t tw0 = nt0 * 32 * K + lw.w0 * 4, tw1 = nt0 * 32 * K + lw.w1 * 4;
        const uint32_t tring = ring_s + static_cast<uint32_t>(CFG::ring_bytes) + ktl * TROW;
        for (int s = 0; s < total; ++s) {
            const int st = s % PF_STAGES, ts = s % TS;
            mbar_wait(&B.tfull[ts], (s / TS) & 1, status);
            uint32_t a[TPW][4];
            if (L.dec_valid) {
                const uint32_t tr = tring + ts * CFG::tslot;
                uint32_t w[TPW][2];
#pragma unroll
                for (int t = 0; t < TPW; ++t) {
                    w[t][0] = lds32(tr + t * 32 * K + tw0);
                    w[t][1] = lds32(tr + t * 32 * K + tw1);
                }
                // two-word decode, 4 windows extracted on the FMA pipe and, below K = 4, pairs packed
                // by integer multiply-adds (the ALU pipe carries the rest of the decode)
#pragma unroll
                for (int t = 0; t < TPW; ++t) decode_afrag_ww<K, 4, (K == 4)>(w[t][0], w[t][1], lw, a[t]);
            }
            // the words are in registers (the decode consumed them): release the trellis slot
            __syncwarp();
            if (lane == 0) mbar_arrive(&B.tempty[ts]);
            mbar_wait(&B.empty[st], ((s / PF_STAGES) & 1) ^ 1, status);   // the MMA is done with the ring stage
            if (L.dec_valid) {
                const uint32_t bt = ring_s + st * PF_STAGE + A_BYTES;
#pragma unroll
                for (int t = 0; t < TPW; ++t) stsm_x4(bt + so[t], a[t]);
                fence_proxy_async_smem();
            }
            __syncwarp();
            if (lane == 0) {
                if (L.rank == 0) mbar_arrive(&B.bfull[st]);
                else mbar_arrive_remote(mapa_rank(&B.bfull[st], 0));
            }
        }
    }
}

// TMEM accumulator (columns col0 .. col0 + 127) -> smem tile [128][PF_EPI_LD] by warps 0-3
// (warp w reads TMEM lanes 32 w .. 32 w + 31).
__device__ __forceinline__ void pf_tmem_to_smem(uint32_t tmem, int col0, float* tile, int warp, int lane)
{
    const int row = warp * 32 + lane;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + col0 + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) tile[row * PF_EPI_LD + c * 32 + i] = v[i];
    }
}

// Epilogue rows in the lane-strided order: lane l holds elements l, l + 32, l + 64, l + 96 of a
// 128-column chunk, so that a warp's reads of a 129-float tile row hit 32 different banks (a lane
// holding 4 consecutive elements would share banks four ways). had128_warp is applied to this order
// unchanged: the Sylvester transform commutes with any permutation of the index bits applied to input
// and output alike, and here the register index is bits 5-6 and the lane bits 0-4.
__device__ __forceinline__ void load4s_half(const __half* p, int lane, float (&v)[4])
{
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __half2float(__ldg(p + lane + 32 * i));
}

__device__ __forceinline__ void store4s_half(__half* p, int lane, const float (&v)[4])
{
#pragma unroll
    for (int i = 0; i < 4; ++i) p[lane + 32 * i] = __float2half_rn(v[i]);
}

// Half-height tiles (M = 128 pair MMAs): a CTA's 64 rows x 256 columns lie folded in its TMEM, lane
// l < 64 holding row l, columns 0..127 and lane 64 + l row l, columns 128..255 (from col0). Chunk c
// (the pair's columns 128 c .. 128 c + 127) -> smem tile [64][PF_EPI_LD] by warps 2 c and 2 c + 1.
__device__ __forceinline__ void pf_tmem_to_smem_half(uint32_t tmem, int col0, int c, float* tile, int warp, int lane)
{
    if ((warp >> 1) != c) return;
    const int row = (warp & 1) * 32 + lane;
#pragma unroll 1
    for (int cc = 0; cc < 4; ++cc) {
        float v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + col0 + cc * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) tile[row * PF_EPI_LD + cc * 32 + i] = v[i];
    }
}

// Row sums for the raw-codebook correction, gathered once per CTA in parallel (L threads per row,
// each a fixed sequence of the row's per-chunk partial sums, then a fixed shuffle tree): out[r] =
// sum over c < nchunk of part[(row0 + r) * stride + c] for the CTA's rows r < rows.
template <int L>
__device__ __forceinline__ void pf_row_sums(const float* part, size_t stride, int nchunk, int row0, int rows,
                                            float* out, int nthreads)
{
    static_assert(L == 2 || L == 4, "threads per row");
    for (int t0 = 0; t0 < PF_BM * L; t0 += nthreads) {
        const int t = t0 + static_cast<int>(threadIdx.x);
        const int r = t / L, q = t % L;
        float s = 0.0f;
        if (t < PF_BM * L && r < rows)
            for (int c = q; c < nchunk; c += L) s += __ldcg(part + static_cast<size_t>(row0 + r) * stride + c);
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        if (L == 4) s += __shfl_xor_sync(0xffffffffu, s, 2);
        if (t < PF_BM * L && q == 0) out[r] = s;
    }
}

template <int NS>
struct PfSmem {
    PfBars<NS> bars;
    uint32_t tmem;
};

__device__ __forceinline__ uint8_t* pf_ring(uint8_t* raw)
{
    const uint32_t a = smem_u32(raw);
    return raw + ((1024 - (a & 1023)) & 1023);
}

// Both CTAs of the pair: barriers, the pair's TMEM allocation (one warp per CTA, same warp), and a
// cluster barrier so that no CTA signals the other's barriers before they exist.
template <class CFG>
__device__ __forceinline__ void pf_setup(PfSmem<CFG::stages>& S, int warp, int ncols)
{
    if (threadIdx.x == 0) {
        PfBars<CFG::stages>& B = S.bars;
        for (int i = 0; i < CFG::stages; ++i) {
            mbar_init(&B.afull[i], 1);
            mbar_init(&B.bfull[i], 2 * CFG::dec);
            mbar_init(&B.empty[i], 1);
        }
        for (int i = 0; i < CFG::tslots; ++i) {
            mbar_init(&B.tfull[i], 1);
            mbar_init(&B.tempty[i], CFG::dec);
        }
        mbar_init(&B.accb, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S.tmem)), "r"(ncols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
}

template <int NS>
__device__ __forceinline__ void pf_teardown(PfSmem<NS>& S, int warp, int ncols)
{
    tc_fence_before();
    cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(S.tmem), "r"(ncols));
    }
}

// ---------------------------------------------------------------------------------------------
// pf_gateup: gate and up of one (expert tile of up to 256 rows, 256 columns of I), CTA pair

template <int KR, int KS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PfGateCfg::threads, PfGateCfg::min_blocks)
    pf_gateup(const PfParams p, const __grid_constant__ CUtensorMap mg, const __grid_constant__ CUtensorMap mu)
{
    using CFG = PfGateCfg;
    constexpr int PF_THREADS = CFG::threads;
    extern __shared__ uint8_t smem_raw[];
    __shared__ PfSmem<CFG::stages> S;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    PfTile t;
    if (!pf_tile(p, blockIdx.y, t)) return;               // both CTAs of the pair agree
    const int I_e = t.shared ? p.I_sh : p.I;
    const int nch = I_e / 128;
    const int pc = blockIdx.x >> 1;
    if (2 * pc >= nch) return;                             // both CTAs of the pair agree
    const uint32_t rank = cluster_ctarank();
    const int Ke = t.shared ? KS : KR;
    uint8_t* ring = pf_ring(smem_raw);
    constexpr int NCOLS = 2 * PF_PAIR_N;
    pf_setup<CFG>(S, warp, NCOLS);

    PfLoop L;
    L.amap[0] = &mg;
    L.amap[1] = &mu;
    L.tmap[0] = p.tmaps + t.e * 3;
    L.tmap[1] = p.tmaps + t.e * 3 + 1;
    L.chunk = 2 * pc + static_cast<int>(rank);
    L.dec_valid = L.chunk < nch;
    L.nproj = 2;
    L.nkb = p.H / (PF_BK * CFG::ksub);                     // H is a multiple of 128
    L.half = t.rows <= PF_BM;
    const int cta_rows = L.half ? PF_BM / 2 : PF_BM;
    L.row0 = t.row0 + static_cast<int>(rank) * cta_rows;
    L.rank = rank;
    if (Ke == KR) pf_mainloop<KR, CFG>(L, ring, S.bars, S.tmem, warp, lane, p.status);
    else pf_mainloop<KS, CFG>(L, ring, S.bars, S.tmem, warp, lane, p.status);

    // epilogue: this CTA's 128 rows x the pair's 256 columns, one 128-column chunk at a time
    mbar_wait(&S.bars.accb, 0, p.status);
    tc_fence_after();
    float* G = reinterpret_cast<float*>(ring);
    float* U = G + PF_BM * PF_EPI_LD;
    const int rows = min(cta_rows, t.rows - static_cast<int>(rank) * cta_rows);
    const int mode = t.shared ? p.act_shared : p.act_routed;
    // raw codebook: x . w = c0 (x . h) + c1 sum(x), sum(x) over the row's stored fp16 inputs
    __shared__ float rsum[2][PF_BM];
    {
        const int nchH = p.H / 128;
        constexpr int RS_THREADS = PF_THREADS < PF_BM * 4 ? PF_THREADS : PF_BM * 4;   // the threads that gather
        if (threadIdx.x < RS_THREADS) {
            pf_row_sums<4>(p.xsum, nchH, nchH, L.row0, rows, rsum[0], RS_THREADS);
            pf_row_sums<4>(p.xsum + (static_cast<size_t>(p.S_cap) + p.M) * nchH, nchH, nchH, L.row0, rows, rsum[1], RS_THREADS);
        }
    }
    for (int c = 0; c < 2; ++c) {
        const int chunk = 2 * pc + c;
        if (chunk >= nch) break;
        if (warp < 4) {
            if (L.half) {
                pf_tmem_to_smem_half(S.tmem, 0, c, G, warp, lane);
                pf_tmem_to_smem_half(S.tmem, PF_PAIR_N, c, U, warp, lane);
            } else {
                pf_tmem_to_smem(S.tmem, c * PF_BN, G, warp, lane);
                pf_tmem_to_smem(S.tmem, PF_PAIR_N + c * PF_BN, U, warp, lane);
            }
        }
        __syncthreads();
        const int col = chunk * 128;   // lane-strided rows (load4s_half)
        float svg[4], svu[4], sud[4];
        load4s_half(reinterpret_cast<const __half*>(pf_ptr(p, t, 2)) + col, lane, svg);
        load4s_half(reinterpret_cast<const __half*>(pf_ptr(p, t, 5)) + col, lane, svu);
        load4s_half(reinterpret_cast<const __half*>(pf_ptr(p, t, 7)) + col, lane, sud);
        for (int r = warp; r < rows; r += PF_THREADS / 32) {
            const int pos = L.row0 + r;
            const float sg = rsum[0][r], su = rsum[1][r];
            float g[4], u[4], a[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                g[i] = CB_C0 * G[r * PF_EPI_LD + lane + 32 * i] + CB_C1 * sg;
                u[i] = CB_C0 * U[r * PF_EPI_LD + lane + 32 * i] + CB_C1 * su;
            }
            had128_warp(g, lane);
            had128_warp(u, lane);
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = act_gated(g[i] * svg[i], u[i] * svu[i], p.limit, mode) * sud[i];
            had128_warp(a, lane);
            store4s_half(p.ap + static_cast<size_t>(pos) * p.imax + col, lane, a);
            float sa = 0.0f;   // sum of the values as stored (fp16), for the down projection's correction
#pragma unroll
            for (int i = 0; i < 4; ++i) sa += __half2float(__float2half_rn(a[i]));
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sa += __shfl_xor_sync(0xffffffffu, sa, o);
            if (lane == 0) p.asum[static_cast<size_t>(pos) * (p.imax / 128) + chunk] = sa;
        }
        __syncthreads();
    }
    pf_teardown(S, warp, NCOLS);
}

// ---------------------------------------------------------------------------------------------
// pf_down: down projection of one (expert tile, 256 columns of H), weighted per-slot rows, CTA pair

template <int KR, int KS>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PfDownCfg::threads, PfDownCfg::min_blocks)
    pf_down(const PfParams p, const __grid_constant__ CUtensorMap ma)
{
    using CFG = PfDownCfg;
    constexpr int PF_THREADS = CFG::threads;
    extern __shared__ uint8_t smem_raw[];
    __shared__ PfSmem<CFG::stages> S;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    PfTile t;
    if (!pf_tile(p, blockIdx.y, t)) return;
    const int I_e = t.shared ? p.I_sh : p.I;
    const int pc = blockIdx.x >> 1;
    const uint32_t rank = cluster_ctarank();
    const int Ke = t.shared ? KS : KR;
    uint8_t* ring = pf_ring(smem_raw);
    constexpr int NCOLS = PF_PAIR_N;
    pf_setup<CFG>(S, warp, NCOLS);

    PfLoop L;
    L.amap[0] = L.amap[1] = &ma;
    L.tmap[0] = L.tmap[1] = p.tmaps + t.e * 3 + 2;
    L.chunk = 2 * pc + static_cast<int>(rank);
    L.dec_valid = 1;                                       // H is a multiple of 256
    L.nproj = 1;
    L.nkb = I_e / (PF_BK * CFG::ksub);
    L.half = t.rows <= PF_BM;
    const int cta_rows = L.half ? PF_BM / 2 : PF_BM;
    L.row0 = t.row0 + static_cast<int>(rank) * cta_rows;
    L.rank = rank;
    if (Ke == KR) pf_mainloop<KR, CFG>(L, ring, S.bars, S.tmem, warp, lane, p.status);
    else pf_mainloop<KS, CFG>(L, ring, S.bars, S.tmem, warp, lane, p.status);

    mbar_wait(&S.bars.accb, 0, p.status);
    tc_fence_after();
    float* D = reinterpret_cast<float*>(ring);
    const int rows = min(cta_rows, t.rows - static_cast<int>(rank) * cta_rows);
    // raw codebook correction with the sums of the rows' stored fp16 down inputs
    __shared__ float rsum[PF_BM];
    if (threadIdx.x < PF_BM * 2) pf_row_sums<2>(p.asum, p.imax / 128, I_e / 128, L.row0, rows, rsum, PF_BM * 2);
    for (int c = 0; c < 2; ++c) {
        if (warp < 4) {
            if (L.half) pf_tmem_to_smem_half(S.tmem, 0, c, D, warp, lane);
            else pf_tmem_to_smem(S.tmem, c * PF_BN, D, warp, lane);
        }
        __syncthreads();
        const int col = (2 * pc + c) * 128;   // lane-strided rows (load4s_half)
        float svd[4];
        load4s_half(reinterpret_cast<const __half*>(pf_ptr(p, t, 8)) + col, lane, svd);
        for (int r = warp; r < rows; r += PF_THREADS / 32) {
            const int slot = pf_row_slot(p, L.row0 + r);
            const float w = t.shared ? 1.0f : p.rw[slot];
            const float sa = rsum[r];
            float v[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = CB_C0 * D[r * PF_EPI_LD + lane + 32 * i] + CB_C1 * sa;
            had128_warp(v, lane);
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] *= svd[i] * w;
            float* dst = p.dpart + static_cast<size_t>(slot) * p.H + col;
#pragma unroll
            for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = v[i];
        }
        __syncthreads();
    }
    pf_teardown(S, warp, NCOLS);
}

// ---------------------------------------------------------------------------------------------
// pf_maps: the trellis tensor maps of every expert (and the shared expert), one warp per expert:
// the template of its shape with the expert's projection address, published for the tensor-map
// proxy (the GEMM kernels acquire before their first copy). Unbound experts (address 0) own no tiles.

struct PfMapTemplates {
    CUtensorMap gu, dn, sgu, sdn;   // routed gate/up (8 k-tile rows per box), down (4), shared gate/up, down
};

__global__ void __launch_bounds__(32) pf_maps(const PfParams p, const __grid_constant__ PfMapTemplates tm, CUtensorMap* maps)
{
    __shared__ __align__(128) CUtensorMap edit[3];
    const int e = blockIdx.x, lane = threadIdx.x;
    const bool shared = e == p.n_local;
    for (int j = 0; j < 3; ++j) {
        const int row = j == 0 ? 0 : (j == 1 ? 3 : 6);
        const int64_t addr = shared ? p.sh[row] : p.tables[row][e];
        const CUtensorMap* t = j < 2 ? (shared ? &tm.sgu : &tm.gu) : (shared ? &tm.sdn : &tm.dn);
        reinterpret_cast<uint32_t*>(&edit[j])[lane] = reinterpret_cast<const uint32_t*>(t)[lane];
        __syncwarp();
        if (lane == 0 && addr != 0 && (addr & 15) == 0) tmap_replace_addr(&edit[j], reinterpret_cast<const void*>(addr));
        __syncwarp();
        tmap_copy_release(maps + e * 3 + j, &edit[j]);
    }
}

// ---------------------------------------------------------------------------------------------
// pf_combine: warp per (token, 128 chunk)

__device__ __forceinline__ void pf_combine_item(const PfParams& p, int tok, int c, int lane);

__global__ void __launch_bounds__(256) pf_combine(const PfParams p)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nch = p.H / 128;
    const long long n_items = static_cast<long long>(p.M) * nch;
    for (long long item = static_cast<long long>(blockIdx.x) * 8 + warp; item < n_items;
         item += static_cast<long long>(gridDim.x) * 8)
        pf_combine_item(p, static_cast<int>(item / nch), static_cast<int>(item % nch), lane);
}

__device__ __forceinline__ void pf_combine_item(const PfParams& p, int tok, int c, int lane)
{
    const int col = c * 128 + lane * 4;
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < p.topk; ++k) {
        const int s = tok * p.topk + k;
        if (!p.slot_act[s]) continue;
        const float4 d = *reinterpret_cast<const float4*>(p.dpart + static_cast<size_t>(s) * p.H + col);
        o[0] += d.x;
        o[1] += d.y;
        o[2] += d.z;
        o[3] += d.w;
    }
    if (p.has_shared && tok >= p.sh0 && tok < p.sh0 + p.shn) {
        const float4 d = *reinterpret_cast<const float4*>(p.dpart + (static_cast<size_t>(p.S_cap) + tok) * p.H + col);
        o[0] += d.x;
        o[1] += d.y;
        o[2] += d.z;
        o[3] += d.w;
    }
    const size_t oi = static_cast<size_t>(tok) * p.H + col;
    if (p.out_f32) *reinterpret_cast<float4*>(p.out_f32 + oi) = make_float4(o[0], o[1], o[2], o[3]);
    if (p.out_bf16) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(o[0], o[1]);
        __nv_bfloat162 hi = __floats2bfloat162_rn(o[2], o[3]);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&lo);
        u.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(p.out_bf16 + oi) = u;
    }
}

// ---------------------------------------------------------------------------------------------
// host side

// Trellis [in/16][out/16][16K] int16 of one projection as [in/16][out/16 x 4K] 8-byte elements, box
// 8 tiles (one 128-column chunk) x rows k-tile rows; base: any 16-byte aligned device address.
static bool make_trellis_map(CUtensorMap* m, void* base, int in, int out, int K, int rows)
{
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(out / 16) * 4 * K, static_cast<cuuint64_t>(in / 16)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(out / 16) * 32 * K};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(NT_PF * 4 * K), static_cast<cuuint32_t>(rows)};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

// fp16 [rows][cols] row-major, box 64 x 128, 128B swizzle
static bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols)
{
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {PF_BK, PF_BM};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

using GateUpKernel = void (*)(PfParams, CUtensorMap, CUtensorMap);
using DownKernel = void (*)(PfParams, CUtensorMap);

template <int A, int B>
static void pick(int kr, int ks, GateUpKernel& g, DownKernel& d)
{
    if (kr == A && ks == B) {
        g = pf_gateup<A, B>;
        d = pf_down<A, B>;
    }
}

cudaError_t launch_prefill(const ExpertsArgs& a, cudaStream_t stream)
{
    const EvaMoeShape& s = *a.shape;
    const WsLayout& L = a.L;
    uint8_t* ws = static_cast<uint8_t*>(a.ws);
    PfParams p{};
    p.M = a.M;
    p.H = s.hidden;
    p.I = s.inter;
    p.I_sh = s.shared_inter;
    p.topk = s.topk;
    p.S_cap = a.M * s.topk;
    p.n_local = s.n_experts;
    p.K = s.bits;
    p.K_sh = s.shared_inter ? s.shared_bits : s.bits;
    p.has_shared = s.shared_inter > 0;
    p.sh0 = a.sh0;
    p.shn = p.has_shared ? a.shn : 0;
    p.imax = L.imax;
    p.act_routed = s.act_routed;
    p.act_shared = s.act_shared;
    p.limit = s.swiglu_limit;
    p.x = a.x;
    p.x_bf16 = a.x_bf16;
    p.rw = a.rw;
    for (int i = 0; i < 9; ++i) {
        p.tables[i] = a.tables[i];
        p.sh[i] = a.shared[i];
    }
    p.runs = reinterpret_cast<const int*>(ws + L.runs);
    p.estart = reinterpret_cast<const int*>(ws + L.estart);
    p.tstart = reinterpret_cast<const int*>(ws + L.tstart);
    p.sel = a.sel;
    p.sel64 = a.sel64;
    p.xg = reinterpret_cast<__half*>(ws + L.pxg);
    p.xu = reinterpret_cast<__half*>(ws + L.pxu);
    p.ap = reinterpret_cast<__half*>(ws + L.pap);
    p.dpart = reinterpret_cast<float*>(ws + L.dpart);
    p.xsum = reinterpret_cast<float*>(ws + L.xsum);
    p.asum = reinterpret_cast<float*>(ws + L.asum);
    p.slot_act = reinterpret_cast<const int*>(ws + L.slot_act);
    p.out_f32 = a.out_f32;
    p.out_bf16 = static_cast<__nv_bfloat16*>(a.out_bf16);
    p.status = reinterpret_cast<int*>(ws + L.status);
    CUtensorMap* maps = reinterpret_cast<CUtensorMap*>(ws + L.tmaps);
    p.tmaps = maps;

    PfMapTemplates tmpl;
    const int ish = p.I_sh ? p.I_sh : p.I;
    if (!make_trellis_map(&tmpl.gu, ws, p.H, p.I, p.K, 4 * PfGateCfg::ksub) ||
        !make_trellis_map(&tmpl.dn, ws, p.I, p.H, p.K, 4 * PfDownCfg::ksub) ||
        !make_trellis_map(&tmpl.sgu, ws, p.H, ish, p.K_sh, 4 * PfGateCfg::ksub) ||
        !make_trellis_map(&tmpl.sdn, ws, ish, p.H, p.K_sh, 4 * PfDownCfg::ksub))
        return cudaErrorInvalidValue;

    const uint64_t rows = static_cast<uint64_t>(p.S_cap) + p.M;
    CUtensorMap mg, mu, ma;
    if (!make_map(&mg, p.xg, rows, p.H) || !make_map(&mu, p.xu, rows, p.H) || !make_map(&ma, p.ap, rows, p.imax))
        return cudaErrorInvalidValue;

    GateUpKernel kg = nullptr;
    DownKernel kd = nullptr;
    pick<2, 2>(p.K, p.K_sh, kg, kd);
    pick<2, 3>(p.K, p.K_sh, kg, kd);
    pick<2, 4>(p.K, p.K_sh, kg, kd);
    pick<3, 2>(p.K, p.K_sh, kg, kd);
    pick<3, 3>(p.K, p.K_sh, kg, kd);
    pick<3, 4>(p.K, p.K_sh, kg, kd);
    pick<4, 2>(p.K, p.K_sh, kg, kd);
    pick<4, 3>(p.K, p.K_sh, kg, kd);
    pick<4, 4>(p.K, p.K_sh, kg, kd);
    if (!kg || !kd) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(kg, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(PfGateCfg::smem));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kd, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(PfDownCfg::smem));
    if (e != cudaSuccess) return e;

    const int small_grid = num_sms() * 8;
    pf_maps<<<p.n_local + (p.has_shared ? 1 : 0), 32, 0, stream>>>(p, tmpl, maps);
    pf_rotate<<<small_grid, 256, 0, stream>>>(p);
    // tile upper bound: sum over experts of ceil(n_e / T) <= S / T + E, plus the shared tiles
    const int max_tiles = (p.S_cap + PF_TILE_ROWS - 1) / PF_TILE_ROWS + p.n_local +
                          (p.has_shared ? (p.shn + PF_TILE_ROWS - 1) / PF_TILE_ROWS : 0);
    const int pairs_gu = (L.imax / 128 + 1) / 2;          // 256-column pairs of the widest I (odd: last pair half used)
    kg<<<dim3(2 * pairs_gu, max_tiles), PfGateCfg::threads, PfGateCfg::smem, stream>>>(p, mg, mu);
    kd<<<dim3(2 * (p.H / 256), max_tiles), PfDownCfg::threads, PfDownCfg::smem, stream>>>(p, ma);
    const long long comb = static_cast<long long>(p.M) * (p.H / 128);
    pf_combine<<<static_cast<unsigned>(std::min<long long>((comb + 7) / 8, small_grid)), 256, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace eva
