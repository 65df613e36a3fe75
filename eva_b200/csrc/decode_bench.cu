// Measurement and self-test kernels for the EXL3 decode loop (no counterpart in the reference).
//
// eva_decode_microbench times the decode loop of the expert kernels on trellis tiles resident in
// shared memory (no HBM traffic), one persistent CTA per SM, clock64 per CTA, and reports decoded
// weights per SM clock: the issue-bound ceiling of a decode design, against the 62 weights per SM
// clock that streaming K = 3 records at the measured HBM rate needs (6.54 TB/s / 0.375 B / 148 SMs
// / 1.9 GHz). Variants:
//   0  mma.sync decode of the fused decode kernel: 4 words + 2 funnel shifts + 8 windows per lane
//      and tile, mul1 byte sums, fp16 pairs, mma.m16n8k16 (16 warps, 4 k-rows x 4 tiles each)
//   1  two-word decode -> mul1 products -> tcgen05.st into TMEM (i8 operand form), no MMA
//   2  two-word decode -> raw codebook fp16 -> tcgen05.st into TMEM (f16 operand form), no MMA
//   3  variant 1 + tcgen05.mma.kind::i8 from TMEM (M 128, N 16) through a 7-slot TMEM ring with
//      mbarrier hand-offs between 4 decoding warpgroups and one issuing thread
//   4  variant 2 + tcgen05.mma.kind::f16 from TMEM, same ring
//   5  variant 1 without the ALU/FMA balancing of the window extraction
//   6  two-word decode + mma.m16n8k16 (pairs packed by IMAD, all windows shift + mask)
//   7  6 with pairs packed by PRMT
//   8  7 with 2 windows extracted as multiply + shift (FMA pipe)
//   9  6 with 2 windows extracted as multiply + shift
//  10  7 with 4 windows extracted as multiply + shift
//  11  8 with a stage's bookkeeping around each pass (B from shared memory, mbarrier arrive + wait)
//  12  the fused kernel's ring: a producer warp streams 32 trellis rows + 8 B rows per stage from a
//      1 GB buffer (HBM) into 4 stages, 16 decoding warps as variant 8
//  13  12 with a 32 MB source (resident in L2)
//  14  12 with 5 ring stages
//  15  12 with decoders not waiting for the data (contention only)
//  16  12 with one contiguous copy per stage instead of 32 row copies
//  17  12 with one 2-D tensor copy (TMA tensor map, rows row_stride apart) per stage
//  18  12 with the stage copied by cp.async 16-byte copies from the producer warp
//  19  8 with the byte sum left to 8-bit MMAs (m16n8k32 u8 x s8 / u8 x u8, two activation digits)
// eva_tc_selftest checks the TMEM layouts those designs rely on: the 16x256b store mapping, and
// kind::i8 / kind::f16 MMAs whose A operand is read from TMEM.
#include <cuda_runtime.h>

#include "common.cuh"
#include "decode_tc.cuh"
#include "internal.h"
#include "tc.cuh"

namespace eva {
namespace {

constexpr int MB_ROWS = 32;                    // k-tile rows of the resident stage
constexpr int MB_NT = 8;                       // 16-column tiles per row
constexpr int MB_NSLOT = 7;                    // TMEM ring slots of 64 columns
constexpr int MB_DEC = 16;                     // decoding warps
constexpr int MB_THREADS = (MB_DEC + 1) * 32;

__device__ __forceinline__ uint32_t hash32(uint32_t x)
{
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

// ---------------------------------------------------------------------------------------------
// variant 0: the mma.sync decode loop (same device code as the fused decode kernel)

// POL: 0 the fused kernel's decode_raw (4 words per lane-tile); 1 + (NB, PRMT) combination: the
// two-word decode with NB windows extracted on the FMA pipe and pairs packed by PRMT or IMAD.
// 8-bit MMAs (m16n8k32, s32 accumulate): A = the weights' mul1 products as 4 unsigned bytes each
// (one weight per 4-byte K group), B = one 8-bit digit of a 16-bit fixed-point activation.
__device__ __forceinline__ void mma_16832_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_16832_u8u8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// POL 2: the byte sum left to 8-bit MMAs. A lane's 8 products (positions j0 (g, 2t) j1 (g, 2t+1) j2
// (g, 2t+8) j3 (g, 2t+9), j4..j7 the same for row g + 8) fill the A fragments of two m16n8k32 MMAs
// (k order permuted, B permuted alike), each run for the two activation digits: no dp4a, no packing.
// STAGE: every pass also does what a stage of the fused kernel does around its tiles (B fragments of
// the 4 rows loaded from shared memory, an mbarrier arrive and wait, a warp barrier).
template <int K, int POL, int NB, bool PRMT, bool STAGE = false>
__global__ void __launch_bounds__(MB_DEC * 32, 1) mb_legacy(int iters, unsigned long long* cyc, uint32_t* sink)
{
    extern __shared__ __align__(1024) uint8_t smem[];
    uint32_t* tr = reinterpret_cast<uint32_t*>(smem);
    __shared__ uint64_t wbar[MB_DEC];
    __shared__ __align__(16) uint32_t bsm[MB_ROWS * 64];
    const int nwords = MB_ROWS * MB_NT * 8 * K;
    for (int i = threadIdx.x; i < nwords; i += blockDim.x) tr[i] = hash32(i * 2654435761u + blockIdx.x);
    for (int i = threadIdx.x; i < MB_ROWS * 64; i += blockDim.x) bsm[i] = hash32(i + 77) & 0x3c003c00u;
    if (threadIdx.x < MB_DEC) mbar_init(&wbar[threadIdx.x], 1);
    fence_barrier_init();
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int quad = warp >> 1, whalf = warp & 1;
    const LaneGrp dg = lane_grp<K>(lane);
    const LaneW dw = lane_w<K>(lane);
    float acc[4][4] = {};
    int iacc[4][2][4] = {};
    uint32_t b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) b[i] = hash32(lane + 99 * i) & (POL == 2 ? 0x7f7f7f7fu : 0x3c003c00u);
    const unsigned long long t0 = clock64();
    for (int it = 0; it < iters; ++it) {
        // a different stage quarter every pass, so the decode cannot be hoisted out of the loop
        const int rbase = (4 * quad + 8 * it) & (MB_ROWS - 1);
        if (STAGE) {
            const uint4* bp = reinterpret_cast<const uint4*>(bsm + rbase * 64 + (lane & 3) * 8);
            const uint4 u0 = bp[0], u1 = bp[1];
            b[0] = u0.x; b[1] = u0.y; b[2] = u0.z; b[3] = u0.w;
            b[4] = u1.x; b[5] = u1.y; b[6] = u1.z; b[7] = u1.w;
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const uint32_t* rowp = tr + (((rbase + r) & (MB_ROWS - 1)) * MB_NT + 4 * whalf) * 8 * K;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                if (POL == 2) {
                    uint32_t st[8];
                    lane_states_w<K, NB>(rowp[t * 8 * K + dw.w0], rowp[t * 8 * K + dw.w1], dw, st);
                    uint32_t pr[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) pr[j] = st[j] * 0x83DCD12Du;
                    mma_16832_u8s8(iacc[t][0], pr[0], pr[4], pr[1], pr[5], b[2 * r], b[2 * r + 1]);
                    mma_16832_u8u8(iacc[t][1], pr[0], pr[4], pr[1], pr[5], b[(2 * r + 2) & 7], b[(2 * r + 3) & 7]);
                    mma_16832_u8s8(iacc[t][0], pr[2], pr[6], pr[3], pr[7], b[(2 * r + 4) & 7], b[(2 * r + 5) & 7]);
                    mma_16832_u8u8(iacc[t][1], pr[2], pr[6], pr[3], pr[7], b[(2 * r + 6) & 7], b[(2 * r + 7) & 7]);
                } else {
                    uint32_t a[4];
                    if (POL == 0) decode_raw<K>(rowp + t * 8 * K, dg, a);
                    else decode_afrag_w<K, NB, PRMT>(rowp + t * 8 * K, dw, a);
                    mma_16816(acc[t], a, b[2 * r], b[2 * r + 1]);
                }
            }
        }
        if (STAGE) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&wbar[warp]);
            mbar_wait(&wbar[warp], it & 1, reinterpret_cast<int*>(sink + 1));
        }
    }
    __syncthreads();
    const unsigned long long t1 = clock64();
    float s = 0.0f;
#pragma unroll
    for (int t = 0; t < 4; ++t)
#pragma unroll
        for (int c = 0; c < 4; ++c) s += acc[t][c] + static_cast<float>(iacc[t][0][c]) + static_cast<float>(iacc[t][1][c]);
    if (s == 12345.678f) sink[0] = 1;
    if (threadIdx.x == 0) atomicMax(cyc, t1 - t0);
}

// ---------------------------------------------------------------------------------------------
// variants 12 / 13: the fused decode kernel's pipeline with a synthetic item stream: one producer
// warp bulk-copies 32 trellis rows (8 tiles each, rows `row_stride` bytes apart, as a gate/up item
// reads them) plus 8 B rows of 1 KB per stage into a 4-stage ring; 16 decoding warps wait for the
// stage, load B from it, decode + MMA their 16 tiles and release it. src: trellis source of
// src_bytes (12: larger than L2, streamed from HBM; 13: 32 MB, resident in L2).

constexpr int MS_STAGE = 32 * 8 * 32 * 4 + 8 * 1024;   // trellis (K <= 4) + 8 B rows

__device__ __forceinline__ void cp_async16_cg(void* dst, const void* src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// Arrive on bar when this thread's earlier cp.async copies have landed (counted in the init count).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar)
{
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// NST ring stages; WAITF: decoders wait for the stage's data (false: they decode whatever the slot
// holds, which separates shared-memory contention from copy latency; then the decoders touch no
// barrier, the producer refills a slot only after its own previous copy into it landed, and it waits
// for its last copies before the CTA exits, so no copy is in flight at exit); MODE: 0 one bulk copy per
// trellis row (32 per stage), 1 one contiguous bulk copy per stage, 2 one 2-D tensor copy per stage
// (rows row_stride apart), 3 cp.async 16-byte copies by the producer warp.
template <int K, int NST, bool WAITF, int MODE>
__global__ void __launch_bounds__((MB_DEC + 1) * 32, 1) mb_stream(int iters, const uint8_t* src, size_t src_bytes,
                                                                 const uint8_t* bsrc, unsigned long long* cyc,
                                                                 int* status, const __grid_constant__ CUtensorMap tmap)
{
    constexpr int MS_NSTAGE = NST;
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ uint64_t full[MS_NSTAGE], empty[MS_NSTAGE];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < MS_NSTAGE; ++i) {
            mbar_init(&full[i], MODE == 3 ? 33 : 1);
            mbar_init(&empty[i], MB_DEC);
        }
        fence_barrier_init();
    }
    __syncthreads();
    constexpr uint32_t row_bytes = 8 * 32 * K;
    const size_t row_stride = static_cast<size_t>(128) * 32 * K;   // 2048 output columns per k-tile row
    const size_t rows_total = src_bytes / row_stride;
    const unsigned long long t0 = clock64();
    if (warp == MB_DEC) {
        for (int it = 0; it < iters; ++it) {
            const int slot = it % MS_NSTAGE;
            if (WAITF) mbar_wait(&empty[slot], ((it / MS_NSTAGE) & 1) ^ 1, status);
            else if (it >= MS_NSTAGE) mbar_wait(&full[slot], ((it / MS_NSTAGE) - 1) & 1, status);   // own copy landed
            // this CTA's stream of 32-row stages, chunk (blockIdx) of the row, rows advancing
            const size_t r0 = (static_cast<size_t>(it) * 32 + static_cast<size_t>(blockIdx.x) * 7919 * 32) % (rows_total - 32);
            const uint8_t* s0 = src + r0 * row_stride + static_cast<size_t>(blockIdx.x % 16) * row_bytes;
            if (lane == 0) mbar_arrive_expect_tx(&full[slot], (MODE == 3 ? 0 : 32 * row_bytes) + 8 * 1024);
            __syncwarp();
            uint8_t* st = smem + slot * MS_STAGE;
            if (MODE == 1) {
                if (lane == 0) bulk_g2s(st, s0, 32 * row_bytes, &full[slot]);
            } else if (MODE == 2) {
                if (lane == 0)
                    tma_load_2d(st, &tmap, static_cast<int>((blockIdx.x % 16) * (row_bytes / 8)), static_cast<int>(r0),
                                &full[slot]);
            } else if (MODE == 3) {
                for (int c = lane; c < 32 * static_cast<int>(row_bytes / 16); c += 32) {
                    const int row = c / (row_bytes / 16), off = (c % (row_bytes / 16)) * 16;
                    cp_async16_cg(st + row * row_bytes + off, s0 + row * row_stride + off);
                }
                cp_async_arrive_noinc(&full[slot]);
            } else {
                bulk_g2s(st + lane * row_bytes, s0 + lane * row_stride, row_bytes, &full[slot]);
            }
            if (lane < 8) bulk_g2s(st + 32 * 8 * 32 * 4 + lane * 1024, bsrc + lane * 1024, 1024, &full[slot]);
        }
        if (!WAITF)   // the last copy of every slot has landed before the CTA may exit
            for (int it = iters > MS_NSTAGE ? iters - MS_NSTAGE : 0; it < iters; ++it)
                mbar_wait(&full[it % MS_NSTAGE], (it / MS_NSTAGE) & 1, status);
    } else {
        const int quad = warp >> 1, whalf = warp & 1;
        const LaneW dw = lane_w<K>(lane);
        float acc[4][4] = {};
        for (int it = 0; it < iters; ++it) {
            const int slot = it % MS_NSTAGE;
            if (WAITF) mbar_wait(&full[slot], (it / MS_NSTAGE) & 1, status);
            const uint8_t* st = smem + slot * MS_STAGE;
            uint32_t b[8];
            const uint4* bp = reinterpret_cast<const uint4*>(st + 32 * 8 * 32 * 4 + (lane >> 2) * 1024 + quad * 128 +
                                                             (lane & 3) * 32);
            const uint4 u0 = bp[0], u1 = bp[1];
            b[0] = u0.x; b[1] = u0.y; b[2] = u0.z; b[3] = u0.w;
            b[4] = u1.x; b[5] = u1.y; b[6] = u1.z; b[7] = u1.w;
            const uint32_t* tr = reinterpret_cast<const uint32_t*>(st);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const uint32_t* rowp = tr + ((4 * quad + r) * MB_NT + 4 * whalf) * 8 * K;
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    uint32_t a[4];
                    decode_afrag_w<K, 2, true>(rowp + t * 8 * K, dw, a);
                    mma_16816(acc[t], a, b[2 * r] & 0x3fff3fffu, b[2 * r + 1] & 0x3fff3fffu);
                }
            }
            __syncwarp();
            if (WAITF && lane == 0) mbar_arrive(&empty[slot]);
        }
        float sm = 0.0f;
#pragma unroll
        for (int t = 0; t < 4; ++t)
#pragma unroll
            for (int c = 0; c < 4; ++c) sm += acc[t][c];
        if (sm == 12345.678f) status[1] = 1;
    }
    __syncthreads();
    const unsigned long long t1 = clock64();
    if (threadIdx.x == 0) atomicMax(cyc, t1 - t0);
}

// ---------------------------------------------------------------------------------------------
// variants 1..5: decode into TMEM (warp 0: TMEM owner and MMA issuer; warps 1..16: decoders)

template <int K, bool I8, bool MMA, bool BAL>
__global__ void __launch_bounds__(MB_THREADS, 1) mb_tmem(int iters, unsigned long long* cyc, int* status)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = align1024(smem_raw);
    uint8_t* bsm = smem;                                            // B operand: 2 KB, 128B swizzle
    uint32_t* tr = reinterpret_cast<uint32_t*>(smem + 2048);        // resident trellis stage
    __shared__ uint64_t full[MB_NSLOT], freeb[MB_NSLOT];
    __shared__ uint32_t tmem_base;
    const int nwords = MB_ROWS * MB_NT * 8 * K;
    for (int i = threadIdx.x; i < nwords; i += blockDim.x) tr[i] = hash32(i * 2654435761u + blockIdx.x);
    for (int i = threadIdx.x; i < 2048 / 4; i += blockDim.x)
        reinterpret_cast<uint32_t*>(bsm)[i] = I8 ? (hash32(i) & 0x03030303u) : (hash32(i) & 0x3c003c00u);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < MB_NSLOT; ++i) {
            mbar_init(&full[i], 4);
            mbar_init(&freeb[i], 1);
        }
        fence_barrier_init();
    }
    if (warp == 0) tmem_alloc(&tmem_base, 512);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = tmem_base;
    // a slot = 64 columns: i8 4 k-tiles x 16 columns, f16 8 k-tiles x 8 columns
    constexpr int KT = I8 ? 4 : 8, CPK = I8 ? 16 : 8;
    const int total_slots = 4 * iters;
    const unsigned long long t0 = clock64();
    if (warp == 0) {
        if (MMA && lane == 0) {
            const uint32_t idesc = I8 ? umma_idesc_u8s8(128, 16) : umma_idesc_f16(128, 16);
            const uint32_t tmem_d = tbase + 448;
            for (int it = 0; it < total_slots; ++it) {
                const int s = it % MB_NSLOT;
                if (!mbar_wait(&full[s], (it / MB_NSLOT) & 1, status)) break;
                tc_fence_after();
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint64_t db = umma_desc_sw128(smem_u32(bsm) + 32 * (j & 3));
                    const uint32_t ta = tbase + s * 64 + 8 * j;
                    if (I8) umma_i8_ta(tmem_d, ta, db, idesc, (it | j) != 0);
                    else umma_f16_ta(tmem_d, ta, db, idesc, (it | j) != 0);
                }
                umma_commit(&freeb[s]);
            }
            // the last commits: every slot free again before TMEM is released
            for (int s = 0; s < MB_NSLOT; ++s) {
                const int uses = total_slots / MB_NSLOT + (s < total_slots % MB_NSLOT ? 1 : 0);
                if (uses) mbar_wait(&freeb[s], (uses - 1) & 1, status);
            }
        }
    } else {
        const int q = (warp - 1) >> 2, sub = warp & 3;
        const LaneW d = lane_w<K>(lane);
        for (int it = q; it < total_slots; it += 4) {
            const int s = it % MB_NSLOT;
            if (MMA && !mbar_wait(&freeb[s], ((it / MB_NSLOT) & 1) ^ 1, status)) break;
#pragma unroll
            for (int kt = 0; kt < KT; ++kt) {
                const int row = (it * KT + kt) & (MB_ROWS - 1);
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                    const uint32_t* tile = tr + (row * MB_NT + 2 * sub + nt) * 8 * K;
                    const uint32_t taddr = tbase + ((32 * sub + 16 * nt) << 16) + s * 64 + kt * CPK;
                    if (I8) {
                        uint32_t r[8];
                        decode_prod_st<K, BAL>(tile, d, r);
                        tmem_st16x256_x2(taddr, r);
                    } else {
                        uint32_t r[4];
                        decode_raw_st<K, BAL>(tile, d, r);
                        tmem_st16x256_x1(taddr, r);
                    }
                }
            }
            if (MMA) {
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);
            }
        }
        tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    const unsigned long long t1 = clock64();
    if (threadIdx.x == 0) atomicMax(cyc, t1 - t0);
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
}

// ---------------------------------------------------------------------------------------------
// self tests (one CTA of 128 threads)

// 0: 16x256b.x2 stores tagged (half << 12 | thread << 4 | register) at lanes 32 w + 16 half, columns
//    0..15, read back with 32x32b.x16 -> out[lane][16]
// 1: D[128][16] s32 = A (u8 [128][32], TMEM) x B^T (s8 [16][32], smem)
// 2: D[128][16] f32 = A (f16 [128][16], TMEM) x B^T (f16 [16][16], smem)
__global__ void __launch_bounds__(128, 1) tc_selftest(int what, const uint32_t* a, const uint32_t* b, uint32_t* out,
                                                      int* status)
{
    __shared__ __align__(1024) uint8_t bsm[2048];
    __shared__ uint64_t done;
    __shared__ uint32_t tmem_base;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = threadIdx.x;
    if (t == 0) {
        mbar_init(&done, 1);
        fence_barrier_init();
    }
    for (int i = t; i < 512; i += 128) reinterpret_cast<uint32_t*>(bsm)[i] = 0;
    __syncthreads();
    if (warp == 0) tmem_alloc(&tmem_base, 64);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tb = tmem_base;
    const uint32_t lane_addr = static_cast<uint32_t>(32 * warp) << 16;
    if (what == 0) {
        for (int half = 0; half < 2; ++half) {
            uint32_t r[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) r[i] = (half << 12) | (lane << 4) | i;
            tmem_st16x256_x2(tb + lane_addr + (static_cast<uint32_t>(16 * half) << 16), r);
        }
        tmem_wait_st();
        uint32_t v[16];
        tmem_ld32x32_x16(tb + lane_addr, v);
        for (int i = 0; i < 16; ++i) out[t * 16 + i] = v[i];
    } else {
        // A row t: 8 words (u8 x 32 or f16 x 16) into TMEM columns 0..7 of lane t
        uint32_t r[8];
        for (int i = 0; i < 8; ++i) r[i] = a[t * 8 + i];
        tmem_st32x32_x8(tb + lane_addr, r);
        tmem_wait_st();
        // B rows n = 0..15, 32 bytes each, into the 128B-swizzled K-major layout
        if (t < 16 * 8) {
            const int n = t >> 3, w = t & 7, kb = 4 * w;   // byte offset kb of row n
            const int off = (n >> 3) * 1024 + (n & 7) * 128 + (((kb >> 4) ^ (n & 7)) << 4) + (kb & 15);
            *reinterpret_cast<uint32_t*>(bsm + off) = b[n * 8 + w];
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (t == 0) {
            const uint64_t db = umma_desc_sw128(smem_u32(bsm));
            if (what == 1) umma_i8_ta(tb + 32, tb, db, umma_idesc_u8s8(128, 16), 0);
            else umma_f16_ta(tb + 32, tb, db, umma_idesc_f16(128, 16), 0);
            umma_commit(&done);
        }
        __syncwarp();
        mbar_wait(&done, 0, status);
        tc_fence_after();
        uint32_t v[16];
        tmem_ld32x32_x16(tb + lane_addr + 32, v);
        for (int i = 0; i < 16; ++i) out[t * 16 + i] = v[i];
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tb, 64);
    }
}

// Dynamic shared memory of every variant: enough that one CTA fills an SM (each CTA allocates all
// 512 TMEM columns, and the rate is per SM).
constexpr size_t MB_SMEM = 120 * 1024;

template <int K>
cudaError_t run_micro(int variant, int iters, unsigned long long* cyc, int* status, uint32_t* sink, cudaStream_t st,
                      int sms)
{
    static_assert(1024 + 2048 + static_cast<size_t>(MB_ROWS) * MB_NT * 8 * 4 * 4 <= MB_SMEM, "resident stage");
    if (variant >= 12 && variant <= 18) {
        const size_t bytes = variant == 13 ? (static_cast<size_t>(32) << 20) : (static_cast<size_t>(1) << 30);
        uint8_t* src = nullptr;
        if (cudaMallocAsync(&src, bytes + 8192, st) != cudaSuccess) return cudaErrorMemoryAllocation;
        cudaMemsetAsync(src, 0x5b, bytes + 8192, st);
        void (*k)(int, const uint8_t*, size_t, const uint8_t*, unsigned long long*, int*, const CUtensorMap) = nullptr;
        int nst = 4;
        switch (variant) {
            case 12: case 13: k = mb_stream<K, 4, true, 0>; break;
            case 14: k = mb_stream<K, 5, true, 0>; nst = 5; break;
            case 15: k = mb_stream<K, 4, false, 0>; break;
            case 16: k = mb_stream<K, 4, true, 1>; break;
            case 17: k = mb_stream<K, 4, true, 2>; break;
            case 18: k = mb_stream<K, 4, true, 3>; break;
            default: return cudaErrorInvalidValue;
        }
        // 2-D map of the source as [rows][row_stride bytes] in 8-byte elements, box = 8 tiles x 32 rows
        CUtensorMap tmap{};
        {
            const size_t row_stride = static_cast<size_t>(128) * 32 * K;
            const cuuint64_t dims[2] = {row_stride / 8, bytes / row_stride};
            const cuuint64_t strides[1] = {row_stride};
            const cuuint32_t box[2] = {static_cast<cuuint32_t>(8 * 32 * K / 8), 32};
            const cuuint32_t estr[2] = {1, 1};
            auto fn = encode_fn();
            if (!fn || fn(&tmap, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, src, dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
                cudaFreeAsync(src, st);
                return cudaErrorInvalidValue;
            }
        }
        const size_t smem = static_cast<size_t>(nst) * MS_STAGE;
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        k<<<sms, (MB_DEC + 1) * 32, smem, st>>>(iters, src, bytes, src + bytes, cyc, status, tmap);
        const cudaError_t e = cudaGetLastError();
        cudaFreeAsync(src, st);
        return e;
    }
    if (variant == 0 || variant >= 6) {
        void (*k)(int, unsigned long long*, uint32_t*) = nullptr;
        switch (variant) {
            case 0: k = mb_legacy<K, 0, 0, false>; break;
            case 6: k = mb_legacy<K, 1, 0, false>; break;
            case 7: k = mb_legacy<K, 1, 0, true>; break;
            case 8: k = mb_legacy<K, 1, 2, true>; break;
            case 9: k = mb_legacy<K, 1, 2, false>; break;
            case 10: k = mb_legacy<K, 1, 4, true>; break;
            case 11: k = mb_legacy<K, 1, 2, true, true>; break;
            case 19: k = mb_legacy<K, 2, 2, true>; break;
            default: return cudaErrorInvalidValue;
        }
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(MB_SMEM));
        k<<<sms, MB_DEC * 32, MB_SMEM, st>>>(iters, cyc, sink);
        return cudaGetLastError();
    }
    const size_t smem = MB_SMEM;
    void (*k)(int, unsigned long long*, int*) = nullptr;
    switch (variant) {
        case 1: k = mb_tmem<K, true, false, true>; break;
        case 2: k = mb_tmem<K, false, false, true>; break;
        case 3: k = mb_tmem<K, true, true, true>; break;
        case 4: k = mb_tmem<K, false, true, true>; break;
        case 5: k = mb_tmem<K, true, false, false>; break;
        default: return cudaErrorInvalidValue;
    }
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    k<<<sms, MB_THREADS, smem, st>>>(iters, cyc, status);
    return cudaGetLastError();
}

}  // namespace
}  // namespace eva

using namespace eva;

extern "C" int eva_decode_microbench(int32_t variant, int32_t bits, int32_t iters, double* out, void* stream)
{
    if (!out || variant < 0 || variant > 19 || bits < 2 || bits > 4 || iters < 1 || iters > (1 << 24))
        return EVA_ERR_INVALID;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned long long* cyc = nullptr;
    if (cudaMallocAsync(&cyc, 64, st) != cudaSuccess) return EVA_ERR_CUDA;
    cudaMemsetAsync(cyc, 0, 64, st);
    int* status = reinterpret_cast<int*>(cyc + 2);
    uint32_t* sink = reinterpret_cast<uint32_t*>(cyc + 4);
    const int sms = num_sms();
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, st);
    cudaError_t e = bits == 2 ? run_micro<2>(variant, iters, cyc, status, sink, st, sms)
                  : bits == 3 ? run_micro<3>(variant, iters, cyc, status, sink, st, sms)
                              : run_micro<4>(variant, iters, cyc, status, sink, st, sms);
    cudaEventRecord(e1, st);
    unsigned long long h[3] = {0, 0, 0};
    if (e == cudaSuccess) e = cudaMemcpyAsync(h, cyc, 24, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    float ms = 0.0f;
    if (e == cudaSuccess) cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaFreeAsync(cyc, st);
    if (e != cudaSuccess) return EVA_ERR_CUDA;
    // weights per CTA: variant 0: 16 warps x iters x 16 tiles; TMEM variants: 4 x iters slots of
    // 4 warps x 2 n-tiles x KT k-tiles (i8 KT = 4, f16 KT = 8)
    const bool i8 = variant == 1 || variant == 3 || variant == 5;
    const bool legacy = variant == 0 || (variant >= 6 && variant <= 11) || variant == 19;
    const double tiles = variant >= 12 ? 16.0 * iters * 16 : legacy ? 16.0 * iters * 16 : 4.0 * iters * 4 * 2 * (i8 ? 4 : 8);
    out[0] = tiles * 256.0 / static_cast<double>(h[0] ? h[0] : 1);   // weights per SM clock
    out[1] = static_cast<double>(h[0]);                               // SM clocks (max over CTAs)
    out[2] = tiles * 256.0 * sms;                                     // weights decoded
    out[3] = static_cast<double>(static_cast<int>(h[2] & 0xffffffffu));   // device status bits
    out[4] = ms;                                                      // event time of the launch
    return EVA_OK;
}

extern "C" int eva_tc_selftest(int32_t what, const uint32_t* a, const uint32_t* b, uint32_t* out, int32_t* status,
                               void* stream)
{
    if (what < 0 || what > 4 || !out || !status || ((what == 1 || what == 2) && (!a || !b))) return EVA_ERR_INVALID;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (what >= 3) return pf_pair_selftest_launch(what == 3 ? 256 : 128, out, status, st) == cudaSuccess ? EVA_OK : EVA_ERR_CUDA;
    tc_selftest<<<1, 128, 0, st>>>(what, a, b, out, status);
    return cudaGetLastError() == cudaSuccess ? EVA_OK : EVA_ERR_CUDA;
}
