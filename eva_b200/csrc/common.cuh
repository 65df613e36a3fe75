// Device helpers shared by the eva_b200 MoE kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/eva_moe.h"

namespace eva {

// Device status bits (OR-ed into the workspace status word).
constexpr int ST_BAD_EXPERT = EVA_STATUS_BAD_EXPERT;     // expert id outside the tables / unbound pointer
constexpr int ST_TIMEOUT = EVA_STATUS_TIMEOUT;           // a bounded wait gave up
constexpr int ST_CAPACITY = EVA_STATUS_CAPACITY;         // more work than the workspace was sized for

constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;         // 2 s for any spin on another CTA / the TMA

__device__ __forceinline__ uint64_t globaltimer()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------------
// mbarrier + bulk copy (TMA, 1-D, no multicast)

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase. Returns false (and flags ST_TIMEOUT) when it gives up.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - t0 > WAIT_LIMIT_NS) {
            atomicOr(status, ST_TIMEOUT);
            return false;
        }
    }
    return true;
}

// Global -> shared bulk copy completing on an mbarrier. dst, src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// ---------------------------------------------------------------------------------------------
// Cross-CTA flags

__device__ __forceinline__ int ld_acquire(const int* p)
{
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Spin until *p >= target (acquire). Bounded; on timeout flags ST_TIMEOUT and returns false.
__device__ __forceinline__ bool wait_geq(const int* p, int target, int* status)
{
    if (ld_acquire(p) >= target) return true;
    const uint64_t t0 = globaltimer();
    while (ld_acquire(p) < target) {
        __nanosleep(64);
        if (globaltimer() - t0 > WAIT_LIMIT_NS) {
            atomicOr(status, ST_TIMEOUT);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void named_sync(int id, int threads)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------------------------------------
// 128-point Hadamard across a warp: lane l holds elements 4l..4l+3. Natural (Sylvester) order,
// scaled by 1/sqrt(128): out[i] = sum_j (-1)^popcount(i & j) in[j] / sqrt(128).

__device__ __forceinline__ void had128_warp(float (&v)[4], int lane)
{
    // in-register butterflies over the two low index bits
    float a = v[0] + v[1], b = v[0] - v[1], c = v[2] + v[3], d = v[2] - v[3];
    v[0] = a + c;
    v[1] = b + d;
    v[2] = a - c;
    v[3] = b - d;
    // butterflies over the 5 lane bits
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const bool upper = (lane & m) != 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float o = __shfl_xor_sync(0xffffffffu, v[i], m);
            v[i] = upper ? (o - v[i]) : (v[i] + o);
        }
    }
    const float s = 0.08838834764831845f;   // 1/sqrt(128)
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] *= s;
}

// ---------------------------------------------------------------------------------------------
// Half/bf16 helpers

__device__ __forceinline__ void load4_half(const __half* p, float (&v)[4])
{
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __half2 a = *reinterpret_cast<const __half2*>(&u.x);
    const __half2 b = *reinterpret_cast<const __half2*>(&u.y);
    v[0] = __low2float(a);
    v[1] = __high2float(a);
    v[2] = __low2float(b);
    v[3] = __high2float(b);
}

__device__ __forceinline__ void load4_half_ro(const __half* p, float (&v)[4])
{
    const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
    const __half2 a = *reinterpret_cast<const __half2*>(&u.x);
    const __half2 b = *reinterpret_cast<const __half2*>(&u.y);
    v[0] = __low2float(a);
    v[1] = __high2float(a);
    v[2] = __low2float(b);
    v[3] = __high2float(b);
}

__device__ __forceinline__ void store4_half(__half* p, const float (&v)[4])
{
    const __half2 a = __floats2half2_rn(v[0], v[1]);
    const __half2 b = __floats2half2_rn(v[2], v[3]);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = u;
}

// x row element loads: bf16 (is_bf16) or fp16
__device__ __forceinline__ void load4_x(const void* x, size_t off, int is_bf16, float (&v)[4])
{
    if (is_bf16) {
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(x) + off));
        const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
        const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
        v[0] = __low2float(a);
        v[1] = __high2float(a);
        v[2] = __low2float(b);
        v[3] = __high2float(b);
    } else {
        load4_half_ro(static_cast<const __half*>(x) + off, v);
    }
}

// ---------------------------------------------------------------------------------------------
// EXL3 trellis decode (mul1 codebook)
//
// A 16x16 tile holds 256 K-bit codes in 8K 32-bit words, bits MSB-first through the words. The
// 16-bit state of position p is the window ending at bit (p+1)K, circular modulo 256K. State ->
// weight: byte sum of state * 0x83DCD12D added to the fp16 pattern of 1024.0 (exact fp16 1024 +
// sum), then one fp16 FMA with the constants 0x1eee, 0xc931 (codebook format of the reference's
// vendored ExLlamaV3 headers; see DESIGN.md "format constants").
//
// Lane l decodes positions 8l..8l+7. With p = 8l + j the position is weight (k, n) of the tile:
// n = l/4 + 8(j/4), k = 2(l%4) + (j%2) + 8((j/2)%2). That is exactly the A fragment of
// mma.m16n8k16 with A[m = n][k]: reg0 = (j0,j1), reg1 = (j4,j5), reg2 = (j2,j3), reg3 = (j6,j7).

__device__ __forceinline__ uint32_t mul1_sum(uint32_t state)
{
    return __dp4a(state * 0x83DCD12Du, 0x01010101u, 0x6400u);
}

__device__ __forceinline__ uint32_t mul1_pair(uint32_t s0, uint32_t s1)
{
    const uint32_t h = __byte_perm(mul1_sum(s0), mul1_sum(s1), 0x5410);
    const __half2 k0 = __halves2half2(__ushort_as_half(0x1eee), __ushort_as_half(0x1eee));
    const __half2 k1 = __halves2half2(__ushort_as_half(0xc931), __ushort_as_half(0xc931));
    const __half2 r = __hfma2(*reinterpret_cast<const __half2*>(&h), k0, k1);
    return *reinterpret_cast<const uint32_t*>(&r);
}

// The 8 states of lane `lane` from the tile's words (smem or global).
template <int K>
__device__ __forceinline__ void lane_states(const uint32_t* tile, int lane, uint32_t (&st)[8])
{
    constexpr int NB = 256 * K, NW = 8 * K;
    int start = (8 * lane + 1) * K - 16;
    if (start < 0) start += NB;
    const int w0 = start >> 5, off = start & 31;
    const uint32_t hi = tile[w0];
    const uint32_t lo = tile[(w0 + 1 == NW) ? 0 : w0 + 1];
    const uint64_t v = (static_cast<uint64_t>(hi) << 32) | lo;
#pragma unroll
    for (int j = 0; j < 8; ++j) st[j] = static_cast<uint32_t>(v >> (48 - off - j * K)) & 0xffffu;
}

// A fragment (4 x half2) of lane `lane` for one tile.
template <int K>
__device__ __forceinline__ void decode_afrag(const uint32_t* tile, int lane, uint32_t (&a)[4])
{
    uint32_t st[8];
    lane_states<K>(tile, lane, st);
    a[0] = mul1_pair(st[0], st[1]);
    a[1] = mul1_pair(st[4], st[5]);
    a[2] = mul1_pair(st[2], st[3]);
    a[3] = mul1_pair(st[6], st[7]);
}

// D[16 x 8] += A[16 x 16] (fp16, row) * B[16 x 8] (fp16, col), fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Gated activation. mode 0: silu(g) then clamp (u to +-limit, the activation to <= limit) when
// limit != 0 (the MoE coop kernels' act_gate). mode 1: clamp g (<= limit) and u (+-limit) first
// when limit > 0, then silu(g) * u (torch swiglu, used for the shared expert).
__device__ __forceinline__ float act_gated(float g, float u, float limit, int mode)
{
    if (mode == 1) {
        if (limit > 0.0f) {
            u = fminf(fmaxf(u, -limit), limit);
            g = fminf(g, limit);
        }
        return g / (1.0f + expf(-g)) * u;
    }
    float a = g / (1.0f + expf(-g));
    if (limit != 0.0f) {
        u = fminf(fmaxf(u, -limit), limit);
        a = fminf(a, limit);
    }
    return a * u;
}

}  // namespace eva
