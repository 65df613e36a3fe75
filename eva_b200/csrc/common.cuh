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
// mbarrier + bulk copy (TMA, 1-D, one CTA per copy)

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

__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// Bounded wait on an mbarrier phase. Returns false (and flags ST_TIMEOUT) when it gives up. Once
// any wait of the launch has given up, later waits return at once, so a systematic failure costs
// one wait limit, not one per stage.
// try_wait suspends the thread in hardware for a while, so the loop is not hot; the clock and the
// global status word are only read every 32 unsuccessful tries (a global load per try would put
// every briefly waiting warp behind a memory round trip).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status)
{
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = 0;
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 31) == 0) {
            const uint64_t t = globaltimer();
            if (t0 == 0) {
                t0 = t;
                if (ld_volatile(status) & ST_TIMEOUT) return false;
            } else if (t - t0 > WAIT_LIMIT_NS || (ld_volatile(status) & ST_TIMEOUT)) {
                atomicOr(status, ST_TIMEOUT);
                return false;
            }
        }
    }
}

// mbar_wait for warps that are not on the critical path (they sleep ns nanoseconds between tries, so a
// long wait does not take issue slots from the warps doing the work). Same bound and status rules.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, int* status, uint32_t ns)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    if (ld_volatile(status) & ST_TIMEOUT) return false;
    for (;;) {
        __nanosleep(ns);
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer() - t0 > WAIT_LIMIT_NS || (ld_volatile(status) & ST_TIMEOUT)) {
            atomicOr(status, ST_TIMEOUT);
            return false;
        }
    }
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
    if (ld_volatile(status) & ST_TIMEOUT) return false;
    const uint64_t t0 = globaltimer();
    while (ld_acquire(p) < target) {
        __nanosleep(64);
        if (globaltimer() - t0 > WAIT_LIMIT_NS || (ld_volatile(status) & ST_TIMEOUT)) {
            atomicOr(status, ST_TIMEOUT);
            return false;
        }
    }
    return true;
}

// Ampere-style async copy of 8 bytes global -> shared (L1-cached; only for data not written during
// the kernel), with group commit / wait.
__device__ __forceinline__ void cp_async8(void* dst, const void* src)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void named_sync(int id, int threads)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------------------------------------
// Packed fp32 pairs (sm_100's two-wide FADD / FMUL / FFMA): each half is rounded exactly as the
// scalar operation rounds it, so a butterfly written on pairs gives the scalar code's bits with
// half the instructions. a - b is fma(b, -1, a): the product is exact, the one rounding is a - b's.

__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 sub2(float2 a, float2 b) { return __ffma2_rn(b, make_float2(-1.0f, -1.0f), a); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// ---------------------------------------------------------------------------------------------
// 128-point Hadamard across a warp: lane l holds elements 4l..4l+3. Natural (Sylvester) order,
// scaled by 1/sqrt(128): out[i] = sum_j (-1)^popcount(i & j) in[j] / sqrt(128).

__device__ __forceinline__ void had128_warp(float (&v)[4], int lane)
{
    // in-register butterflies over the two low index bits: bit 0 inside the pairs (v0, v1) and
    // (v2, v3), bit 1 between the pairs as packed operations
    const float2 p = make_float2(v[0] + v[1], v[0] - v[1]), q = make_float2(v[2] + v[3], v[2] - v[3]);
    float2 lo = add2(p, q), hi = sub2(p, q);   // new (v0, v1) = p + q, new (v2, v3) = p - q
    // butterflies over the 5 lane bits: lower lane v + o, upper lane o - v, both as one fma with the
    // lane's sign (exactly the same roundings as the add / subtract)
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const float s1 = (lane & m) ? -1.0f : 1.0f;
        const float2 sg = make_float2(s1, s1);
        const float2 olo = make_float2(__shfl_xor_sync(0xffffffffu, lo.x, m), __shfl_xor_sync(0xffffffffu, lo.y, m));
        const float2 ohi = make_float2(__shfl_xor_sync(0xffffffffu, hi.x, m), __shfl_xor_sync(0xffffffffu, hi.y, m));
        lo = fma2(lo, sg, olo);
        hi = fma2(hi, sg, ohi);
    }
    const float2 s = make_float2(0.08838834764831845f, 0.08838834764831845f);   // 1/sqrt(128)
    lo = mul2(lo, s);
    hi = mul2(hi, s);
    v[0] = lo.x;
    v[1] = lo.y;
    v[2] = hi.x;
    v[3] = hi.y;
}

// Explicit shared-space accesses for decoding warps (generic accesses wait on the long scoreboard).
__device__ __forceinline__ uint32_t lds32(uint32_t addr)
{
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ uint4 lds128(uint32_t addr)
{
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ void sts32(uint32_t addr, uint32_t v)
{
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
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
// sum), then one fp16 FMA with the constants 0x1eee, 0xc931. These constants define the EXL3 mul1
// codebook (ExLlamaV3, vendored by the reference at runtime/ds41/csrc/moe_coop2048/vendor/quant/
// codebook.cuh:86-99); the stored weights only mean anything under them.
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

// Per-lane decode constants of a K-bit tile: the two words that hold the lane's 8 windows (wrap
// resolved) and the bit offset of the first window inside them.
struct LaneDec {
    int w0, w1, off;
};

template <int K>
__device__ __forceinline__ LaneDec lane_dec(int lane)
{
    constexpr int NB = 256 * K, NW = 8 * K;
    int start = (8 * lane + 1) * K - 16;
    if (start < 0) start += NB;
    LaneDec d;
    d.w0 = start >> 5;
    d.w1 = d.w0 + 1 == NW ? 0 : d.w0 + 1;
    d.off = start & 31;
    return d;
}

// The 8 states of one tile for a lane: the 16-bit windows ending at bits (8 lane + j + 1) K lie
// within two consecutive words (16 + 7K <= 44 bits, offset <= 27 for K <= 4).
template <int K>
__device__ __forceinline__ void lane_states(const uint32_t* tile, const LaneDec& d, uint32_t (&st)[8])
{
    const uint64_t v = (static_cast<uint64_t>(tile[d.w0]) << 32) | tile[d.w1];
#pragma unroll
    for (int j = 0; j < 8; ++j) st[j] = static_cast<uint32_t>(v >> (48 - d.off - j * K)) & 0xffffu;
}

template <int K>
__device__ __forceinline__ void lane_states(const uint32_t* tile, int lane, uint32_t (&st)[8])
{
    lane_states<K>(tile, lane_dec<K>(lane), st);
}

// Raw-codebook decode for the GEMV (decode_raw): the MMA takes h = 1024 + bytesum as an exact fp16
// value and the affine map w = c0 h + c1 (c0, c1 = fp16 0x1eee, 0xc931) is applied to the sums:
// sum_k x_k w_k = c0 sum_k x_k h_k + c1 sum_k x_k. This drops the per-weight fp16 FMA; the weights
// used are c0 h + c1 before their single fp16 rounding (|difference| <= half an fp16 ulp).
constexpr float CB_C0 = 0.00676727294921875f;   // fp16 0x1eee
constexpr float CB_C1 = -10.3828125f;           // fp16 0xc931

// The two groups of 4 windows (0-3 and 4-7) each span 16 + 3K <= 28 bits, so one funnel shift
// (amount < 32) of the two words around the group's end puts its last window in bits 0-15 and
// the others K, 2K, 3K bits higher.
struct LaneGrp {
    int b0, b1, a0, a1;   // word indices (wrap resolved) of group 0-3 (b) and 4-7 (a)
    int shb, sha;
};

template <int K>
__device__ __forceinline__ LaneGrp lane_grp(int lane)
{
    constexpr int NW = 8 * K;
    LaneGrp g;
    const int eb = (8 * lane + 4) * K, ea = (8 * lane + 8) * K;   // end bits of windows 3 and 7
    const int wb = (eb + 31) / 32 - 2, wa = (ea + 31) / 32 - 2;
    g.shb = 32 * (wb + 2) - eb;
    g.sha = 32 * (wa + 2) - ea;
    g.b0 = wb < 0 ? wb + NW : wb;
    g.a0 = wa < 0 ? wa + NW : wa;
    g.b1 = g.b0 + 1 == NW ? 0 : g.b0 + 1;
    g.a1 = g.a0 + 1 == NW ? 0 : g.a0 + 1;
    return g;
}

__device__ __forceinline__ uint32_t imad_pack(uint32_t hi, uint32_t lo)
{
    uint32_t r;
    asm("mad.lo.u32 %0, %1, 65536, %2;" : "=r"(r) : "r"(hi), "r"(lo));
    return r;
}

template <int K>
__device__ __forceinline__ void decode_raw(const uint32_t* tile, const LaneGrp& g, uint32_t (&a)[4])
{
    const uint32_t wb = __funnelshift_r(tile[g.b1], tile[g.b0], g.shb);
    const uint32_t wa = __funnelshift_r(tile[g.a1], tile[g.a0], g.sha);
    uint32_t h[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        h[3 - j] = mul1_sum((wb >> (j * K)) & 0xffffu);
        h[7 - j] = mul1_sum((wa >> (j * K)) & 0xffffu);
    }
    // pack pairs with a multiply-add (FMA pipe) instead of a byte permute (ALU pipe, the busier one):
    // h < 2^16, so hi * 2^16 + lo is the packed pair
    a[0] = imad_pack(h[1], h[0]);
    a[1] = imad_pack(h[5], h[4]);
    a[2] = imad_pack(h[3], h[2]);
    a[3] = imad_pack(h[7], h[6]);
}

// A fragment of one tile for a lane from the words of its two window groups (see LaneGrp): each
// group is one funnel shift, each window one shift + mask. RAW: the raw codebook values
// h = 1024 + bytesum (exact fp16, as decode_raw; the affine map is applied to the products);
// otherwise exact fp16 weights (the codebook FMA on the packed pairs).
template <int K, bool RAW = false>
__device__ __forceinline__ void decode_afrag_grp(uint32_t b0, uint32_t b1, uint32_t a0, uint32_t a1, const LaneGrp& g,
                                                 uint32_t (&a)[4])
{
    const uint32_t wb = __funnelshift_r(b1, b0, g.shb);
    const uint32_t wa = __funnelshift_r(a1, a0, g.sha);
    uint32_t h[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        h[3 - j] = mul1_sum((wb >> (j * K)) & 0xffffu);
        h[7 - j] = mul1_sum((wa >> (j * K)) & 0xffffu);
    }
    const __half2 k0 = __halves2half2(__ushort_as_half(0x1eee), __ushort_as_half(0x1eee));
    const __half2 k1 = __halves2half2(__ushort_as_half(0xc931), __ushort_as_half(0xc931));
    const uint32_t p[4] = {imad_pack(h[1], h[0]), imad_pack(h[5], h[4]), imad_pack(h[3], h[2]), imad_pack(h[7], h[6])};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if (RAW) {
            a[i] = p[i];
        } else {
            const __half2 r = __hfma2(*reinterpret_cast<const __half2*>(&p[i]), k0, k1);
            a[i] = *reinterpret_cast<const uint32_t*>(&r);
        }
    }
}

// A fragment (4 x half2) of one tile for a lane: exact fp16 weights.
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
    // the routed experts' SiLU with the fast exponential and reciprocal, as the reference's coop
    // kernels evaluate it (exl3_moe_coop_kernel.cuh:80-84): a few ulp from the correctly rounded value,
    // an eighth of the instructions of expf and an IEEE division
    float a = g * __fdividef(1.0f, 1.0f + __expf(-g));
    if (limit != 0.0f) {
        u = fminf(fmaxf(u, -limit), limit);
        a = fminf(a, limit);
    }
    return a * u;
}

}  // namespace eva
