// EXL3 decode into tensor memory: helpers for feeding tcgen05.mma with the weight operand (A) held in
// TMEM, written by the decoding warps with tcgen05.st.
//
// A lane of a decoding warp decodes the 8 trellis positions 8 l .. 8 l + 7 of a 16 x 16 tile (lane
// l), which are the weights (n, k) with n in {g, g + 8} (g = l / 4) and k in {2 t, 2 t + 1, 2 t + 8,
// 2 t + 9} (t = l % 4) (the position map of the format, see common.cuh). Those are exactly the
// cells the 16x256b shape of tcgen05.st gives a thread (TMEM lanes g and g + 8, columns 2 t, 2 t + 1
// of each 8-column block), so a tile goes to TMEM without any exchange between lanes:
//   * i8 form: each weight is stored as its 32-bit mul1 product P = state * 0x83DCD12D, whose four
//     bytes sum to the raw codebook value h - 1024. Row n of the A operand holds P(n, k) in column
//     k (k = 0..15 per tile): one column = four K positions of kind::i8, so the MMA forms the byte
//     sum itself when every byte of a column meets the same activation (B replicated 4 times along
//     K). Instruction count per weight: window extraction, one multiply, 1/8 of a store.
//   * f16 form: each weight is stored as the fp16 raw codebook value h = 1024 + bytesum (exact).
//     Column c holds the k pair (c, c + 1) for even c and (c + 7, c + 8) for odd c, so the B
//     operand's K order within each 16 is [0 1 8 9 2 3 10 11 4 5 12 13 6 7 14 15].
// The windows of a lane lie in two consecutive 32-bit words of the tile (off + 7K + 16 <= 64 bits
// for K <= 4), so a tile costs a lane two shared-memory loads.
#pragma once

#include "common.cuh"

namespace eva {

// Per-lane constants of the two-word decode: the two words (wrap resolved) and the funnel shifts
// that give G_b = stream bits [start, start + 32) and G_a = the 32 bits ending at the end of
// window 7 (start = first bit of window 0).
struct LaneW {
    int w0, w1, sb, sa;
};

template <int K>
__device__ __forceinline__ LaneW lane_w(int lane)
{
    constexpr int NB = 256 * K, NW = 8 * K;
    int start = (8 * lane + 1) * K - 16;
    if (start < 0) start += NB;
    LaneW d;
    d.w0 = start >> 5;
    d.w1 = d.w0 + 1 == NW ? 0 : d.w0 + 1;
    const int off = start & 31;                 // 1 <= off <= 27 for K = 2, 3, 4
    d.sb = 32 - off;
    d.sa = 64 - (off + 7 * K + 16);             // K = 2 uses G_b only
    return d;
}

// x << s as a multiply (the FMA pipe's IMAD), so that window extraction can be split between the
// ALU and FMA pipes: (x >> s) & 0xffff == (x * 2^(16 - s)) >> 16 for s <= 16.
__device__ __forceinline__ uint32_t mul_shl(uint32_t x, uint32_t m)
{
    uint32_t r;
    asm("mad.lo.u32 %0, %1, %2, 0;" : "=r"(r) : "r"(x), "r"(m));
    return r;
}

// The 8 trellis states of a lane, j = 0..7 (window j ends at bit (8 lane + j + 1) K of the tile).
// NB windows (0, 2 or 4: windows 1, 5, then 2, 6) are extracted as multiply + shift (FMA + ALU pipe)
// instead of shift + mask (2 ALU), to balance the two integer pipes.
template <int K, int NB>
__device__ __forceinline__ void lane_states_w(uint32_t w0, uint32_t w1, const LaneW& d, uint32_t (&s)[8])
{
    const uint32_t gb = __funnelshift_r(w1, w0, d.sb);
    if constexpr (K == 2) {
        s[0] = gb >> 16;
#pragma unroll
        for (int j = 1; j < 8; ++j) {
            const bool bal = (NB >= 2 && (j == 1 || j == 5)) || (NB >= 4 && (j == 3 || j == 7));
            if (bal) s[j] = mul_shl(gb, 1u << (2 * j)) >> 16;
            else s[j] = (gb >> (16 - 2 * j)) & 0xffffu;
        }
    } else {
        const uint32_t ga = __funnelshift_r(w1, w0, d.sa);
        s[0] = gb >> 16;
#pragma unroll
        for (int j = 1; j < 4; ++j) {
            const bool bal = (NB >= 2 && j == 1) || (NB >= 4 && j == 2);
            if (bal) s[j] = mul_shl(gb, 1u << (j * K)) >> 16;
            else s[j] = (gb >> (16 - j * K)) & 0xffffu;
        }
#pragma unroll
        for (int j = 4; j < 7; ++j) {
            const bool bal = (NB >= 2 && j == 5) || (NB >= 4 && j == 6);
            if (bal) s[j] = mul_shl(ga, 1u << (16 - (7 - j) * K)) >> 16;
            else s[j] = (ga >> ((7 - j) * K)) & 0xffffu;
        }
        s[7] = ga & 0xffffu;
    }
}

// A fragment of mma.m16n8k16 (weights as A[m = n][k]) for one tile, from the lane's two words: raw codebook values
// h = 1024 + bytesum as exact fp16 pairs, reg0 (g; 2t, 2t+1) reg1 (g+8; 2t, 2t+1) reg2 (g; 2t+8, 2t+9)
// reg3 (g+8; 2t+8, 2t+9). PRMT: pack pairs with a byte permute (ALU) instead of a multiply-add (FMA).
template <int K, int NB, bool PRMT>
__device__ __forceinline__ void decode_afrag_ww(uint32_t w0, uint32_t w1, const LaneW& d, uint32_t (&a)[4])
{
    uint32_t s[8];
    lane_states_w<K, NB>(w0, w1, d, s);
    uint32_t h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) h[j] = mul1_sum(s[j]);
    if (PRMT) {
        a[0] = __byte_perm(h[0], h[1], 0x5410);
        a[1] = __byte_perm(h[4], h[5], 0x5410);
        a[2] = __byte_perm(h[2], h[3], 0x5410);
        a[3] = __byte_perm(h[6], h[7], 0x5410);
    } else {
        a[0] = imad_pack(h[1], h[0]);
        a[1] = imad_pack(h[5], h[4]);
        a[2] = imad_pack(h[3], h[2]);
        a[3] = imad_pack(h[7], h[6]);
    }
}

// The same from the tile in shared memory (words d.w0, d.w1).
template <int K, int NB, bool PRMT>
__device__ __forceinline__ void decode_afrag_w(const uint32_t* tile, const LaneW& d, uint32_t (&a)[4])
{
    decode_afrag_ww<K, NB, PRMT>(tile[d.w0], tile[d.w1], d, a);
}

// i8 form: the eight mul1 products in 16x256b.x2 register order
// r0 (g, k 2t) r1 (g, 2t+1) r2 (g+8, 2t) r3 (g+8, 2t+1) r4 (g, 2t+8) r5 (g, 2t+9) r6 (g+8, 2t+8) r7 (g+8, 2t+9)
template <int K, bool BAL>
__device__ __forceinline__ void decode_prod_st(const uint32_t* tile, const LaneW& d, uint32_t (&r)[8])
{
    uint32_t s[8];
    lane_states_w<K, BAL ? 4 : 0>(tile[d.w0], tile[d.w1], d, s);
    // position j of the lane: j0 (g, 2t) j1 (g, 2t+1) j2 (g, 2t+8) j3 (g, 2t+9) j4..j7 the same for g + 8
    r[0] = s[0] * 0x83DCD12Du;
    r[1] = s[1] * 0x83DCD12Du;
    r[2] = s[4] * 0x83DCD12Du;
    r[3] = s[5] * 0x83DCD12Du;
    r[4] = s[2] * 0x83DCD12Du;
    r[5] = s[3] * 0x83DCD12Du;
    r[6] = s[6] * 0x83DCD12Du;
    r[7] = s[7] * 0x83DCD12Du;
}

// f16 form: raw codebook pairs in 16x256b.x1 register order r0 (g, col 2t) r1 (g, 2t+1) r2 (g+8, 2t)
// r3 (g+8, 2t+1); column 2t holds k (2t, 2t+1), column 2t+1 holds k (2t+8, 2t+9).
template <int K, bool BAL>
__device__ __forceinline__ void decode_raw_st(const uint32_t* tile, const LaneW& d, uint32_t (&r)[4])
{
    uint32_t s[8];
    lane_states_w<K, BAL ? 4 : 0>(tile[d.w0], tile[d.w1], d, s);
    uint32_t h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) h[j] = mul1_sum(s[j]);
    r[0] = __byte_perm(h[0], h[1], 0x5410);
    r[1] = __byte_perm(h[2], h[3], 0x5410);
    r[2] = __byte_perm(h[4], h[5], 0x5410);
    r[3] = __byte_perm(h[6], h[7], 0x5410);
}

// ---------------------------------------------------------------------------------------------
// tcgen05 forms with A in tensor memory

__device__ __forceinline__ void tmem_st16x256_x1(uint32_t taddr, const uint32_t (&r)[4])
{
    asm volatile("tcgen05.st.sync.aligned.16x256b.x1.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(r[0]), "r"(r[1]),
                 "r"(r[2]), "r"(r[3])
                 : "memory");
}

__device__ __forceinline__ void tmem_st16x256_x2(uint32_t taddr, const uint32_t (&r)[8])
{
    asm volatile("tcgen05.st.sync.aligned.16x256b.x2.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}

__device__ __forceinline__ void tmem_st32x32_x8(uint32_t taddr, const uint32_t (&r)[8])
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32x32_x8(uint32_t taddr, uint32_t (&r)[8])
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32x32_x16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
        "[%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// kind::i8 instruction descriptor: u8 A, s8 B (K-major), s32 accumulator, M x N
__host__ __device__ constexpr uint32_t umma_idesc_u8s8(int M, int N)
{
    return (2u << 4) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// D[tmem] (+)= A[tmem] * B[smem]^T, one CTA
__device__ __forceinline__ void umma_i8_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc, uint32_t acc)
{
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n}\n" ::"r"(
            tmem_d),
        "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_f16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc, uint32_t acc)
{
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(
            tmem_d),
        "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc));
}

}  // namespace eva
