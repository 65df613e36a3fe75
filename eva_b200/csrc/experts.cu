// Fused EXL3 expert kernel (decode-shaped, bandwidth bound): one persistent launch runs, for every
// expert run (<= 8 slots that picked one expert) and the shared expert,
//     rotate:   x' = fp16(H128(x * suh))                       for gate and up
//     gate/up:  h = x' W'  (EXL3 tiles decoded in registers)    per 128-column chunk of I
//     epilogue: g, u = H128(h) * svh; a = act(g, u); a' = fp16(H128(a * suh_down))
//     down:     y = a' W'_down                                  per 128-column chunk of H
//     epilogue: v = H128(y) * svh_down * routing weight; the last arrival of a (token, chunk)
//               sums the token's slots in slot order, then the shared expert, and stores the row.
//
// Work items are claimed from a global counter in phase order (all rotations, then all gate/up
// chunks, then all down chunks). An item only ever waits (bounded) on items with smaller indices,
// which were claimed earlier by running CTAs, so the schedule cannot deadlock; an epilogue never
// waits on anything but its own CTA's partial sums.
//
// Per CTA (warp specialised):
//   warp 16      producer: claims items and streams each stage of their trellis rows (32 k-tile rows x
//                128 columns) with one 2-D TMA tensor copy into a shared-memory ring (5 stages when the
//                launch's widest trellis is K <= 3, else 4), writing each item's geometry, run and slots
//                into the stage header; the last warp copies the run's B rows of each stage
//   warps 0..15  decoders: each decodes 4 rows x 4 tiles per stage in registers (two words and two
//                funnel shifts per lane and tile, window extraction split between the ALU and FMA
//                pipes) and runs mma.m16n8k16 with the weights as the 16 x 16 A operand (rows =
//                output columns) and up to 8 tokens as B, accumulating in fp32. The MMA takes the
//                raw codebook values h = 1024 + bytesum and the codebook's affine map is applied to
//                the sums (see decode_raw). At a projection's end they store their partial sums
//                and go straight on; rotation items are done by these 16 warps together.
//   warps 17..   epilogue (2, or 4 for short or split items): sum the 8 k-quads of a projection's
//                partials (mbarrier hand-off, the partial buffer is released right after), then the
//                item's epilogue (split-k publication, Hadamard / scales / activation or the
//                combine) while the decoders already run the next item.
//
// Reference behaviour (paths within Findddx/eva, runtime/ds41/csrc/moe_coop2048/vendor/quant/):
//   exl3_moe_coop_kernel.cuh:634-671 (rotation), :680-809 (gate/up GEMV + epilogue),
//   :816-963 (down GEMV + combine + shared merge); exl3_dq.cuh / codebook.cuh (decode).
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "decode_tc.cuh"
#include "internal.h"
#include "tc.cuh"

namespace eva {

constexpr int NCW = 16;                    // decoding warps (warps 0..15)
// Epilogue warps (warps 17 .. 16 + NEW; warp 16 is the trellis producer, warp 17 + NEW the B
// producer): 2 where items are long (a gate/up item spans more than 4096 input columns), so the
// decoders keep more of the SM's issue slots; 4 where they are short or split (per item the
// epilogue warps' share, the split-k reduction and the rows' epilogues, is then larger).
// Measured (experts launch): V3 batch 8 0.569 ms with 2 vs 0.579 with 4; V3 batch 1 (split 2)
// 0.144 vs 0.132; V2-Lite (H 2048) batch 16 0.148 vs 0.140.
template <int NEW>
struct DecWarps {
    static constexpr int bpw = NCW + 1 + NEW;              // the B producer warp
    static constexpr int threads = (NCW + 2 + NEW) * 32;
};
constexpr int DEC_SHORT_ITEM_COLS = 4096;  // gate/up input columns per item at or below which NEW = 4
constexpr int STAGE_KT = 32;               // k-tile rows per stage (4 per decoding warp pair)
constexpr int NT = 8;                      // 16-column tiles per item (128 output columns)
constexpr int BROW_BYTES = STAGE_KT * 32;              // one token row of B for the stage's k-tile rows (fp16)
constexpr int RES_FLOATS = 2 * RUN_ROWS * 128;
constexpr int PART_F4 = NCW * 4 * 32;      // one projection's partial sums: [warp][tile][lane] float4

// The ring of a launch whose largest trellis width is KMAX: stages sized for KMAX, and one stage more
// where that leaves room (K <= 3), so the copies run further ahead of the decoders.
template <int KMAX>
struct DecRing {
    static constexpr int nstage = KMAX <= 3 ? 5 : 4;
    static constexpr int stage_bytes = STAGE_KT * NT * 32 * KMAX;
    static constexpr int stage_total = stage_bytes + RUN_ROWS * BROW_BYTES;
    static constexpr size_t smem =
        static_cast<size_t>(nstage) * stage_total + PART_F4 * 16 + RES_FLOATS * 4 + (3 * nstage + 2) * 8;
    static_assert(nstage + 1 <= DEC_MAP_SETS, "an item's tensor-map set is reused only after nstage + 1 items");
    static_assert(stage_total % 1024 == 0, "stage alignment");
};
constexpr int DEC_NSTAGE_MAX = 5;

struct KParams {
    // shape
    int M, H, I, topk, n_local, K, I_sh, K_sh, has_shared, S_cap, imax, split_a, hpad, ipad;
    int sh0, shn;   // the shared expert's tokens: sh0 .. sh0 + shn - 1
    int act_routed, act_shared;
    float limit;
    // inputs
    const void* x;
    int x_bf16;
    const float* rw;
    const int64_t* tables[9];
    int64_t sh[9];
    const int* runs;          // reference-layout run table
    const int* run_expert;
    const int* slot_act;
    const int* tok_expect;
    // scratch
    __half* xrot;             // [2][S_tot][hpad] rotated gate/up inputs, fragment layout
    __half* act;              // [S_tot][ipad] down inputs, fragment layout
    float* dpart;             // [S_tot][H]
    float* partA;             // [PARTA_ITEMS][2][8][128]
    float* xsum;              // [2][S_tot][H/128] sums of the fp16 rotated inputs per 128 chunk
    float* asum;              // [S_tot][imax/128] sums of the fp16 down inputs per 128 chunk
    int* ctr_work;
    int* ctr0;
    int* ctrA;
    int* ctrAk;
    int* ctrB;
    int* status;
    // outputs
    float* out_f32;
    __nv_bfloat16* out_bf16;
    CUtensorMap* tmaps;       // [grid][DEC_MAP_SETS][2] per-item tensor maps (workspace)
};

struct RunInfo {
    int nrows, expert, I, K;   // expert -1: shared
    bool shared;
};

struct Geo {
    int type;      // 0 rotate, 1 gate/up, 2 down, -1 none
    int run, chunk, ks;
    int nstages;
    int kb, ke;    // k-tile range (type 1: per projection)
    int nsp;       // stages per projection (type 1)
};

__device__ __forceinline__ int n_runs_routed(const KParams& p) { return p.runs[0]; }
__device__ __forceinline__ int n_runs_shared(const KParams& p) { return p.has_shared ? (p.shn + RUN_ROWS - 1) / RUN_ROWS : 0; }

__device__ __forceinline__ RunInfo run_info(const KParams& p, int r)
{
    RunInfo ri;
    const int nr = n_runs_routed(p);
    if (r < nr) {
        ri.shared = false;
        ri.nrows = p.runs[2 + r + 1] - p.runs[2 + r];
        ri.expert = p.run_expert[r];
        ri.I = p.I;
        ri.K = p.K;
    } else {
        ri.shared = true;
        const int j = r - nr;
        ri.nrows = min(RUN_ROWS, p.shn - j * RUN_ROWS);
        ri.expert = -1;
        ri.I = p.I_sh;
        ri.K = p.K_sh;
    }
    return ri;
}

// slot id of row t of run r (routed: table order; shared: S_cap + token)
__device__ __forceinline__ int run_slot(const KParams& p, int r, int t)
{
    const int nr = n_runs_routed(p);
    if (r < nr) return p.runs[2 + p.S_cap + 1 + p.runs[2 + r] + t];
    return p.S_cap + p.sh0 + (r - nr) * RUN_ROWS + t;
}

__device__ __forceinline__ int slot_token(const KParams& p, int s) { return s < p.S_cap ? s / p.topk : s - p.S_cap; }

__device__ __forceinline__ const void* tensor_ptr(const KParams& p, const RunInfo& ri, int row)
{
    return reinterpret_cast<const void*>(ri.shared ? p.sh[row] : p.tables[row][ri.expert]);
}

__device__ __forceinline__ Geo item_geo(const KParams& p, int item)
{
    Geo g;
    g.type = -1;
    const int nr = n_runs_routed(p), ns = n_runs_shared(p);
    const int R = nr + ns;
    if (item < R) {
        g.type = 0;
        g.run = item;
        g.chunk = g.ks = 0;
        g.nstages = 1;
        g.kb = g.ke = g.nsp = 0;
        return g;
    }
    item -= R;
    const int chA = p.I / 128, chAs = p.I_sh / 128;
    const int nA = (nr * chA + ns * chAs) * p.split_a;
    if (item < nA) {
        g.type = 1;
        g.ks = item % p.split_a;
        int j = item / p.split_a;
        if (j < nr * chA) {
            g.run = j / chA;
            g.chunk = j % chA;
        } else {
            j -= nr * chA;
            g.run = nr + j / chAs;
            g.chunk = j % chAs;
        }
        const int nkt = p.H / 16;
        g.kb = nkt * g.ks / p.split_a;
        g.ke = nkt * (g.ks + 1) / p.split_a;
        g.nsp = (g.ke - g.kb + STAGE_KT - 1) / STAGE_KT;
        g.nstages = 2 * g.nsp;
        return g;
    }
    item -= nA;
    const int chH = p.H / 128;
    if (item < R * chH) {
        g.type = 2;
        g.run = item / chH;
        g.chunk = item % chH;
        g.ks = 0;
        const RunInfo ri = run_info(p, g.run);
        g.kb = 0;
        g.ke = ri.I / 16;
        g.nsp = (g.ke + STAGE_KT - 1) / STAGE_KT;
        g.nstages = g.nsp;
    }
    return g;
}

__device__ __forceinline__ int total_items(const KParams& p)
{
    const int nr = n_runs_routed(p), ns = n_runs_shared(p);
    return (nr + ns) + (nr * (p.I / 128) + ns * (p.I_sh / 128)) * p.split_a + (nr + ns) * (p.H / 128);
}

// ---------------------------------------------------------------------------------------------
// Fragment layout of a GEMV input row: every 64 elements (4 k-tile rows) form one 128-byte block in
// which lane q of a token's lane group finds the B fragments of the 4 rows contiguously:
// half offset (q * 4 + r) * 4 + w * 2 + sub holds element k = 16 (4 b + r) + 8 w + 2 q + sub.
__device__ __forceinline__ int frag_offset(int k)
{
    const int b = k >> 6, r = (k >> 4) & 3, k16 = k & 15;
    const int q = (k16 & 7) >> 1, w = k16 >> 3, sub = k16 & 1;
    return b * 64 + (q * 4 + r) * 4 + w * 2 + sub;
}

// Store 4 consecutive elements k0..k0+3 (k0 % 4 == 0) as fp16 in fragment layout: two 4-byte stores.
__device__ __forceinline__ void store4_frag(__half* row, int k0, const float (&v)[4])
{
    const __half2 a = __floats2half2_rn(v[0], v[1]);
    const __half2 b = __floats2half2_rn(v[2], v[3]);
    *reinterpret_cast<__half2*>(row + frag_offset(k0)) = a;
    *reinterpret_cast<__half2*>(row + frag_offset(k0 + 2)) = b;
}

// ---------------------------------------------------------------------------------------------
// Decoding warps. A stage holds 32 k-tile rows x 8 tiles (128 output columns). Warp w takes k-tile
// rows 4 (w / 2) .. 4 (w / 2) + 3 of the stage and tiles 4 (w % 2) .. 4 (w % 2) + 3, i.e. 16 tiles
// and 16 fp32 accumulator registers; the eight warps of one column half split k. At the end of a
// projection each warp stores its partial sums to shared memory and goes on with the next stage;
// the epilogue warps sum the eight k-quads and run the item's epilogue meanwhile.

constexpr int WT = 4;   // tiles per warp per k-tile row
constexpr int WR = 4;   // k-tile rows per warp per stage

// B fragments of the 4 k-tile rows 4 g .. 4 g + 3 of a stage for lane `lane`: one 32-byte contiguous
// shared-memory read from the stage's copy of the lane's token row (fragment layout).
__device__ __forceinline__ void load_b4_smem(const uint8_t* brow, int g, int lane, uint32_t (&b)[2 * WR])
{
    const uint32_t a = smem_u32(brow + g * 128 + (lane & 3) * 32);
    const uint4 u0 = lds128(a), u1 = lds128(a + 16);
    b[0] = u0.x; b[1] = u0.y; b[2] = u0.z; b[3] = u0.w;
    b[4] = u1.x; b[5] = u1.y; b[6] = u1.z; b[7] = u1.w;
}


// One k-tile row of a warp's stage: its WT tiles' words (explicit shared-memory loads, all issued
// before the first decode), then decode + MMA per tile. tiles: shared-memory address of the row's
// first tile.
template <int K>
__device__ __forceinline__ void gemv_row_w(uint32_t tiles, const LaneW& d, uint32_t b0, uint32_t b1,
                                           float (&acc)[WT][4])
{
    uint32_t w[WT][2];
#pragma unroll
    for (int t = 0; t < WT; ++t) {
        w[t][0] = lds32(tiles + (t * 8 * K + d.w0) * 4);
        w[t][1] = lds32(tiles + (t * 8 * K + d.w1) * 4);
    }
#pragma unroll
    for (int t = 0; t < WT; ++t) {
        uint32_t a[4];
        // 4 of the 8 windows extracted and, below K = 4, the pairs packed on the FMA pipe: the ALU pipe
        // is the busier one in this kernel (measured best: 2 or 6 windows, or byte-permute packs, are slower)
        decode_afrag_ww<K, 4, (K == 4)>(w[t][0], w[t][1], d, a);
        mma_16816(acc[t], a, b0, b1);
    }
}

// One GEMV stage of a decoding warp: k-tile rows 4 quad .. 4 quad + 3 of the stage (those below ke)
// x tiles 4 whalf .. 4 whalf + 3, B fragments of those rows in b.
template <int K>
__device__ __forceinline__ void gemv_stage(const uint32_t* buf, const LaneW& d, int quad, int whalf, int r0, int ke,
                                           const uint32_t (&b)[2 * WR], float (&acc)[WT][4])
{
    const uint32_t rowp = smem_u32(buf + ((WR * quad) * NT + WT * whalf) * 8 * K);
    if (r0 + WR <= ke) {
#pragma unroll
        for (int r = 0; r < WR; ++r) gemv_row_w<K>(rowp + r * NT * 8 * K * 4, d, b[2 * r], b[2 * r + 1], acc);
    } else {
#pragma unroll
        for (int r = 0; r < WR; ++r)
            if (r0 + r < ke) gemv_row_w<K>(rowp + r * NT * 8 * K * 4, d, b[2 * r], b[2 * r + 1], acc);
    }
}

// Item state of one warp (each warp follows the item sequence on its own).
struct WarpItem {
    Geo g;
    RunInfo ri;
    int slot[RUN_ROWS];
};

// Ring stage header written by the producer: the item and its stage, and at the item's first stage
// its geometry, run and the run's slots (the producer has them already; the decoding warps read
// them from here instead of each repeating the chain of dependent global loads).
struct StageHdr {
    int item, s;
    WarpItem wi;
};

// What the decoding warps hand to the epilogue warps with each projection's partial sums.
struct PartInfo {
    int item, proj, last;   // item -1: no more work; last: the item's final projection
    WarpItem wi;
};

// Gate/up epilogue of row t (one warp): g, u = H128(res) * svh (+ the codebook's affine term when
// with_corr), a = act(g, u), a' = fp16(H128(a * suh_down)) stored in fragment layout with its
// per-chunk sum, then the run's gate/up completion counter.
__device__ __forceinline__ void epi_gateup_row(const KParams& p, const WarpItem& wi, const float* res, int t,
                                               bool with_corr, int lane)
{
    const Geo& g = wi.g;
    const RunInfo& ri = wi.ri;
    const size_t S_tot = static_cast<size_t>(p.S_cap) + p.M;
    const int nchH = p.H / 128;
    const int sl = wi.slot[t];
    const int col = g.chunk * 128 + lane * 4;
    float gv[4], uv[4], sv[4];
    float t0 = 0.0f, t1 = 0.0f;
    if (with_corr) {
        const float* xs0 = p.xsum + static_cast<size_t>(sl) * nchH;
        const float* xs1 = p.xsum + (S_tot + sl) * nchH;
        for (int c = g.kb / 8 + lane; c < g.ke / 8; c += 32) {
            t0 += __ldcg(xs0 + c);
            t1 += __ldcg(xs1 + c);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            t0 += __shfl_xor_sync(0xffffffffu, t0, o);
            t1 += __shfl_xor_sync(0xffffffffu, t1, o);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        gv[i] = res[t * 128 + lane * 4 + i] + CB_C1 * t0;
        uv[i] = res[RUN_ROWS * 128 + t * 128 + lane * 4 + i] + CB_C1 * t1;
    }
    had128_warp(gv, lane);
    had128_warp(uv, lane);
    load4_half_ro(static_cast<const __half*>(tensor_ptr(p, ri, 2)) + col, sv);
#pragma unroll
    for (int i = 0; i < 4; ++i) gv[i] *= sv[i];
    load4_half_ro(static_cast<const __half*>(tensor_ptr(p, ri, 5)) + col, sv);
#pragma unroll
    for (int i = 0; i < 4; ++i) uv[i] *= sv[i];
    const int mode = ri.shared ? p.act_shared : p.act_routed;
    float av[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) av[i] = act_gated(gv[i], uv[i], p.limit, mode);
    load4_half_ro(static_cast<const __half*>(tensor_ptr(p, ri, 7)) + col, sv);
#pragma unroll
    for (int i = 0; i < 4; ++i) av[i] *= sv[i];
    had128_warp(av, lane);
    store4_frag(p.act + static_cast<size_t>(sl) * p.ipad, col, av);
    float sm = 0.0f;   // sum of the values as stored (fp16)
#pragma unroll
    for (int i = 0; i < 4; ++i) sm += __half2float(__float2half_rn(av[i]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
    if (lane == 0) p.asum[static_cast<size_t>(sl) * (p.imax / 128) + g.chunk] = sm;
    __threadfence();
    __syncwarp();
    if (lane == 0) atomicAdd(&p.ctrA[g.run], 1);
}

// Down epilogue of row t (one warp): v = H128(res + affine term) * svh_down * routing weight into the
// slot's partial row; the last arrival of (token, chunk) sums the token's slots in slot order, then
// the shared expert, and stores the output row.
__device__ __forceinline__ void epi_down_row(const KParams& p, const WarpItem& wi, const float* res, int t, int lane)
{
    const Geo& g = wi.g;
    const RunInfo& ri = wi.ri;
    const int sl = wi.slot[t];
    const int tok = slot_token(p, sl);
    const int col = g.chunk * 128 + lane * 4;
    const float* as = p.asum + static_cast<size_t>(sl) * (p.imax / 128);
    float t0 = 0.0f;
    for (int c = lane; c < ri.I / 128; c += 32) t0 += __ldcg(as + c);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t0 += __shfl_xor_sync(0xffffffffu, t0, o);
    float v[4], sv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = res[t * 128 + lane * 4 + i] + CB_C1 * t0;
    had128_warp(v, lane);
    load4_half_ro(static_cast<const __half*>(tensor_ptr(p, ri, 8)) + col, sv);
    const float wgt = ri.shared ? 1.0f : p.rw[sl];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = v[i] * sv[i] * wgt;
    *reinterpret_cast<float4*>(p.dpart + static_cast<size_t>(sl) * p.H + col) = make_float4(v[0], v[1], v[2], v[3]);
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) {
        const int old = atomicAdd(&p.ctrB[tok * (p.H / 128) + g.chunk], 1);
        last = old == p.tok_expect[tok] - 1;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence();
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < p.topk; ++k) {
        const int s2 = tok * p.topk + k;
        if (!p.slot_act[s2]) continue;
        const float4 d = __ldcg(reinterpret_cast<const float4*>(p.dpart + static_cast<size_t>(s2) * p.H + col));
        o[0] += d.x;
        o[1] += d.y;
        o[2] += d.z;
        o[3] += d.w;
    }
    if (p.has_shared && tok >= p.sh0 && tok < p.sh0 + p.shn) {
        const float4 d =
            __ldcg(reinterpret_cast<const float4*>(p.dpart + (static_cast<size_t>(p.S_cap) + tok) * p.H + col));
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

// Template tensor maps of the trellis of one projection, viewed as [in/16 k-tile rows][out/16 x 32K
// bytes] in 8-byte elements with a box of 8 tiles (one 128-column chunk) x STAGE_KT rows: routed
// gate/up, routed down, shared gate/up, shared down. Their global address is replaced per item.
struct TrellisMaps {
    CUtensorMap gu, dn, sgu, sdn;
};

template <int KR, int KS, int NEW>
__global__ void __launch_bounds__(DecWarps<NEW>::threads, 1)
    experts_kernel(const KParams p, const __grid_constant__ TrellisMaps tm)
{
    constexpr int BPW = DecWarps<NEW>::bpw;
    using R = DecRing<(KR > KS ? KR : KS)>;
    constexpr int NSTAGE = R::nstage, STAGE_BYTES = R::stage_bytes, STAGE_TOTAL = R::stage_total;
    static_assert(NSTAGE <= DEC_NSTAGE_MAX, "stage headers");
    extern __shared__ __align__(1024) uint8_t smem[];
    uint32_t* ring = reinterpret_cast<uint32_t*>(smem);
    float4* part = reinterpret_cast<float4*>(smem + static_cast<size_t>(NSTAGE) * STAGE_TOTAL);   // [warp][t][lane]
    float* res = reinterpret_cast<float*>(part + PART_F4);                                         // [2][8][128]
    // full: the stage's trellis and B rows landed (arrivals of both producers, with their bytes)
    uint64_t* full = reinterpret_cast<uint64_t*>(res + RES_FLOATS);
    uint64_t* empty = full + NSTAGE;       // the decoders are done with the stage
    uint64_t* hready = empty + NSTAGE;     // the stage header is written (trellis producer -> B producer)
    uint64_t* pfull = hready + NSTAGE;     // decoders -> epilogue warps: one projection's partial sums written
    uint64_t* pfree = pfull + 1;           // epilogue warps -> decoders: partial sums consumed
    __shared__ StageHdr hdr[DEC_NSTAGE_MAX];
    __shared__ PartInfo pinfo;
    __shared__ PartInfo epi;               // the epilogue warps' copy of the item they finish
    __shared__ WarpItem wi0;               // decoder warp 0's copy of its current item
    __shared__ int sh_flag;
    __shared__ __align__(128) CUtensorMap tm_edit[2];   // the producer's staging copies of an item's maps

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < NSTAGE; ++i) {
            mbar_init(&full[i], 2);
            mbar_init(&empty[i], NCW);
            mbar_init(&hready[i], 1);
        }
        mbar_init(pfull, NCW);
        mbar_init(pfree, NEW);
        fence_barrier_init();
    }
    __syncthreads();

    const int total = total_items(p);

    if (warp == NCW) {
        // ------------------------------------------------------------------ producer
        // One 2-D tensor copy per stage (32 strided trellis rows of the item's 128-column chunk): many
        // small bulk copies per stage throttle the copy engine. Per item the projection's tensor
        // map(s) are written into this CTA's slot set (item_seq % DEC_MAP_SETS); a set is rewritten
        // only after NSTAGE + 1 later items, by which time every copy that read it has landed (each
        // item has at least one stage and a stage slot is refilled only after its decoders released it).
        uint32_t q = 0, item_seq = 0;
        for (;; ++item_seq) {
            int item = 0;
            if (lane == 0) item = atomicAdd(p.ctr_work, 1);
            item = __shfl_sync(0xffffffffu, item, 0);
            if (item >= total) item = -1;
            Geo g;
            RunInfo ri;
            if (item >= 0) {
                g = item_geo(p, item);
                ri = run_info(p, g.run);
            } else {
                g.nstages = 1;
                g.type = -1;
            }
            const CUtensorMap* maps = nullptr;
            if (g.type == 1 || g.type == 2) {
                CUtensorMap* gm = p.tmaps + (static_cast<size_t>(blockIdx.x) * DEC_MAP_SETS + item_seq % DEC_MAP_SETS) * 2;
                const CUtensorMap* tmpl = g.type == 1 ? (ri.shared ? &tm.sgu : &tm.gu) : (ri.shared ? &tm.sdn : &tm.dn);
                const int nmap = g.type == 1 ? 2 : 1;
                for (int j = 0; j < nmap; ++j)
                    reinterpret_cast<uint32_t*>(&tm_edit[j])[lane] = reinterpret_cast<const uint32_t*>(tmpl)[lane];
                __syncwarp();
                if (lane == 0)
                    for (int j = 0; j < nmap; ++j) tmap_replace_addr(&tm_edit[j], tensor_ptr(p, ri, (g.type == 1 ? j : 2) * 3));
                __syncwarp();
                for (int j = 0; j < nmap; ++j) tmap_copy_release(gm + j, &tm_edit[j]);
                if (lane == 0)
                    for (int j = 0; j < nmap; ++j) tmap_acquire(gm + j);
                __syncwarp();
                maps = gm;
            }
            for (int s = 0; s < g.nstages; ++s, ++q) {
                const int slot = q % NSTAGE;
                const uint32_t ph = (q / NSTAGE) & 1;
                mbar_wait_sleep(&empty[slot], ph ^ 1, p.status, 100);
                int kt0 = 0, proj = 0;
                uint32_t stage_bytes = 0;
                if (g.type == 1 || g.type == 2) {
                    proj = g.type == 2 ? 0 : s / g.nsp;                  // map index: 0 gate / down, 1 up
                    kt0 = g.kb + (s % g.nsp) * STAGE_KT;
                    stage_bytes = STAGE_KT * NT * 32 * ri.K;             // the full box (rows past the tensor read 0)
                }
                if (lane == 0) {
                    hdr[slot].item = item;
                    hdr[slot].s = s;
                    if (item >= 0 && s == 0) {
                        hdr[slot].wi.g = g;
                        hdr[slot].wi.ri = ri;
                    }
                }
                if (item >= 0 && s == 0 && lane < RUN_ROWS)
                    hdr[slot].wi.slot[lane] = lane < ri.nrows ? run_slot(p, g.run, lane) : run_slot(p, g.run, 0);
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&hready[slot]);
                    mbar_arrive_expect_tx(&full[slot], stage_bytes);
                    if (stage_bytes)
                        tma_load_2d(ring + slot * (STAGE_TOTAL / 4), maps + proj, g.chunk * NT * 4 * ri.K, kt0, &full[slot]);
                }
                __syncwarp();
            }
            if (item < 0) break;
        }
        return;
    }

    if (warp == BPW) {
        // ------------------------------------------------------------------ B producer
        // Follows the stage headers. At an item's start it waits (bounded) for the item's inputs,
        // which other items write (rotation, gate/up epilogues), so that the trellis producer never
        // blocks on them; then per stage it copies the run's 8 token rows of B for the stage's k-tile
        // rows into the stage (lane t: row t; rows past the run repeat row 0).
        int cur_item = -2, type = -1, bslot = 0, kb = 0, ke = 0, nsp = 1;
        for (uint32_t q = 0;; ++q) {
            const int slot = q % NSTAGE;
            const uint32_t ph = (q / NSTAGE) & 1;
            mbar_wait_sleep(&hready[slot], ph, p.status, 32);
            const int item = hdr[slot].item;
            const int s = hdr[slot].s;
            if (item < 0) {
                if (lane == 0) mbar_arrive(&full[slot]);   // the end marker's stage completes without B rows
                break;
            }
            if (item != cur_item) {
                cur_item = item;
                const WarpItem& hw = hdr[slot].wi;
                type = hw.g.type;
                kb = hw.g.kb;
                ke = hw.g.ke;
                nsp = hw.g.nsp;
                bslot = hw.slot[lane < RUN_ROWS ? lane : 0];
                if (type != 0 && lane == 0) {
                    if (type == 1) wait_geq(&p.ctr0[hw.g.run], 1, p.status);
                    else wait_geq(&p.ctrA[hw.g.run], (hw.ri.I / 128) * hw.ri.nrows, p.status);
                    // written by generic-proxy stores of other CTAs, read below by bulk copies (async proxy)
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                }
                __syncwarp();
            }
            if (type != 1 && type != 2) {
                if (lane == 0) mbar_arrive(&full[slot]);
                continue;
            }
            const int proj = type == 2 ? 0 : s / nsp;
            const int kt0 = kb + (s % nsp) * STAGE_KT;
            const int nvalid = min(STAGE_KT, ke - kt0);
            const __half* brow = type == 1 ? p.xrot + (static_cast<size_t>(proj) * (p.S_cap + p.M) + bslot) * p.hpad
                                           : p.act + static_cast<size_t>(bslot) * p.ipad;
            if (lane == 0) mbar_arrive_expect_tx(&full[slot], nvalid * RUN_ROWS * 32);
            __syncwarp();
            if (lane < RUN_ROWS)
                bulk_g2s(ring + slot * (STAGE_TOTAL / 4) + (STAGE_BYTES + lane * BROW_BYTES) / 4,
                         brow + static_cast<size_t>(kt0) * 16, nvalid * 32, &full[slot]);
        }
        return;
    }

    if (warp > NCW) {
        // ------------------------------------------------------------------ epilogue warps
        // Per projection end: sum the 8 k-quads' partials into res, release the partial buffer, and
        // after an item's last projection run its epilogue (split-k publication, row epilogues).
        const int ew = warp - NCW - 1, etid = tid - (NCW + 1) * 32;
        for (uint32_t pe = 0;; ++pe) {
            if (!mbar_wait_sleep(pfull, pe & 1, p.status, 500)) break;
            static_assert(sizeof(PartInfo) % 4 == 0 && sizeof(PartInfo) / 4 <= NEW * 32, "PartInfo copy");
            if (etid < static_cast<int>(sizeof(PartInfo) / 4))
                reinterpret_cast<int*>(&epi)[etid] = reinterpret_cast<const int*>(&pinfo)[etid];
            named_sync(2, NEW * 32);
            if (epi.item < 0) break;
            float* rs = res + epi.proj * RUN_ROWS * 128;
            for (int cmb = etid; cmb < 2 * WT * 32; cmb += NEW * 32) {
                const int wh = cmb >> 7, t = (cmb >> 5) & 3, l = cmb & 31;
                float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int qd = 0; qd < NCW / 2; ++qd) {
                    const float4 v = part[((2 * qd + wh) * WT + t) * 32 + l];
                    a.x += v.x;
                    a.y += v.y;
                    a.z += v.z;
                    a.w += v.w;
                }
                // D fragment of mma.m16n8k16: c0 (col g, tok 2t') c1 (g, 2t'+1) c2 (g+8, 2t') c3 (g+8, 2t'+1)
                const int col = (wh * WT + t) * 16 + (l >> 2), tok = 2 * (l & 3);
                rs[tok * 128 + col] = CB_C0 * a.x;
                rs[(tok + 1) * 128 + col] = CB_C0 * a.y;
                rs[tok * 128 + col + 8] = CB_C0 * a.z;
                rs[(tok + 1) * 128 + col + 8] = CB_C0 * a.w;
            }
            named_sync(2, NEW * 32);
            if (lane == 0) mbar_arrive(pfree);
            if (!epi.last) continue;
            const WarpItem& wi = epi.wi;
            const Geo& g = wi.g;
            const int nrows = wi.ri.nrows;
            if (g.type == 1) {
                bool with_corr = true;
                if (p.split_a > 1) {
                    // this split's sums (with the affine term of its k range) to global; the last split
                    // of (run, chunk) sums them and runs the row epilogues
                    const size_t S_tot = static_cast<size_t>(p.S_cap) + p.M;
                    const int nchH = p.H / 128;
                    for (int t = ew; t < nrows; t += NEW) {
                        const int sl = wi.slot[t];
                        float t0 = 0.0f, t1 = 0.0f;
                        for (int c = g.kb / 8 + lane; c < g.ke / 8; c += 32) {
                            t0 += __ldcg(p.xsum + static_cast<size_t>(sl) * nchH + c);
                            t1 += __ldcg(p.xsum + (S_tot + sl) * nchH + c);
                        }
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) {
                            t0 += __shfl_xor_sync(0xffffffffu, t0, o);
                            t1 += __shfl_xor_sync(0xffffffffu, t1, o);
                        }
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            res[t * 128 + lane * 4 + i] += CB_C1 * t0;
                            res[RUN_ROWS * 128 + t * 128 + lane * 4 + i] += CB_C1 * t1;
                        }
                    }
                    named_sync(2, NEW * 32);
                    const int pidx = (g.run * (p.imax / 128) + g.chunk) * p.split_a + g.ks;
                    float* dst = p.partA + static_cast<size_t>(pidx) * RES_FLOATS;
                    for (int i = etid; i < RES_FLOATS; i += NEW * 32) dst[i] = res[i];
                    __threadfence();
                    named_sync(2, NEW * 32);
                    if (etid == 0) {
                        const int old = atomicAdd(&p.ctrAk[g.run * (p.imax / 128) + g.chunk], 1);
                        sh_flag = old == p.split_a - 1;
                    }
                    named_sync(2, NEW * 32);
                    const int last = sh_flag;
                    named_sync(2, NEW * 32);
                    if (!last) continue;
                    __threadfence();
                    const float* base =
                        p.partA + static_cast<size_t>((g.run * (p.imax / 128) + g.chunk) * p.split_a) * RES_FLOATS;
                    for (int i = etid; i < RES_FLOATS; i += NEW * 32) {
                        float a = 0.0f;
                        for (int k = 0; k < p.split_a; ++k) a += __ldcg(base + static_cast<size_t>(k) * RES_FLOATS + i);
                        res[i] = a;
                    }
                    named_sync(2, NEW * 32);
                    with_corr = false;
                }
                for (int t = ew; t < nrows; t += NEW) epi_gateup_row(p, wi, res, t, with_corr, lane);
            } else {
                for (int t = ew; t < nrows; t += NEW) epi_down_row(p, wi, res, t, lane);
            }
            named_sync(2, NEW * 32);   // res is read by the row epilogues until here
        }
        return;
    }

    // ---------------------------------------------------------------------- decoders
    float acc[WT][4];
#pragma unroll
    for (int t = 0; t < WT; ++t)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[t][c] = 0.0f;

    const LaneW dR = lane_w<KR>(lane);
    const LaneW dS = lane_w<KS>(lane);
    const int quad = warp >> 1, whalf = warp & 1;
    const size_t S_tot = static_cast<size_t>(p.S_cap) + p.M;
    const int nchH = p.H / 128;
    uint32_t q = 0, pq = 0;
    uint32_t bc[2 * WR];               // B fragments of this warp's WR rows of the stage
    int cur_item = -2;
    // the current item, in registers
    int type = -1, run = 0, nsp = 1, kb = 0, ke = 0, nstages = 1;
    bool shared_run = false;
    int sp = 0, proj = 0;              // stage within the projection, projection (0 gate / 1 up)
    for (;; ++q) {
        const int slot = q % NSTAGE;
        const uint32_t ph = (q / NSTAGE) & 1;
        mbar_wait(&full[slot], ph, p.status);
        const int item = hdr[slot].item;
        const int s = hdr[slot].s;
        if (item < 0) break;
        const WarpItem& hw = hdr[slot].wi;
        if (item != cur_item) {
            // item start: geometry into registers, the B row, the dependency
            cur_item = item;
            type = hw.g.type;
            run = hw.g.run;
            nsp = hw.g.nsp;
            kb = hw.g.kb;
            ke = hw.g.ke;
            nstages = hw.g.nstages;
            shared_run = hw.ri.shared;
            sp = 0;
            proj = 0;
            if (warp == 0) {
                if (lane < RUN_ROWS) wi0.slot[lane] = hw.slot[lane];
                if (lane == 0) {
                    wi0.g = hw.g;
                    wi0.ri = hw.ri;
                }
            }
        }

        if (type == 0) {
            // rotation of the run's rows for gate (suh row 1) and up (suh row 4); decoders only
            const RunInfo ri = hw.ri;
            const int nch = p.H / 128;
            const int units = ri.nrows * 2 * nch;
            for (int u = warp; u < units; u += NCW) {
                const int t = u / (2 * nch), rem = u % (2 * nch), pj = rem / nch, c = rem % nch;
                const int sl = hw.slot[t];
                const int tok = slot_token(p, sl);
                const int col = c * 128 + lane * 4;
                float v[4], su[4];
                load4_x(p.x, static_cast<size_t>(tok) * p.H + col, p.x_bf16, v);
                load4_half_ro(static_cast<const __half*>(tensor_ptr(p, ri, pj == 0 ? 1 : 4)) + col, su);
#pragma unroll
                for (int i = 0; i < 4; ++i) v[i] *= su[i];
                had128_warp(v, lane);
                store4_frag(p.xrot + (static_cast<size_t>(pj) * S_tot + sl) * p.hpad, col, v);
                float sm = 0.0f;   // sum of the values as stored (fp16)
#pragma unroll
                for (int i = 0; i < 4; ++i) sm += __half2float(__float2half_rn(v[i]));
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
                if (lane == 0) p.xsum[(static_cast<size_t>(pj) * S_tot + sl) * nchH + c] = sm;
            }
            __threadfence();
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            named_sync(1, NCW * 32);
            if (tid == 0) atomicAdd(&p.ctr0[run], 1);
            continue;
        }

        // GEMV stage: rows 4 quad .. 4 quad + 3 of the stage; B from the stage's copy of the run's rows
        const int kt0 = kb + sp * STAGE_KT;
        const int r0 = kt0 + WR * quad;
        const uint8_t* stage_base = reinterpret_cast<const uint8_t*>(ring + slot * (STAGE_TOTAL / 4));
        load_b4_smem(stage_base + STAGE_BYTES + (lane >> 2) * BROW_BYTES, quad, lane, bc);
        const int sp1 = sp + 1 == nsp ? 0 : sp + 1;
        const int proj1 = sp + 1 == nsp ? proj + 1 : proj;
        {
            const uint32_t* buf = reinterpret_cast<const uint32_t*>(stage_base);
            if (!shared_run || KR == KS) gemv_stage<KR>(buf, dR, quad, whalf, r0, ke, bc, acc);
            else gemv_stage<KS>(buf, dS, quad, whalf, r0, ke, bc, acc);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);

        const bool proj_end = sp + 1 == nsp;
        const int cproj = proj;
        sp = sp1;
        proj = proj1;
        if (!proj_end) continue;
        // hand this projection's partial sums to the epilogue warps
        mbar_wait(pfree, (pq & 1) ^ 1, p.status);
#pragma unroll
        for (int t = 0; t < WT; ++t) {
            part[(warp * WT + t) * 32 + lane] = make_float4(acc[t][0], acc[t][1], acc[t][2], acc[t][3]);
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[t][c] = 0.0f;
        }
        if (warp == 0) {
            if (lane < static_cast<int>(sizeof(WarpItem) / 4))
                reinterpret_cast<int*>(&pinfo.wi)[lane] = reinterpret_cast<const int*>(&wi0)[lane];
            if (lane == 0) {
                pinfo.item = cur_item;
                pinfo.proj = cproj;
                pinfo.last = s == nstages - 1;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(pfull);
        ++pq;
    }
    // no more items: tell the epilogue warps
    mbar_wait(pfree, (pq & 1) ^ 1, p.status);
    if (warp == 0 && lane == 0) pinfo.item = -1;
    __syncwarp();
    if (lane == 0) mbar_arrive(pfull);
}

using ExpertsKernel = void (*)(KParams, TrellisMaps);

// Template map of a projection's trellis [in/16][out/16][16K] int16 as [in/16][out/16 x 4K] 8-byte
// elements, box 8 tiles x STAGE_KT rows; base: any 16-byte aligned device address (replaced per item).
static bool encode_trellis_map(CUtensorMap* m, void* base, int in, int out, int K)
{
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(out / 16) * 4 * K, static_cast<cuuint64_t>(in / 16)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(out / 16) * 32 * K};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(NT * 4 * K), STAGE_KT};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

template <int NEW>
static ExpertsKernel pick_kernel(int kr, int ks)
{
#define EVA_K(a, b) \
    if (kr == a && ks == b) return experts_kernel<a, b, NEW>;
    EVA_K(2, 2) EVA_K(2, 3) EVA_K(2, 4) EVA_K(3, 2) EVA_K(3, 3) EVA_K(3, 4) EVA_K(4, 2) EVA_K(4, 3) EVA_K(4, 4)
#undef EVA_K
    return nullptr;
}

cudaError_t launch_experts(const ExpertsArgs& a, cudaStream_t stream)
{
    const EvaMoeShape& s = *a.shape;
    const WsLayout& L = a.L;
    const CtrLayout C = ctr_layout(L);
    uint8_t* ws = static_cast<uint8_t*>(a.ws);
    int32_t* ctr = reinterpret_cast<int32_t*>(ws + L.counters);
    KParams p{};
    p.M = a.M;
    p.H = s.hidden;
    p.I = s.inter;
    p.topk = s.topk;
    p.n_local = s.n_experts;
    p.K = s.bits;
    p.I_sh = s.shared_inter;
    p.K_sh = s.shared_inter ? s.shared_bits : s.bits;
    p.has_shared = s.shared_inter > 0;
    p.sh0 = a.sh0;
    p.shn = p.has_shared ? a.shn : 0;
    p.S_cap = a.M * s.topk;
    p.imax = L.imax;
    p.hpad = L.hpad;
    p.ipad = L.ipad;
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
    p.run_expert = reinterpret_cast<const int*>(ws + L.run_expert);
    p.slot_act = reinterpret_cast<const int*>(ws + L.slot_act);
    p.tok_expect = reinterpret_cast<const int*>(ws + L.tok_expect);
    p.xrot = reinterpret_cast<__half*>(ws + L.xrot);
    p.act = reinterpret_cast<__half*>(ws + L.act);
    p.dpart = reinterpret_cast<float*>(ws + L.dpart);
    p.partA = reinterpret_cast<float*>(ws + L.partA);
    p.xsum = reinterpret_cast<float*>(ws + L.xsum);
    p.asum = reinterpret_cast<float*>(ws + L.asum);
    p.ctr_work = ctr + C.work;
    p.ctr0 = ctr + C.ctr0;
    p.ctrA = ctr + C.ctrA;
    p.ctrAk = ctr + C.ctrAk;
    p.ctrB = ctr + C.ctrB;
    p.status = reinterpret_cast<int*>(ws + L.status);
    p.out_f32 = a.out_f32;
    p.out_bf16 = static_cast<__nv_bfloat16*>(a.out_bf16);
    p.tmaps = reinterpret_cast<CUtensorMap*>(ws + L.tmaps);

    // split the gate/up k range when there are too few gate/up items to fill the GPU
    const int sms = num_sms();
    const int r_max = a.M * s.topk + (p.has_shared ? (p.shn + RUN_ROWS - 1) / RUN_ROWS : 0);
    const int items_a = r_max * (L.imax / 128);
    int split = 1;
    // a split boundary must fall on a 128 chunk of the input (per-chunk input sums)
    while (split < L.max_split && items_a * split * 2 <= 2 * sms && items_a * split * 2 <= PARTA_ITEMS &&
           (s.hidden / 128) % (split * 2) == 0)
        split *= 2;
    p.split_a = split;

    TrellisMaps tm;
    const int ish = p.I_sh ? p.I_sh : p.I;
    if (!encode_trellis_map(&tm.gu, ws, p.H, p.I, p.K) || !encode_trellis_map(&tm.dn, ws, p.I, p.H, p.K) ||
        !encode_trellis_map(&tm.sgu, ws, p.H, ish, p.K_sh) || !encode_trellis_map(&tm.sdn, ws, ish, p.H, p.K_sh))
        return cudaErrorInvalidValue;
    const bool short_items = s.hidden / split <= DEC_SHORT_ITEM_COLS;
    const ExpertsKernel kern = short_items ? pick_kernel<4>(p.K, p.K_sh) : pick_kernel<2>(p.K, p.K_sh);
    const int threads = short_items ? DecWarps<4>::threads : DecWarps<2>::threads;
    if (!kern) return cudaErrorInvalidValue;
    const int kmax = std::max(p.K, p.K_sh);
    const size_t smem = kmax <= 2 ? DecRing<2>::smem : (kmax == 3 ? DecRing<3>::smem : DecRing<4>::smem);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    kern<<<std::min(sms, DEC_MAX_CTAS), threads, smem, stream>>>(p, tm);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// Standalone dequantisation (one warp per 16x16 tile), same decode path as the fused kernel.

template <int K>
__global__ void __launch_bounds__(256) dequant_kernel(const uint32_t* __restrict__ tr, int in, int out, __half* __restrict__ w)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntn = out / 16;
    const long long tile = static_cast<long long>(blockIdx.x) * 8 + warp;
    if (tile >= static_cast<long long>(in / 16) * ntn) return;
    const int kt = static_cast<int>(tile / ntn), nt = static_cast<int>(tile % ntn);
    uint32_t a[4];
    decode_afrag<K>(tr + tile * 8 * K, lane, a);
    const int n0 = lane >> 2, k0 = 2 * (lane & 3);
    // reg0: (n0, k0..k0+1), reg1: (n0+8, k0..), reg2: (n0, k0+8..), reg3: (n0+8, k0+8..)
    const int nn[4] = {n0, n0 + 8, n0, n0 + 8};
    const int kk[4] = {k0, k0, k0 + 8, k0 + 8};
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const __half2 h = *reinterpret_cast<const __half2*>(&a[r]);
        w[static_cast<size_t>(kt * 16 + kk[r]) * out + nt * 16 + nn[r]] = __low2half(h);
        w[static_cast<size_t>(kt * 16 + kk[r] + 1) * out + nt * 16 + nn[r]] = __high2half(h);
    }
}

cudaError_t launch_dequant(const void* trellis, int in, int out, int K, uint16_t* w, cudaStream_t stream)
{
    const long long tiles = static_cast<long long>(in / 16) * (out / 16);
    const unsigned grid = static_cast<unsigned>((tiles + 7) / 8);
    const uint32_t* tr = static_cast<const uint32_t*>(trellis);
    __half* wo = reinterpret_cast<__half*>(w);
    switch (K) {
        case 2: dequant_kernel<2><<<grid, 256, 0, stream>>>(tr, in, out, wo); break;
        case 3: dequant_kernel<3><<<grid, 256, 0, stream>>>(tr, in, out, wo); break;
        case 4: dequant_kernel<4><<<grid, 256, 0, stream>>>(tr, in, out, wo); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace eva
