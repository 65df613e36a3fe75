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
// which were claimed earlier by running CTAs, so the schedule cannot deadlock.
//
// Per CTA: 1 producer warp streams the item's trellis rows with 1-D bulk copies (TMA, one
// CTA per copy) into a 4-stage shared-memory ring (32 k-tile rows x 128 columns per stage); 16
// consumer warps each decode 4 rows x 4 tiles per stage in registers and run mma.m16n8k16 with
// the weights as the 16 x 16 A operand (rows = output columns) and up to 8 tokens as the B
// operand, accumulating in fp32. The MMA takes the raw codebook values h = 1024 + bytesum and the
// affine map of the codebook is applied to the sums (see decode_raw). Each warp follows the item
// sequence on its own; the only CTA-wide barriers are the cross-warp k reduction at the end of a
// projection, the rotation items and the split-k hand-off. The epilogue of a run row is done by
// one warp while the others go on to the next item.
//
// Reference behaviour (paths within Findddx/eva, runtime/ds41/csrc/moe_coop2048/vendor/quant/):
//   exl3_moe_coop_kernel.cuh:634-671 (rotation), :680-809 (gate/up GEMV + epilogue),
//   :816-963 (down GEMV + combine + shared merge); exl3_dq.cuh / codebook.cuh (decode).
#include <cuda_runtime.h>

#include "common.cuh"
#include "internal.h"

namespace eva {

constexpr int NCW = 16;                    // consumer warps
constexpr int THREADS = (NCW + 1) * 32;    // + producer warp
constexpr int NSTAGE = 4;
constexpr int STAGE_KT = 32;               // k-tile rows per stage (4 per consumer warp pair)
constexpr int NT = 8;                      // 16-column tiles per item (128 output columns)
constexpr int STAGE_BYTES = STAGE_KT * NT * 32 * 4;   // sized for K = 4
constexpr int RED_FLOATS = NCW * 4 * 4 * 32;  // [warp][tile][c][lane]
constexpr int RES_FLOATS = 2 * RUN_ROWS * 128;
constexpr size_t SMEM_BYTES = static_cast<size_t>(NSTAGE) * STAGE_BYTES + RED_FLOATS * 4 + RES_FLOATS * 4 + 1024;

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
// Consumers. A stage holds 32 k-tile rows x 8 tiles (128 output columns). Warp w takes k-tile rows
// 4 (w / 2) .. 4 (w / 2) + 3 of the stage and tiles 4 (w % 2) .. 4 (w % 2) + 3, i.e. 16 tiles and
// 16 fp32 accumulator registers; the eight warps of one column half split k and are summed at the
// end of a projection.

constexpr int WT = 4;   // tiles per warp per k-tile row
constexpr int WR = 4;   // k-tile rows per warp per stage

// B fragments of the 4 k-tile rows 4 g .. 4 g + 3 for lane `lane`: one 32-byte contiguous read
// (row = fragment-layout input row of the lane's token).
__device__ __forceinline__ void load_b4(const __half* row, int g, int lane, uint32_t (&b)[2 * WR])
{
    const uint4* p = reinterpret_cast<const uint4*>(row + g * 64 + (lane & 3) * 16);
    const uint4 u0 = __ldcg(p), u1 = __ldcg(p + 1);
    b[0] = u0.x; b[1] = u0.y; b[2] = u0.z; b[3] = u0.w;
    b[4] = u1.x; b[5] = u1.y; b[6] = u1.z; b[7] = u1.w;
}

template <int K>
__device__ __forceinline__ void gemv_row(const uint32_t* tiles, const LaneGrp& d, uint32_t b0, uint32_t b1,
                                         float (&acc)[WT][4])
{
#pragma unroll
    for (int t = 0; t < WT; ++t) {
        uint32_t a[4];
        decode_raw<K>(tiles + t * 8 * K, d, a);
        mma_16816(acc[t], a, b0, b1);
    }
}

// Sum of the 8 k-split accumulators of each column half into res[tok][col] (natural layout).
__device__ __forceinline__ void reduce_acc(float (&acc)[WT][4], float* red, float* res, int tid, int warp, int lane)
{
#pragma unroll
    for (int t = 0; t < WT; ++t)
#pragma unroll
        for (int c = 0; c < 4; ++c) red[((warp * WT + t) * 4 + c) * 32 + lane] = acc[t][c];
    named_sync(1, NCW * 32);
    for (int v = tid; v < 2 * WT * 4 * 32; v += NCW * 32) {
        const int half = v >> 9, r = v & 511;        // r = (t * 4 + c) * 32 + lane
        float sum = 0.0f;
#pragma unroll
        for (int pr = 0; pr < NCW / 2; ++pr) sum += red[(2 * pr + half) * WT * 4 * 32 + r];
        const int l = r & 31, c = (r >> 5) & 3, t = r >> 7;
        const int col = (half * WT + t) * 16 + (l >> 2) + 8 * (c >> 1);
        const int tok = 2 * (l & 3) + (c & 1);
        res[tok * 128 + col] = CB_C0 * sum;
    }
    named_sync(1, NCW * 32);
#pragma unroll
    for (int t = 0; t < WT; ++t)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[t][c] = 0.0f;
}

// Item state of one consumer warp (each warp follows the item sequence on its own).
struct WarpItem {
    Geo g;
    RunInfo ri;
    int slot[RUN_ROWS];
};

// Ring stage header written by the producer: the item and its stage, and at the item's first stage
// its geometry, run and the run's slots (the producer has them already; the 16 consumer warps copy
// them instead of each repeating the chain of dependent global loads).
struct StageHdr {
    int item, s;
    WarpItem wi;
};

// Epilogue operands prefetched at item start by the warp that runs the epilogue of row `warp`:
// type 1: svh_gate, svh_up, suh_down of the chunk; type 2: svh_down (fp16 x 4 per lane).
struct EpiOps {
    uint2 v[3][32];
};

template <int KR, int KS>
__global__ void __launch_bounds__(THREADS, 1) experts_kernel(const KParams p)
{
    extern __shared__ __align__(1024) uint8_t smem[];
    uint32_t* ring = reinterpret_cast<uint32_t*>(smem);
    float* red = reinterpret_cast<float*>(smem + static_cast<size_t>(NSTAGE) * STAGE_BYTES);
    float* res = red + RED_FLOATS;   // [2][8][128]
    uint64_t* full = reinterpret_cast<uint64_t*>(res + RES_FLOATS);
    uint64_t* empty = full + NSTAGE;
    __shared__ StageHdr hdr[NSTAGE];
    __shared__ WarpItem wis[NCW];
    __shared__ EpiOps eps[RUN_ROWS];
    __shared__ int sh_flag;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < NSTAGE; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], NCW);
        }
        fence_barrier_init();
    }
    __syncthreads();

    const int total = total_items(p);

    if (warp == NCW) {
        // ------------------------------------------------------------------ producer
        uint32_t q = 0;
        for (;;) {
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
            for (int s = 0; s < g.nstages; ++s, ++q) {
                const int slot = q % NSTAGE;
                const uint32_t ph = (q / NSTAGE) & 1;
                mbar_wait(&empty[slot], ph ^ 1, p.status);
                int nvalid = 0;
                const uint8_t* src = nullptr;
                size_t row_stride = 0;
                uint32_t row_bytes = 0;
                if (g.type == 1 || g.type == 2) {
                    const int proj = g.type == 2 ? 2 : s / g.nsp;      // 0 gate, 1 up, 2 down
                    const int kt0 = g.kb + (s % g.nsp) * STAGE_KT;
                    nvalid = min(STAGE_KT, g.ke - kt0);
                    const int out = g.type == 2 ? p.H : ri.I;
                    row_bytes = NT * 32 * ri.K;                          // 8 tiles of 32K bytes
                    row_stride = static_cast<size_t>(out / 16) * 32 * ri.K;
                    src = static_cast<const uint8_t*>(tensor_ptr(p, ri, proj * 3)) + static_cast<size_t>(kt0) * row_stride +
                          static_cast<size_t>(g.chunk) * row_bytes;
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
                if (lane == 0) mbar_arrive_expect_tx(&full[slot], nvalid * row_bytes);
                __syncwarp();
                if (lane < nvalid)
                    bulk_g2s(ring + slot * (STAGE_BYTES / 4) + lane * (row_bytes / 4), src + lane * row_stride, row_bytes,
                             &full[slot]);
            }
            if (item < 0) break;
        }
        return;
    }

    // ---------------------------------------------------------------------- consumers
    float acc[WT][4];
#pragma unroll
    for (int t = 0; t < WT; ++t)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[t][c] = 0.0f;

    const LaneGrp dR = lane_grp<KR>(lane);
    const LaneGrp dS = lane_grp<KS>(lane);
    const int quad = warp >> 1, whalf = warp & 1;
    const size_t S_tot = static_cast<size_t>(p.S_cap) + p.M;
    const int nchH = p.H / 128;
    WarpItem& wi = wis[warp];
    uint32_t q = 0;
    uint32_t bc[2 * WR], bn[2 * WR];   // B of this warp's WR rows: current stage / next stage
#pragma unroll
    for (int i = 0; i < 2 * WR; ++i) bc[i] = bn[i] = 0;
    float tsp[2] = {0.0f, 0.0f};       // epilogue warps: per-lane partial input sums (gate/up or down)
    int cur_item = -2;
    int sp = 0, proj = 0;              // stage within the projection, projection (0 gate / 1 up)
    const __half* brow = nullptr;      // this lane's token row of the B input (projection 0)
    size_t bproj = 0;                  // element offset from the gate to the up input
    for (;; ++q) {
        const int slot = q % NSTAGE;
        const uint32_t ph = (q / NSTAGE) & 1;
        mbar_wait(&full[slot], ph, p.status);
        const int item = hdr[slot].item;
        const int s = hdr[slot].s;
        if (item < 0) break;
        if (item != cur_item) {
            // item start, per warp: geometry, the run's slots, the dependency, epilogue prefetch
            cur_item = item;
            if (lane == 0) {
                wi.g = hdr[slot].wi.g;
                wi.ri = hdr[slot].wi.ri;
            }
            if (lane < RUN_ROWS) wi.slot[lane] = hdr[slot].wi.slot[lane];
            __syncwarp();
            const Geo g = wi.g;
            const RunInfo ri = wi.ri;
            sp = 0;
            proj = 0;
            __syncwarp();
            {
                const int bs = wi.slot[lane >> 2];   // this lane's token row (rows past the run repeat row 0)
                if (g.type == 1) {
                    brow = p.xrot + static_cast<size_t>(bs) * p.hpad;
                    bproj = S_tot * p.hpad;
                } else {
                    brow = p.act + static_cast<size_t>(bs) * p.ipad;
                    bproj = 0;
                }
            }
            if (lane == 0) {
                if (g.type == 1) wait_geq(&p.ctr0[g.run], 1, p.status);
                if (g.type == 2) wait_geq(&p.ctrA[g.run], (ri.I / 128) * ri.nrows, p.status);
            }
            __syncwarp();
            if (g.type != 0 && warp < ri.nrows) {
                const int sl = wi.slot[warp];
                const int col = g.chunk * 128 + lane * 4;
                if (g.type == 1) {
                    cp_async8(&eps[warp].v[0][lane], static_cast<const __half*>(tensor_ptr(p, ri, 2)) + col);
                    cp_async8(&eps[warp].v[1][lane], static_cast<const __half*>(tensor_ptr(p, ri, 5)) + col);
                    cp_async8(&eps[warp].v[2][lane], static_cast<const __half*>(tensor_ptr(p, ri, 7)) + col);
                    const float* xs0 = p.xsum + static_cast<size_t>(sl) * nchH;
                    const float* xs1 = p.xsum + (S_tot + sl) * nchH;
                    tsp[0] = tsp[1] = 0.0f;
                    for (int c = g.kb / 8 + lane; c < g.ke / 8; c += 32) {
                        tsp[0] += __ldcg(xs0 + c);
                        tsp[1] += __ldcg(xs1 + c);
                    }
                } else {
                    cp_async8(&eps[warp].v[0][lane], static_cast<const __half*>(tensor_ptr(p, ri, 8)) + col);
                    const float* as = p.asum + static_cast<size_t>(sl) * (p.imax / 128);
                    tsp[0] = 0.0f;
                    for (int c = lane; c < ri.I / 128; c += 32) tsp[0] += __ldcg(as + c);
                }
                cp_async_commit();
            }
        }
        const int type = wi.g.type;

        if (type == 0) {
            // rotation of the run's rows for gate (suh row 1) and up (suh row 4); CTA-wide
            const RunInfo ri = wi.ri;
            const int nch = p.H / 128;
            const int units = ri.nrows * 2 * nch;
            for (int u = warp; u < units; u += NCW) {
                const int t = u / (2 * nch), rem = u % (2 * nch), pj = rem / nch, c = rem % nch;
                const int sl = wi.slot[t];
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
            if (lane == 0) mbar_arrive(&empty[slot]);
            named_sync(1, NCW * 32);
            if (tid == 0) atomicAdd(&p.ctr0[wi.g.run], 1);
            continue;
        }

        // GEMV stage: rows 4 quad .. 4 quad + 3 of the stage, B fragments prefetched one stage ahead
        const int nsp = wi.g.nsp, kb = wi.g.kb, ke = wi.g.ke, nstages = wi.g.nstages;
        const bool shared_run = wi.ri.shared;
        const int kt0 = kb + sp * STAGE_KT;
        const int r0 = kt0 + WR * quad;
        if (s == 0) {
            load_b4(brow, (kt0 >> 2) + quad, lane, bc);
        } else {
#pragma unroll
            for (int i = 0; i < 2 * WR; ++i) bc[i] = bn[i];
        }
        const int sp1 = sp + 1 == nsp ? 0 : sp + 1;
        const int proj1 = sp + 1 == nsp ? proj + 1 : proj;
        if (s + 1 < nstages) load_b4(brow + proj1 * bproj, ((kb + sp1 * STAGE_KT) >> 2) + quad, lane, bn);
        {
            const uint32_t* buf = ring + slot * (STAGE_BYTES / 4);
            if (!shared_run || KR == KS) {
                const uint32_t* rowp = buf + ((WR * quad) * NT + WT * whalf) * 8 * KR;
#pragma unroll
                for (int r = 0; r < WR; ++r)
                    if (r0 + r < ke) gemv_row<KR>(rowp + r * NT * 8 * KR, dR, bc[2 * r], bc[2 * r + 1], acc);
            } else {
                const uint32_t* rowp = buf + ((WR * quad) * NT + WT * whalf) * 8 * KS;
#pragma unroll
                for (int r = 0; r < WR; ++r)
                    if (r0 + r < ke) gemv_row<KS>(rowp + r * NT * 8 * KS, dS, bc[2 * r], bc[2 * r + 1], acc);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);

        const bool proj_end = sp + 1 == nsp;
        const int cproj = proj;
        sp = sp1;
        proj = proj1;
        if (!proj_end) continue;
        reduce_acc(acc, red, res + cproj * RUN_ROWS * 128, tid, warp, lane);
        if (s != nstages - 1) continue;

        // ------------------------------------------------------------- item epilogues
        const Geo g = wi.g;
        const RunInfo ri = wi.ri;
        if (type == 1) {
            if (p.split_a > 1) {
                // publish this split's partial sums (input-sum correction included); the last
                // split of (run, chunk) finishes. CTA-wide.
                if (warp < ri.nrows) {
                    float t0 = tsp[0], t1 = tsp[1];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        t0 += __shfl_xor_sync(0xffffffffu, t0, o);
                        t1 += __shfl_xor_sync(0xffffffffu, t1, o);
                    }
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        res[warp * 128 + lane * 4 + i] += CB_C1 * t0;
                        res[RUN_ROWS * 128 + warp * 128 + lane * 4 + i] += CB_C1 * t1;
                    }
                    tsp[0] = tsp[1] = 0.0f;
                }
                named_sync(1, NCW * 32);
                const int pidx = (g.run * (p.imax / 128) + g.chunk) * p.split_a + g.ks;
                float* dst = p.partA + static_cast<size_t>(pidx) * RES_FLOATS;
                for (int i = tid; i < RES_FLOATS; i += NCW * 32) dst[i] = res[i];
                __threadfence();
                named_sync(1, NCW * 32);
                if (tid == 0) {
                    const int old = atomicAdd(&p.ctrAk[g.run * (p.imax / 128) + g.chunk], 1);
                    sh_flag = old == p.split_a - 1;
                }
                named_sync(1, NCW * 32);
                const int last = sh_flag;
                named_sync(1, NCW * 32);
                if (!last) {
                    if (warp < ri.nrows) cp_async_wait_all();
                    continue;
                }
                __threadfence();
                const float* base = p.partA + static_cast<size_t>((g.run * (p.imax / 128) + g.chunk) * p.split_a) * RES_FLOATS;
                for (int i = tid; i < RES_FLOATS; i += NCW * 32) {
                    float a = 0.0f;
                    for (int k = 0; k < p.split_a; ++k) a += __ldcg(base + static_cast<size_t>(k) * RES_FLOATS + i);
                    res[i] = a;
                }
                named_sync(1, NCW * 32);
            }
            if (warp < ri.nrows) {
                // this warp's row: output rotation, scales, activation, down-input rotation
                const int t = warp, sl = wi.slot[t];
                const int col = g.chunk * 128 + lane * 4;
                float t0 = tsp[0], t1 = tsp[1];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    t0 += __shfl_xor_sync(0xffffffffu, t0, o);
                    t1 += __shfl_xor_sync(0xffffffffu, t1, o);
                }
                float gv[4], uv[4], sv[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    gv[i] = res[t * 128 + lane * 4 + i] + CB_C1 * t0;
                    uv[i] = res[RUN_ROWS * 128 + t * 128 + lane * 4 + i] + CB_C1 * t1;
                }
                cp_async_wait_all();
                __syncwarp();
                had128_warp(gv, lane);
                had128_warp(uv, lane);
                load4_half(reinterpret_cast<const __half*>(&eps[t].v[0][lane]), sv);
#pragma unroll
                for (int i = 0; i < 4; ++i) gv[i] *= sv[i];
                load4_half(reinterpret_cast<const __half*>(&eps[t].v[1][lane]), sv);
#pragma unroll
                for (int i = 0; i < 4; ++i) uv[i] *= sv[i];
                const int mode = ri.shared ? p.act_shared : p.act_routed;
                float av[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) av[i] = act_gated(gv[i], uv[i], p.limit, mode);
                load4_half(reinterpret_cast<const __half*>(&eps[t].v[2][lane]), sv);
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
        } else if (warp < ri.nrows) {
            // down epilogue of this warp's row: rotate, scale, weight; the last arrival of
            // (token, chunk) combines the token's slots in slot order, then the shared expert
            const int t = warp, sl = wi.slot[t];
            const int tok = slot_token(p, sl);
            const int col = g.chunk * 128 + lane * 4;
            float t0 = tsp[0];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) t0 += __shfl_xor_sync(0xffffffffu, t0, o);
            float v[4], sv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = res[t * 128 + lane * 4 + i] + CB_C1 * t0;
            cp_async_wait_all();
            __syncwarp();
            had128_warp(v, lane);
            load4_half(reinterpret_cast<const __half*>(&eps[t].v[0][lane]), sv);
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
            if (last) {
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
                    const float4 d = __ldcg(reinterpret_cast<const float4*>(
                        p.dpart + (static_cast<size_t>(p.S_cap) + tok) * p.H + col));
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
        }
    }
    cp_async_wait_all();
}

using ExpertsKernel = void (*)(KParams);

static ExpertsKernel pick_kernel(int kr, int ks)
{
#define EVA_K(a, b) \
    if (kr == a && ks == b) return experts_kernel<a, b>;
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

    const ExpertsKernel kern = pick_kernel(p.K, p.K_sh);
    if (!kern) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(SMEM_BYTES));
    if (e != cudaSuccess) return e;
    kern<<<sms, THREADS, SMEM_BYTES, stream>>>(p);
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
