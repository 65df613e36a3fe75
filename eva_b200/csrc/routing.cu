// Router (FP32 logits, scoring, biased / group-limited top-k) and the token permutation.
//
// Reference behaviour (paths within Findddx/eva):
//   router:      runtime/ds41/model.py:404-416 (sqrt(softplus) + bias top-k, weights normalised and
//                scaled). The softmax (DeepSeek-V2-Lite) and sigmoid group-limited (DeepSeek-V3) forms
//                follow the published DeepSeek gating; the reference has neither.
//   permutation: runtime/ds41/csrc/moe_coop2048/prepare_runs.cuh:8-66 and the CPU fixture
//                runtime/ds41/moe_coop2048.py:69-111: active slots (rw != 0) sorted by (expert, slot),
//                runs of at most 8 slots of one expert, table [n_runs, 0, run_start[S+1], order[S]].
//                The reference ranks every slot against every other (O(S^2), one CTA); here a
//                histogram + exclusive scan + chunked stable scatter does it in O(S + E) per CTA.
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace eva {

// ---------------------------------------------------------------------------------------------
// Router logits, small M: per 512-element k slice, partial sums of every (token, expert).

// A block takes 32 experts x one 512-element k slice: each warp holds 4 experts' weight slices in
// registers (16 float4 per lane, all loads in flight at once), the slice of 8 tokens' x at a time is
// staged in shared memory as FP32, and every (expert, token) partial is a warp reduction.
constexpr int RG_EXPERTS = 32;

__global__ void __launch_bounds__(256) router_gemv_kernel(const void* __restrict__ x, int x_bf16, int M, int H, int E,
                                                          const float* __restrict__ W, float* __restrict__ part, int KS)
{
    __shared__ __align__(16) float xs[8 * ROUTER_KSLICE];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ks = blockIdx.y;
    const int k0 = ks * ROUTER_KSLICE, klen = min(H - k0, ROUTER_KSLICE);
    const int eb = blockIdx.x * RG_EXPERTS + warp * 4;
    float4 w[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int k = lane * 4 + 128 * i;
            w[j][i] = (eb + j < E && k < klen) ? __ldg(reinterpret_cast<const float4*>(W + static_cast<size_t>(eb + j) * H + k0 + k))
                                               : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    for (int m0 = 0; m0 < M; m0 += 8) {
        __syncthreads();
        for (int v = threadIdx.x; v < 8 * (ROUTER_KSLICE / 4); v += blockDim.x) {
            const int t = v / (ROUTER_KSLICE / 4), k = (v % (ROUTER_KSLICE / 4)) * 4;
            float xv[4] = {0.f, 0.f, 0.f, 0.f};
            if (m0 + t < M && k < klen) load4_x(x, static_cast<size_t>(m0 + t) * H + k0 + k, x_bf16, xv);
            *reinterpret_cast<float4*>(xs + t * ROUTER_KSLICE + k) = make_float4(xv[0], xv[1], xv[2], xv[3]);
        }
        __syncthreads();
        float acc[4][8];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int t = 0; t < 8; ++t) acc[j][t] = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                const float4 xv = *reinterpret_cast<const float4*>(xs + t * ROUTER_KSLICE + lane * 4 + 128 * i);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    acc[j][t] = fmaf(w[j][i].x, xv.x, acc[j][t]);
                    acc[j][t] = fmaf(w[j][i].y, xv.y, acc[j][t]);
                    acc[j][t] = fmaf(w[j][i].z, xv.z, acc[j][t]);
                    acc[j][t] = fmaf(w[j][i].w, xv.w, acc[j][t]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                float v = acc[j][t];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (lane == 0 && m0 + t < M && eb + j < E) part[(static_cast<size_t>(ks) * M + m0 + t) * E + eb + j] = v;
            }
    }
}

// Router logits, large M when the tensor-core path does not apply (fp16 activations, H not a
// multiple of 64): 64 tokens x 64 experts per CTA, k chunks of 32 through shared memory,
// each thread 4 x 4 outputs; full sums (one slice).
__global__ void __launch_bounds__(256) router_gemm_kernel(const void* __restrict__ x, int x_bf16, int M, int H, int E,
                                                          const float* __restrict__ W, float* __restrict__ out)
{
    __shared__ __align__(16) float xs[32][64 + 4];
    __shared__ __align__(16) float wsm[32][64 + 4];
    const int tid = threadIdx.x;
    const int m0 = blockIdx.y * 64, e0 = blockIdx.x * 64;
    const int tm = (tid / 16) * 4, te = (tid % 16) * 4;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < H; k0 += 32) {
        // stage 64 x 32 of x and of W (transposed to [k][row])
        for (int i = tid; i < 64 * 8; i += 256) {
            const int r = i / 8, c = (i % 8) * 4;
            float v[4] = {0.f, 0.f, 0.f, 0.f};
            if (m0 + r < M) load4_x(x, static_cast<size_t>(m0 + r) * H + k0 + c, x_bf16, v);
            xs[c + 0][r] = v[0];
            xs[c + 1][r] = v[1];
            xs[c + 2][r] = v[2];
            xs[c + 3][r] = v[3];
            float4 w4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (e0 + r < E) w4 = __ldg(reinterpret_cast<const float4*>(W + static_cast<size_t>(e0 + r) * H + k0 + c));
            wsm[c + 0][r] = w4.x;
            wsm[c + 1][r] = w4.y;
            wsm[c + 2][r] = w4.z;
            wsm[c + 3][r] = w4.w;
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < 32; ++k) {
            // two 16-byte shared loads per 16 FMAs (rows are 68 floats: 16-byte aligned)
            const float4 x4 = *reinterpret_cast<const float4*>(&xs[k][tm]);
            const float4 w4 = *reinterpret_cast<const float4*>(&wsm[k][te]);
            const float xa[4] = {x4.x, x4.y, x4.z, x4.w}, wb[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xa[i], wb[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (m0 + tm + i < M && e0 + te + j < E) out[static_cast<size_t>(m0 + tm + i) * E + e0 + te + j] = acc[i][j];
}

cudaError_t launch_router_logits(const void* x, int x_bf16, int M, int H, int E, const float* W, float* part,
                                 void* wsplit, int* status, int* ks_used, cudaStream_t stream)
{
    if (router_tc_usable(x, x_bf16, M, H, E, wsplit))
        return launch_router_tc(x, M, H, E, W, wsplit, part, status, ks_used, stream);
    if (M < ROUTER_TC_MIN_ROWS) {
        const int KS = (H + ROUTER_KSLICE - 1) / ROUTER_KSLICE;
        *ks_used = KS;
        router_gemv_kernel<<<dim3((E + RG_EXPERTS - 1) / RG_EXPERTS, KS), 256, 0, stream>>>(x, x_bf16, M, H, E, W, part, KS);
    } else {
        *ks_used = 1;
        dim3 grid((E + 63) / 64, (M + 63) / 64);
        router_gemm_kernel<<<grid, 256, 0, stream>>>(x, x_bf16, M, H, E, W, part);
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// Scoring + top-k: one warp per token. Score functions are evaluated in double and rounded once
// to float, so the result is the correctly rounded value in all but vanishingly rare cases and
// matches a CPU evaluation of the same definition bit for bit.

__device__ __forceinline__ float score_of(float l, int router)
{
    const double d = static_cast<double>(l);
    if (router == EVA_ROUTER_SIGMOID) return static_cast<float>(1.0 / (1.0 + exp(-d)));
    if (router == EVA_ROUTER_SQRTSOFTPLUS) {
        const float sp = static_cast<float>(d > 20.0 ? d : log1p(exp(d)));   // softplus, threshold 20
        return sqrtf(sp);
    }
    return l;   // softmax: handled by the caller (needs the row max and sum)
}

// larger value first; equal values: lower index first
__device__ __forceinline__ bool better(float a, int ia, float b, int ib)
{
    return a > b || (a == b && ia < ib);
}

__device__ __forceinline__ void warp_argmax(float& v, int& i)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (better(ov, oi, v, i)) {
            v = ov;
            i = oi;
        }
    }
}

// One block per token: the block sums the slice partials and evaluates the scores (a thread per
// expert, E <= 1024), then warp 0 does the group-limited selection and the top-k from shared memory.
__global__ void __launch_bounds__(1024) topk_kernel(EvaMoeShape s, const float* __restrict__ part, int KS, int M,
                                                    const float* __restrict__ bias, float* __restrict__ logits_out,
                                                    int32_t* __restrict__ idx_out, float* __restrict__ w_out)
{
    extern __shared__ float smem_f[];
    __shared__ float red_f[32];
    __shared__ double red_d[32];
    const int E = s.n_experts;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    const int m = blockIdx.x;
    float* sc = smem_f;                  // unbiased scores
    float* ch = sc + E;                  // selection values
    // logits = sum of the slice partials in slice order
    float lmax = -INFINITY;
    for (int e = tid; e < E; e += blockDim.x) {
        float l = 0.0f;
        for (int k = 0; k < KS; ++k) l += part[(static_cast<size_t>(k) * M + m) * E + e];
        if (logits_out) logits_out[static_cast<size_t>(m) * E + e] = l;
        sc[e] = l;
        lmax = fmaxf(lmax, l);
    }
    if (s.router == EVA_ROUTER_SOFTMAX) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
        if (lane == 0) red_f[warp] = lmax;
        __syncthreads();
        lmax = red_f[0];
        for (int i = 1; i < nw; ++i) lmax = fmaxf(lmax, red_f[i]);
        double sum = 0.0;
        for (int e = tid; e < E; e += blockDim.x) sum += exp(static_cast<double>(sc[e]) - static_cast<double>(lmax));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) red_d[warp] = sum;
        __syncthreads();
        sum = 0.0;
        for (int i = 0; i < nw; ++i) sum += red_d[i];
        for (int e = tid; e < E; e += blockDim.x) {
            const float l = sc[e];
            ch[e] = l;   // softmax is monotonic: select on the logits
            sc[e] = static_cast<float>(exp(static_cast<double>(l) - static_cast<double>(lmax)) / sum);
        }
    } else {
        for (int e = tid; e < E; e += blockDim.x) {
            const float v = score_of(sc[e], s.router);
            sc[e] = v;
            ch[e] = v + (bias ? bias[e] : 0.0f);
        }
    }
    __syncthreads();
    if (warp != 0) return;
    // group-limited selection: keep the topk_group groups with the largest top-2 sums
    if (s.n_group > 1) {
        const int gsz = E / s.n_group;
        float gscore = -INFINITY;   // lane g holds group g's score (n_group <= 32)
        for (int g = 0; g < s.n_group; ++g) {
            float b1 = -INFINITY, b2 = -INFINITY;
            for (int j = lane; j < gsz; j += 32) {
                const float v = ch[g * gsz + j];
                if (v > b1) {
                    b2 = b1;
                    b1 = v;
                } else if (v > b2) {
                    b2 = v;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float o1 = __shfl_xor_sync(0xffffffffu, b1, o);
                const float o2 = __shfl_xor_sync(0xffffffffu, b2, o);
                // merge two sorted pairs
                const float n1 = fmaxf(b1, o1);
                const float n2 = fmaxf(fminf(b1, o1), fmaxf(b2, o2));
                b1 = n1;
                b2 = n2;
            }
            if (lane == g) gscore = b1 + b2;
        }
        unsigned keep = 0;
        for (int t = 0; t < s.topk_group; ++t) {
            float v = (lane < s.n_group && !((keep >> lane) & 1)) ? gscore : -INFINITY;
            int i = lane < s.n_group ? lane : 1 << 30;
            warp_argmax(v, i);
            keep |= 1u << i;
        }
        for (int e = lane; e < E; e += 32)
            if (!((keep >> (e / gsz)) & 1)) ch[e] = -INFINITY;
        __syncwarp();
    }
    // top-k: k rounds of a warp argmax over the remaining candidates
    float wsel = 0.0f;   // lane k keeps the k-th selection's score
    int isel = 0;
    float wsum = 0.0f;
    for (int k = 0; k < s.topk; ++k) {
        float v = -INFINITY;
        int i = 1 << 30;
        for (int e = lane; e < E; e += 32) {
            const float c = ch[e];
            if (better(c, e, v, i)) {
                v = c;
                i = e;
            }
        }
        warp_argmax(v, i);
        const float sv = sc[i];
        if (lane == k) {
            isel = i;
            wsel = sv;
        }
        wsum += sv;
        __syncwarp();
        if (lane == 0) ch[i] = -INFINITY;
        __syncwarp();
    }
    if (lane < s.topk) {
        float w = wsel;
        if (s.norm_topk) w = w / (wsum + 1e-20f);
        w = w * s.route_scale;
        idx_out[static_cast<size_t>(m) * s.topk + lane] = isel;
        w_out[static_cast<size_t>(m) * s.topk + lane] = w;
    }
}

cudaError_t launch_topk(const EvaMoeShape& s, const float* part, int ks, int M, const float* bias,
                        float* logits_out, int32_t* idx, float* w, cudaStream_t stream)
{
    const size_t smem = static_cast<size_t>(2) * s.n_experts * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    const int threads = std::min(1024, (s.n_experts + 31) / 32 * 32);
    topk_kernel<<<M, threads, smem, stream>>>(s, part, ks, M, bias, logits_out, idx, w);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// Permutation: one CTA of 1024 threads.
//   1. per-expert histogram of active slots (and per-token active counts)
//   2. exclusive scans: slot start and run start per expert
//   3. stable scatter in chunks of 1024 slots: in-warp rank by __match_any_sync, cross-warp offsets
//      by a per-chunk [warp][expert] count table and a running per-expert cursor.

constexpr int PERM_THREADS = 1024;

// Expert e's 9 table entries are all bound (non-zero) and 16-byte aligned (true without tables).
__device__ __forceinline__ bool expert_bound(const PermuteArgs& a, int e)
{
    bool ok = true;
    if (a.tables[0]) {
#pragma unroll
        for (int r = 0; r < 9; ++r) {
            const int64_t p = a.tables[r][e];
            ok = ok && p != 0 && (p & 15) == 0;
        }
    }
    return ok;
}

// bound: [E] per-expert expert_bound results (shared memory), filled before the first call
__device__ __forceinline__ int slot_expert(const PermuteArgs& a, int s, bool flag_errors, int32_t* status,
                                           const unsigned char* bound)
{
    const int m = s / a.topk;
    if (m >= a.M) return -1;
    if (a.rw[s] == 0.0f) return -1;
    const long long e = a.sel64 ? static_cast<const long long*>(a.sel)[s] : static_cast<const int32_t*>(a.sel)[s];
    const bool ok = e >= 0 && e < a.n_local && bound[e];
    if (!ok) {
        if (flag_errors && status) atomicOr(status, ST_BAD_EXPERT);
        return -1;
    }
    return static_cast<int>(e);
}

__global__ void __launch_bounds__(PERM_THREADS) permute_kernel(PermuteArgs a)
{
    extern __shared__ int smem_i[];
    const int E = a.n_local;
    int* hist = smem_i;              // [E]
    int* estart = hist + E;          // [E + 1]
    int* rstart = estart + E + 1;    // [E + 1]
    int* tsh = rstart + E + 1;       // [E + 1] tile prefix
    int* cursor = tsh + E + 1;       // [E]
    int* wcnt = cursor + E;          // [32][E]
    unsigned char* bound = reinterpret_cast<unsigned char*>(wcnt + 32 * E);   // [E]
    __shared__ int sh_tot[2];
    __shared__ int scan_tmp[32];
    __shared__ int scan_tmp2[32];
    __shared__ int scan_tmp3[32];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int S_cap = a.capacity * a.topk;
    const int S = a.M * a.topk;

    for (int i = tid; i < E; i += PERM_THREADS) {
        hist[i] = 0;
        cursor[i] = 0;
        bound[i] = expert_bound(a, i) ? 1 : 0;
    }
    if (a.counters)
        for (int i = tid; i < a.n_counters; i += PERM_THREADS) a.counters[i] = 0;
    if (a.tok_expect)
        for (int i = tid; i < a.M; i += PERM_THREADS) a.tok_expect[i] = 0;
    __syncthreads();

    // 1. histogram
    for (int s = tid; s < S; s += PERM_THREADS) {
        const int e = slot_expert(a, s, true, a.status, bound);
        if (a.slot_act) a.slot_act[s] = e >= 0;
        if (e >= 0) {
            atomicAdd(&hist[e], 1);
            if (a.tok_expect) atomicAdd(&a.tok_expect[s / a.topk], 1);
        }
    }
    __syncthreads();

    // 2. exclusive scans over experts (E <= 1024 = one element per thread)
    {
        const int h = tid < E ? hist[tid] : 0;
        const int r = (h + RUN_ROWS - 1) / RUN_ROWS;
        const int mt = (h + PF_TILE_ROWS - 1) / PF_TILE_ROWS;
        int v0 = h, v1 = r, v2 = mt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n0 = __shfl_up_sync(0xffffffffu, v0, o);
            const int n1 = __shfl_up_sync(0xffffffffu, v1, o);
            const int n2 = __shfl_up_sync(0xffffffffu, v2, o);
            if (lane >= o) {
                v0 += n0;
                v1 += n1;
                v2 += n2;
            }
        }
        if (lane == 31) {
            scan_tmp[warp] = v0;
            scan_tmp2[warp] = v1;
            scan_tmp3[warp] = v2;
        }
        __syncthreads();
        int b0 = 0, b1 = 0, b2 = 0, t0 = 0, t1 = 0, t2 = 0;
        for (int w = 0; w < 32; ++w) {
            if (w < warp) {
                b0 += scan_tmp[w];
                b1 += scan_tmp2[w];
                b2 += scan_tmp3[w];
            }
            t0 += scan_tmp[w];
            t1 += scan_tmp2[w];
            t2 += scan_tmp3[w];
        }
        if (tid < E) {
            estart[tid] = b0 + v0 - h;
            rstart[tid] = b1 + v1 - r;
            tsh[tid] = b2 + v2 - mt;
        }
        if (tid == 0) {
            estart[E] = t0;
            rstart[E] = t1;
            tsh[E] = t2;
            sh_tot[0] = t0;   // active slots
            sh_tot[1] = t1;   // runs
        }
    }
    __syncthreads();
    const int n_active = sh_tot[0], n_runs = sh_tot[1];
    int* run_start = a.runs + 2;
    int* order = a.runs + 2 + S_cap + 1;

    // 3. stable scatter
    for (int c0 = 0; c0 < S; c0 += PERM_THREADS) {
        const int s = c0 + tid;
        const int e = s < S ? slot_expert(a, s, false, nullptr, bound) : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        const bool leader = rank == 0;
        for (int i = tid; i < 32 * E; i += PERM_THREADS) wcnt[i] = 0;
        __syncthreads();
        if (leader && e >= 0) wcnt[warp * E + e] = __popc(peers);
        __syncthreads();
        for (int x = tid; x < E; x += PERM_THREADS) {
            int run = cursor[x];
            for (int w = 0; w < 32; ++w) {
                const int v = wcnt[w * E + x];
                wcnt[w * E + x] = run;
                run += v;
            }
            cursor[x] = run;
        }
        __syncthreads();
        if (e >= 0) {
            const int pe = wcnt[warp * E + e] + rank;
            const int pos = estart[e] + pe;
            order[pos] = s;
            if (pe % RUN_ROWS == 0) {
                const int rid = rstart[e] + pe / RUN_ROWS;
                run_start[rid] = pos;
                if (a.run_expert) a.run_expert[rid] = e;
            }
        }
        __syncthreads();
    }

    // 4. table tail and zero fill
    for (int i = n_runs + 1 + tid; i <= S_cap; i += PERM_THREADS) run_start[i] = 0;
    for (int i = n_active + tid; i < S_cap; i += PERM_THREADS) order[i] = 0;
    if (tid == 0) {
        a.runs[0] = n_runs;
        a.runs[1] = 0;
        run_start[n_runs] = n_active;
    }
    if (a.estart)
        for (int i = tid; i <= E; i += PERM_THREADS) a.estart[i] = estart[i];
    if (a.tstart) {
        for (int i = tid; i <= E; i += PERM_THREADS) a.tstart[i] = tsh[i];
        if (tid == 0) a.tstart[E + 1] = tsh[E] + (a.has_shared ? (a.shn + PF_TILE_ROWS - 1) / PF_TILE_ROWS : 0);
    }
    __syncthreads();

    // 5. expected combine arrivals; rows nobody will write are zeroed here
    if (a.tok_expect) {
        for (int m = tid; m < a.M; m += PERM_THREADS) {
            const bool sh = a.has_shared && m >= a.sh0 && m < a.sh0 + a.shn;
            a.tok_expect[m] += sh ? 1 : 0;
        }
        __syncthreads();
        {
            // warp per row; only rows without arrivals are written (H is a multiple of 256)
            for (int m = warp; m < a.M; m += PERM_THREADS / 32) {
                if (a.tok_expect[m] != 0) continue;
                const size_t row = static_cast<size_t>(m) * a.H;
                if (a.out_f32)
                    for (int c = lane * 4; c < a.H; c += 128)
                        *reinterpret_cast<float4*>(a.out_f32 + row + c) = make_float4(0.f, 0.f, 0.f, 0.f);
                if (a.out_bf16)   // 8-byte aligned
                    for (int c = lane * 4; c < a.H; c += 128)
                        *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(a.out_bf16) + row + c) = make_uint2(0, 0);
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Permutation, multi-CTA form for large batches: the same table in three launches.
//   count:   CTA per chunk of PERM_TOK_CHUNK tokens (thread per token): per-chunk expert counts,
//            slot_act, per-token arrival counts, work counters zeroed
//   scan:    one CTA: per expert, the chunks' exclusive prefix (each chunk's base inside its
//            expert's segment), then the expert / run / tile starts and the table header
//   scatter: CTA per chunk: stable in-chunk ranks (as permute_kernel's step 3) from the chunk's
//            bases, the table's zero tail, rows with no arrivals zeroed
// Scratch (ints): [n_chunks][E] counts -> bases, [E + 1] slot starts, [E + 1] run starts.

__global__ void __launch_bounds__(PERM_TOK_CHUNK) permute_count_kernel(PermuteArgs a)
{
    extern __shared__ int smem_i[];
    const int E = a.n_local;
    int* hist = smem_i;                                               // [E]
    unsigned char* bound = reinterpret_cast<unsigned char*>(hist + E);   // [E]
    const int tid = threadIdx.x, c = blockIdx.x;
    for (int i = tid; i < E; i += blockDim.x) {
        hist[i] = 0;
        bound[i] = expert_bound(a, i) ? 1 : 0;
    }
    if (a.counters)
        for (int i = blockIdx.x * blockDim.x + tid; i < a.n_counters; i += gridDim.x * blockDim.x) a.counters[i] = 0;
    __syncthreads();
    const int m = c * PERM_TOK_CHUNK + tid;
    if (m < a.M) {
        int n = 0;
        for (int k = 0; k < a.topk; ++k) {
            const int s = m * a.topk + k;
            const int e = slot_expert(a, s, true, a.status, bound);
            if (a.slot_act) a.slot_act[s] = e >= 0;
            if (e >= 0) {
                atomicAdd(&hist[e], 1);
                ++n;
            }
        }
        if (a.tok_expect) a.tok_expect[m] = n + ((a.has_shared && m >= a.sh0 && m < a.sh0 + a.shn) ? 1 : 0);
    }
    __syncthreads();
    for (int i = tid; i < E; i += blockDim.x) a.scratch[static_cast<size_t>(c) * E + i] = hist[i];
}

__global__ void __launch_bounds__(PERM_THREADS) permute_scan_kernel(PermuteArgs a, int n_chunks)
{
    __shared__ int scan_tmp[3][32];
    const int E = a.n_local;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int* sc_estart = a.scratch + static_cast<size_t>(n_chunks) * E;
    int* sc_rstart = sc_estart + E + 1;
    // per expert: exclusive prefix over the chunks (loads batched for memory-level parallelism)
    int h = 0;
    if (tid < E) {
        int* col = a.scratch + tid;
        int c = 0;
        for (; c + 8 <= n_chunks; c += 8) {
            int v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = col[static_cast<size_t>(c + i) * E];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                col[static_cast<size_t>(c + i) * E] = h;
                h += v[i];
            }
        }
        for (; c < n_chunks; ++c) {
            const int v = col[static_cast<size_t>(c) * E];
            col[static_cast<size_t>(c) * E] = h;
            h += v;
        }
    }
    // exclusive scans over experts (E <= 1024 = one element per thread): slots, runs, tiles
    const int r = (h + RUN_ROWS - 1) / RUN_ROWS;
    const int mt = (h + PF_TILE_ROWS - 1) / PF_TILE_ROWS;
    int v0 = h, v1 = r, v2 = mt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n0 = __shfl_up_sync(0xffffffffu, v0, o);
        const int n1 = __shfl_up_sync(0xffffffffu, v1, o);
        const int n2 = __shfl_up_sync(0xffffffffu, v2, o);
        if (lane >= o) {
            v0 += n0;
            v1 += n1;
            v2 += n2;
        }
    }
    if (lane == 31) {
        scan_tmp[0][warp] = v0;
        scan_tmp[1][warp] = v1;
        scan_tmp[2][warp] = v2;
    }
    __syncthreads();
    int b0 = 0, b1 = 0, b2 = 0, t0 = 0, t1 = 0, t2 = 0;
    for (int w = 0; w < PERM_THREADS / 32; ++w) {
        if (w < warp) {
            b0 += scan_tmp[0][w];
            b1 += scan_tmp[1][w];
            b2 += scan_tmp[2][w];
        }
        t0 += scan_tmp[0][w];
        t1 += scan_tmp[1][w];
        t2 += scan_tmp[2][w];
    }
    if (tid < E) {
        sc_estart[tid] = b0 + v0 - h;
        sc_rstart[tid] = b1 + v1 - r;
        if (a.estart) a.estart[tid] = b0 + v0 - h;
        if (a.tstart) a.tstart[tid] = b2 + v2 - mt;
    }
    if (tid == 0) {
        const int S_cap = a.capacity * a.topk;
        sc_estart[E] = t0;
        sc_rstart[E] = t1;
        if (a.estart) a.estart[E] = t0;
        if (a.tstart) {
            a.tstart[E] = t2;
            a.tstart[E + 1] = t2 + (a.has_shared ? (a.shn + PF_TILE_ROWS - 1) / PF_TILE_ROWS : 0);
        }
        a.runs[0] = t1;
        a.runs[1] = 0;
        a.runs[2 + t1] = t0;   // run_start[n_runs] = n_active
        (void)S_cap;
    }
}

__global__ void __launch_bounds__(PERM_THREADS) permute_scatter_kernel(PermuteArgs a, int n_chunks)
{
    extern __shared__ int smem_i[];
    const int E = a.n_local;
    int* cursor = smem_i;                 // [E] next position inside the expert's segment
    int* wcnt = cursor + E;               // [32][E]
    int* estart = wcnt + 32 * E;          // [E]
    int* rstart = estart + E;             // [E]
    unsigned char* bound = reinterpret_cast<unsigned char*>(rstart + E);   // [E]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, c = blockIdx.x;
    const int* sc_estart = a.scratch + static_cast<size_t>(n_chunks) * E;
    const int* sc_rstart = sc_estart + E + 1;
    for (int i = tid; i < E; i += PERM_THREADS) {
        cursor[i] = a.scratch[static_cast<size_t>(c) * E + i];
        estart[i] = sc_estart[i];
        rstart[i] = sc_rstart[i];
        bound[i] = expert_bound(a, i) ? 1 : 0;
    }
    __syncthreads();
    const int S_cap = a.capacity * a.topk;
    const int S = a.M * a.topk;
    int* run_start = a.runs + 2;
    int* order = a.runs + 2 + S_cap + 1;
    const int s_lo = c * PERM_TOK_CHUNK * a.topk, s_hi = min(S, s_lo + PERM_TOK_CHUNK * a.topk);
    for (int c0 = s_lo; c0 < s_hi; c0 += PERM_THREADS) {
        const int s = c0 + tid;
        const int e = s < s_hi ? slot_expert(a, s, false, nullptr, bound) : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, e);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        for (int i = tid; i < 32 * E; i += PERM_THREADS) wcnt[i] = 0;
        __syncthreads();
        if (rank == 0 && e >= 0) wcnt[warp * E + e] = __popc(peers);
        __syncthreads();
        for (int x = tid; x < E; x += PERM_THREADS) {
            int run = cursor[x];
            for (int w = 0; w < 32; ++w) {
                const int v = wcnt[w * E + x];
                wcnt[w * E + x] = run;
                run += v;
            }
            cursor[x] = run;
        }
        __syncthreads();
        if (e >= 0) {
            const int pe = wcnt[warp * E + e] + rank;
            const int pos = estart[e] + pe;
            order[pos] = s;
            if (pe % RUN_ROWS == 0) {
                const int rid = rstart[e] + pe / RUN_ROWS;
                run_start[rid] = pos;
                if (a.run_expert) a.run_expert[rid] = e;
            }
        }
        __syncthreads();
    }
    // the table's zero tail, over the whole grid
    const int n_runs = sc_rstart[E], n_active = sc_estart[E];
    const int gt = blockIdx.x * PERM_THREADS + tid, gs = gridDim.x * PERM_THREADS;
    for (int i = n_runs + 1 + gt; i <= S_cap; i += gs) run_start[i] = 0;
    for (int i = n_active + gt; i < S_cap; i += gs) order[i] = 0;
    // rows nobody will write (no active slot, no shared expert) are zeroed; warp per row
    if (a.tok_expect) {
        const int m_hi = min(a.M, (c + 1) * PERM_TOK_CHUNK);
        for (int m = c * PERM_TOK_CHUNK + warp; m < m_hi; m += PERM_THREADS / 32) {
            if (a.tok_expect[m] != 0) continue;
            const size_t row = static_cast<size_t>(m) * a.H;
            if (a.out_f32)
                for (int cc = lane * 4; cc < a.H; cc += 128)
                    *reinterpret_cast<float4*>(a.out_f32 + row + cc) = make_float4(0.f, 0.f, 0.f, 0.f);
            if (a.out_bf16)
                for (int cc = lane * 4; cc < a.H; cc += 128)
                    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(a.out_bf16) + row + cc) = make_uint2(0, 0);
        }
    }
}

cudaError_t launch_permute(const PermuteArgs& a, cudaStream_t stream)
{
    const int E = a.n_local;
    if (a.scratch && a.M > 2 * PERM_TOK_CHUNK) {
        const int n_chunks = (a.M + PERM_TOK_CHUNK - 1) / PERM_TOK_CHUNK;
        const size_t smem1 = static_cast<size_t>(E) * sizeof(int) + E;
        const size_t smem3 = (static_cast<size_t>(E) * 35) * sizeof(int) + E;
        cudaError_t e = cudaFuncSetAttribute(permute_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem3));
        if (e != cudaSuccess) return e;
        permute_count_kernel<<<n_chunks, PERM_TOK_CHUNK, smem1, stream>>>(a);
        permute_scan_kernel<<<1, PERM_THREADS, 0, stream>>>(a, n_chunks);
        permute_scatter_kernel<<<n_chunks, PERM_THREADS, smem3, stream>>>(a, n_chunks);
        return cudaGetLastError();
    }
    const size_t smem = (static_cast<size_t>(E) * 5 + 3 + 32 * static_cast<size_t>(E)) * sizeof(int) + static_cast<size_t>(E);
    cudaError_t e = cudaFuncSetAttribute(permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    permute_kernel<<<1, PERM_THREADS, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace eva
