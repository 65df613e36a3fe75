/*
 * Float32 CPU path of the MoE layer — BENCHMARK INFRASTRUCTURE ONLY.
 *
 * bench.py's CPU baseline and its reference arm time this function on the host cores; the tests check
 * it against eo_moe_forward (exl3_oracle.c, the float64 restatement that pins parity). The product
 * (eva_b200) never links or calls it.
 *
 * Same steps and summation order as eo_moe_forward (routed slots in slot order, then the shared
 * expert; per linear: x * suh -> 128-point Hadamard -> fp16 -> GEMV -> Hadamard -> * svh; the coop
 * activation for routed experts, torch swiglu for the shared one), in float32 instead of float64, with
 * the dequantization fused into the GEMV: each 16x16 trellis tile's 256 sixteen-bit windows are looked
 * up in a 65,536-entry float table of the mul1 codebook (filled from eo_mul1_decode) and accumulated
 * straight into the outputs. Threads split each linear's output columns (16-column tiles), so no
 * weight matrix is materialised and no partial sums are reduced.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

uint16_t eo_mul1_decode(uint32_t state);
void eo_tile_pos(int p, int* k, int* n);
double eo_f16_to_double(uint16_t h);
uint16_t eo_f16_from_double(double v);

#define CF_ROWS 32          /* rows per pass over a linear's tiles */

static float cf_cb[65536];   /* trellis state -> codebook value */
static float cf_f16[65536];  /* fp16 bits -> float */
static uint8_t cf_lw0[5][32], cf_lw1[5][32], cf_loff[5][32];  /* per group of 8 positions: its two words
                                                                 * and the bit offset of its first window */
static uint8_t cf_dst[256];  /* position p -> k * 16 + n inside the tile */
static int cf_ready;

static void cf_init(void)
{
    if (cf_ready) return;
    for (uint32_t s = 0; s < 65536; ++s) cf_f16[s] = (float) eo_f16_to_double((uint16_t) s);
    for (uint32_t s = 0; s < 65536; ++s) cf_cb[s] = cf_f16[eo_mul1_decode(s)];
    /* positions 8l .. 8l+7 end at bits (8l + j + 1) K: their windows span 16 + 7K bits starting at
     * bit (8l + 1) K - 16 (circular), which lie inside two consecutive words for K <= 4 */
    for (int K = 2; K <= 4; ++K) {
        const int nbits = 256 * K, words = 8 * K;
        for (int l = 0; l < 32; ++l) {
            int start = (8 * l + 1) * K - 16;
            if (start < 0) start += nbits;
            cf_lw0[K][l] = (uint8_t) (start >> 5);
            cf_lw1[K][l] = (uint8_t) (((start >> 5) + 1) % words);
            cf_loff[K][l] = (uint8_t) (start & 31);
        }
    }
    for (int p = 0; p < 256; ++p) {
        int k, n;
        eo_tile_pos(p, &k, &n);
        cf_dst[p] = (uint8_t) (k * 16 + n);
    }
    cf_ready = 1;
}

static inline float cf_round16(float v) { return cf_f16[eo_f16_from_double((double) v)]; }

static void cf_had128(float* v, int n)
{
    const float s = (float) (1.0 / sqrt(128.0));
    for (int c = 0; c + 128 <= n; c += 128) {
        float* b = v + c;
        for (int h = 1; h < 128; h <<= 1)
            for (int i = 0; i < 128; i += 2 * h)
                for (int j = i; j < i + h; ++j) {
                    const float a = b[j], d = b[j + h];
                    b[j] = a + d;
                    b[j + h] = a - d;
                }
        for (int i = 0; i < 128; ++i) b[i] *= s;
    }
}

/* acc[r][c] += sum_k x[r][k] * tile[k][c] for one 16x16 tile already decoded into wt[k * 16 + c]. */
__attribute__((target_clones("avx2", "default")))
static void cf_tile_fma(const float* wt, const float* x, int ldx, int n, float* acc)
{
    for (int r = 0; r < n; ++r) {
        float* a = acc + r * 16;
        const float* xr = x + (size_t) r * ldx;
        for (int k = 0; k < 16; ++k) {
            const float xv = xr[k];
            for (int c = 0; c < 16; ++c) a[c] += xv * wt[k * 16 + c];
        }
    }
}

/* The 256 codebook values of one K-bit tile, stored at wt[k * 16 + n]. */
static inline void cf_decode_tile(const uint32_t* t, int K, float* wt)
{
    const uint8_t *w0 = cf_lw0[K], *w1 = cf_lw1[K], *off = cf_loff[K];
    for (int l = 0; l < 32; ++l) {
        const uint64_t v = ((uint64_t) t[w0[l]] << 32) | t[w1[l]];
        const int top = 48 - off[l];
        const uint8_t* dst = cf_dst + 8 * l;
        for (int j = 0; j < 8; ++j) wt[dst[j]] = cf_cb[(uint32_t) (v >> (top - j * K)) & 0xffffu];
    }
}

/* y[r][j] = sum_i x[r][i] * W[i][j], r < n; W (in x out) decoded from the trellis on the fly. */
static void cf_gemv(const uint32_t* trellis, int in, int out, int K, const float* x, int n, float* y)
{
    const int kt_n = in / 16, nt_n = out / 16, words = 8 * K;
    #pragma omp parallel for schedule(static)
    for (int nt = 0; nt < nt_n; ++nt) {
        float wt[256], acc[CF_ROWS * 16];
        for (int r0 = 0; r0 < n; r0 += CF_ROWS) {
            const int nr = n - r0 < CF_ROWS ? n - r0 : CF_ROWS;
            memset(acc, 0, sizeof(float) * 16 * nr);
            for (int kt = 0; kt < kt_n; ++kt) {
                cf_decode_tile(trellis + ((size_t) kt * nt_n + nt) * words, K, wt);
                cf_tile_fma(wt, x + (size_t) r0 * in + kt * 16, in, nr, acc);
            }
            for (int r = 0; r < nr; ++r) memcpy(y + (size_t) (r0 + r) * out + nt * 16, acc + r * 16, 64);
        }
    }
}

/* One EXL3 linear on n rows: x float [n][in] -> y float [n][out]. xr: scratch [n][in]. */
static void cf_linear(const float* x, int n, int in, int out, const uint16_t* suh, const uint16_t* svh,
                      const void* trellis, int K, float* xr, float* y)
{
    for (int r = 0; r < n; ++r) {
        float* v = xr + (size_t) r * in;
        const float* s = x + (size_t) r * in;
        for (int i = 0; i < in; ++i) v[i] = s[i] * cf_f16[suh[i]];
        cf_had128(v, in);
        for (int i = 0; i < in; ++i) v[i] = cf_round16(v[i]);
    }
    cf_gemv((const uint32_t*) trellis, in, out, K, xr, n, y);
    for (int r = 0; r < n; ++r) {
        float* v = y + (size_t) r * out;
        cf_had128(v, out);
        for (int j = 0; j < out; ++j) v[j] *= cf_f16[svh[j]];
    }
}

static inline float cf_act(float g, float u, float limit, int mode)
{
    if (mode == 1) {
        if (limit > 0) {
            u = u < -limit ? -limit : (u > limit ? limit : u);
            if (g > limit) g = limit;
        }
        return g / (1.0f + expf(-g)) * u;
    }
    float a = g / (1.0f + expf(-g));
    if (limit != 0.0f) {
        u = u < -limit ? -limit : (u > limit ? limit : u);
        if (a > limit) a = limit;
    }
    return a * u;
}

/* gate/up -> activation -> down on n rows; 9 pointers in the reference handle order. */
static void cf_expert(const float* x, int n, int H, int I, const void* const* p, int K, float limit, int mode,
                      float* xr, float* g, float* u, float* y)
{
    cf_linear(x, n, H, I, (const uint16_t*) p[1], (const uint16_t*) p[2], p[0], K, xr, g);
    cf_linear(x, n, H, I, (const uint16_t*) p[4], (const uint16_t*) p[5], p[3], K, xr, u);
    for (size_t i = 0; i < (size_t) n * I; ++i) g[i] = cf_act(g[i], u[i], limit, mode);
    cf_linear(g, n, I, H, (const uint16_t*) p[7], (const uint16_t*) p[8], p[6], K, xr, y);
}

/* Arguments as eo_moe_forward (exl3_oracle.c); bf16 output omitted. Returns 2 when a selected expert
 * has no trellis pointer. */
int cf_moe_forward(const uint16_t* x, int x_is_f16, int M, int H, int I, int topk, int E,
                   const int32_t* sel, const float* rw, const void* const* ptrs, int K,
                   const void* const* sh_ptrs, int sh_I, int sh_K, double limit, float* out, int threads)
{
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void) threads;
#endif
    if (K < 2 || K > 4 || (sh_ptrs && (sh_K < 2 || sh_K > 4))) return 1;
    cf_init();
    const int Imax = I > sh_I ? I : sh_I;
    const int W = H > Imax ? H : Imax;
    /* a row may select one expert in several slots: up to M * topk rows per expert */
    const size_t R = (size_t) (M > 0 ? M : 1) * (topk > 0 ? topk : 1);
    float* xf = (float*) malloc(sizeof(float) * (size_t) (M > 0 ? M : 1) * H);
    float* xs = (float*) malloc(sizeof(float) * R * H);
    float* xr = (float*) malloc(sizeof(float) * R * W);
    float* g = (float*) malloc(sizeof(float) * R * Imax);
    float* u = (float*) malloc(sizeof(float) * R * Imax);
    float* ys = (float*) malloc(sizeof(float) * R * H);
    float* slot_out = (float*) calloc(R * H, sizeof(float));
    int* rows = (int*) malloc(sizeof(int) * R);
    int* ks = (int*) malloc(sizeof(int) * R);
    int status = 0;
    for (size_t i = 0; i < (size_t) M * H; ++i) {
        uint32_t b = x[i];
        if (x_is_f16) {
            xf[i] = cf_f16[b];
        } else {
            b <<= 16;
            float f;
            memcpy(&f, &b, 4);
            xf[i] = f;
        }
    }
    for (int e = 0; e < E && !status; ++e) {
        int n = 0;
        for (int m = 0; m < M; ++m)
            for (int k = 0; k < topk; ++k)
                if (sel[m * topk + k] == e && rw[m * topk + k] != 0.0f) { rows[n] = m; ks[n] = k; ++n; }
        if (!n) continue;
        const void* const* p = ptrs + (size_t) e * 9;
        if (!p[0] || !p[3] || !p[6]) { status = 2; break; }
        for (int r = 0; r < n; ++r) memcpy(xs + (size_t) r * H, xf + (size_t) rows[r] * H, sizeof(float) * H);
        cf_expert(xs, n, H, I, p, K, (float) limit, 0, xr, g, u, ys);
        for (int r = 0; r < n; ++r) {
            const float w = rw[rows[r] * topk + ks[r]];
            float* dst = slot_out + ((size_t) rows[r] * topk + ks[r]) * H;
            for (int h = 0; h < H; ++h) dst[h] = w * ys[(size_t) r * H + h];
        }
    }
    if (!status) {
        for (int m = 0; m < M; ++m) {
            float* o = out + (size_t) m * H;
            memset(o, 0, sizeof(float) * H);
            for (int k = 0; k < topk; ++k) {
                const float* s = slot_out + ((size_t) m * topk + k) * H;
                for (int h = 0; h < H; ++h) o[h] += s[h];
            }
        }
        if (sh_ptrs && M > 0) {
            cf_expert(xf, M, H, sh_I, sh_ptrs, sh_K, (float) limit, 1, xr, g, u, ys);
            for (size_t i = 0; i < (size_t) M * H; ++i) out[i] += ys[i];
        }
    }
    free(xf); free(xs); free(xr); free(g); free(u); free(ys); free(slot_out); free(rows); free(ks);
    return status;
}
