/*
 * CPU restatement of the EXL3 expert arithmetic on eva's DeepSeek MoE path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the CUDA kernels in
 * eva_b200/csrc. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it.
 * The product path never links or calls it.
 *
 * Everything here is restated from the reference's behaviour, not copied. Citations are paths
 * within the Findddx/eva project:
 *   - bitstream window of a trellis position:   runtime/ds41/csrc/moe_coop2048/vendor/quant/exl3_dq.cuh:15-31
 *   - mul1 codebook (one fp16 FMA):             .../vendor/quant/codebook.cuh:86-99
 *   - integer identity of mul1:                 runtime/ds41/cpu_precision_reference.py:43-45
 *   - position -> (k, n) inside a 16x16 tile:   .../vendor/quant/exl3_moe_coop_kernel.cuh:458-495 (B fragment of
 *                                               mma.m16n8k16, decode of lane<<3 positions)
 *   - 128-point Hadamard, natural order:        .../exl3_moe_coop_kernel.cuh:132-147, hadamard_inner.cuh:17-44
 *   - linear y = H(H(x*suh) W') * svh:          .../exl3_moe_coop_kernel.cuh:612-629 (input), :785-786 (output)
 *   - gated activation with act_limit:          .../exl3_moe_coop_kernel.cuh:115-129
 *   - torch swiglu (shared expert):             runtime/ds41/kernels.py:213-217
 *   - routed combine + shared merge:            .../exl3_moe_coop_kernel.cuh:906-949, runtime/ds41/model.py:498
 *
 * Numerics: the decoded weights are exact fp16 values (one rounding, as the reference's __hfma).
 * Rotated inputs and the down-projection input are rounded to fp16 as the reference stores them
 * (store_h4, exl3_moe_coop_kernel.cuh:176-184). Everything else accumulates in double.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------------------------------------
 * IEEE binary16 helpers (own implementation: round to nearest even from double)
 */
static uint16_t eo_f64_to_f16(double v)
{
    uint16_t sign = 0;
    if (signbit(v)) { sign = 0x8000; v = -v; }
    if (isnan(v)) return 0x7e00;
    if (v >= 65520.0) return sign | 0x7c00;          /* rounds to infinity */
    if (v == 0.0) return sign;
    int e;
    double m = frexp(v, &e);                          /* v = m * 2^e, m in [0.5, 1) */
    int exp16 = e - 1 + 15;                           /* biased exponent of 1.xxx * 2^(e-1) */
    double scaled;
    uint32_t q;
    if (exp16 <= 0) {
        /* subnormal: units of 2^-24 */
        scaled = ldexp(v, 24);
        double fl = floor(scaled);
        double rem = scaled - fl;
        q = (uint32_t) fl;
        if (rem > 0.5 || (rem == 0.5 && (q & 1))) q++;
        return sign | (uint16_t) q;                   /* q == 1024 becomes the smallest normal */
    }
    scaled = ldexp(m, 11);                            /* 11 significant bits incl. the hidden one */
    double fl = floor(scaled);
    double rem = scaled - fl;
    q = (uint32_t) fl;
    if (rem > 0.5 || (rem == 0.5 && (q & 1))) q++;
    if (q == 2048) { q = 1024; exp16++; }
    if (exp16 >= 31) return sign | 0x7c00;
    return sign | (uint16_t) ((exp16 << 10) | (q - 1024));
}

static double eo_f16_to_f64(uint16_t h)
{
    int sign = h >> 15, exp16 = (h >> 10) & 31, man = h & 1023;
    double v;
    if (exp16 == 0) v = ldexp((double) man, -24);
    else if (exp16 == 31) v = man ? NAN : INFINITY;
    else v = ldexp((double) (1024 + man), exp16 - 25);
    return sign ? -v : v;
}

static double eo_f16_table[65536];
static int eo_f16_table_ready = 0;

static void eo_init_table(void)
{
    if (eo_f16_table_ready) return;
    for (int i = 0; i < 65536; ++i) eo_f16_table[i] = eo_f16_to_f64((uint16_t) i);
    eo_f16_table_ready = 1;
}

__attribute__((constructor)) static void eo_ctor(void) { eo_init_table(); }

#define F16(h) (eo_f16_table[(uint16_t) (h)])

uint16_t eo_f16_from_double(double v) { return eo_f64_to_f16(v); }
double eo_f16_to_double(uint16_t h) { return eo_f16_to_f64(h); }

/* bf16 round to nearest even from float */
static uint16_t eo_f32_to_bf16(float f)
{
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t) ((u >> 16) | 0x40);
    uint32_t lsb = (u >> 16) & 1;
    u += 0x7fffu + lsb;
    return (uint16_t) (u >> 16);
}

static float eo_bf16_to_f32(uint16_t h)
{
    uint32_t u = ((uint32_t) h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* ---------------------------------------------------------------------------------------------
 * EXL3 mul1 codebook
 */

/* 32-bit product of a 16-bit trellis state with the codebook multiplier. */
static inline uint32_t eo_mul1_product(uint32_t state) { return (state & 0xffffu) * 0x83DCD12Du; }

static inline uint32_t eo_bytesum(uint32_t x) { return (x & 255) + ((x >> 8) & 255) + ((x >> 16) & 255) + (x >> 24); }

/* Integer identity of the codebook: byte sum of the product minus 510
 * (cpu_precision_reference.py:43-45). */
int eo_mul1_integer(uint32_t state) { return (int) eo_bytesum(eo_mul1_product(state)) - 510; }

/* fp16 bits of the decoded weight. The byte sum s added to the fp16 pattern of 1024.0 is the
 * exact fp16 value 1024 + s; the fp16 FMA with the two codebook constants (fp16 bit patterns
 * 0x1eee and 0xc931) rounds once. Here the exact value (1024 + s) * c0 + c1 is formed in double
 * (exact: both constants are fp16 numbers and the sum needs < 53 bits) and rounded once. */
uint16_t eo_mul1_decode(uint32_t state)
{
    const double c0 = eo_f16_to_f64(0x1eee);
    const double c1 = eo_f16_to_f64(0xc931);
    const double h = 1024.0 + (double) eo_bytesum(eo_mul1_product(state));
    return eo_f64_to_f16(h * c0 + c1);
}

/* ---------------------------------------------------------------------------------------------
 * Trellis bitstream
 *
 * One 16x16 tile is 256 * K bits in 8 * K little-endian uint32 words (two int16 per word). Bits
 * are numbered MSB-first through consecutive words. The state of position p is the 16-bit window
 * that ends at bit (p + 1) * K, read circularly modulo 256 * K (exl3_dq.cuh:15-31).
 */
uint32_t eo_tile_state(const uint32_t* tile, int K, int p)
{
    const int nbits = 256 * K;
    const int end = (p + 1) * K;
    uint32_t v = 0;
    for (int i = 0; i < 16; ++i) {
        int g = end - 16 + i;
        g %= nbits;
        if (g < 0) g += nbits;
        uint32_t bit = (tile[g >> 5] >> (31 - (g & 31))) & 1u;
        v = (v << 1) | bit;
    }
    return v;
}

/* Same window from the two words that hold it (the 16 bits never span more than two words). */
static inline uint32_t eo_tile_state2(const uint32_t* tile, int K, int p)
{
    const int nbits = 256 * K, words = 8 * K;
    int start = (p + 1) * K - 16;
    if (start < 0) start += nbits;
    const int w0 = start >> 5, off = start & 31;
    const uint64_t v = ((uint64_t) tile[w0] << 32) | tile[(w0 + 1) % words];
    return (uint32_t) (v >> (48 - off)) & 0xffffu;
}

uint32_t eo_tile_state_fast(const uint32_t* tile, int K, int p) { return eo_tile_state2(tile, K, p); }

/* Position p inside a tile -> (k, n) of the 16x16 weight block. Lane l = p / 8 of the MMA
 * decodes positions 8l..8l+7 into the B fragment of mma.m16n8k16 (k = 2(l%4) + {0,1} [+8],
 * n = l/4 [+8]). */
void eo_tile_pos(int p, int* k, int* n)
{
    const int l = p >> 3, j = p & 7;
    *n = (l >> 2) + 8 * (j >> 2);
    *k = 2 * (l & 3) + (j & 1) + 8 * ((j >> 1) & 1);
}

/* eo_mul1_decode of every 16-bit state, filled once (the dequantization reads it per weight). */
static uint16_t eo_mul1_table[65536];

__attribute__((constructor)) static void eo_mul1_ctor(void)
{
    for (uint32_t s = 0; s < 65536; ++s) eo_mul1_table[s] = eo_mul1_decode(s);
}

/* Dequantize a whole projection. trellis: int16 [in/16][out/16][16K]; w: fp16 bits [in][out]. */
void eo_dequant(const int16_t* trellis, int in, int out, int K, uint16_t* w)
{
    const int kt_n = in / 16, nt_n = out / 16, words = 8 * K;
    int kk[256], nn[256];
    for (int p = 0; p < 256; ++p) eo_tile_pos(p, &kk[p], &nn[p]);
    #pragma omp parallel for schedule(static)
    for (int kt = 0; kt < kt_n; ++kt)
        for (int nt = 0; nt < nt_n; ++nt) {
            const uint32_t* tile = (const uint32_t*) (trellis) + ((size_t) kt * nt_n + nt) * words;
            for (int p = 0; p < 256; ++p) {
                uint16_t h = eo_mul1_table[eo_tile_state2(tile, K, p)];
                w[(size_t) (kt * 16 + kk[p]) * out + nt * 16 + nn[p]] = h;
            }
        }
}

/* ---------------------------------------------------------------------------------------------
 * Blockwise 128-point Sylvester Hadamard, natural order, scaled by 1/sqrt(128)
 */
static void eo_had128(double* v)
{
    for (int h = 1; h < 128; h <<= 1)
        for (int i = 0; i < 128; i += 2 * h)
            for (int j = i; j < i + h; ++j) {
                double a = v[j], b = v[j + h];
                v[j] = a + b;
                v[j + h] = a - b;
            }
    const double s = 1.0 / sqrt(128.0);
    for (int i = 0; i < 128; ++i) v[i] *= s;
}

void eo_had128_blocks(double* v, int n)
{
    for (int c = 0; c + 128 <= n; c += 128) eo_had128(v + c);
}

/* ---------------------------------------------------------------------------------------------
 * One EXL3 linear on M rows. x: double [M][in]; w: dequantized fp16 [in][out]; y: double [M][out].
 * round_in: round the rotated input to fp16 (the reference stores it as fp16).
 */
void eo_linear(const double* x, int M, int in, int out, const uint16_t* suh, const uint16_t* svh,
               const uint16_t* w, int round_in, double* y)
{
    double* xr = (double*) malloc(sizeof(double) * in);
    double* acc = (double*) malloc(sizeof(double) * out);
    for (int m = 0; m < M; ++m) {
        for (int i = 0; i < in; ++i) xr[i] = x[(size_t) m * in + i] * F16(suh[i]);
        eo_had128_blocks(xr, in);
        if (round_in)
            for (int i = 0; i < in; ++i) xr[i] = F16(eo_f64_to_f16(xr[i]));
        /* each output column sums its products in input order; columns are split over threads */
        #pragma omp parallel for schedule(static)
        for (int j0 = 0; j0 < out; j0 += 256) {
            const int j1 = j0 + 256 < out ? j0 + 256 : out;
            for (int j = j0; j < j1; ++j) acc[j] = 0.0;
            for (int i = 0; i < in; ++i) {
                const double xi = xr[i];
                if (xi == 0.0) continue;
                const uint16_t* wr = w + (size_t) i * out;
                for (int j = j0; j < j1; ++j) acc[j] += xi * F16(wr[j]);
            }
        }
        eo_had128_blocks(acc, out);
        for (int j = 0; j < out; ++j) y[(size_t) m * out + j] = acc[j] * F16(svh[j]);
    }
    free(xr);
    free(acc);
}

/* ---------------------------------------------------------------------------------------------
 * Gated activations
 *   mode 0: coop semantics (exl3_moe_coop_kernel.cuh:115-129): a = silu(g); clamp u to +-limit and a
 *           to <= limit when limit != 0; return a * u.
 *   mode 1: torch swiglu (kernels.py:213-217): clamp u to +-limit and g to <= limit when limit > 0,
 *           then silu(g) * u.
 */
double eo_act(double g, double u, double limit, int mode)
{
    if (mode == 1) {
        if (limit > 0) {
            if (u < -limit) u = -limit;
            if (u > limit) u = limit;
            if (g > limit) g = limit;
        }
        return g / (1.0 + exp(-g)) * u;
    }
    double a = g / (1.0 + exp(-g));
    if (limit != 0.0) {
        if (u < -limit) u = -limit;
        if (u > limit) u = limit;
        if (a > limit) a = limit;
    }
    return a * u;
}

/* ---------------------------------------------------------------------------------------------
 * One expert MLP on M rows: gate/up -> act -> fp16 -> down.
 * wg/wu: fp16 [H][I]; wd: fp16 [I][Ho]. x: double [M][H]; y: double [M][Ho].
 */
void eo_expert(const double* x, int M, int H, int I, int Ho,
               const uint16_t* g_suh, const uint16_t* g_svh, const uint16_t* wg,
               const uint16_t* u_suh, const uint16_t* u_svh, const uint16_t* wu,
               const uint16_t* d_suh, const uint16_t* d_svh, const uint16_t* wd,
               double limit, int act_mode, double* y)
{
    double* g = (double*) malloc(sizeof(double) * (size_t) M * I);
    double* u = (double*) malloc(sizeof(double) * (size_t) M * I);
    eo_linear(x, M, H, I, g_suh, g_svh, wg, 1, g);
    eo_linear(x, M, H, I, u_suh, u_svh, wu, 1, u);
    for (size_t i = 0; i < (size_t) M * I; ++i) g[i] = eo_act(g[i], u[i], limit, act_mode);
    eo_linear(g, M, I, Ho, d_suh, d_svh, wd, 1, y);
    free(g);
    free(u);
}

/* ---------------------------------------------------------------------------------------------
 * Routed MoE forward from EXL3 tensors (dequantized on the fly, one expert at a time).
 *
 *   x:        bf16 bits [M][H] (x_is_f16 = 0) or fp16 bits (x_is_f16 = 1)
 *   sel:      int32 [M][topk] global expert ids (< E)
 *   rw:       float [M][topk] routing weights (0 = inactive slot)
 *   ptrs:     host pointers, 9 per expert in the reference handle order
 *             [g.trellis, g.suh, g.svh, u.trellis, u.suh, u.svh, d.trellis, d.suh, d.svh]
 *             (runtime/ds41/cache.py:1864-1887); the routed experts' arrays are E x 9.
 *   sh_ptrs:  9 host pointers of the shared expert, or NULL; sh_I its intermediate width
 *   out_f32:  float [M][H] (may be NULL); out_bf16: bf16 bits [M][H] (may be NULL)
 *   threads:  OpenMP threads for the dequantization (<= 0: library default)
 *
 * Order of the sum: routed slots k = 0..topk-1 in order, then the shared expert
 * (exl3_moe_coop_kernel.cuh:906-949, model.py:498).
 */
int eo_moe_forward(const uint16_t* x, int x_is_f16, int M, int H, int I, int topk, int E,
                   const int32_t* sel, const float* rw, const void* const* ptrs, int K,
                   const void* const* sh_ptrs, int sh_I, int sh_K,
                   double limit, float* out_f32, uint16_t* out_bf16, int threads)
{
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void) threads;
#endif
    double* xd = (double*) malloc(sizeof(double) * (size_t) M * H);
    double* acc = (double*) calloc((size_t) M * H, sizeof(double));
    for (size_t i = 0; i < (size_t) M * H; ++i) xd[i] = x_is_f16 ? F16(x[i]) : eo_bf16_to_f32(x[i]);

    uint16_t* wg = (uint16_t*) malloc(sizeof(uint16_t) * (size_t) H * (I > sh_I ? I : sh_I));
    uint16_t* wu = (uint16_t*) malloc(sizeof(uint16_t) * (size_t) H * (I > sh_I ? I : sh_I));
    uint16_t* wd = (uint16_t*) malloc(sizeof(uint16_t) * (size_t) H * (I > sh_I ? I : sh_I));
    /* a row may select one expert in several slots: up to M * topk rows per expert */
    const size_t R = (size_t) (M > 0 ? M : 1) * (topk > 0 ? topk : 1);
    double* xs = (double*) malloc(sizeof(double) * R * H);
    double* ys = (double*) malloc(sizeof(double) * R * H);
    int* rows = (int*) malloc(sizeof(int) * R);
    int* ks = (int*) malloc(sizeof(int) * R);
    int status = 0;

    /* per token, per slot contribution, summed in slot order: keep per-slot outputs */
    double* slot_out = (double*) calloc((size_t) M * topk * H, sizeof(double));
    for (int e = 0; e < E; ++e) {
        int n = 0;
        for (int m = 0; m < M; ++m)
            for (int k = 0; k < topk; ++k)
                if (sel[m * topk + k] == e && rw[m * topk + k] != 0.0f) { rows[n] = m; ks[n] = k; ++n; }
        if (!n) continue;
        const void* const* p = ptrs + (size_t) e * 9;
        if (!p[0] || !p[3] || !p[6]) { status = 2; break; }
        eo_dequant((const int16_t*) p[0], H, I, K, wg);
        eo_dequant((const int16_t*) p[3], H, I, K, wu);
        eo_dequant((const int16_t*) p[6], I, H, K, wd);
        for (int r = 0; r < n; ++r) memcpy(xs + (size_t) r * H, xd + (size_t) rows[r] * H, sizeof(double) * H);
        eo_expert(xs, n, H, I, H, (const uint16_t*) p[1], (const uint16_t*) p[2], wg,
                  (const uint16_t*) p[4], (const uint16_t*) p[5], wu,
                  (const uint16_t*) p[7], (const uint16_t*) p[8], wd, limit, 0, ys);
        for (int r = 0; r < n; ++r) {
            const double w = rw[rows[r] * topk + ks[r]];
            double* dst = slot_out + ((size_t) rows[r] * topk + ks[r]) * H;
            for (int h = 0; h < H; ++h) dst[h] = w * ys[(size_t) r * H + h];
        }
    }
    if (!status) {
        for (int m = 0; m < M; ++m)
            for (int k = 0; k < topk; ++k) {
                const double* src = slot_out + ((size_t) m * topk + k) * H;
                for (int h = 0; h < H; ++h) acc[(size_t) m * H + h] += src[h];
            }
        if (sh_ptrs) {
            eo_dequant((const int16_t*) sh_ptrs[0], H, sh_I, sh_K, wg);
            eo_dequant((const int16_t*) sh_ptrs[3], H, sh_I, sh_K, wu);
            eo_dequant((const int16_t*) sh_ptrs[6], sh_I, H, sh_K, wd);
            eo_expert(xd, M, H, sh_I, H, (const uint16_t*) sh_ptrs[1], (const uint16_t*) sh_ptrs[2], wg,
                      (const uint16_t*) sh_ptrs[4], (const uint16_t*) sh_ptrs[5], wu,
                      (const uint16_t*) sh_ptrs[7], (const uint16_t*) sh_ptrs[8], wd, limit, 1, ys);
            for (size_t i = 0; i < (size_t) M * H; ++i) acc[i] += ys[i];
        }
        for (size_t i = 0; i < (size_t) M * H; ++i) {
            if (out_f32) out_f32[i] = (float) acc[i];
            if (out_bf16) out_bf16[i] = eo_f32_to_bf16((float) acc[i]);
        }
    }
    free(slot_out);
    free(rows); free(ks); free(xs); free(ys);
    free(wg); free(wu); free(wd);
    free(xd); free(acc);
    return status;
}
