/* CPU oracle for the MXFP6 GEMM path — TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load this library, and
 * only to check or time against; the product (libmxfp6gemm) never calls it and has no CPU path.
 *
 * A plain-C restatement of the reference's CPU algorithm (eeezio/mxfp6-gemm, paths within that
 * project), pinned against the reference itself: tests/golden/ holds vectors produced by the
 * reference's own functions (compiled from its sources by oracle/Makefile into oracle/_ref/),
 * and tests/test_oracle.py checks this file against them.
 *
 *   oracle_fp6_to_float      include/mxfp6/types.hpp:13-24   E2M3 decode
 *   oracle_float_to_fp6      include/mxfp6/types.hpp:26-72   nearest E2M3, ties to even, sat 7.5
 *   oracle_e8m0_to_float     include/mxfp6/types.hpp:78-81   2^(c-127), 255 = NaN
 *   oracle_float_to_e8m0     include/mxfp6/types.hpp:83-92   log-domain nearest power of two
 *   oracle_quantize          include/mxfp6/preprocess.hpp:51-97  per-32 ceil-pow2 scale
 *   oracle_dequantize        include/mxfp6/preprocess.hpp:100-109
 *   oracle_gemm_rows         tests/reference.hpp:14-29        dequantise, then for each (m,n)
 *                            acc = 0; for k in 0..K-1: acc += a[m][k]*b[n][k]  (FP32, in order)
 *
 * Build with -ffp-contract=off so a*b+acc is never fused: the reference's loop is a separate
 * FP32 multiply and add. Rows are independent, so the threaded versions are bit-identical to a
 * single thread.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---- codecs ---------------------------------------------------------------------------------- */

float oracle_fp6_to_float(uint8_t c) {
    int e = (c >> 3) & 3, m = c & 7;
    float v = e == 0 ? (float)m * 0.125f : ldexpf(1.0f + (float)m * 0.125f, e - 1);
    return (c & 0x20) ? -v : v;
}

float oracle_e8m0_to_float(uint8_t c) {
    return c == 255 ? NAN : ldexpf(1.0f, (int)c - 127);
}

/* q >= 0 exact; nearest integer, ties to even */
static int rne_int(float q) {
    float f = floorf(q);
    float d = q - f;
    int b = (int)f;
    if (d > 0.5f) return b + 1;
    if (d < 0.5f) return b;
    return b + (b & 1);
}

uint8_t oracle_float_to_fp6(float v) {
    uint8_t s = 0;
    if (v < 0.0f) {
        s = 0x20;
        v = -v;
    }
    if (v == 0.0f) return s;
    if (isnan(v)) return 0x18; /* what the reference's (int)roundf(NaN) path yields on x86-64 */
    if (v > 7.5f) v = 7.5f;
    if (v < 1.0f) {
        int m = rne_int(v * 8.0f);
        if (m <= 0) return s;
        if (m >= 8) return (uint8_t)(s | 0x08);
        return (uint8_t)(s | m);
    }
    int e = v < 2.0f ? 1 : (v < 4.0f ? 2 : 3);
    float frac = v / (float)(1 << (e - 1)) - 1.0f;
    int m = rne_int(frac * 8.0f);
    if (m >= 8) {
        m = 0;
        if (++e > 3) return (uint8_t)(s | 0x1F);
    }
    return (uint8_t)(s | (e << 3) | m);
}

uint8_t oracle_float_to_e8m0(float v) {
    if (isnan(v)) return 255;
    if (v <= 0.0f) return 0;
    int e2;
    float m = frexpf(v, &e2);
    int e = e2 - 1;
    if (m * 2.0f >= 1.41421356f) e++;
    int c = e + 127;
    return (uint8_t)(c < 0 ? 0 : (c > 254 ? 254 : c));
}

uint8_t oracle_block_scale(float max_abs) {
    if (max_abs == 0.0f) return 127;
    int e2;
    float m = frexpf(max_abs / 7.5f, &e2);
    int e = (m == 0.5f) ? e2 - 1 : e2;
    int c = e + 127;
    return (uint8_t)(c < 0 ? 0 : (c > 254 ? 254 : c));
}

/* ---- packing ---------------------------------------------------------------------------------- */

static void pack4(const uint8_t* in, uint8_t* out) {
    uint32_t g = (uint32_t)(in[0] & 63) | ((uint32_t)(in[1] & 63) << 6) | ((uint32_t)(in[2] & 63) << 12) |
                 ((uint32_t)(in[3] & 63) << 18);
    out[0] = (uint8_t)g;
    out[1] = (uint8_t)(g >> 8);
    out[2] = (uint8_t)(g >> 16);
}

static uint8_t code_at(const uint8_t* row, int k) {
    const uint8_t* g = row + (k >> 2) * 3;
    uint32_t w = (uint32_t)g[0] | ((uint32_t)g[1] << 8) | ((uint32_t)g[2] << 16);
    return (uint8_t)((w >> (6 * (k & 3))) & 63);
}

/* ---- quantise / dequantise ------------------------------------------------------------------- */

/* mat [rows][cols] (cols % 32 == 0) -> packed [rows][3*cols/4], scales [rows][cols/32] */
void oracle_quantize(const float* mat, int rows, int cols, uint8_t* packed, uint8_t* scales) {
    const int rb = cols / 4 * 3, sc = cols / 32;
    uint8_t codes[32];
    for (int r = 0; r < rows; r++)
        for (int b = 0; b < sc; b++) {
            const float* x = mat + (size_t)r * cols + 32 * b;
            float mx = 0.0f;
            for (int k = 0; k < 32; k++) {
                float a = fabsf(x[k]);
                if (a > mx) mx = a;
            }
            uint8_t s = oracle_block_scale(mx);
            scales[(size_t)r * sc + b] = s;
            float sv = oracle_e8m0_to_float(s);
            for (int k = 0; k < 32; k++) codes[k] = oracle_float_to_fp6(x[k] / sv);
            for (int k = 0; k < 32; k += 4) pack4(codes + k, packed + (size_t)r * rb + 24 * b + 3 * (k / 4));
        }
}

/* packed rows (row_bytes stride) + raw scales [rows][cols/32] -> float [rows][cols] */
void oracle_dequantize(const uint8_t* packed, int row_bytes, const uint8_t* scales, int rows, int cols,
                       float* out) {
    const int sc = cols / 32;
    for (int r = 0; r < rows; r++) {
        const uint8_t* row = packed + (size_t)r * row_bytes;
        for (int k = 0; k < cols; k++)
            out[(size_t)r * cols + k] =
                oracle_fp6_to_float(code_at(row, k)) * oracle_e8m0_to_float(scales[(size_t)r * sc + k / 32]);
    }
}

/* ---- GEMM ---------------------------------------------------------------------------------------- */

typedef struct {
    const float* a;  /* dequantised A rows [nrows][K] */
    const float* b;  /* dequantised B^T [N][K] */
    float* d32;      /* [nrows][N] or NULL */
    double* d64;     /* [nrows][N] or NULL */
    int nrows, N, K, t, nt;
} job_t;

static void* gemm_worker(void* arg) {
    job_t* j = (job_t*)arg;
    for (int i = j->t; i < j->nrows; i += j->nt) {
        const float* a = j->a + (size_t)i * j->K;
        for (int n = 0; n < j->N; n++) {
            const float* b = j->b + (size_t)n * j->K;
            if (j->d32) {
                float acc = 0.0f;
                for (int k = 0; k < j->K; k++) acc += a[k] * b[k];
                j->d32[(size_t)i * j->N + n] = acc;
            } else {
                double acc = 0.0;
                for (int k = 0; k < j->K; k++) acc += (double)a[k] * (double)b[k];
                j->d64[(size_t)i * j->N + n] = acc;
            }
        }
    }
    return NULL;
}

/* D rows for the A rows listed in `rows` (or 0..nrows-1 when rows == NULL):
 *   out[i][n] = sum_k dequant(A)[rows[i]][k] * dequant(B^T)[n][k]
 * A: packed [M][A_row_bytes], raw scales [M][K/32]; B^T: packed [N][B_row_bytes], scales
 * [N][K/32]. f64 != 0 accumulates in double into out64 (an error-bound companion), otherwise
 * the reference's FP32 order into out32. Returns 0, or -1 on allocation failure. */
int oracle_gemm_rows(const uint8_t* A, int A_row_bytes, const uint8_t* sA, const uint8_t* B, int B_row_bytes,
                     const uint8_t* sB, int N, int K, const int* rows, int nrows, float* out32, double* out64,
                     int nthreads) {
    const int sc = K / 32;
    float* a = (float*)malloc((size_t)nrows * K * sizeof(float));
    float* b = (float*)malloc((size_t)N * K * sizeof(float));
    if (!a || !b) {
        free(a);
        free(b);
        return -1;
    }
    for (int i = 0; i < nrows; i++) {
        int r = rows ? rows[i] : i;
        oracle_dequantize(A + (size_t)r * A_row_bytes, A_row_bytes, sA + (size_t)r * sc, 1, K, a + (size_t)i * K);
    }
    oracle_dequantize(B, B_row_bytes, sB, N, K, b);
    if (nthreads < 1) nthreads = 1;
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nthreads);
    job_t* jobs = (job_t*)malloc(sizeof(job_t) * nthreads);
    for (int t = 0; t < nthreads; t++) {
        job_t j = {a, b, out64 ? NULL : out32, out64, nrows, N, K, t, nthreads};
        jobs[t] = j;
        if (t > 0) pthread_create(&th[t], NULL, gemm_worker, &jobs[t]);
    }
    gemm_worker(&jobs[0]);
    for (int t = 1; t < nthreads; t++) pthread_join(th[t], NULL);
    free(th);
    free(jobs);
    free(a);
    free(b);
    return 0;
}

/* ---- output rounding (what the GEMM's FP16 / BF16 store must equal) ------------------------------ */

/* float -> IEEE binary16 bits, round to nearest even, overflow to Inf, NaN kept quiet. */
uint16_t oracle_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7FFFFFFFu;
    if (absx > 0x7F800000u) return (uint16_t)(sign | 0x7E00u);
    if (absx >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* >= 65520 rounds to Inf */
    if (absx < 0x33000001u) return (uint16_t)sign;              /* <= 2^-25 rounds to 0 */
    int e = (int)(absx >> 23) - 127;
    uint32_t mant = (absx & 0x7FFFFFu) | 0x800000u;
    uint32_t h;
    if (e >= -14) { /* normal half */
        uint32_t shift = 13;
        uint32_t q = mant >> shift, rem = mant & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q++;
        h = ((uint32_t)(e + 15) << 10) + (q - 0x400u); /* carry into exponent is correct */
    } else {                                          /* subnormal half */
        uint32_t shift = (uint32_t)(13 + (-14 - e));
        uint32_t q = mant >> shift, rem = mant & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1))) q++;
        h = q;
    }
    return (uint16_t)(sign | h);
}

/* float -> bfloat16 bits, round to nearest even, NaN kept quiet. */
uint16_t oracle_f32_to_bf16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((x >> 16) | 0x40u);
    uint32_t lsb = (x >> 16) & 1u;
    x += 0x7FFFu + lsb;
    return (uint16_t)(x >> 16);
}

void oracle_round_f16(const float* in, uint16_t* out, long long n) {
    for (long long i = 0; i < n; i++) out[i] = oracle_f32_to_f16(in[i]);
}

void oracle_round_bf16(const float* in, uint16_t* out, long long n) {
    for (long long i = 0; i < n; i++) out[i] = oracle_f32_to_bf16(in[i]);
}
