/*
 * qlinear_ref.c -- CPU oracle for the quantized-linear hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker: tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / --impl reference legs load it. The product path
 * (open_rknpu2_lm_infer_b200 and libqlinear_b200.so) never links, loads or calls it.
 *
 * It restates, in plain C, the only CPU implementation of the path that the reference
 * holds: the `oracle` function of src/npu.rs:1097-1121 (open_rknpu2_lm_infer v0.6.1).
 * Its arithmetic, per row m of an f32 input [rows][K] and a weight QuantMatrix with
 * codes [K][N] (index k*N+n, src/npu.rs:1115) and f32 scales [N]:
 *
 *   amax   = max_k |x[m,k]|  folded from 0.0 with f32::max, which ignores NaN   (:1101)
 *   scale  = amax == 0 ? 1.0 : max(amax / 127, FLT_MIN)                          (:1102-1106)
 *   q[k]   = clamp(round(x[m,k] * (1 / scale)), -127, 127) as i32                (:1107-1110)
 *            round = f32::round, ties away from zero; NaN -> 0 by the `as` cast
 *   acc[n] = sum_k q[k] * codes[k*N+n]              exact in i32                (:1111-1116)
 *   y[m,n] = (acc[n] as f32 * scale) * scales[n]    two RN f32 multiplies        (:1117)
 *
 * plus the fused SwiGLU expectation of src/npu.rs:1202-1208:
 *   mid[m,j] = gate / (1 + exp(-gate)) * up,  gate = y[m,j], up = y[m,N/2+j]
 *
 * Rounding: QREF_ROUND_AWAY (default) is the reference's f32::round. QREF_ROUND_EVEN
 * (round half to even) exists only because one benchmark description names it; the
 * reference itself never uses it.
 *
 * Build: gcc -O3 -march=native -fopenmp -ffp-contract=off (no -ffast-math): the two
 * multiplies of the epilogue and x*inv must stay separately rounded f32 operations.
 * The integer dot product is evaluated k-outer / n-inner so that it vectorises over n;
 * integer addition is associative, so any order gives the same i32.
 */
#include <math.h>
#include <float.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define QREF_ROUND_AWAY 0
#define QREF_ROUND_EVEN 1

/* f32::round (ties away from zero) or round-half-even, then clamp and `as i32`. */
static inline int32_t quant_code(float v, int round_mode)
{
    float r = (round_mode == QREF_ROUND_EVEN) ? nearbyintf(v) : roundf(v);
    if (isnan(r)) return 0;                 /* Rust: NaN.clamp(..) is NaN, `NaN as i32` = 0 */
    if (r < -127.0f) r = -127.0f;
    if (r > 127.0f) r = 127.0f;
    return (int32_t)r;
}

/* Rust f32::max(a, b): returns the non-NaN operand when one is NaN (src/npu.rs:1101). */
static inline float rust_max(float a, float b)
{
    if (isnan(a)) return b;
    if (isnan(b)) return a;
    return a > b ? a : b;
}

/* Exact IEEE binary16 -> binary32 widening (every half is representable in f32). */
float qref_half_to_float(uint16_t h)
{
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal half: normalise */
            int e = -1;
            do { man <<= 1; e++; } while ((man & 0x400u) == 0);
            man &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* One row of the activation quantisation (src/npu.rs:1099-1110). Returns the scale. */
static float quant_row(const float *a, int64_t k, int round_mode, int8_t *codes, int32_t *rowsum)
{
    float maximum = 0.0f;
    for (int64_t i = 0; i < k; i++) maximum = rust_max(maximum, fabsf(a[i]));
    float scale;
    if (maximum == 0.0f) {
        scale = 1.0f;
    } else {
        scale = rust_max(maximum / 127.0f, FLT_MIN);
    }
    volatile float one = 1.0f;              /* keep `1.0 / scale` a real IEEE division */
    float inv = one / scale;
    int32_t sum = 0;
    for (int64_t i = 0; i < k; i++) {
        int32_t q = quant_code(a[i] * inv, round_mode);
        codes[i] = (int8_t)q;
        sum += q;
    }
    if (rowsum) *rowsum = sum;
    return scale;
}

/* Activation quantisation of an f32 [rows][k] matrix: codes [rows][k], scales [rows].
 * rowsums (may be NULL) receives sum_k q[m,k]. */
int qref_act_quant_f32(const float *x, int64_t rows, int64_t k, int round_mode,
                       int8_t *codes, float *scales, int32_t *rowsums)
{
    if (!x || !codes || !scales || rows < 0 || k <= 0) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < rows; m++)
        scales[m] = quant_row(x + m * k, k, round_mode, codes + m * k, rowsums ? rowsums + m : NULL);
    return 0;
}

/* Same for fp16 input bits [rows][k], widened exactly to f32 first. */
int qref_act_quant_f16(const uint16_t *x, int64_t rows, int64_t k, int round_mode,
                       int8_t *codes, float *scales, int32_t *rowsums)
{
    if (!x || !codes || !scales || rows < 0 || k <= 0) return -1;
#pragma omp parallel
    {
        float *row = (float *)malloc(sizeof(float) * (size_t)k);
#pragma omp for schedule(static)
        for (int64_t m = 0; m < rows; m++) {
            for (int64_t i = 0; i < k; i++) row[i] = qref_half_to_float(x[m * k + i]);
            scales[m] = quant_row(row, k, round_mode, codes + m * k, rowsums ? rowsums + m : NULL);
        }
        free(row);
    }
    return 0;
}

/* Integer GEMM acc[m][n] = sum_k codes_a[m][k] * codes_w[k][n] (src/npu.rs:1111-1116).
 * Blocked 16 rows x 256 columns so each 256-byte weight segment is reused from L1 by 16
 * rows; integer sums are exact, so the blocking does not change any result. */
int qref_int_gemm(const int8_t *qa, int64_t rows, int64_t k, const int8_t *w_kn, int64_t n,
                  int32_t *acc)
{
    if (!qa || !w_kn || !acc || rows < 0 || k <= 0 || n <= 0) return -1;
    enum { RB = 16, NB = 256 };
    int64_t rblocks = (rows + RB - 1) / RB, nblocks = (n + NB - 1) / NB;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t rb = 0; rb < rblocks; rb++) {
        for (int64_t b = 0; b < nblocks; b++) {
            int32_t tile[RB][NB];
            int64_t r0 = rb * RB, r1 = r0 + RB < rows ? r0 + RB : rows;
            int64_t n0 = b * NB, n1 = n0 + NB < n ? n0 + NB : n, w = n1 - n0;
            memset(tile, 0, sizeof(tile));
            for (int64_t kk = 0; kk < k; kk++) {
                const int8_t *wr = w_kn + kk * n + n0;
                for (int64_t r = r0; r < r1; r++) {
                    int32_t q = qa[r * k + kk];
                    if (q == 0) continue;
                    int32_t *t = tile[r - r0];
                    for (int64_t j = 0; j < w; j++) t[j] += q * (int32_t)wr[j];
                }
            }
            for (int64_t r = r0; r < r1; r++)
                memcpy(acc + r * n + n0, tile[r - r0], sizeof(int32_t) * (size_t)w);
        }
    }
    return 0;
}

/* Dequant epilogue y = (f32(acc) * s_a) * s_w (src/npu.rs:1117). */
int qref_dequant(const int32_t *acc, int64_t rows, int64_t n, const float *sa, const float *sw,
                 float *y)
{
    if (!acc || !sa || !sw || !y) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < rows; m++) {
        float s = sa[m];
        for (int64_t j = 0; j < n; j++) {
            float t = (float)acc[m * n + j] * s;   /* two separately rounded products */
            y[m * n + j] = t * sw[j];
        }
    }
    return 0;
}

/* The whole oracle (src/npu.rs:1097-1121): f32 input [rows][k], QuantMatrix codes [k][n]
 * and scales [n] -> f32 output [rows][n]. acc_out (may be NULL) receives the i32 sums. */
int qref_linear_f32(const int8_t *w_kn, const float *w_scales, int64_t k, int64_t n,
                    const float *x, int64_t rows, int round_mode, float *y, int32_t *acc_out)
{
    if (!w_kn || !w_scales || !x || !y || rows < 0 || k <= 0 || n <= 0) return -1;
    if (rows == 0) return 0;
    int8_t *qa = (int8_t *)malloc((size_t)(rows * k));
    float *sa = (float *)malloc(sizeof(float) * (size_t)rows);
    int32_t *acc = acc_out ? acc_out : (int32_t *)malloc(sizeof(int32_t) * (size_t)(rows * n));
    if (!qa || !sa || !acc) { free(qa); free(sa); if (!acc_out) free(acc); return -2; }
    qref_act_quant_f32(x, rows, k, round_mode, qa, sa, NULL);
    qref_int_gemm(qa, rows, k, w_kn, n, acc);
    qref_dequant(acc, rows, n, sa, w_scales, y);
    free(qa); free(sa);
    if (!acc_out) free(acc);
    return 0;
}

/* Same with fp16 input bits (widened exactly). */
int qref_linear_f16(const int8_t *w_kn, const float *w_scales, int64_t k, int64_t n,
                    const uint16_t *x, int64_t rows, int round_mode, float *y, int32_t *acc_out)
{
    if (!w_kn || !w_scales || !x || !y || rows < 0 || k <= 0 || n <= 0) return -1;
    if (rows == 0) return 0;
    int8_t *qa = (int8_t *)malloc((size_t)(rows * k));
    float *sa = (float *)malloc(sizeof(float) * (size_t)rows);
    int32_t *acc = acc_out ? acc_out : (int32_t *)malloc(sizeof(int32_t) * (size_t)(rows * n));
    if (!qa || !sa || !acc) { free(qa); free(sa); if (!acc_out) free(acc); return -2; }
    qref_act_quant_f16(x, rows, k, round_mode, qa, sa, NULL);
    qref_int_gemm(qa, rows, k, w_kn, n, acc);
    qref_dequant(acc, rows, n, sa, w_scales, y);
    free(qa); free(sa);
    if (!acc_out) free(acc);
    return 0;
}

/* SwiGLU expectation of src/npu.rs:1202-1208 over y [rows][n]:
 * mid[r][j] = gate / (1 + exp(-gate)) * up, gate = y[r][j], up = y[r][n/2 + j]. */
int qref_swiglu(const float *y, int64_t rows, int64_t n, float *mid)
{
    if (!y || !mid || n % 2) return -1;
    int64_t h = n / 2;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        for (int64_t j = 0; j < h; j++) {
            float gate = y[r * n + j];
            float up = y[r * n + h + j];
            mid[r * h + j] = gate / (1.0f + expf(-gate)) * up;
        }
    }
    return 0;
}

int qref_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void qref_set_threads(int n)
{
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
