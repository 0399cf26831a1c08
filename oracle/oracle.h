/*
 * TEST INFRASTRUCTURE ONLY. This is the CPU oracle: an FP64 restatement of the
 * reference's independent CPU references. Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg may load it, and only as a checker or as the
 * timed CPU baseline. No product code links it.
 *
 * Every function names the reference file:line whose behaviour it restates
 * (paths are relative to the reference project root, demier-demier/jade-compute).
 * Parity pins: the golden vectors in the reference's own unit tests
 * (validation.rs:102-112, metal_lab.rs:471-484, metal.rs:820-822,893-912,971-985,
 * workloads.rs:530-539) and the exhaustive FP16 test (native/fp16_test.cpp),
 * checked by tests/test_oracle.py.
 */
#ifndef JADE_ORACLE_H
#define JADE_ORACLE_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* workloads.rs:17-27: xorshift32 (<<13, >>17, <<5) mapped to ((s>>8)/2^24*2-1)*scale.
 * validation.rs:5-21 is the same stream with scale 1. */
void or_values(float *out, size_t len, uint32_t seed, float scale);

/* workloads.rs:28-32: FP64 row-major dot, out[i] = sum_p a[i/n*k+p]*b[p*n+i%n]. */
void or_dot(size_t m, size_t n, size_t k, const double *a, const double *b, double *out);

/* metal_lab.rs:18-31: FP64 GEMM from FP32 inputs, (row, p, col) traversal.
 * threads > 1 splits rows over OpenMP threads (same arithmetic per row). */
void or_gemm_reference(size_t m, size_t n, size_t k, const float *a, const float *b,
                       double *out, int threads);

/* FP64 GEMM restricted to listed rows (for sampled checks at large sizes). */
void or_gemm_rows(size_t n, size_t k, const float *a, const float *b,
                  const int64_t *rows, size_t nrows, double *out, int threads);
/* The same chain with h = silu(g)*u rounded to BF16 when round_h != 0 (where a
 * BF16 pipeline stores it), and optionally mag[r*width+c] = sum_p |h_p*wd[p][c]|
 * + |x_c|, the magnitude of the down projection and residual sums. */
void or_mlp_rows_ex(size_t width, size_t hidden, const float *x, const float *norm_weight,
                    const float *wg, const float *wu, const float *wd, double eps,
                    const int64_t *rows, size_t nrows, int round_h, double *out, double *mag,
                    int threads);

/* ir.rs:524-557: the reference's generated FP32 GEMM kernels accumulate each output
 * sequentially over p=0..k-1 with fmaf starting from 0.0f. Bit-exact restatement. */
void or_gemm_fp32_sequential(size_t m, size_t n, size_t k, const float *a, const float *b,
                             float *out, int threads);

/* validation.rs:35-91: budgeted evenly spread FP64 sampled check.
 * Returns 0 when every sample is inside 2e-5 + coef*sum|ab| (coef 0.0012 for the
 * FP16/BF16 input allowance, else max(2*k*eps32, 2e-6)); 1 on mismatch, 2 on a
 * non-finite output, 3 on bad arguments. coef_override > 0 replaces coef. */
typedef struct or_validation {
    size_t checked_elements, total_elements;
    double max_abs_error, max_scaled_error;
    int64_t first_bad_index;
    double max_magnitude_error; /* max |out - expected| / sum|a*b| over the sample */
} or_validation;
int or_validation_check(size_t m, size_t n, size_t k, const float *a, const float *b,
                        const float *out, size_t budget, int fp16, double coef_override,
                        or_validation *result);

/* workloads.rs:224-243: every element finite and |a-e| <= atol + rtol*|e|.
 * Returns 0 ok, 1 mismatch, 2 non-finite. max_rel = max err/max(|e|,atol). */
typedef struct or_check {
    size_t elements;
    double max_abs_error, max_relative_error;
    int64_t first_bad_index;
} or_check;
int or_compare(const float *actual, const double *expected, size_t n, double atol,
               double rtol, or_check *result);

/* workloads.rs:36-43 stable sigmoid; workloads.rs:96-100 g*sigmoid(g)*u. */
double or_sigmoid(double x);
void or_swiglu(size_t n, const float *gate, const float *up, double *out);

/* workloads.rs:44-55: x*inv*w with inv = 1/sqrt(sum x^2/cols + eps), FP64. */
void or_normalize(size_t rows, size_t cols, const float *x, const float *weight,
                  double eps, double *out, int threads);

/* workloads.rs:134-141: max in FP32, exp and sum in FP64. */
void or_softmax(size_t rows, size_t cols, const float *x, double *out, int threads);

/* workloads.rs:58-90: -0.375*a+b and a+b in FP64; fmaf / FP32 add are the
 * device's bit-exact targets (ir.rs:485-486). */
void or_axpy(size_t n, float alpha, const float *a, const float *b, double *out);
void or_axpy_fp32(size_t n, float alpha, const float *a, const float *b, float *out);
void or_add_fp32(size_t n, const float *a, const float *b, float *out);

/* metal_lab.rs:33-73: materialized FP64 attention, layout [batch*heads, seq, dim],
 * scale 1/sqrt(dim), causal rows see keys 0..row. */
void or_attention(size_t bh, size_t seq, size_t dim, int causal, const float *q,
                  const float *k, const float *v, double *out, int threads);
/* Same arithmetic for listed (bh, row) pairs; out is [npairs, dim]. */
void or_attention_rows(size_t seq, size_t dim, int causal, const float *q, const float *k,
                       const float *v, const int64_t *bh_idx, const int64_t *row_idx,
                       size_t npairs, double *out, int threads);
/* The same rows plus mag[t*dim+d] = sum_col p[col]*|v[col][d]| (softmax weights p):
 * the magnitude that scales the rounding error of the weighted sum. */
void or_attention_rows_bound(size_t seq, size_t dim, int causal, const float *q, const float *k,
                             const float *v, const int64_t *bh_idx, const int64_t *row_idx,
                             size_t npairs, double *out, double *mag, int threads);

/* workloads.rs:466-479: FP64 chain normalize -> gate/up dot -> g*sigmoid(g)*u ->
 * down dot -> +x for listed token rows. Weights row-major: wg, wu [width, hidden],
 * wd [hidden, width] (the reference's K x N layout). out is [nrows, width]. */
void or_mlp_rows(size_t width, size_t hidden, const float *x, const float *norm_weight,
                 const float *wg, const float *wu, const float *wd, double eps,
                 const int64_t *rows, size_t nrows, double *out, int threads);

/* Rounding helpers (IEEE RNE, own restatement). native/fp16.hpp:11-44 is the
 * reference's binary32->binary16 converter; or_f32_to_f16 matches it bit for bit
 * (NaN canonicalised to 0x7e00). */
uint16_t or_f32_to_bf16(float x);
float or_bf16_to_f32(uint16_t h);
uint16_t or_f32_to_f16(float x);
float or_f16_to_f32(uint16_t h);
void or_round_bf16_array(float *x, size_t n);

int or_omp_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
