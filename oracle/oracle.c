/*
 * TEST INFRASTRUCTURE ONLY: FP64 CPU oracle (see oracle.h). Restates the
 * reference's CPU reference arithmetic in plain C; it is the checker for the
 * CUDA path and the timed CPU baseline, never part of the product.
 */
#include "oracle.h"
#include <math.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int or_omp_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

static int clamp_threads(int threads) { return threads < 1 ? 1 : threads; }

/* workloads.rs:17-27 */
void or_values(float *out, size_t len, uint32_t seed, float scale) {
    uint32_t s = seed;
    for (size_t i = 0; i < len; ++i) {
        s ^= s << 13;
        s ^= s >> 17;
        s ^= s << 5;
        out[i] = ((float)(s >> 8) / 16777216.0f * 2.0f - 1.0f) * scale;
    }
}

/* workloads.rs:28-32 */
void or_dot(size_t m, size_t n, size_t k, const double *a, const double *b, double *out) {
    for (size_t i = 0; i < m * n; ++i) {
        double s = 0.0;
        for (size_t p = 0; p < k; ++p) s += a[i / n * k + p] * b[p * n + i % n];
        out[i] = s;
    }
}

/* metal_lab.rs:18-31: for row { for p { av = a[row,p]; for col { out[row,col] += av*b[p,col] } } } */
void or_gemm_reference(size_t m, size_t n, size_t k, const float *a, const float *b,
                       double *out, int threads) {
    memset(out, 0, m * n * sizeof(double));
    long long rows = (long long)m;
#pragma omp parallel for num_threads(clamp_threads(threads)) schedule(static)
    for (long long row = 0; row < rows; ++row) {
        double *o = out + (size_t)row * n;
        for (size_t p = 0; p < k; ++p) {
            const double av = (double)a[(size_t)row * k + p];
            const float *br = b + p * n;
            for (size_t col = 0; col < n; ++col) o[col] += av * (double)br[col];
        }
    }
}

void or_gemm_rows(size_t n, size_t k, const float *a, const float *b, const int64_t *rows,
                  size_t nrows, double *out, int threads) {
    memset(out, 0, nrows * n * sizeof(double));
    long long cnt = (long long)nrows;
#pragma omp parallel for num_threads(clamp_threads(threads)) schedule(static)
    for (long long r = 0; r < cnt; ++r) {
        const size_t row = (size_t)rows[r];
        double *o = out + (size_t)r * n;
        for (size_t p = 0; p < k; ++p) {
            const double av = (double)a[row * k + p];
            const float *br = b + p * n;
            for (size_t col = 0; col < n; ++col) o[col] += av * (double)br[col];
        }
    }
}

/* ir.rs:524-530 (naive) and ir.rs:531-557 (register32): each output is
 * acc = fmaf(a[row,p], b[p,col], acc) for p = 0..k-1, acc starting at 0.0f. */
void or_gemm_fp32_sequential(size_t m, size_t n, size_t k, const float *a, const float *b,
                             float *out, int threads) {
    long long rows = (long long)m;
#pragma omp parallel for num_threads(clamp_threads(threads)) schedule(static)
    for (long long row = 0; row < rows; ++row) {
        for (size_t col = 0; col < n; ++col) {
            float acc = 0.0f;
            for (size_t p = 0; p < k; ++p) acc = fmaf(a[(size_t)row * k + p], b[p * n + col], acc);
            out[(size_t)row * n + col] = acc;
        }
    }
}

/* validation.rs:35-91 */
int or_validation_check(size_t m, size_t n, size_t k, const float *a, const float *b,
                        const float *out, size_t budget, int fp16, double coef_override,
                        or_validation *r) {
    memset(r, 0, sizeof(*r));
    r->first_bad_index = -1;
    if (!budget || !m || !n || !k) return 3;
    const size_t len = m * n;
    r->total_elements = len;
    for (size_t i = 0; i < len; ++i) {
        if (!isfinite(out[i])) {
            r->first_bad_index = (int64_t)i;
            return 2;
        }
    }
    const size_t count = budget < len ? budget : len;
    r->checked_elements = count;
    double coefficient;
    if (coef_override > 0) coefficient = coef_override;
    else if (fp16) coefficient = 0.0012;
    else {
        coefficient = (double)k * (double)1.1920928955078125e-07 * 2.0;
        if (coefficient < 2e-6) coefficient = 2e-6;
    }
    for (size_t sample = 0; sample < count; ++sample) {
        const size_t idx = count <= 1 ? 0 : sample * (len - 1) / (count - 1);
        const size_t row = idx / n, col = idx % n;
        double expected = 0.0, sum_abs = 0.0;
        for (size_t inner = 0; inner < k; ++inner) {
            const double product = (double)a[row * k + inner] * (double)b[inner * n + col];
            expected += product;
            sum_abs += fabs(product);
        }
        const double error = fabs((double)out[idx] - expected);
        const double tolerance = 2e-5 + coefficient * sum_abs;
        if (error > r->max_abs_error) r->max_abs_error = error;
        if (error / tolerance > r->max_scaled_error) r->max_scaled_error = error / tolerance;
        if (sum_abs > 0 && error / sum_abs > r->max_magnitude_error) r->max_magnitude_error = error / sum_abs;
        if (!(error <= tolerance)) {
            r->first_bad_index = (int64_t)idx;
            return 1;
        }
    }
    return 0;
}

/* workloads.rs:224-243 */
int or_compare(const float *actual, const double *expected, size_t n, double atol, double rtol,
               or_check *r) {
    memset(r, 0, sizeof(*r));
    r->elements = n;
    r->first_bad_index = -1;
    for (size_t i = 0; i < n; ++i) {
        const double a = (double)actual[i], e = expected[i];
        if (!isfinite(a) || !isfinite(e)) {
            r->first_bad_index = (int64_t)i;
            return 2;
        }
        const double error = fabs(a - e);
        if (!(error <= atol + rtol * fabs(e))) {
            r->first_bad_index = (int64_t)i;
            if (error > r->max_abs_error) r->max_abs_error = error;
            return 1;
        }
        if (error > r->max_abs_error) r->max_abs_error = error;
        const double denom = fabs(e) > atol ? fabs(e) : atol;
        if (error / denom > r->max_relative_error) r->max_relative_error = error / denom;
    }
    return 0;
}

/* workloads.rs:36-43 */
double or_sigmoid(double x) {
    if (x >= 0.0) return 1.0 / (1.0 + exp(-x));
    const double e = exp(x);
    return e / (1.0 + e);
}

/* workloads.rs:96-100 */
void or_swiglu(size_t n, const float *gate, const float *up, double *out) {
    for (size_t i = 0; i < n; ++i) {
        const double g = (double)gate[i];
        out[i] = g * or_sigmoid(g) * (double)up[i];
    }
}

/* workloads.rs:44-55 */
void or_normalize(size_t rows, size_t cols, const float *x, const float *weight, double eps,
                  double *out, int threads) {
    long long nr = (long long)rows;
#pragma omp parallel for num_threads(clamp_threads(threads)) schedule(static)
    for (long long row = 0; row < nr; ++row) {
        const size_t off = (size_t)row * cols;
        double square = 0.0;
        for (size_t c = 0; c < cols; ++c) square += (double)x[off + c] * (double)x[off + c];
        const double inv = 1.0 / sqrt(square / (double)cols + eps);
        for (size_t c = 0; c < cols; ++c) out[off + c] = (double)x[off + c] * inv * (double)weight[c];
    }
}

/* workloads.rs:134-141 */
void or_softmax(size_t rows, size_t cols, const float *x, double *out, int threads) {
    long long nr = (long long)rows;
#pragma omp parallel for num_threads(clamp_threads(threads)) schedule(static)
    for (long long row = 0; row < nr; ++row) {
        const float *s = x + (size_t)row * cols;
        float mx = -INFINITY;
        for (size_t c = 0; c < cols; ++c) mx = fmaxf(mx, s[c]);
        const double max = (double)mx;
        double sum = 0.0;
        for (size_t c = 0; c < cols; ++c) sum += exp((double)s[c] - max);
        for (size_t c = 0; c < cols; ++c) out[(size_t)row * cols + c] = exp((double)s[c] - max) / sum;
    }
}

/* workloads.rs:58-75 and 76-90 */
void or_axpy(size_t n, float alpha, const float *a, const float *b, double *out) {
    for (size_t i = 0; i < n; ++i) out[i] = (double)alpha * (double)a[i] + (double)b[i];
}
void or_axpy_fp32(size_t n, float alpha, const float *a, const float *b, float *out) {
    for (size_t i = 0; i < n; ++i) out[i] = fmaf(alpha, a[i], b[i]);
}
void or_add_fp32(size_t n, const float *a, const float *b, float *out) {
    for (size_t i = 0; i < n; ++i) {
        volatile float s = a[i] + b[i]; /* FP32 add, no widening */
        out[i] = s;
    }
}

/* metal_lab.rs:33-73, one (head, row). When mag is given it also receives, per
 * output element d, sum_col p[col]*|v[col][d]| (p the softmax weights): the
 * magnitude that scales the rounding error of a weighted sum (validation.rs:35-91
 * uses sum|a*b| the same way for GEMM). */
static void attention_one(size_t seq, size_t dim, int causal, const float *qh, const float *kh,
                          const float *vh, size_t row, double *scores, double *o, double *mag) {
    const size_t count = causal ? row + 1 : seq;
    const double sd = sqrt((double)dim);
    for (size_t col = 0; col < count; ++col) {
        double s = 0.0;
        for (size_t d = 0; d < dim; ++d) s += (double)qh[row * dim + d] * (double)kh[col * dim + d];
        scores[col] = s / sd;
    }
    double max = -INFINITY;
    for (size_t col = 0; col < count; ++col) max = fmax(max, scores[col]);
    for (size_t col = 0; col < count; ++col) scores[col] = exp(scores[col] - max);
    double denom = 0.0;
    for (size_t col = 0; col < count; ++col) denom += scores[col];
    for (size_t d = 0; d < dim; ++d) {
        double acc = 0.0, size = 0.0;
        for (size_t col = 0; col < count; ++col) {
            const double p = scores[col] / denom, v = (double)vh[col * dim + d];
            acc += p * v;
            size += p * fabs(v);
        }
        o[d] = acc;
        if (mag) mag[d] = size;
    }
}

#include <stdlib.h>
void or_attention(size_t bh, size_t seq, size_t dim, int causal, const float *q, const float *k,
                  const float *v, double *out, int threads) {
    long long total = (long long)(bh * seq);
#pragma omp parallel num_threads(clamp_threads(threads))
    {
        double *scores = (double *)malloc(seq * sizeof(double));
#pragma omp for schedule(dynamic, 16)
        for (long long t = 0; t < total; ++t) {
            const size_t h = (size_t)t / seq, row = (size_t)t % seq;
            const size_t base = h * seq * dim;
            attention_one(seq, dim, causal, q + base, k + base, v + base, row, scores,
                          out + base + row * dim, NULL);
        }
        free(scores);
    }
}

void or_attention_rows_bound(size_t seq, size_t dim, int causal, const float *q, const float *k,
                             const float *v, const int64_t *bh_idx, const int64_t *row_idx,
                             size_t npairs, double *out, double *mag, int threads) {
    long long total = (long long)npairs;
#pragma omp parallel num_threads(clamp_threads(threads))
    {
        double *scores = (double *)malloc(seq * sizeof(double));
#pragma omp for schedule(dynamic, 1)
        for (long long t = 0; t < total; ++t) {
            const size_t base = (size_t)bh_idx[t] * seq * dim;
            attention_one(seq, dim, causal, q + base, k + base, v + base, (size_t)row_idx[t],
                          scores, out + (size_t)t * dim, mag ? mag + (size_t)t * dim : NULL);
        }
        free(scores);
    }
}

void or_attention_rows(size_t seq, size_t dim, int causal, const float *q, const float *k,
                       const float *v, const int64_t *bh_idx, const int64_t *row_idx,
                       size_t npairs, double *out, int threads) {
    or_attention_rows_bound(seq, dim, causal, q, k, v, bh_idx, row_idx, npairs, out, NULL, threads);
}

float or_bf16_to_f32(uint16_t h);
uint16_t or_f32_to_bf16(float x);

/* workloads.rs:466-479 for a subset of token rows. round_h != 0 rounds the
 * activation h = silu(g)*u to BF16 before the down projection, the point where a
 * BF16 pipeline stores it; mag (optional) receives per output element
 * sum_p |h_p*wd[p][c]| + |x_c|, the magnitude of the down projection and
 * residual sums. */
void or_mlp_rows_ex(size_t width, size_t hidden, const float *x, const float *norm_weight,
                    const float *wg, const float *wu, const float *wd, double eps,
                    const int64_t *rows, size_t nrows, int round_h, double *out, double *mag,
                    int threads) {
    long long cnt = (long long)nrows;
#pragma omp parallel num_threads(clamp_threads(threads))
    {
        double *nrm = (double *)malloc(width * sizeof(double));
        double *g = (double *)malloc(hidden * sizeof(double));
        double *u = (double *)malloc(hidden * sizeof(double));
#pragma omp for schedule(dynamic, 1)
        for (long long r = 0; r < cnt; ++r) {
            const float *xr = x + (size_t)rows[r] * width;
            double square = 0.0;
            for (size_t c = 0; c < width; ++c) square += (double)xr[c] * (double)xr[c];
            const double inv = 1.0 / sqrt(square / (double)width + eps);
            for (size_t c = 0; c < width; ++c) nrm[c] = (double)xr[c] * inv * (double)norm_weight[c];
            for (size_t j = 0; j < hidden; ++j) { g[j] = 0.0; u[j] = 0.0; }
            /* dot(m,h,w): output j = sum_p nrm[p]*W[p*h+j], p ascending */
            for (size_t p = 0; p < width; ++p) {
                const double a = nrm[p];
                const float *wgr = wg + p * hidden, *wur = wu + p * hidden;
                for (size_t j = 0; j < hidden; ++j) {
                    g[j] += a * (double)wgr[j];
                    u[j] += a * (double)wur[j];
                }
            }
            for (size_t j = 0; j < hidden; ++j) {
                g[j] = g[j] * or_sigmoid(g[j]) * u[j];
                if (round_h) g[j] = (double)or_bf16_to_f32(or_f32_to_bf16((float)g[j]));
            }
            double *o = out + (size_t)r * width;
            double *mg = mag ? mag + (size_t)r * width : NULL;
            for (size_t c = 0; c < width; ++c) o[c] = 0.0;
            if (mg)
                for (size_t c = 0; c < width; ++c) mg[c] = fabs((double)xr[c]);
            for (size_t p = 0; p < hidden; ++p) {
                const double a = g[p];
                const float *wdr = wd + p * width;
                for (size_t c = 0; c < width; ++c) o[c] += a * (double)wdr[c];
                if (mg)
                    for (size_t c = 0; c < width; ++c) mg[c] += fabs(a * (double)wdr[c]);
            }
            for (size_t c = 0; c < width; ++c) o[c] += (double)xr[c];
        }
        free(nrm);
        free(g);
        free(u);
    }
}

void or_mlp_rows(size_t width, size_t hidden, const float *x, const float *norm_weight,
                 const float *wg, const float *wu, const float *wd, double eps,
                 const int64_t *rows, size_t nrows, double *out, int threads) {
    or_mlp_rows_ex(width, hidden, x, norm_weight, wg, wu, wd, eps, rows, nrows, 0, out, NULL, threads);
}

/* IEEE round-to-nearest-even narrowing, restated from the binary formats. */
uint16_t or_f32_to_bf16(float x) {
    uint32_t bits;
    memcpy(&bits, &x, 4);
    if ((bits & 0x7f800000u) == 0x7f800000u && (bits & 0x7fffffu)) return (uint16_t)((bits >> 16) | 0x40u);
    const uint32_t lsb = (bits >> 16) & 1u;
    bits += 0x7fffu + lsb;
    return (uint16_t)(bits >> 16);
}
float or_bf16_to_f32(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}
void or_round_bf16_array(float *x, size_t n) {
    for (size_t i = 0; i < n; ++i) x[i] = or_bf16_to_f32(or_f32_to_bf16(x[i]));
}

/* binary32 -> binary16 RNE: scale into the half range, then round the dropped bits. */
uint16_t or_f32_to_f16(float x) {
    uint32_t bits;
    memcpy(&bits, &x, 4);
    const uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    const uint32_t ex = (bits >> 23) & 0xffu, frac = bits & 0x7fffffu;
    if (ex == 0xffu) return (uint16_t)(sign | (frac ? 0x7e00u : 0x7c00u));
    const int e = (int)ex - 127;
    if (e > 15) return (uint16_t)(sign | 0x7c00u);
    if (e < -25) return sign;
    uint32_t sig, drop, out_base;
    if (e >= -14) { /* normal half */
        sig = frac;
        drop = 13;
        out_base = (uint32_t)(e + 15) << 10;
    } else { /* subnormal half: value = sig * 2^-24 with sig = (1.frac) >> (-e-1) */
        sig = frac | 0x800000u;
        drop = (uint32_t)(-e - 1);
        out_base = 0;
    }
    const uint32_t kept = sig >> drop;
    const uint32_t rem = sig & ((1u << drop) - 1u), half = 1u << (drop - 1);
    const uint32_t up = (rem > half) || (rem == half && (kept & 1u));
    return (uint16_t)(sign | (out_base + kept + up)); /* carries into exponent/inf are correct */
}
float or_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t ex = (h >> 10) & 31u, man = h & 1023u;
    float v;
    if (ex == 0) v = ldexpf((float)man, -24);
    else if (ex == 31) v = man ? NAN : INFINITY;
    else v = ldexpf(1.0f + (float)man / 1024.0f, (int)ex - 15);
    uint32_t bits;
    memcpy(&bits, &v, 4);
    bits |= sign;
    memcpy(&v, &bits, 4);
    return v;
}
