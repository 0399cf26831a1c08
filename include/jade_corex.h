/* Fixed-shape GEMM plan ABI v1 - the drop-in for the reference's cuBLAS provider.
 *
 * Replaces native/jade_corex.h:1-37 of the reference (loaded by name through
 * dlopen/dlsym in src/corex.rs:55-84, selected by --corex-library in
 * src/main.rs:25,86). Same symbols, signatures, error codes and messages; the
 * plan runs on this library's sm_100a kernels instead of cuBLAS:
 *   precision 0: FP32 A, B, C - the FFMA GEMM (FP32 products summed in k order);
 *   precision 1: A, B rounded to FP16 on upload (round-to-nearest-even), FP32
 *                accumulation and C - the tcgen05 tensor-core GEMM.
 *
 * Contexts require serial access. Every matrix is dense, row-major:
 * C[m,n] = A[m,k] . B[k,n].
 * 0 = success; 1 = invalid input/state; 2 = runtime; 3 = BLAS (not produced:
 * no BLAS is involved); 4 = allocation.
 * Errors are copied into caller storage and NUL-terminated when capacity > 0.
 * The caller retains all host arrays. Upload/run/download synchronize before
 * returning; no caller-owned pointer is retained. Destroy is null-safe. */
#ifndef JADE_COREX_H
#define JADE_COREX_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define JC_API __attribute__((visibility("default")))
#else
#define JC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* reference native/jade_corex.h:17 - returns 1 */
JC_API uint32_t jade_corex_abi_version(void);
/* reference native/jade_corex.h:18-19 - dimensions 1..INT_MAX, device >= 0,
 * precision 0 or 1; allocates A, B, C on the device and compiles the kernel */
JC_API int jade_corex_create(uint32_t m, uint32_t n, uint32_t k, int device, uint32_t precision, void **out, char *err,
                             size_t cap);
/* reference native/jade_corex.h:20-21 - exact element counts m*k and k*n */
JC_API int jade_corex_upload(void *ctx, const float *a, size_t a_len, const float *b, size_t b_len, char *err,
                             size_t cap);
/* reference native/jade_corex.h:22-24 - elapsed_ms is the total GPU-event time of
 * all iterations, excluding transfers */
JC_API int jade_corex_run(void *ctx, uint32_t iterations, double *elapsed_ms, char *err, size_t cap);
/* reference native/jade_corex.h:25-26 - exact element count m*n, after a run */
JC_API int jade_corex_download(void *ctx, float *out, size_t out_len, char *err, size_t cap);
/* reference native/jade_corex.h:27-28 - "device=.. name=.. memory_bytes=..
 * multiprocessors=.. runtime_api=.. driver_api=.. blas_api=0 precision=..
 * kernel=.." (blas_api is 0: no BLAS library is used) */
JC_API int jade_corex_device_info(void *ctx, char *out, size_t out_cap, char *err, size_t cap);
/* reference native/jade_corex.h:29 */
JC_API void jade_corex_destroy(void *ctx);

#ifdef __cplusplus
}
#endif
#endif
