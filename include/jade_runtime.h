/*
 * jade_runtime.h - C ABI of the B200 (sm_100a) Jade Compute runtime,
 * libjade_runtime.so.
 *
 * ABI 1 is the reference's native runtime bridge, unchanged: same symbols,
 * signatures, error codes and semantics as native/jade_runtime_corex.h:9-31
 * (implementation native/jade_runtime_corex.cpp:81-224). A caller written for
 * that bridge (src/runtime/corex.rs:206-320, which dlopens it and checks
 * jr_version() == 1) loads this library unchanged.
 *
 * ABI 2 (jr2_version() == 2) adds what the reference's Rust host does above the
 * bridge (src/runtime/ir.rs validation/bindings/emission, corex.rs:439-612
 * compile/execute with full-batch binding validation) and what the B200 build
 * needs beyond it: built-in sm_100a kernels selected from the JSON KernelSpec,
 * a buffer registry for ownership/length/alias checks, per-job device timing,
 * CUDA-graph replay of an ordered batch, host-pinned transfer jobs, and an NCCL
 * communicator with an all-reduce job.
 *
 * Error convention (native/jade_runtime_corex.cpp:15-29): 0 ok, 1 invalid input
 * or state, 2 CUDA runtime error, 3 allocation failure, plus 4 = a device-side
 * bounded wait expired or a collective timed out/aborted. Messages are copied
 * into (err, cap) and NUL-terminated. Contexts require serial access.
 */
#ifndef JADE_RUNTIME_H
#define JADE_RUNTIME_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define JR_API __attribute__((visibility("default")))
#else
#define JR_API
#endif

#define JR_OK 0
#define JR_EINVAL 1
#define JR_ECUDA 2
#define JR_ENOMEM 3
#define JR_ETIMEOUT 4

/* ----------------------------- ABI 1 ---------------------------------- */
/* native/jade_runtime_corex.h:9-14 */
typedef int (*jr_launch_fn)(void *stream, void **buffers);
typedef struct jr_job {
    jr_launch_fn launch;
    void **buffers;
    size_t buffer_count;
} jr_job;

/* native/jade_runtime_corex.h:18 - returns 1. */
JR_API uint32_t jr_version(void);
/* native/jade_runtime_corex.h:19 - one device, one non-blocking stream, timing events. */
JR_API int jr_create(int device, void **out, char *err, size_t cap);
/* native/jade_runtime_corex.h:20 - synchronises, releases every registered buffer. */
JR_API void jr_destroy(void *ctx);
/* native/jade_runtime_corex.h:21 - "device=%d name=%s memory_bytes=%llu runtime_api=%d driver_api=%d". */
JR_API int jr_info(void *ctx, char *out, size_t out_cap, char *err, size_t cap);
/* native/jade_runtime_corex.h:22 - zero-filled device allocation. */
JR_API int jr_alloc(void *ctx, size_t bytes, void **out, char *err, size_t cap);
/* native/jade_runtime_corex.h:23 - synchronises the context stream first. */
JR_API void jr_free(void *ctx, void *ptr);
/* native/jade_runtime_corex.h:24-27 - synchronous exact transfers. */
JR_API int jr_upload(void *ctx, void *device_ptr, const void *host_ptr, size_t bytes, char *err, size_t cap);
JR_API int jr_download(void *ctx, const void *device_ptr, void *host_ptr, size_t bytes, char *err, size_t cap);
/* native/jade_runtime_corex.h:28-31 - ordered jobs replayed `repeats` times on the
 * context stream; one event pair brackets the whole sequence. */
JR_API int jr_execute(void *ctx, const jr_job *jobs, size_t job_count, uint32_t repeats, double *gpu_ms,
               char *err, size_t cap);

/* ----------------------------- ABI 2 ---------------------------------- */
JR_API uint32_t jr2_version(void);
/* Number of visible CUDA devices (0 when there is no driver or GPU). */
JR_API int jr_device_count(void);

/* KernelSpec JSON (src/runtime/ir.rs:6-84 serde form plus optional extension
 * fields). These run on any host; no device is touched. */
/* ir.rs:193-268 */
JR_API int jr_spec_validate(const char *spec_json, char *err, size_t cap);
/* ir.rs:269-339, JSON array of {name, elements, write, dtype}. */
JR_API int jr_spec_bindings(const char *spec_json, char *out, size_t out_cap, char *err, size_t cap);
/* ir.rs:340-367: element counts and buffer identities, one per binding. */
JR_API int jr_spec_validate_bindings(const char *spec_json, const uint64_t *lengths, const uint64_t *ids,
                              size_t count, char *err, size_t cap);
/* ir.rs:368-420, JSON {grid, block} of the reference's emitted kernel. */
JR_API int jr_spec_launch(const char *spec_json, char *out, size_t out_cap, char *err, size_t cap);
/* ir.rs:450-575 (target "corex", byte-exact) or "cuda" (this backend's sm_100a
 * lowering of elementwise expressions). Writes the NUL-terminated text into out
 * when it fits; *needed receives strlen+1 either way. */
JR_API int jr_spec_emit(const char *spec_json, const char *target, char *out, size_t out_cap, size_t *needed,
                 char *err, size_t cap);
/* serde round-trip of a spec (canonical field order). */
JR_API int jr_spec_canonical(const char *spec_json, char *out, size_t out_cap, char *err, size_t cap);

/* Built-in sm_100a kernels (replaces corex.rs:439-542 compile for this backend).
 * A kernel belongs to the context that compiled it. */
typedef struct jr_kernel jr_kernel;
JR_API int jr_compile(void *ctx, const char *spec_json, jr_kernel **out, char *err, size_t cap);
JR_API void jr_kernel_release(jr_kernel *kernel);
/* JSON {name, spec, bindings, path} describing the implementation chosen. */
JR_API int jr_kernel_info(jr_kernel *kernel, char *out, size_t out_cap, char *err, size_t cap);

typedef struct jr_dispatch {
    jr_kernel *kernel;
    void **buffers;
    size_t buffer_count;
} jr_dispatch;

#define JR_EXEC_GRAPH 1u /* capture one pass as a CUDA graph, replay it `repeats` times */
/* Dependency-scheduled streams (not with JR_EXEC_GRAPH): host-to-device copy jobs
 * run on a transfer-in stream, device-to-host copy jobs on a transfer-out stream,
 * all_reduce jobs on a collective stream (so that the all-reduce of one row block
 * overlaps the kernels of the next), every other job on the context stream;
 * each job first waits for the jobs it
 * conflicts with on its bindings (read after write, write after write, write after
 * read), so results equal in-order execution while transfers overlap compute and
 * each other (e.g. one repeat's result read-back with the next repeat's uploads).
 * No counterpart in the reference (its execute is strictly in order). */
#define JR_EXEC_STREAMS 2u

/* Validates every job (context ownership, registered buffers, exact byte sizes,
 * output aliasing - corex.rs:557-569, ir.rs:340-367) before any work is
 * submitted, then runs jobs x repeats in order on the context stream.
 * gpu_ms: event time of the whole sequence. job_ms (optional, job_count entries,
 * not with JR_EXEC_GRAPH): per-job event time summed over repeats. */
JR_API int jr_execute2(void *ctx, const jr_dispatch *jobs, size_t job_count, uint32_t repeats, uint32_t flags,
                double *gpu_ms, double *job_ms, char *err, size_t cap);

/* Registry queries and pinned host memory for transfer jobs (spec op "copy"). */
JR_API int jr_buffer_bytes(void *ctx, const void *ptr, size_t *bytes);
JR_API int jr_host_alloc(void *ctx, size_t bytes, void **out, char *err, size_t cap);
JR_API void jr_host_free(void *ctx, void *ptr);

/* Collectives over NCCL (loaded at first use). One process per GPU:
 * jr_comm_unique_id on rank 0, broadcast the 128 bytes, jr_comm_init on every
 * rank. One process, many GPUs: jr_comm_init_all. timeout_ms bounds each
 * execute that contains an all_reduce job (0 = 60 s); on expiry the communicator
 * is aborted and JR_ETIMEOUT returned. */
JR_API int jr_comm_unique_id(unsigned char id[128], char *err, size_t cap);
JR_API int jr_comm_init(void *ctx, int nranks, int rank, const unsigned char id[128], uint32_t timeout_ms,
                 char *err, size_t cap);
JR_API int jr_comm_init_all(void **ctxs, int count, uint32_t timeout_ms, char *err, size_t cap);
JR_API int jr_comm_destroy(void *ctx);

/* Peer memory over NVLink for the collectives that run without NCCL (the gemm
 * "scatter" epilogue, shard_reduce, shard_gather). No counterpart in the
 * reference (it has no multi-device code). One process per GPU: every rank
 * exports the buffer with jr_peer_handle, the host gathers the 64-byte handles
 * in rank order, and every rank calls jr_peer_attach with all of them; each
 * rank's buffer must have the same size. nranks 1..8; with nranks 1 no handle is
 * opened. The mappings close when the context is destroyed. */
JR_API int jr_peer_handle(void *ctx, const void *ptr, unsigned char handle[64], char *err, size_t cap);
JR_API int jr_peer_attach(void *ctx, const void *ptr, const unsigned char *handles, int nranks, int rank, char *err,
                          size_t cap);

/* Allocation-free TF32 GEMM: out[m,n] (FP32) = a[m,k] . b[k,n], a and b FP32
 * row-major, computed on the tensor cores in TF32 with FP32 accumulation - the
 * same kernels as a compiled {"op":"gemm","dtype":"tf32"} spec with the default
 * b_layout "kn". No counterpart in the reference.
 *
 * For callers that cannot allocate device memory when they call: code running
 * inside a host framework that owns every device allocation through its own
 * pool, or a latency-critical loop where cudaMalloc's implicit device-wide
 * synchronisation is not acceptable. The compiled path obtains its B-transpose
 * workspace with cudaMalloc; this entry point instead uses a static 16 MiB
 * device array built into the library, so it calls no cudaMalloc, cudaFree or
 * other allocating routine, and needs no jr_create context.
 *
 *  - Limit: k * n <= 4,194,304 elements (16 MiB of FP32); larger shapes are
 *    rejected with JR_EINVAL and a message. k must be a multiple of 4 and a, b
 *    and out 16-byte aligned (rejected with JR_EINVAL before any launch
 *    otherwise). Every GPU that loads the library holds the 16 MiB until the
 *    process exits.
 *  - Runs on the current device. The first call on each device performs a
 *    one-time set-up there (it looks up the array's device address); make that
 *    first call before any stream capture.
 *  - Enqueues on `stream` (NULL = the legacy default stream) and synchronises
 *    that stream before returning (the error word is read back on it too, so
 *    no other stream is synchronised); returns JR_ETIMEOUT if a device-side
 *    bounded wait expired.
 *  - Every call on a device shares the one array and it keeps the last call's
 *    contents: calls whose GPU work overlaps (several host threads or streams at
 *    once) race on it and must be serialised by the caller. */
JR_API int jr_gemm_tf32_kn_noalloc(const float *a, const float *b, float *out, uint32_t m, uint32_t n, uint32_t k,
                                   void *stream, char *err, size_t cap);

#ifdef __cplusplus
}
#endif
#endif
