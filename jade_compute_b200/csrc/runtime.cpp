// C ABI of the B200 runtime (include/jade_runtime.h).
//
// ABI 1 follows native/jade_runtime_corex.cpp:81-224 exactly: one device, one
// non-blocking stream, two timing events, zero-filled allocations, synchronous
// exact transfers, and an ordered execute that validates every job before it
// submits any and brackets the whole repeats x jobs sequence with one event pair.
// ABI 2 adds a buffer registry (so ownership, exact sizes and write aliasing are
// checked natively, as src/runtime/corex.rs:557-569 does in the caller), the
// JSON KernelSpec front end, built-in sm_100a kernels, per-job timing, CUDA-graph
// replay, and collectives.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <chrono>
#include <map>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <thread>

#include "../../include/jade_runtime.h"
#include "internal.hpp"

using jade::Context;

namespace {

int fail(int code, char *err, size_t cap, const char *format, ...) {
    if (err && cap) {
        va_list args;
        va_start(args, format);
        std::vsnprintf(err, cap, format, args);
        va_end(args);
        err[cap - 1] = '\0';
    }
    return code;
}
void clear(char *err, size_t cap) {
    if (err && cap) err[0] = '\0';
}
int cuda_fail(cudaError_t status, char *err, size_t cap, const char *operation) {
    return fail(JR_ECUDA, err, cap, "%s: %s (%d)", operation, cudaGetErrorString(status), static_cast<int>(status));
}
int select(Context *ctx, char *err, size_t cap) {
    if (!ctx) return fail(JR_EINVAL, err, cap, "null runtime context");
    const auto status = cudaSetDevice(ctx->device);
    return status == cudaSuccess ? 0 : cuda_fail(status, err, cap, "cudaSetDevice");
}
void destroy(Context *ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    jade::comm_destroy(ctx);
    jade::cublas_destroy(ctx);
    jade::rtc_destroy(ctx);
    for (auto &a : ctx->allocations) {
        if (a.second.host) cudaFreeHost(reinterpret_cast<void *>(a.first));
        else cudaFree(reinterpret_cast<void *>(a.first));
    }
    for (auto e : ctx->job_events) cudaEventDestroy(e);
    for (auto e : ctx->dep_events) cudaEventDestroy(e);
    if (ctx->copy_in) cudaStreamDestroy(ctx->copy_in);
    if (ctx->copy_out) cudaStreamDestroy(ctx->copy_out);
    if (ctx->err_host) cudaFreeHost(ctx->err_host);
    if (ctx->start) cudaEventDestroy(ctx->start);
    if (ctx->stop) cudaEventDestroy(ctx->stop);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
}
int copy_out(const std::string &s, char *out, size_t out_cap, char *err, size_t cap) {
    if (!out || !out_cap) return fail(JR_EINVAL, err, cap, "missing output buffer");
    if (s.size() + 1 > out_cap) {
        out[0] = '\0';
        return fail(JR_EINVAL, err, cap, "output buffer too small (%zu bytes needed)", s.size() + 1);
    }
    memcpy(out, s.c_str(), s.size() + 1);
    return 0;
}

// Reads and clears the device error word written by bounded waits.
int check_device_error(Context *ctx, char *err, size_t cap) {
    if (!ctx->err_host) return 0;
    const int code = *reinterpret_cast<volatile int *>(ctx->err_host);
    if (!code) return 0;
    *reinterpret_cast<volatile int *>(ctx->err_host) = 0;
    static const char *what[] = {"", "MMA wait for a TMA stage", "producer wait for a free stage", "epilogue wait for an accumulator",
                                 "MMA wait for a drained accumulator", "softmax wait for scores", "MMA wait for probabilities",
                                 "correction wait for P.V", "exit wait for copies in flight", "launch geometry mismatch"};
    return fail(JR_ETIMEOUT, err, cap, "device-side bounded wait expired: %s (code %d)", code > 0 && code < 10 ? what[code] : "unknown",
                code);
}

}  // namespace

namespace jade {
void *driver_entry(const char *name) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion(name, &fn, 12000, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
        return nullptr;
    return fn;
}
}  // namespace jade

// ============================================================== ABI 1
namespace {
// 16-bit attention kernel choice: JADE_ATTENTION_KERNEL=pair or two_tile forces one
// (read when a kernel is compiled); otherwise the measured rule of
// attention_prefers_pair decides.
bool attention_use_pair(const jade::Spec &s, int sm_count) {
    const char *force = std::getenv("JADE_ATTENTION_KERNEL");
    if (!force || !*force) return jade::attention_prefers_pair(s, sm_count);
    if (std::strcmp(force, "two_tile") == 0) return false;
    if (std::strcmp(force, "pair") != 0) throw jade::IrError("JADE_ATTENTION_KERNEL must be pair or two_tile");
    if (s.dim != 128) throw jade::IrError("the pair attention kernel needs head dim 128");
    return true;
}
}  // namespace

extern "C" uint32_t jr_version(void) { return 1; }

extern "C" int jr_create(int device, void **out, char *err, size_t cap) {
    clear(err, cap);
    if (!out) return fail(JR_EINVAL, err, cap, "null output handle");
    *out = nullptr;
    if (device < 0) return fail(JR_EINVAL, err, cap, "negative device index");
    int count = 0;
    auto status = cudaGetDeviceCount(&count);
    if (status != cudaSuccess) return cuda_fail(status, err, cap, "cudaGetDeviceCount");
    if (device >= count) return fail(JR_EINVAL, err, cap, "device %d outside device count %d", device, count);
    auto *ctx = new (std::nothrow) Context;
    if (!ctx) return fail(JR_ENOMEM, err, cap, "runtime context allocation failed");
    ctx->device = device;
    int rc = select(ctx, err, cap);
    if (rc) {
        destroy(ctx);
        return rc;
    }
    status = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (status == cudaSuccess) status = cudaEventCreate(&ctx->start);
    if (status == cudaSuccess) status = cudaEventCreate(&ctx->stop);
    if (status == cudaSuccess) status = cudaHostAlloc(reinterpret_cast<void **>(&ctx->err_host), 64, cudaHostAllocMapped);
    if (status == cudaSuccess) status = cudaHostGetDevicePointer(reinterpret_cast<void **>(&ctx->err_dev), ctx->err_host, 0);
    if (status == cudaSuccess) status = cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
    if (status != cudaSuccess) {
        rc = cuda_fail(status, err, cap, "create stream/timing events");
        destroy(ctx);
        return rc;
    }
    memset(ctx->err_host, 0, 64);
    *out = ctx;
    return 0;
}

extern "C" void jr_destroy(void *ctx) { destroy(static_cast<Context *>(ctx)); }

extern "C" int jr_info(void *handle, char *out, size_t out_cap, char *err, size_t cap) {
    clear(err, cap);
    if (out && out_cap) out[0] = '\0';
    if (!out || !out_cap) return fail(JR_EINVAL, err, cap, "missing device-info output");
    auto *ctx = static_cast<Context *>(handle);
    const int rc = select(ctx, err, cap);
    if (rc) return rc;
    cudaDeviceProp prop{};
    auto status = cudaGetDeviceProperties(&prop, ctx->device);
    if (status != cudaSuccess) return cuda_fail(status, err, cap, "cudaGetDeviceProperties");
    int runtime = 0, driver = 0;
    status = cudaRuntimeGetVersion(&runtime);
    if (status == cudaSuccess) status = cudaDriverGetVersion(&driver);
    if (status != cudaSuccess) return cuda_fail(status, err, cap, "runtime/driver version");
    const int n = std::snprintf(out, out_cap, "device=%d name=%.255s memory_bytes=%llu runtime_api=%d driver_api=%d", ctx->device, prop.name,
                                static_cast<unsigned long long>(prop.totalGlobalMem), runtime, driver);
    if (n < 0 || static_cast<size_t>(n) >= out_cap) {
        out[out_cap - 1] = '\0';
        return fail(JR_EINVAL, err, cap, "device-info output too small");
    }
    return 0;
}

extern "C" int jr_alloc(void *handle, size_t bytes, void **out, char *err, size_t cap) {
    clear(err, cap);
    if (!out) return fail(JR_EINVAL, err, cap, "null allocation output");
    *out = nullptr;
    if (!bytes) return fail(JR_EINVAL, err, cap, "allocation must be nonempty");
    auto *ctx = static_cast<Context *>(handle);
    const int rc = select(ctx, err, cap);
    if (rc) return rc;
    auto status = cudaMalloc(out, bytes);
    if (status != cudaSuccess) {
        cudaGetLastError();
        *out = nullptr;
        return fail(status == cudaErrorMemoryAllocation ? JR_ENOMEM : JR_ECUDA, err, cap, "cudaMalloc: %s (%d)", cudaGetErrorString(status),
                    (int)status);
    }
    // Public allocations contain defined zeros, even before the first upload.
    status = cudaMemsetAsync(*out, 0, bytes, ctx->stream);
    const auto sync = cudaStreamSynchronize(ctx->stream);
    if (status != cudaSuccess || sync != cudaSuccess) {
        cudaFree(*out);
        *out = nullptr;
        return cuda_fail(status != cudaSuccess ? status : sync, err, cap, "initialize allocation");
    }
    ctx->allocations[reinterpret_cast<uintptr_t>(*out)] = jade::Allocation{bytes, false};
    return 0;
}

extern "C" void jr_free(void *handle, void *ptr) {
    if (!handle || !ptr) return;
    auto *ctx = static_cast<Context *>(handle);
    if (cudaSetDevice(ctx->device) != cudaSuccess) return;
    cudaStreamSynchronize(ctx->stream);
    auto it = ctx->allocations.find(reinterpret_cast<uintptr_t>(ptr));
    if (it != ctx->allocations.end()) {
        if (it->second.host) return;  // host buffers are released by jr_host_free
        ctx->allocations.erase(it);
    }
    cudaFree(ptr);
}

extern "C" int jr_upload(void *handle, void *device_ptr, const void *host_ptr, size_t bytes, char *err, size_t cap) {
    clear(err, cap);
    if (!device_ptr || !host_ptr || !bytes) return fail(JR_EINVAL, err, cap, "invalid upload buffers/size");
    auto *ctx = static_cast<Context *>(handle);
    const int rc = select(ctx, err, cap);
    if (rc) return rc;
    const auto status = cudaMemcpyAsync(device_ptr, host_ptr, bytes, cudaMemcpyHostToDevice, ctx->stream);
    const auto sync = cudaStreamSynchronize(ctx->stream);
    if (status != cudaSuccess) return cuda_fail(status, err, cap, "upload");
    return sync == cudaSuccess ? 0 : cuda_fail(sync, err, cap, "upload synchronization");
}

extern "C" int jr_download(void *handle, const void *device_ptr, void *host_ptr, size_t bytes, char *err, size_t cap) {
    clear(err, cap);
    if (!device_ptr || !host_ptr || !bytes) return fail(JR_EINVAL, err, cap, "invalid download buffers/size");
    auto *ctx = static_cast<Context *>(handle);
    const int rc = select(ctx, err, cap);
    if (rc) return rc;
    const auto status = cudaMemcpyAsync(host_ptr, device_ptr, bytes, cudaMemcpyDeviceToHost, ctx->stream);
    const auto sync = cudaStreamSynchronize(ctx->stream);
    if (status != cudaSuccess) return cuda_fail(status, err, cap, "download");
    return sync == cudaSuccess ? 0 : cuda_fail(sync, err, cap, "download synchronization");
}

extern "C" int jr_execute(void *handle, const jr_job *jobs, size_t job_count, uint32_t repeats, double *gpu_ms, char *err, size_t cap) {
    clear(err, cap);
    if (gpu_ms) *gpu_ms = 0;
    if (!jobs || !job_count || !repeats || !gpu_ms) return fail(JR_EINVAL, err, cap, "empty dispatch sequence or missing timing output");
    // Validate every job before any work is submitted.
    for (size_t j = 0; j < job_count; ++j) {
        if (!jobs[j].launch || !jobs[j].buffers || !jobs[j].buffer_count) return fail(JR_EINVAL, err, cap, "invalid job %zu", j);
        for (size_t b = 0; b < jobs[j].buffer_count; ++b)
            if (!jobs[j].buffers[b]) return fail(JR_EINVAL, err, cap, "null buffer in job %zu", j);
    }
    auto *ctx = static_cast<Context *>(handle);
    const int rc = select(ctx, err, cap);
    if (rc) return rc;
    auto status = cudaEventRecord(ctx->start, ctx->stream);
    if (status != cudaSuccess) return cuda_fail(status, err, cap, "record start event");
    for (uint32_t repeat = 0; repeat < repeats; ++repeat) {
        for (size_t j = 0; j < job_count; ++j) {
            status = static_cast<cudaError_t>(jobs[j].launch(static_cast<void *>(ctx->stream), jobs[j].buffers));
            if (status != cudaSuccess) {
                cudaStreamSynchronize(ctx->stream);
                return cuda_fail(status, err, cap, "generated kernel launch");
            }
        }
    }
    status = cudaEventRecord(ctx->stop, ctx->stream);
    if (status != cudaSuccess) {
        cudaStreamSynchronize(ctx->stream);
        return cuda_fail(status, err, cap, "record stop event");
    }
    status = cudaEventSynchronize(ctx->stop);
    if (status != cudaSuccess) return cuda_fail(status, err, cap, "kernel synchronization");
    float elapsed = 0;
    status = cudaEventElapsedTime(&elapsed, ctx->start, ctx->stop);
    if (status != cudaSuccess) return cuda_fail(status, err, cap, "event elapsed time");
    if (!std::isfinite(elapsed) || elapsed < 0) return fail(JR_ECUDA, err, cap, "invalid GPU-event duration");
    *gpu_ms = static_cast<double>(elapsed);
    return 0;
}

// ============================================================== ABI 2
extern "C" uint32_t jr2_version(void) { return 2; }

extern "C" int jr_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

#define IR_GUARD(body)                                                  \
    try {                                                               \
        body                                                            \
    } catch (const std::exception &e) {                                 \
        return fail(JR_EINVAL, err, cap, "%s", e.what());               \
    }

extern "C" int jr_spec_validate(const char *spec_json, char *err, size_t cap) {
    clear(err, cap);
    if (!spec_json) return fail(JR_EINVAL, err, cap, "null spec");
    IR_GUARD(jade::validate(jade::parse_spec_text(spec_json)); return 0;)
}

extern "C" int jr_spec_bindings(const char *spec_json, char *out, size_t out_cap, char *err, size_t cap) {
    clear(err, cap);
    if (!spec_json) return fail(JR_EINVAL, err, cap, "null spec");
    IR_GUARD({
        auto bs = jade::bindings(jade::parse_spec_text(spec_json));
        jade::Json arr = jade::Json::array();
        for (auto &b : bs) arr.push(jade::binding_to_json(b));
        return copy_out(jade::to_string_compact(arr), out, out_cap, err, cap);
    })
}

extern "C" int jr_spec_validate_bindings(const char *spec_json, const uint64_t *lengths, const uint64_t *ids, size_t count, char *err,
                                         size_t cap) {
    clear(err, cap);
    if (!spec_json || (count && (!lengths || !ids))) return fail(JR_EINVAL, err, cap, "null spec or bindings");
    IR_GUARD({
        jade::validate_bindings(jade::parse_spec_text(spec_json), std::vector<uint64_t>(lengths, lengths + count),
                                std::vector<uint64_t>(ids, ids + count));
        return 0;
    })
}

extern "C" int jr_spec_launch(const char *spec_json, char *out, size_t out_cap, char *err, size_t cap) {
    clear(err, cap);
    if (!spec_json) return fail(JR_EINVAL, err, cap, "null spec");
    IR_GUARD(return copy_out(jade::to_string_compact(jade::launch_to_json(jade::launch(jade::parse_spec_text(spec_json)))), out, out_cap,
                             err, cap);)
}

extern "C" int jr_spec_emit(const char *spec_json, const char *target, char *out, size_t out_cap, size_t *needed, char *err, size_t cap) {
    clear(err, cap);
    if (needed) *needed = 0;
    if (!spec_json || !target) return fail(JR_EINVAL, err, cap, "null spec or target");
    IR_GUARD({
        const jade::Spec s = jade::parse_spec_text(spec_json);
        std::string src;
        if (!strcmp(target, "corex")) src = jade::corex_source(s);
        else if (!strcmp(target, "cuda")) src = jade::cuda_elementwise_source(s);
        else if (!strcmp(target, "metal")) src = jade::metal_source(s);
        else return fail(JR_EINVAL, err, cap, "unknown emit target `%s` (corex, metal, cuda)", target);
        if (needed) *needed = src.size() + 1;
        return copy_out(src, out, out_cap, err, cap);
    })
}

extern "C" int jr_spec_canonical(const char *spec_json, char *out, size_t out_cap, char *err, size_t cap) {
    clear(err, cap);
    if (!spec_json) return fail(JR_EINVAL, err, cap, "null spec");
    IR_GUARD(return copy_out(jade::to_string_pretty(jade::spec_to_json(jade::parse_spec_text(spec_json))), out, out_cap, err, cap);)
}

extern "C" int jr_compile(void *handle, const char *spec_json, jr_kernel **out, char *err, size_t cap) {
    clear(err, cap);
    if (!out) return fail(JR_EINVAL, err, cap, "null kernel output");
    *out = nullptr;
    if (!spec_json) return fail(JR_EINVAL, err, cap, "null spec");
    auto *ctx = static_cast<Context *>(handle);
    const int rc = select(ctx, err, cap);
    if (rc) return rc;
    auto *k = new (std::nothrow) jr_kernel;
    if (!k) return fail(JR_ENOMEM, err, cap, "kernel allocation failed");
    try {
        k->ctx = ctx;
        k->spec = jade::parse_spec_text(spec_json);
        k->binds = jade::bindings(k->spec);
        using jade::Op;
        const jade::Spec &s = k->spec;
        std::string why;
        switch (s.op) {
            case Op::Elementwise: k->run = jade::make_elementwise_rtc(ctx, s, k->impl); k->path = "nvrtc"; break;
            case Op::Axpy: case Op::Add: case Op::SwiGlu: case Op::RmsNorm: case Op::Softmax: case Op::RmsInv:
                k->run = jade::make_row_kernel(ctx, s, k->impl);
                k->path = "simt";
                break;
            case Op::Gemm: case Op::GemmSimd:
                if (s.op == Op::Gemm && s.dtype != jade::DType::F32 && jade::gemm_tc_supports(s, why)) {
                    k->run = jade::make_gemm_tc(ctx, s, k->impl);
                    k->path = "tcgen05";
                } else {
                    k->run = jade::make_gemm_simt(ctx, s, k->impl);
                    k->path = "simt";
                }
                break;
            case Op::GemmMps: k->run = jade::make_cublas_gemm(ctx, s, k->impl); k->path = "cublas"; break;
            case Op::AttentionOnline: case Op::AttentionScores: case Op::AttentionApply:
                if (s.dtype == jade::DType::F32) {
                    k->run = jade::make_attention_simt(ctx, s, k->impl);
                    k->path = "simt";
                } else if (s.op == Op::AttentionOnline && attention_use_pair(s, ctx->sm_count)) {
                    try {
                        k->run = jade::make_attention_pair(ctx, s, k->impl);
                    } catch (const jade::IrError &) {  // more work items than the pair kernel's list holds
                        k->run = jade::make_attention_tc(ctx, s, k->impl);
                    }
                    k->path = "tcgen05";
                } else {
                    k->run = jade::make_attention_tc(ctx, s, k->impl);
                    k->path = "tcgen05";
                }
                break;
            case Op::Fill: case Op::L2Flush: k->run = jade::make_misc_kernel(ctx, s, k->impl); k->path = "simt"; break;
            case Op::AllReduce:
                k->run = jade::make_all_reduce(ctx, s, k->impl);
                k->path = "nccl";
                k->collective = true;
                break;
            case Op::Copy: {
                const cudaMemcpyKind kind = s.direction == "h2d" ? cudaMemcpyHostToDevice
                                            : s.direction == "d2h" ? cudaMemcpyDeviceToHost
                                                                   : cudaMemcpyDeviceToDevice;
                const size_t bytes = s.bytes;
                k->run = [kind, bytes](cudaStream_t st, void **b) { return cudaMemcpyAsync(b[1], b[0], bytes, kind, st); };
                k->impl = "copy_" + s.direction;
                k->path = "copy";
                break;
            }
        }
    } catch (const std::exception &e) {
        delete k;
        return fail(JR_EINVAL, err, cap, "%s", e.what());
    }
    const auto st = cudaGetLastError();
    if (st != cudaSuccess) {
        delete k;
        return cuda_fail(st, err, cap, "kernel setup");
    }
    *out = k;
    return 0;
}

extern "C" void jr_kernel_release(jr_kernel *kernel) { delete kernel; }

extern "C" int jr_kernel_info(jr_kernel *k, char *out, size_t out_cap, char *err, size_t cap) {
    clear(err, cap);
    if (!k) return fail(JR_EINVAL, err, cap, "null kernel");
    jade::Json j = jade::Json::object();
    j.set("name", jade::Json::str(jade::spec_name(k->spec))).set("impl", jade::Json::str(k->impl)).set("path", jade::Json::str(k->path));
    j.set("spec", jade::spec_to_json(k->spec));
    jade::Json arr = jade::Json::array();
    for (auto &b : k->binds) arr.push(jade::binding_to_json(b));
    j.set("bindings", arr);
    return copy_out(jade::to_string_compact(j), out, out_cap, err, cap);
}

namespace {
int validate_dispatch(Context *ctx, const jr_dispatch *jobs, size_t n, char *err, size_t cap) {
    for (size_t j = 0; j < n; ++j) {
        const jr_dispatch &d = jobs[j];
        if (!d.kernel) return fail(JR_EINVAL, err, cap, "job %zu: null kernel", j);
        if (d.kernel->ctx != ctx) return fail(JR_EINVAL, err, cap, "job %zu: kernel belongs to another runtime/device context", j);
        const auto &binds = d.kernel->binds;
        if (!d.buffers || d.buffer_count != binds.size())
            return fail(JR_EINVAL, err, cap, "job %zu: %s expects %zu bindings", j, jade::spec_name(d.kernel->spec), binds.size());
        for (size_t b = 0; b < binds.size(); ++b) {
            const void *p = d.buffers[b];
            if (!p) return fail(JR_EINVAL, err, cap, "job %zu: null buffer %zu", j, b);
            auto it = ctx->allocations.find(reinterpret_cast<uintptr_t>(p));
            if (it == ctx->allocations.end())
                return fail(JR_EINVAL, err, cap, "job %zu: buffer %s belongs to another runtime/device context", j, binds[b].name.c_str());
            if (it->second.host != binds[b].host)
                return fail(JR_EINVAL, err, cap, "job %zu: buffer %s must be %s memory", j, binds[b].name.c_str(),
                            binds[b].host ? "pinned host" : "device");
            const uint64_t want = binds[b].elements * jade::dtype_size(binds[b].dtype);
            if (it->second.bytes != want)
                return fail(JR_EINVAL, err, cap, "job %zu: %s binding %s expected %llu bytes (%llu %s), got %zu", j,
                            jade::spec_name(d.kernel->spec), binds[b].name.c_str(), (unsigned long long)want,
                            (unsigned long long)binds[b].elements, jade::dtype_name(binds[b].dtype), it->second.bytes);
            if (binds[b].write)
                for (size_t o = 0; o < binds.size(); ++o)
                    if (o != b && d.buffers[o] == p) return fail(JR_EINVAL, err, cap, "job %zu: output binding must not alias another binding", j);
        }
    }
    return 0;
}

// Waits for `ev` without blocking forever when collectives are in flight.
int wait_event(Context *ctx, cudaEvent_t ev, bool collective, char *err, size_t cap);
}  // namespace

namespace jade {
int comm_poll_abort(Context *ctx, char *err, size_t cap);  // comm.cpp
}

namespace {
int wait_event(Context *ctx, cudaEvent_t ev, bool collective, char *err, size_t cap) {
    if (!collective) {
        const auto st = cudaEventSynchronize(ev);
        return st == cudaSuccess ? 0 : cuda_fail(st, err, cap, "kernel synchronization");
    }
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        const auto st = cudaEventQuery(ev);
        if (st == cudaSuccess) return 0;
        if (st != cudaErrorNotReady) return cuda_fail(st, err, cap, "kernel synchronization");
        const int rc = jade::comm_poll_abort(ctx, err, cap);
        if (rc) return rc;
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
        if ((uint64_t)ms > ctx->comm_timeout_ms) {
            jade::comm_destroy(ctx);  // aborts the communicator so queued collectives return
            cudaStreamSynchronize(ctx->stream);
            return fail(JR_ETIMEOUT, err, cap, "collective did not complete within %u ms; communicator aborted", ctx->comm_timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}
}  // namespace

extern "C" int jr_execute2(void *handle, const jr_dispatch *jobs, size_t job_count, uint32_t repeats, uint32_t flags, double *gpu_ms,
                           double *job_ms, char *err, size_t cap) {
    clear(err, cap);
    if (gpu_ms) *gpu_ms = 0;
    if (!jobs || !job_count || !repeats || !gpu_ms) return fail(JR_EINVAL, err, cap, "empty dispatch sequence or missing timing output");
    const bool graph = flags & JR_EXEC_GRAPH, streams = flags & JR_EXEC_STREAMS;
    if (flags & ~(JR_EXEC_GRAPH | JR_EXEC_STREAMS)) return fail(JR_EINVAL, err, cap, "unknown execution flags 0x%x", flags);
    if (graph && job_ms) return fail(JR_EINVAL, err, cap, "per-job timing is not available with graph replay");
    if (graph && streams) return fail(JR_EINVAL, err, cap, "graph replay and dependency-scheduled streams cannot be combined");
    auto *ctx = static_cast<Context *>(handle);
    if (!ctx) return fail(JR_EINVAL, err, cap, "null runtime context");
    int rc = validate_dispatch(ctx, jobs, job_count, err, cap);
    if (rc) return rc;
    rc = select(ctx, err, cap);
    if (rc) return rc;
    bool collective = false;
    for (size_t j = 0; j < job_count; ++j) collective |= jobs[j].kernel->collective;
    if (job_ms) {
        for (size_t j = 0; j < job_count; ++j) job_ms[j] = 0;
        const size_t need = 2 * job_count * repeats;
        if (need > 65536) return fail(JR_EINVAL, err, cap, "per-job timing supports at most 32768 job launches per call");
        while (ctx->job_events.size() < need) {
            cudaEvent_t e;
            const auto st = cudaEventCreate(&e);
            if (st != cudaSuccess) return cuda_fail(st, err, cap, "create job events");
            ctx->job_events.push_back(e);
        }
    }
    if (streams) {
        const size_t need = job_count * repeats;
        if (need > 65536) return fail(JR_EINVAL, err, cap, "dependency-scheduled streams support at most 65536 job launches per call");
        cudaError_t st = cudaSuccess;
        if (!ctx->copy_in) st = cudaStreamCreateWithFlags(&ctx->copy_in, cudaStreamNonBlocking);
        if (st == cudaSuccess && !ctx->copy_out) st = cudaStreamCreateWithFlags(&ctx->copy_out, cudaStreamNonBlocking);
        while (st == cudaSuccess && ctx->dep_events.size() < need) {
            cudaEvent_t e;
            st = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
            if (st == cudaSuccess) ctx->dep_events.push_back(e);
        }
        if (st != cudaSuccess) return cuda_fail(st, err, cap, "create transfer streams/dependency events");
    }
    cudaError_t status;
    cudaGraphExec_t exec = nullptr;
    cudaGraph_t g = nullptr;
    if (graph) {
        status = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal);
        if (status != cudaSuccess) return cuda_fail(status, err, cap, "begin graph capture");
        for (size_t j = 0; j < job_count && status == cudaSuccess; ++j) status = jobs[j].kernel->run(ctx->stream, jobs[j].buffers);
        const auto end = cudaStreamEndCapture(ctx->stream, &g);
        if (status != cudaSuccess || end != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            cudaGetLastError();
            return cuda_fail(status != cudaSuccess ? status : end, err, cap, "graph capture");
        }
        status = cudaGraphInstantiate(&exec, g, 0);
        if (status != cudaSuccess) {
            cudaGraphDestroy(g);
            return cuda_fail(status, err, cap, "graph instantiate");
        }
    }
    status = cudaEventRecord(ctx->start, ctx->stream);
    if (status != cudaSuccess) return cuda_fail(status, err, cap, "record start event");
    // JR_EXEC_STREAMS: stream 0 = context stream, 1 = transfers in, 2 = transfers out.
    // Per buffer, the last writing launch and the last reading launch on each stream
    // since that write (launches on one stream are ordered, so the last one suffices).
    struct Access {
        long write = -1;
        long read[3] = {-1, -1, -1};
    };
    std::map<const void *, Access> access;
    std::vector<int> launch_stream;
    long waited[3][3];  // [stream][source stream]: latest launch already waited for
    long last_on[3] = {-1, -1, -1};
    cudaStream_t stream_of[3] = {ctx->stream, ctx->copy_in, ctx->copy_out};
    if (streams) {
        for (auto &w : waited)
            for (long &x : w) x = -1;
        launch_stream.reserve(job_count * repeats);
        status = cudaStreamWaitEvent(ctx->copy_in, ctx->start, 0);
        if (status == cudaSuccess) status = cudaStreamWaitEvent(ctx->copy_out, ctx->start, 0);
    }
    size_t ev = 0;
    long launch = 0;
    for (uint32_t r = 0; r < repeats && status == cudaSuccess; ++r) {
        if (graph) {
            status = cudaGraphLaunch(exec, ctx->stream);
            continue;
        }
        for (size_t j = 0; j < job_count; ++j) {
            int sid = 0;
            if (streams) {
                const jade::Spec &sp = jobs[j].kernel->spec;
                if (sp.op == jade::Op::Copy) sid = sp.direction == "h2d" ? 1 : sp.direction == "d2h" ? 2 : 0;
                long need[3] = {-1, -1, -1};
                const auto &binds = jobs[j].kernel->binds;
                for (size_t b = 0; b < binds.size(); ++b) {
                    const Access &a = access[jobs[j].buffers[b]];
                    if (a.write >= 0) need[launch_stream[a.write]] = std::max(need[launch_stream[a.write]], a.write);
                    if (binds[b].write)
                        for (int t = 0; t < 3; ++t) need[t] = std::max(need[t], a.read[t]);
                }
                for (int t = 0; t < 3 && status == cudaSuccess; ++t)
                    if (t != sid && need[t] > waited[sid][t]) {
                        status = cudaStreamWaitEvent(stream_of[sid], ctx->dep_events[need[t]], 0);
                        waited[sid][t] = need[t];
                    }
                if (status != cudaSuccess) break;
            }
            cudaStream_t st = stream_of[sid];
            if (job_ms) cudaEventRecord(ctx->job_events[ev++], st);
            status = jobs[j].kernel->run(st, jobs[j].buffers);
            if (job_ms) cudaEventRecord(ctx->job_events[ev++], st);
            if (status != cudaSuccess) break;
            if (streams) {
                status = cudaEventRecord(ctx->dep_events[launch], st);
                launch_stream.push_back(sid);
                last_on[sid] = launch;
                const auto &binds = jobs[j].kernel->binds;
                for (size_t b = 0; b < binds.size(); ++b) {
                    Access &a = access[jobs[j].buffers[b]];
                    if (binds[b].write) {
                        a.write = launch;
                        a.read[0] = a.read[1] = a.read[2] = -1;
                    } else {
                        a.read[sid] = launch;
                    }
                }
                ++launch;
                if (status != cudaSuccess) break;
            }
        }
    }
    if (streams)  // the context stream joins the transfer streams before the stop event
        for (int t = 1; t < 3 && status == cudaSuccess; ++t)
            if (last_on[t] >= 0) status = cudaStreamWaitEvent(ctx->stream, ctx->dep_events[last_on[t]], 0);
    if (status != cudaSuccess) {
        if (streams) {
            cudaStreamSynchronize(ctx->copy_in);
            cudaStreamSynchronize(ctx->copy_out);
        }
        cudaStreamSynchronize(ctx->stream);
        if (exec) cudaGraphExecDestroy(exec);
        if (g) cudaGraphDestroy(g);
        return cuda_fail(status, err, cap, "kernel launch");
    }
    status = cudaEventRecord(ctx->stop, ctx->stream);
    if (status != cudaSuccess) {
        cudaStreamSynchronize(ctx->stream);
        return cuda_fail(status, err, cap, "record stop event");
    }
    rc = wait_event(ctx, ctx->stop, collective, err, cap);
    if (exec) cudaGraphExecDestroy(exec);
    if (g) cudaGraphDestroy(g);
    if (rc) return rc;
    rc = check_device_error(ctx, err, cap);
    if (rc) return rc;
    float elapsed = 0;
    status = cudaEventElapsedTime(&elapsed, ctx->start, ctx->stop);
    if (status != cudaSuccess) return cuda_fail(status, err, cap, "event elapsed time");
    if (!std::isfinite(elapsed) || elapsed < 0) return fail(JR_ECUDA, err, cap, "invalid GPU-event duration");
    *gpu_ms = elapsed;
    if (job_ms) {
        ev = 0;
        for (uint32_t r = 0; r < repeats; ++r)
            for (size_t j = 0; j < job_count; ++j) {
                float t = 0;
                cudaEventElapsedTime(&t, ctx->job_events[ev], ctx->job_events[ev + 1]);
                ev += 2;
                job_ms[j] += t;
            }
    }
    return 0;
}

extern "C" int jr_buffer_bytes(void *handle, const void *ptr, size_t *bytes) {
    auto *ctx = static_cast<Context *>(handle);
    if (!ctx || !ptr || !bytes) return JR_EINVAL;
    auto it = ctx->allocations.find(reinterpret_cast<uintptr_t>(ptr));
    if (it == ctx->allocations.end()) return JR_EINVAL;
    *bytes = it->second.bytes;
    return 0;
}

extern "C" int jr_host_alloc(void *handle, size_t bytes, void **out, char *err, size_t cap) {
    clear(err, cap);
    if (!out) return fail(JR_EINVAL, err, cap, "null allocation output");
    *out = nullptr;
    if (!bytes) return fail(JR_EINVAL, err, cap, "allocation must be nonempty");
    auto *ctx = static_cast<Context *>(handle);
    const int rc = select(ctx, err, cap);
    if (rc) return rc;
    const auto status = cudaMallocHost(out, bytes);
    if (status != cudaSuccess) {
        cudaGetLastError();
        *out = nullptr;
        return fail(JR_ENOMEM, err, cap, "cudaMallocHost: %s", cudaGetErrorString(status));
    }
    memset(*out, 0, bytes);
    ctx->allocations[reinterpret_cast<uintptr_t>(*out)] = jade::Allocation{bytes, true};
    return 0;
}

extern "C" void jr_host_free(void *handle, void *ptr) {
    auto *ctx = static_cast<Context *>(handle);
    if (!ctx || !ptr) return;
    auto it = ctx->allocations.find(reinterpret_cast<uintptr_t>(ptr));
    if (it == ctx->allocations.end() || !it->second.host) return;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    ctx->allocations.erase(it);
    cudaFreeHost(ptr);
}
