// C ABI of the B200 runtime (include/jade_runtime.h).
//
// A context is one device with one non-blocking stream, a timing-event pair, a
// mapped error word written by the kernels' bounded waits, and a registry of
// every buffer it handed out. ABI 1 (jr_version() == 1) is the reference
// bridge's surface over that context: raw launcher jobs run in order between the
// event pair. ABI 2 builds on the same pieces: the JSON KernelSpec front end,
// built-in sm_100a kernels, registry checks of every job before any launch (as
// src/runtime/corex.rs:557-569 does in the caller), per-job timing, CUDA-graph
// replay, dependency-scheduled transfer streams and collectives.
//
// Every exported function is a jade::c_entry body (cabi.hpp): failures are
// thrown as jade::Fault and turned into the return code and message there.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <thread>

#include "../../include/jade_runtime.h"
#include "cabi.hpp"
#include "internal.hpp"

using jade::check_cuda;
using jade::Context;
using jade::Fault;
using jade::raise;
using jade::require;

namespace jade {
void *driver_entry(const char *name) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion(name, &fn, 12000, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
        return nullptr;
    return fn;
}
void comm_poll_abort(Context *ctx);  // comm.cpp: throws JR_ETIMEOUT on an asynchronous NCCL error
}  // namespace jade

namespace {

// ------------------------------------------------------------ context plumbing

// The context behind a caller's handle, with its device made current.
Context &enter(void *handle) {
    auto *ctx = static_cast<Context *>(handle);
    require(ctx != nullptr, "null runtime context");
    check_cuda(cudaSetDevice(ctx->device), "cudaSetDevice");
    return *ctx;
}

// Teardown never reports: it runs from jr_destroy and from a failed jr_create.
// Queued work finishes first, then the collective, libraries, registered
// buffers, events and streams go, in that order.
void teardown(Context *ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    jade::comm_destroy(ctx);
    jade::cublas_destroy(ctx);
    jade::rtc_destroy(ctx);
    while (!ctx->peers.empty()) jade::peer_detach(ctx, reinterpret_cast<void *>(ctx->peers.begin()->first));
    for (const auto &entry : ctx->allocations) {
        void *p = reinterpret_cast<void *>(entry.first);
        if (entry.second.host) cudaFreeHost(p);
        else cudaFree(p);
    }
    ctx->allocations.clear();
    for (cudaEvent_t e : ctx->job_events) cudaEventDestroy(e);
    for (cudaEvent_t e : ctx->dep_events) cudaEventDestroy(e);
    for (cudaEvent_t e : {ctx->start, ctx->stop})
        if (e) cudaEventDestroy(e);
    for (cudaStream_t s : {ctx->copy_in, ctx->copy_out, ctx->collective, ctx->stream})
        if (s) cudaStreamDestroy(s);
    if (ctx->err_host) cudaFreeHost(ctx->err_host);
    delete ctx;
}

// A fresh context on `device`: its stream, timing events, mapped error word and
// SM count. Throws with everything created so far released.
Context *build_context(int device) {
    std::unique_ptr<Context, void (*)(Context *)> ctx(new (std::nothrow) Context, teardown);
    if (!ctx) raise(JR_ENOMEM, "runtime context allocation failed");
    ctx->device = device;
    check_cuda(cudaSetDevice(device), "cudaSetDevice");
    cudaError_t st = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    for (cudaEvent_t *e : {&ctx->start, &ctx->stop})
        if (st == cudaSuccess) st = cudaEventCreate(e);
    if (st == cudaSuccess) st = cudaHostAlloc(reinterpret_cast<void **>(&ctx->err_host), 64, cudaHostAllocMapped);
    if (st == cudaSuccess) st = cudaHostGetDevicePointer(reinterpret_cast<void **>(&ctx->err_dev), ctx->err_host, 0);
    if (st == cudaSuccess) st = cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
    check_cuda(st, "create stream/timing events");
    std::memset(ctx->err_host, 0, 64);
    return ctx.release();
}

// Device memory registered with the context and zero-filled before it is
// returned, so a buffer never exposes stale contents.
void *device_buffer(Context &ctx, size_t bytes) {
    void *p = nullptr;
    const cudaError_t st = cudaMalloc(&p, bytes);
    if (st != cudaSuccess) {
        cudaGetLastError();
        raise(st == cudaErrorMemoryAllocation ? JR_ENOMEM : JR_ECUDA, "cudaMalloc: %s (%d)", cudaGetErrorString(st), (int)st);
    }
    const cudaError_t zero = cudaMemsetAsync(p, 0, bytes, ctx.stream);
    const cudaError_t done = cudaStreamSynchronize(ctx.stream);
    if (zero != cudaSuccess || done != cudaSuccess) {
        cudaFree(p);
        check_cuda(zero != cudaSuccess ? zero : done, "initialize allocation");
    }
    ctx.allocations[reinterpret_cast<uintptr_t>(p)] = jade::Allocation{bytes, false};
    return p;
}

// One blocking transfer on the context stream; `name` is "upload" or "download".
void blocking_copy(Context &ctx, void *dst, const void *src, size_t bytes, cudaMemcpyKind kind, const char *name) {
    const cudaError_t issued = cudaMemcpyAsync(dst, src, bytes, kind, ctx.stream);
    const cudaError_t done = cudaStreamSynchronize(ctx.stream);
    check_cuda(issued, name);
    check_cuda(done, (std::string(name) + " synchronization").c_str());
}

// Reads and clears the error word the kernels' bounded waits write (first
// expiry wins), as JR_ETIMEOUT naming the wait that gave up.
void raise_device_wait_error(Context &ctx) {
    if (!ctx.err_host) return;
    volatile int *word = reinterpret_cast<volatile int *>(ctx.err_host);
    const int code = *word;
    if (!code) return;
    *word = 0;
    static const char *const site[] = {"",
                                       "MMA wait for a TMA stage",
                                       "producer wait for a free stage",
                                       "epilogue wait for an accumulator",
                                       "MMA wait for a drained accumulator",
                                       "softmax wait for scores",
                                       "MMA wait for probabilities",
                                       "correction wait for P.V",
                                       "exit wait for copies in flight",
                                       "launch geometry mismatch",
                                       "wait probe (a wait that nothing satisfies)"};
    const bool known = code > 0 && code < (int)(sizeof site / sizeof site[0]);
    raise(JR_ETIMEOUT, "device-side bounded wait expired: %s (code %d)", known ? site[code] : "unknown", code);
}

// Blocks until `ev` completes. With a collective in flight the wait polls NCCL's
// asynchronous error state and gives up after the context's collective timeout,
// aborting the communicator so that queued collectives return.
void await_event(Context &ctx, cudaEvent_t ev, bool collective) {
    if (!collective) {
        check_cuda(cudaEventSynchronize(ev), "kernel synchronization");
        return;
    }
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(ctx.comm_timeout_ms);
    for (;;) {
        const cudaError_t st = cudaEventQuery(ev);
        if (st == cudaSuccess) return;
        if (st != cudaErrorNotReady) check_cuda(st, "kernel synchronization");
        jade::comm_poll_abort(&ctx);
        if (std::chrono::steady_clock::now() > deadline) {
            jade::comm_destroy(&ctx);
            cudaStreamSynchronize(ctx.stream);
            raise(JR_ETIMEOUT, "collective did not complete within %u ms; communicator aborted", ctx.comm_timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

// Milliseconds between the context's start and stop events, already completed.
double bracket_ms(Context &ctx) {
    float ms = 0;
    check_cuda(cudaEventElapsedTime(&ms, ctx.start, ctx.stop), "event elapsed time");
    if (!std::isfinite(ms) || ms < 0) raise(JR_ECUDA, "invalid GPU-event duration");
    return ms;
}

// 16-bit attention kernel choice: JADE_ATTENTION_KERNEL=pair or two_tile forces
// one (read when a kernel is compiled); otherwise the measured rule of
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

// ============================================================== ABI 1
extern "C" uint32_t jr_version(void) { return 1; }

extern "C" int jr_create(int device, void **out, char *err, size_t cap) {
    return jade::c_entry(err, cap, [&] {
        require(out != nullptr, "null output handle");
        *out = nullptr;
        require(device >= 0, "negative device index");
        int visible = 0;
        check_cuda(cudaGetDeviceCount(&visible), "cudaGetDeviceCount");
        if (device >= visible) raise(JR_EINVAL, "device %d outside device count %d", device, visible);
        *out = build_context(device);
    });
}

extern "C" void jr_destroy(void *ctx) { teardown(static_cast<Context *>(ctx)); }

extern "C" int jr_info(void *handle, char *out, size_t out_cap, char *err, size_t cap) {
    if (out && out_cap) out[0] = '\0';
    return jade::c_entry(err, cap, [&] {
        require(out && out_cap, "missing device-info output");
        Context &ctx = enter(handle);
        cudaDeviceProp prop{};
        check_cuda(cudaGetDeviceProperties(&prop, ctx.device), "cudaGetDeviceProperties");
        int runtime = 0, driver = 0;
        cudaError_t st = cudaRuntimeGetVersion(&runtime);
        if (st == cudaSuccess) st = cudaDriverGetVersion(&driver);
        check_cuda(st, "runtime/driver version");
        const int n = std::snprintf(out, out_cap, "device=%d name=%.255s memory_bytes=%llu runtime_api=%d driver_api=%d", ctx.device,
                                    prop.name, static_cast<unsigned long long>(prop.totalGlobalMem), runtime, driver);
        if (n < 0 || static_cast<size_t>(n) >= out_cap) {
            out[out_cap - 1] = '\0';
            raise(JR_EINVAL, "device-info output too small");
        }
    });
}

extern "C" int jr_alloc(void *handle, size_t bytes, void **out, char *err, size_t cap) {
    return jade::c_entry(err, cap, [&] {
        require(out != nullptr, "null allocation output");
        *out = nullptr;
        require(bytes != 0, "allocation must be nonempty");
        *out = device_buffer(enter(handle), bytes);
    });
}

extern "C" void jr_free(void *handle, void *ptr) {
    auto *ctx = static_cast<Context *>(handle);
    if (!ctx || !ptr || cudaSetDevice(ctx->device) != cudaSuccess) return;
    cudaStreamSynchronize(ctx->stream);
    const auto it = ctx->allocations.find(reinterpret_cast<uintptr_t>(ptr));
    if (it != ctx->allocations.end()) {
        if (it->second.host) return;  // pinned host buffers go through jr_host_free
        ctx->allocations.erase(it);
    }
    jade::peer_detach(ctx, ptr);  // a later allocation at this address is not attached
    cudaFree(ptr);
}

extern "C" int jr_upload(void *handle, void *device_ptr, const void *host_ptr, size_t bytes, char *err, size_t cap) {
    return jade::c_entry(err, cap, [&] {
        require(device_ptr && host_ptr && bytes, "invalid upload buffers/size");
        blocking_copy(enter(handle), device_ptr, host_ptr, bytes, cudaMemcpyHostToDevice, "upload");
    });
}

extern "C" int jr_download(void *handle, const void *device_ptr, void *host_ptr, size_t bytes, char *err, size_t cap) {
    return jade::c_entry(err, cap, [&] {
        require(device_ptr && host_ptr && bytes, "invalid download buffers/size");
        blocking_copy(enter(handle), host_ptr, device_ptr, bytes, cudaMemcpyDeviceToHost, "download");
    });
}

extern "C" int jr_execute(void *handle, const jr_job *jobs, size_t job_count, uint32_t repeats, double *gpu_ms, char *err, size_t cap) {
    if (gpu_ms) *gpu_ms = 0;
    return jade::c_entry(err, cap, [&] {
        require(jobs && job_count && repeats && gpu_ms, "empty dispatch sequence or missing timing output");
        // The whole sequence is checked before the device sees any of it.
        for (size_t j = 0; j < job_count; ++j) {
            const jr_job &job = jobs[j];
            if (!job.launch || !job.buffers || !job.buffer_count) raise(JR_EINVAL, "invalid job %zu", j);
            if (std::find(job.buffers, job.buffers + job.buffer_count, nullptr) != job.buffers + job.buffer_count)
                raise(JR_EINVAL, "null buffer in job %zu", j);
        }
        Context &ctx = enter(handle);
        check_cuda(cudaEventRecord(ctx.start, ctx.stream), "record start event");
        for (uint64_t launch = 0, total = (uint64_t)repeats * job_count; launch < total; ++launch) {
            const jr_job &job = jobs[launch % job_count];
            const auto st = static_cast<cudaError_t>(job.launch(static_cast<void *>(ctx.stream), job.buffers));
            if (st != cudaSuccess) {
                cudaStreamSynchronize(ctx.stream);
                check_cuda(st, "generated kernel launch");
            }
        }
        const cudaError_t stop = cudaEventRecord(ctx.stop, ctx.stream);
        if (stop != cudaSuccess) {
            cudaStreamSynchronize(ctx.stream);
            check_cuda(stop, "record stop event");
        }
        check_cuda(cudaEventSynchronize(ctx.stop), "kernel synchronization");
        *gpu_ms = bracket_ms(ctx);
    });
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

// KernelSpec front end: parse/validate errors (jade::IrError) become JR_EINVAL
// with the reference's message text.
extern "C" int jr_spec_validate(const char *spec_json, char *err, size_t cap) {
    return jade::c_entry(err, cap, [&] {
        require(spec_json != nullptr, "null spec");
        jade::validate(jade::parse_spec_text(spec_json));
    });
}

extern "C" int jr_spec_bindings(const char *spec_json, char *out, size_t out_cap, char *err, size_t cap) {
    return jade::c_entry(err, cap, [&] {
        require(spec_json != nullptr, "null spec");
        jade::Json list = jade::Json::array();
        for (const auto &b : jade::bindings(jade::parse_spec_text(spec_json))) list.push(jade::binding_to_json(b));
        jade::put_output(jade::to_string_compact(list), out, out_cap);
    });
}

extern "C" int jr_spec_validate_bindings(const char *spec_json, const uint64_t *lengths, const uint64_t *ids, size_t count, char *err,
                                         size_t cap) {
    return jade::c_entry(err, cap, [&] {
        require(spec_json && (!count || (lengths && ids)), "null spec or bindings");
        jade::validate_bindings(jade::parse_spec_text(spec_json), std::vector<uint64_t>(lengths, lengths + count),
                                std::vector<uint64_t>(ids, ids + count));
    });
}

extern "C" int jr_spec_launch(const char *spec_json, char *out, size_t out_cap, char *err, size_t cap) {
    return jade::c_entry(err, cap, [&] {
        require(spec_json != nullptr, "null spec");
        jade::put_output(jade::to_string_compact(jade::launch_to_json(jade::launch(jade::parse_spec_text(spec_json)))), out, out_cap);
    });
}

extern "C" int jr_spec_emit(const char *spec_json, const char *target, char *out, size_t out_cap, size_t *needed, char *err, size_t cap) {
    if (needed) *needed = 0;
    return jade::c_entry(err, cap, [&] {
        require(spec_json && target, "null spec or target");
        const jade::Spec s = jade::parse_spec_text(spec_json);
        std::string text;
        if (!std::strcmp(target, "corex")) text = jade::corex_source(s);
        else if (!std::strcmp(target, "cuda")) text = jade::cuda_source(s);
        else if (!std::strcmp(target, "metal")) text = jade::metal_source(s);
        else raise(JR_EINVAL, "unknown emit target `%s` (corex, metal, cuda)", target);
        if (needed) *needed = text.size() + 1;
        jade::put_output(text, out, out_cap);
    });
}

extern "C" int jr_spec_canonical(const char *spec_json, char *out, size_t out_cap, char *err, size_t cap) {
    return jade::c_entry(err, cap, [&] {
        require(spec_json != nullptr, "null spec");
        jade::put_output(jade::to_string_pretty(jade::spec_to_json(jade::parse_spec_text(spec_json))), out, out_cap);
    });
}

namespace {
// Picks the sm_100a implementation of a validated spec and stores its launch
// closure, implementation name and path in `k`.
void select_implementation(Context *ctx, jr_kernel &k) {
    using jade::Op;
    const jade::Spec &s = k.spec;
    std::string why;
    switch (s.op) {
        case Op::Elementwise:
            k.run = jade::make_elementwise_rtc(ctx, s, k.impl);
            k.path = "nvrtc";
            return;
        case Op::Axpy: case Op::Add: case Op::SwiGlu: case Op::RmsNorm: case Op::Softmax: case Op::RmsInv:
            k.run = jade::make_row_kernel(ctx, s, k.impl);
            k.path = "simt";
            return;
        case Op::Gemm: case Op::GemmSimd:
            if (s.op == Op::Gemm && s.dtype != jade::DType::F32 && jade::gemm_tc_supports(s, why)) {
                k.run = jade::make_gemm_tc(ctx, s, k.impl);
                k.path = "tcgen05";
                if (s.epilogue == "scatter") {  // out (the local receive buffer) and flags
                    k.peer_ranks = s.ranks;
                    k.peer_bindings = {k.binds.size() - 2, k.binds.size() - 1};
                }
            } else {
                k.run = jade::make_gemm_simt(ctx, s, k.impl);
                k.path = "simt";
            }
            return;
        case Op::GemmMps:
            k.run = jade::make_cublas_gemm(ctx, s, k.impl);
            k.path = "cublas";
            return;
        case Op::AttentionOnline: case Op::AttentionScores: case Op::AttentionApply:
            k.path = s.dtype == jade::DType::F32 ? "simt" : "tcgen05";
            if (s.dtype == jade::DType::F32) {
                k.run = jade::make_attention_simt(ctx, s, k.impl);
            } else if (s.op == Op::AttentionOnline && attention_use_pair(s, ctx->sm_count)) {
                try {
                    k.run = jade::make_attention_pair(ctx, s, k.impl);
                } catch (const jade::IrError &) {  // more work items than the pair kernel's list holds
                    k.run = jade::make_attention_tc(ctx, s, k.impl);
                }
            } else {
                k.run = jade::make_attention_tc(ctx, s, k.impl);
            }
            return;
        case Op::Fill: case Op::L2Flush: case Op::WaitProbe:
            k.run = jade::make_misc_kernel(ctx, s, k.impl);
            k.path = "simt";
            return;
        case Op::AllReduce:
            k.run = jade::make_all_reduce(ctx, s, k.impl);
            k.path = "nccl";
            k.collective = true;
            return;
        case Op::ShardReduce: case Op::ShardGather:
            k.run = jade::make_shard_op(ctx, s, k.impl);
            k.path = "nvlink";
            k.peer_ranks = s.ranks;
            if (s.op == Op::ShardReduce) k.peer_bindings = {s.residual ? 2u : 1u, s.residual ? 3u : 2u};  // out, flags
            else k.peer_bindings = {1};                                                                   // flags
            return;
        case Op::Copy: {
            const cudaMemcpyKind kind = s.direction == "h2d"   ? cudaMemcpyHostToDevice
                                        : s.direction == "d2h" ? cudaMemcpyDeviceToHost
                                                               : cudaMemcpyDeviceToDevice;
            const size_t bytes = s.bytes;
            k.run = [kind, bytes](cudaStream_t st, void **b) { return cudaMemcpyAsync(b[1], b[0], bytes, kind, st); };
            k.impl = "copy_" + s.direction;
            k.path = "copy";
            return;
        }
    }
}
}  // namespace

extern "C" int jr_compile(void *handle, const char *spec_json, jr_kernel **out, char *err, size_t cap) {
    return jade::c_entry(err, cap, [&] {
        require(out != nullptr, "null kernel output");
        *out = nullptr;
        require(spec_json != nullptr, "null spec");
        Context &ctx = enter(handle);
        auto k = std::make_unique<jr_kernel>();
        k->ctx = &ctx;
        k->spec = jade::parse_spec_text(spec_json);
        k->binds = jade::bindings(k->spec);
        select_implementation(&ctx, *k);
        check_cuda(cudaGetLastError(), "kernel setup");
        *out = k.release();
    });
}

extern "C" void jr_kernel_release(jr_kernel *kernel) { delete kernel; }

extern "C" int jr_kernel_info(jr_kernel *k, char *out, size_t out_cap, char *err, size_t cap) {
    return jade::c_entry(err, cap, [&] {
        require(k != nullptr, "null kernel");
        jade::Json binds = jade::Json::array();
        for (const auto &b : k->binds) binds.push(jade::binding_to_json(b));
        jade::Json info = jade::Json::object();
        info.set("name", jade::Json::str(jade::spec_name(k->spec)))
            .set("impl", jade::Json::str(k->impl))
            .set("path", jade::Json::str(k->path))
            .set("spec", jade::spec_to_json(k->spec))
            .set("bindings", binds);
        jade::put_output(jade::to_string_compact(info), out, out_cap);
    });
}

namespace {

// Registry checks of one batch, all before any launch: each kernel belongs to
// this context, each binding is a buffer this context allocated, of the memory
// kind and exact byte size the spec declares, and no output aliases another
// binding of its job.
void check_batch(Context &ctx, const jr_dispatch *jobs, size_t n) {
    for (size_t j = 0; j < n; ++j) {
        const jr_dispatch &d = jobs[j];
        if (!d.kernel) raise(JR_EINVAL, "job %zu: null kernel", j);
        if (d.kernel->ctx != &ctx) raise(JR_EINVAL, "job %zu: kernel belongs to another runtime/device context", j);
        const auto &binds = d.kernel->binds;
        const char *kname = jade::spec_name(d.kernel->spec);
        if (!d.buffers || d.buffer_count != binds.size()) raise(JR_EINVAL, "job %zu: %s expects %zu bindings", j, kname, binds.size());
        for (size_t b = 0; b < binds.size(); ++b) {
            const jade::Binding &bind = binds[b];
            const void *p = d.buffers[b];
            if (!p) raise(JR_EINVAL, "job %zu: null buffer %zu", j, b);
            const auto reg = ctx.allocations.find(reinterpret_cast<uintptr_t>(p));
            if (reg == ctx.allocations.end())
                raise(JR_EINVAL, "job %zu: buffer %s belongs to another runtime/device context", j, bind.name.c_str());
            if (reg->second.host != bind.host)
                raise(JR_EINVAL, "job %zu: buffer %s must be %s memory", j, bind.name.c_str(), bind.host ? "pinned host" : "device");
            const uint64_t want = bind.elements * jade::dtype_size(bind.dtype);
            if (reg->second.bytes != want)
                raise(JR_EINVAL, "job %zu: %s binding %s expected %llu bytes (%llu %s), got %zu", j, kname, bind.name.c_str(),
                      (unsigned long long)want, (unsigned long long)bind.elements, jade::dtype_name(bind.dtype), reg->second.bytes);
            if (bind.write && std::count(d.buffers, d.buffers + binds.size(), p) > 1)
                raise(JR_EINVAL, "job %zu: output binding must not alias another binding", j);
        }
        for (size_t b : d.kernel->peer_bindings) {
            const auto peer = ctx.peers.find(reinterpret_cast<uintptr_t>(d.buffers[b]));
            if (peer == ctx.peers.end() || peer->second.size() != d.kernel->peer_ranks)
                raise(JR_EINVAL, "job %zu: buffer %s is not attached to peer memory of %u ranks (jr_peer_attach)", j, binds[b].name.c_str(),
                      d.kernel->peer_ranks);
        }
    }
}

// Per-launch timing events, grown on demand and kept by the context.
void reserve_events(std::vector<cudaEvent_t> &pool, size_t need, unsigned flags, const char *what) {
    while (pool.size() < need) {
        cudaEvent_t e;
        check_cuda(cudaEventCreateWithFlags(&e, flags), what);
        pool.push_back(e);
    }
}

// A captured pass of the batch, instantiated once and released on every path.
struct CapturedPass {
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    ~CapturedPass() {
        if (exec) cudaGraphExecDestroy(exec);
        if (graph) cudaGraphDestroy(graph);
    }
    void capture(cudaStream_t s, const jr_dispatch *jobs, size_t n) {
        check_cuda(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "begin graph capture");
        cudaError_t st = cudaSuccess;
        for (size_t j = 0; j < n && st == cudaSuccess; ++j) st = jobs[j].kernel->run(s, jobs[j].buffers);
        const cudaError_t end = cudaStreamEndCapture(s, &graph);
        if (st != cudaSuccess || end != cudaSuccess) {
            cudaGetLastError();
            check_cuda(st != cudaSuccess ? st : end, "graph capture");
        }
        check_cuda(cudaGraphInstantiate(&exec, graph, 0), "graph instantiate");
    }
};

// JR_EXEC_STREAMS placement: lane 0 is the context stream, lane 1 takes
// host-to-device copies, lane 2 device-to-host copies and lane 3 collectives
// (so that an all-reduce of one block overlaps the kernels of the next, which
// do not touch its buffer). Every launch records
// an event; before a launch, its lane waits for the latest conflicting launch on
// each other lane (a write to a buffer it touches; for an output, also reads of
// it since that write). Launches within a lane are already ordered, so the
// latest conflicting launch per lane is all that needs waiting for.
class LaneScheduler {
  public:
    LaneScheduler(Context &ctx, size_t launches) : ctx_(ctx) {
        lane_stream_[0] = ctx.stream;
        lane_stream_[1] = ctx.copy_in;
        lane_stream_[2] = ctx.copy_out;
        lane_stream_[3] = ctx.collective;
        for (auto &row : waited_) std::fill(std::begin(row), std::end(row), -1L);
        lane_of_.reserve(launches);
        for (int l = 1; l < kLanes; ++l) check_cuda(cudaStreamWaitEvent(lane_stream_[l], ctx.start, 0), "kernel launch");
    }

    // Makes `job`'s lane wait for its hazards, launches it (between the timing
    // events `before` and `after` when given), records its dependency event.
    void launch(const jr_dispatch &job, cudaEvent_t before, cudaEvent_t after) {
        const jade::Spec &sp = job.kernel->spec;
        int lane = 0;
        if (sp.op == jade::Op::Copy) lane = sp.direction == "h2d" ? 1 : sp.direction == "d2h" ? 2 : 0;
        if (job.kernel->collective) lane = 3;
        long hazard[kLanes] = {-1, -1, -1, -1};
        const auto &binds = job.kernel->binds;
        for (size_t b = 0; b < binds.size(); ++b) {
            const Uses &u = uses_[job.buffers[b]];
            if (u.writer >= 0) hazard[lane_of_[u.writer]] = std::max(hazard[lane_of_[u.writer]], u.writer);
            if (binds[b].write)
                for (int l = 0; l < kLanes; ++l) hazard[l] = std::max(hazard[l], u.reader[l]);
        }
        for (int l = 0; l < kLanes; ++l)
            if (l != lane && hazard[l] > waited_[lane][l]) {
                check_cuda(cudaStreamWaitEvent(lane_stream_[lane], ctx_.dep_events[hazard[l]], 0), "kernel launch");
                waited_[lane][l] = hazard[l];
            }
        const long id = (long)lane_of_.size();
        if (before) cudaEventRecord(before, lane_stream_[lane]);
        check_cuda(job.kernel->run(lane_stream_[lane], job.buffers), "kernel launch");
        if (after) cudaEventRecord(after, lane_stream_[lane]);
        check_cuda(cudaEventRecord(ctx_.dep_events[id], lane_stream_[lane]), "kernel launch");
        lane_of_.push_back(lane);
        last_[lane] = id;
        for (size_t b = 0; b < binds.size(); ++b) {
            Uses &u = uses_[job.buffers[b]];
            if (binds[b].write) u = Uses{id, {-1, -1, -1, -1}};
            else u.reader[lane] = id;
        }
    }

    // The context stream joins the transfer lanes (before the stop event).
    void join() {
        for (int l = 1; l < kLanes; ++l)
            if (last_[l] >= 0) check_cuda(cudaStreamWaitEvent(ctx_.stream, ctx_.dep_events[last_[l]], 0), "kernel launch");
    }

    void drain() {
        for (cudaStream_t s : lane_stream_) cudaStreamSynchronize(s);
    }

  private:
    static constexpr int kLanes = 4;
    struct Uses {
        long writer = -1;
        long reader[kLanes] = {-1, -1, -1, -1};
    };
    Context &ctx_;
    cudaStream_t lane_stream_[kLanes];
    std::map<const void *, Uses> uses_;
    std::vector<int> lane_of_;
    long waited_[kLanes][kLanes];
    long last_[kLanes] = {-1, -1, -1, -1};
};

}  // namespace

extern "C" int jr_execute2(void *handle, const jr_dispatch *jobs, size_t job_count, uint32_t repeats, uint32_t flags, double *gpu_ms,
                           double *job_ms, char *err, size_t cap) {
    if (gpu_ms) *gpu_ms = 0;
    return jade::c_entry(err, cap, [&] {
        require(jobs && job_count && repeats && gpu_ms, "empty dispatch sequence or missing timing output");
        const bool graph = flags & JR_EXEC_GRAPH, lanes = flags & JR_EXEC_STREAMS;
        if (flags & ~(JR_EXEC_GRAPH | JR_EXEC_STREAMS)) raise(JR_EINVAL, "unknown execution flags 0x%x", flags);
        require(!(graph && job_ms), "per-job timing is not available with graph replay");
        require(!(graph && lanes), "graph replay and dependency-scheduled streams cannot be combined");
        auto *raw = static_cast<Context *>(handle);
        require(raw != nullptr, "null runtime context");
        check_batch(*raw, jobs, job_count);
        Context &ctx = enter(handle);
        const bool collective = std::any_of(jobs, jobs + job_count, [](const jr_dispatch &d) { return d.kernel->collective; });
        const size_t launches = job_count * (size_t)repeats;
        if (job_ms) {
            std::fill(job_ms, job_ms + job_count, 0.0);
            if (2 * launches > 65536) raise(JR_EINVAL, "per-job timing supports at most 32768 job launches per call");
            reserve_events(ctx.job_events, 2 * launches, cudaEventDefault, "create job events");
        }
        if (lanes) {
            if (launches > 65536) raise(JR_EINVAL, "dependency-scheduled streams support at most 65536 job launches per call");
            const char *what = "create transfer streams/dependency events";
            for (cudaStream_t *s : {&ctx.copy_in, &ctx.copy_out, &ctx.collective})
                if (!*s) check_cuda(cudaStreamCreateWithFlags(s, cudaStreamNonBlocking), what);
            reserve_events(ctx.dep_events, launches, cudaEventDisableTiming, what);
        }
        CapturedPass pass;
        if (graph) pass.capture(ctx.stream, jobs, job_count);
        check_cuda(cudaEventRecord(ctx.start, ctx.stream), "record start event");
        std::unique_ptr<LaneScheduler> sched;
        try {
            if (lanes) sched = std::make_unique<LaneScheduler>(ctx, launches);
            size_t ev = 0;
            for (uint32_t r = 0; r < repeats; ++r) {
                if (graph) {
                    check_cuda(cudaGraphLaunch(pass.exec, ctx.stream), "kernel launch");
                    continue;
                }
                for (size_t j = 0; j < job_count; ++j, ev += 2) {
                    cudaEvent_t before = job_ms ? ctx.job_events[ev] : nullptr;
                    cudaEvent_t after = job_ms ? ctx.job_events[ev + 1] : nullptr;
                    if (sched) {
                        sched->launch(jobs[j], before, after);
                        continue;
                    }
                    if (before) cudaEventRecord(before, ctx.stream);
                    check_cuda(jobs[j].kernel->run(ctx.stream, jobs[j].buffers), "kernel launch");
                    if (after) cudaEventRecord(after, ctx.stream);
                }
            }
            if (sched) sched->join();
        } catch (const Fault &) {
            if (sched) sched->drain();
            cudaStreamSynchronize(ctx.stream);
            throw;
        }
        const cudaError_t stop = cudaEventRecord(ctx.stop, ctx.stream);
        if (stop != cudaSuccess) {
            cudaStreamSynchronize(ctx.stream);
            check_cuda(stop, "record stop event");
        }
        await_event(ctx, ctx.stop, collective);
        raise_device_wait_error(ctx);
        *gpu_ms = bracket_ms(ctx);
        if (job_ms)
            for (size_t launch = 0; launch < launches; ++launch) {
                float t = 0;
                cudaEventElapsedTime(&t, ctx.job_events[2 * launch], ctx.job_events[2 * launch + 1]);
                job_ms[launch % job_count] += t;
            }
    });
}

extern "C" int jr_buffer_bytes(void *handle, const void *ptr, size_t *bytes) {
    auto *ctx = static_cast<Context *>(handle);
    if (!ctx || !ptr || !bytes) return JR_EINVAL;
    const auto it = ctx->allocations.find(reinterpret_cast<uintptr_t>(ptr));
    if (it == ctx->allocations.end()) return JR_EINVAL;
    *bytes = it->second.bytes;
    return JR_OK;
}

extern "C" int jr_host_alloc(void *handle, size_t bytes, void **out, char *err, size_t cap) {
    return jade::c_entry(err, cap, [&] {
        require(out != nullptr, "null allocation output");
        *out = nullptr;
        require(bytes != 0, "allocation must be nonempty");
        Context &ctx = enter(handle);
        void *p = nullptr;
        const cudaError_t st = cudaMallocHost(&p, bytes);
        if (st != cudaSuccess) {
            cudaGetLastError();
            raise(JR_ENOMEM, "cudaMallocHost: %s", cudaGetErrorString(st));
        }
        std::memset(p, 0, bytes);
        ctx.allocations[reinterpret_cast<uintptr_t>(p)] = jade::Allocation{bytes, true};
        *out = p;
    });
}

extern "C" void jr_host_free(void *handle, void *ptr) {
    auto *ctx = static_cast<Context *>(handle);
    if (!ctx || !ptr) return;
    const auto it = ctx->allocations.find(reinterpret_cast<uintptr_t>(ptr));
    if (it == ctx->allocations.end() || !it->second.host) return;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    ctx->allocations.erase(it);
    cudaFreeHost(ptr);
}
