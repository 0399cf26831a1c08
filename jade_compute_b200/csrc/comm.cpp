// NCCL communicator and the all-reduce job. The reference has no collective
// (docs/CUDA_RECONSTRUCTION.md:49 lists multi-GPU as future work); the only one
// this backend needs is the sum all-reduce of the tensor-parallel MLP's
// down-projection partials, enqueued on the context stream inside an ordered
// batch so it shares the batch's timing bracket. NCCL is opened with dlopen.
// Timeouts: an execute containing a collective polls ncclCommGetAsyncError and
// aborts the communicator when the context's timeout expires (JR_ETIMEOUT).
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "../../include/jade_runtime.h"
#include "cabi.hpp"
#include "internal.hpp"

namespace jade {
namespace {

struct Nccl {
    void *lib = nullptr;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*init_all)(ncclComm_t *, int, const int *) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*abort)(ncclComm_t) = nullptr;
    ncclResult_t (*async_error)(ncclComm_t, ncclResult_t *) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};

Nccl &nccl() {
    static Nccl n;
    static bool tried = false;
    if (!tried) {
        tried = true;
        for (const char *name : {"libnccl.so.2", "libnccl.so"}) {
            n.lib = dlopen(name, RTLD_NOW | RTLD_GLOBAL);
            if (n.lib) break;
        }
        if (n.lib) {
            n.get_unique_id = (decltype(n.get_unique_id))dlsym(n.lib, "ncclGetUniqueId");
            n.init_rank = (decltype(n.init_rank))dlsym(n.lib, "ncclCommInitRank");
            n.init_all = (decltype(n.init_all))dlsym(n.lib, "ncclCommInitAll");
            n.all_reduce = (decltype(n.all_reduce))dlsym(n.lib, "ncclAllReduce");
            n.destroy = (decltype(n.destroy))dlsym(n.lib, "ncclCommDestroy");
            n.abort = (decltype(n.abort))dlsym(n.lib, "ncclCommAbort");
            n.async_error = (decltype(n.async_error))dlsym(n.lib, "ncclCommGetAsyncError");
            n.error_string = (decltype(n.error_string))dlsym(n.lib, "ncclGetErrorString");
        }
    }
    return n;
}

const char *nccl_str(ncclResult_t r) { return nccl().error_string ? nccl().error_string(r) : "nccl error"; }
void need_nccl() {
    Nccl &n = nccl();
    require(n.lib && n.get_unique_id && n.init_rank && n.all_reduce && n.abort, "NCCL (libnccl.so.2) is not available");
}
void check_nccl(ncclResult_t r, const char *operation) {
    if (r != ncclSuccess) raise(JR_ECUDA, "%s: %s", operation, nccl_str(r));
}

}  // namespace

// Throws JR_ETIMEOUT (after aborting the communicator) when NCCL reports an
// asynchronous error for this context's communicator.
void comm_poll_abort(Context *ctx) {
    if (!ctx->nccl_comm || !nccl().async_error) return;
    ncclResult_t async = ncclSuccess;
    nccl().async_error(static_cast<ncclComm_t>(ctx->nccl_comm), &async);
    if (async != ncclSuccess && async != ncclInProgress) {
        nccl().abort(static_cast<ncclComm_t>(ctx->nccl_comm));
        ctx->nccl_comm = nullptr;
        raise(JR_ETIMEOUT, "collective failed asynchronously: %s; communicator aborted", nccl_str(async));
    }
}

void comm_destroy(Context *ctx) {
    if (!ctx->nccl_comm) return;
    // Abort (not destroy) so that a communicator whose peers are gone cannot block.
    if (nccl().abort) nccl().abort(static_cast<ncclComm_t>(ctx->nccl_comm));
    ctx->nccl_comm = nullptr;
}

LaunchFn make_all_reduce(Context *ctx, const Spec &s, std::string &impl) {
    if (!ctx->nccl_comm) throw IrError("all_reduce needs a communicator: call jr_comm_init first");
    const size_t count = s.len;
    const ncclDataType_t dt = s.dtype == DType::BF16 ? ncclBfloat16 : s.dtype == DType::F16 ? ncclFloat16 : ncclFloat32;
    impl = std::string("nccl_all_reduce_sum_") + dtype_name(s.dtype);
    return [ctx, count, dt](cudaStream_t st, void **b) {
        if (!ctx->nccl_comm) return cudaErrorInvalidResourceHandle;
        const ncclResult_t r = nccl().all_reduce(b[0], b[0], count, dt, ncclSum, static_cast<ncclComm_t>(ctx->nccl_comm), st);
        return r == ncclSuccess ? cudaSuccess : cudaErrorUnknown;
    };
}

}  // namespace jade

using jade::Context;

extern "C" int jr_comm_unique_id(unsigned char id[128], char *err, size_t cap) {
    return jade::c_entry(err, cap, [&] {
        jade::require(id != nullptr, "null id buffer");
        jade::need_nccl();
        ncclUniqueId u;
        jade::check_nccl(jade::nccl().get_unique_id(&u), "ncclGetUniqueId");
        static_assert(sizeof(u) == 128, "ncclUniqueId is 128 bytes");
        memcpy(id, &u, 128);
    });
}

namespace {
void attach(Context *c, ncclComm_t comm, int nranks, int rank, uint32_t timeout_ms) {
    c->nccl_comm = comm;
    c->nranks = nranks;
    c->rank = rank;
    c->comm_timeout_ms = timeout_ms ? timeout_ms : 60000;
}
}  // namespace

extern "C" int jr_comm_init(void *handle, int nranks, int rank, const unsigned char id[128], uint32_t timeout_ms, char *err, size_t cap) {
    return jade::c_entry(err, cap, [&] {
        auto *ctx = static_cast<Context *>(handle);
        jade::require(ctx && id, "null context or id");
        if (nranks < 1 || rank < 0 || rank >= nranks) jade::raise(JR_EINVAL, "rank %d outside communicator of %d ranks", rank, nranks);
        jade::require(!ctx->nccl_comm, "context already has a communicator");
        jade::need_nccl();
        jade::check_cuda(cudaSetDevice(ctx->device), "cudaSetDevice");
        ncclUniqueId u;
        memcpy(&u, id, 128);
        ncclComm_t comm = nullptr;
        jade::check_nccl(jade::nccl().init_rank(&comm, nranks, u, rank), "ncclCommInitRank");
        attach(ctx, comm, nranks, rank, timeout_ms);
    });
}

extern "C" int jr_comm_init_all(void **ctxs, int count, uint32_t timeout_ms, char *err, size_t cap) {
    return jade::c_entry(err, cap, [&] {
        jade::require(ctxs && count >= 1, "no contexts");
        jade::need_nccl();
        jade::require(jade::nccl().init_all != nullptr, "ncclCommInitAll unavailable");
        std::vector<int> devs;
        for (int i = 0; i < count; ++i) {
            auto *c = static_cast<Context *>(ctxs[i]);
            if (!c) jade::raise(JR_EINVAL, "null context %d", i);
            if (c->nccl_comm) jade::raise(JR_EINVAL, "context %d already has a communicator", i);
            if (std::find(devs.begin(), devs.end(), c->device) != devs.end()) jade::raise(JR_EINVAL, "device %d appears twice", c->device);
            devs.push_back(c->device);
        }
        std::vector<ncclComm_t> comms(count);
        jade::check_nccl(jade::nccl().init_all(comms.data(), count, devs.data()), "ncclCommInitAll");
        for (int i = 0; i < count; ++i) attach(static_cast<Context *>(ctxs[i]), comms[i], count, i, timeout_ms);
    });
}

extern "C" int jr_comm_destroy(void *handle) {
    auto *ctx = static_cast<Context *>(handle);
    if (!ctx) return JR_EINVAL;
    if (ctx->nccl_comm && jade::nccl().destroy) {
        cudaSetDevice(ctx->device);
        cudaStreamSynchronize(ctx->stream);
        jade::nccl().destroy(static_cast<ncclComm_t>(ctx->nccl_comm));
    }
    ctx->nccl_comm = nullptr;
    return 0;
}
