// Runtime internals shared by the C ABI (runtime.cpp) and the kernel families.
#pragma once
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "ir.hpp"

namespace jade {

struct Allocation {
    size_t bytes;
    bool host;  // pinned host memory (copy-job endpoints)
};

struct Context {
    int device = 0;
    int sm_count = 148;
    cudaStream_t stream = nullptr;
    cudaEvent_t start = nullptr, stop = nullptr;
    std::map<uintptr_t, Allocation> allocations;
    int *err_host = nullptr;  // mapped, written by kernels (first error wins)
    int *err_dev = nullptr;
    std::vector<cudaEvent_t> job_events;
    // JR_EXEC_STREAMS: transfer and collective streams (created on first use) and
    // dependency events
    cudaStream_t copy_in = nullptr, copy_out = nullptr, collective = nullptr;
    std::vector<cudaEvent_t> dep_events;
    // NCCL (opaque; see comm.cpp)
    void *nccl_comm = nullptr;
    int nranks = 1, rank = 0;
    uint32_t comm_timeout_ms = 60000;
    // cuBLAS handle for the gemm_mps library comparator (lazy)
    void *cublas = nullptr;
    // peer memory (jr_peer_attach): a local buffer -> every rank's device address
    // of its counterpart (this rank's own entry is the buffer itself; the others
    // are CUDA IPC mappings this context opened and closes with the buffer)
    std::map<uintptr_t, std::vector<void *>> peers;
    // runtime-compiled elementwise modules, keyed by full source text
    std::map<std::string, std::pair<void *, void *>> rtc_modules;  // source -> (CUmodule, CUfunction)
    std::mutex rtc_mutex;
};

using LaunchFn = std::function<cudaError_t(cudaStream_t, void **)>;

}  // namespace jade

struct jr_kernel {
    jade::Context *ctx = nullptr;
    jade::Spec spec;
    std::vector<jade::Binding> binds;
    std::string impl;  // implementation name reported by jr_kernel_info
    std::string path;  // "tcgen05", "simt", "nvrtc", "nccl", "copy", "cublas"
    bool collective = false;
    std::vector<size_t> peer_bindings;  // bindings that must be attached peer buffers (ranks entries)
    uint32_t peer_ranks = 0;
    jade::LaunchFn run;
};

namespace jade {

// Kernel families. Each returns a launch closure for the validated spec, or
// throws IrError when the spec has no implementation on this backend.
LaunchFn make_row_kernel(Context *ctx, const Spec &s, std::string &impl);
LaunchFn make_gemm_simt(Context *ctx, const Spec &s, std::string &impl);
LaunchFn make_gemm_tc(Context *ctx, const Spec &s, std::string &impl);  // tcgen05 path
bool gemm_tc_supports(const Spec &s, std::string &why);
LaunchFn make_attention_simt(Context *ctx, const Spec &s, std::string &impl);
LaunchFn make_attention_tc(Context *ctx, const Spec &s, std::string &impl);
LaunchFn make_attention_pair(Context *ctx, const Spec &s, std::string &impl);  // dim 128, CTA pairs
// Heads per group of the attention work order: groups whose K and V (2 x seq x dim
// x 2 bytes per head) fit in `budget` bytes of L2, split evenly (64 heads under a
// budget for 48 run as 32 + 32, not 48 + 16: a small last group leaves workers idle).
inline int attention_group_heads(long long heads, long long seq, long long dim, long long budget) {
    const long long fit = std::max<long long>(1, budget / (4 * seq * dim));
    const long long groups = (heads + fit - 1) / fit;
    return (int)((heads + groups - 1) / groups);
}
// Which 16-bit attention kernel to run, from measurements on B200. Both deal
// (head, 256-query) work items to persistent workers: the two-tile kernel to one
// CTA per SM, the pair kernel to one CTA pair per two SMs. The two-tile kernel has
// the faster key step (about 9% at long rows) and wins causal attention at every
// length; the pair kernel wins non-causal shapes whose item count leaves the last
// round of the two-tile kernel mostly empty (e.g. 512 items on 148 SMs: 3.46 of 4
// rounds), as it spreads the same items over half as many workers.
inline bool attention_prefers_pair(const Spec &s, int sm_count) {
    if (s.causal || s.dim != 128 || s.seq < 2048 || sm_count < 2) return false;
    const double items = (double)s.batch * s.heads * (double)((s.seq + 255) / 256);
    auto efficiency = [&](double workers) { return items / (std::ceil(items / workers) * workers); };
    return efficiency(sm_count) < 0.92 * efficiency(sm_count / 2);
}
LaunchFn make_elementwise_rtc(Context *ctx, const Spec &s, std::string &impl);
LaunchFn make_misc_kernel(Context *ctx, const Spec &s, std::string &impl);  // fill, l2_flush
LaunchFn make_cublas_gemm(Context *ctx, const Spec &s, std::string &impl);
LaunchFn make_all_reduce(Context *ctx, const Spec &s, std::string &impl);
// Peer collectives over NVLink (peer.cu): shard_reduce and shard_gather, and the
// arrival signal the gemm "scatter" epilogue sends after its stores.
LaunchFn make_shard_op(Context *ctx, const Spec &s, std::string &impl);
struct PeerSet {
    void *p[kMaxPeerRanks];
};
PeerSet peer_set(Context *ctx, const void *local, uint32_t ranks);  // throws if not attached
bool find_peers(Context *ctx, const void *local, uint32_t ranks, PeerSet &out);
cudaError_t launch_peer_signal(cudaStream_t st, const PeerSet &flags, uint32_t ranks, uint32_t rank, int phase);
void cublas_destroy(Context *ctx);
void rtc_destroy(Context *ctx);
void comm_destroy(Context *ctx);
void peer_detach(Context *ctx, const void *local);  // closes the mappings of one attached buffer

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
void *driver_entry(const char *name);

}  // namespace jade
