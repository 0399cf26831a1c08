// Collectives over NVLink peer memory, for the tensor-parallel MLP's
// down-projection: the partial outputs are summed over the ranks without NCCL.
//
//   gemm, epilogue "scatter"  every rank's GEMM writes each 128-row output tile
//                             straight into the receive buffer of the rank that
//                             owns those rows (peer stores, BF16), into the slot
//                             of the writing rank; then signals phase 0
//   shard_reduce              the owner waits for phase 0 from every rank, sums
//                             its rows' slots in rank order in FP32 (+ the
//                             residual), rounds once to BF16 and stores the rows
//                             into every rank's output (peer stores); then
//                             signals phase 1
//   shard_gather              waits for phase 1 from every rank: the output is
//                             complete on this rank
//
// Buffers are shared between the ranks' processes with CUDA IPC
// (jr_peer_handle / jr_peer_attach). Each rank has a 256-byte flag buffer:
// word 8*phase + q holds rank q's latest arrival number for that phase, word
// 16 + phase this rank's own count of its signals of that phase. A rank's k-th
// signal of a phase carries the number k, and a waiter expects its own count,
// so the flags never need resetting; all ranks launch the same sequence. Waits
// run in a one-thread kernel ahead of the kernels that read the peers' data and
// are bounded: on expiry they record kErrWaitPeer in the context's error word
// (JR_ETIMEOUT) and return.
//
// Buffer reuse is ordered by the phases themselves: rank q's next scatter into
// rank r's receive buffer comes after q's shard_gather, which waited for r's
// shard_reduce (phase 1); r's next shard_reduce overwrites rows that q read
// only after q's next scatter arrived (phase 0), i.e. after q's gather.
#include <cuda_bf16.h>

#include "../../include/jade_runtime.h"
#include "cabi.hpp"
#include "common.cuh"
#include "internal.hpp"

namespace jade {
namespace {

constexpr int kErrWaitPeer = 11;
constexpr uint64_t kPeerWaitNs = 5000000000ull;  // 5 s: ranks reach the collective within the batch

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// One thread: the next arrival number of `phase` for this rank, written to every
// rank's flag buffer (this one included). The system-scope fence orders the
// stores of the kernels before it on this stream ahead of the flags.
__global__ void peer_signal_kernel(PeerSet flags, uint32_t ranks, uint32_t rank, int phase) {
    if (threadIdx.x != 0) return;
    uint32_t *local = static_cast<uint32_t *>(flags.p[rank]);
    const uint32_t e = local[16 + phase] + 1;
    local[16 + phase] = e;
    __threadfence_system();
    for (uint32_t q = 0; q < ranks; ++q) st_release_sys(static_cast<uint32_t *>(flags.p[q]) + 8 * phase + rank, e);
}

__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// One thread of one block waits (bounded) until every rank's arrival number of
// `phase` reaches this rank's own count: it polls with relaxed loads and a short
// sleep (many pollers hammering one L2 line slowed the peers' stores landing in
// this GPU's memory), then takes each arrival with an acquire load. The kernels
// after it on the stream read the peers' data.
__global__ void shard_wait_kernel(PeerSet flags, uint32_t ranks, uint32_t rank, int phase, int *err) {
    if (threadIdx.x != 0) return;
    const uint32_t *local = static_cast<const uint32_t *>(flags.p[rank]);
    const uint32_t e = *reinterpret_cast<const volatile uint32_t *>(local + 16 + phase);
    const uint64_t t0 = globaltimer();
    for (uint32_t q = 0; q < ranks; ++q) {
        while ((int)(ld_relaxed_sys(local + 8 * phase + q) - e) < 0) {
            if (globaltimer() - t0 > kPeerWaitNs) {
                if (err) atomicCAS(err, 0, kErrWaitPeer);
                return;
            }
            __nanosleep(64);
        }
        (void)ld_acquire_sys(local + 8 * phase + q);
    }
    __threadfence_system();
}

__device__ __forceinline__ void add_bf16x8(float (&acc)[8], uint4 u) {
    const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
    }
}

// This rank's rows: sum of the ranks' partial slots (rank order) plus the
// residual, one BF16 rounding, stored into every rank's output.
__global__ void __launch_bounds__(256) shard_reduce_kernel(const __nv_bfloat16 *__restrict__ recv, const __nv_bfloat16 *__restrict__ residual,
                                                           PeerSet outs, uint32_t ranks, uint32_t rank, uint32_t rows_per, uint32_t cols) {
    const uint64_t slot = (uint64_t)rows_per * cols;  // elements of one rank's partial rows
    const uint64_t nvec = slot / 8, own = (uint64_t)rank * slot;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t v = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += stride) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (uint32_t q = 0; q < ranks; ++q) add_bf16x8(acc, __ldcs(reinterpret_cast<const uint4 *>(recv + q * slot) + v));
        if (residual) add_bf16x8(acc, __ldg(reinterpret_cast<const uint4 *>(residual + own) + v));
        uint4 o;
        o.x = pack_bf16(acc[0], acc[1]);
        o.y = pack_bf16(acc[2], acc[3]);
        o.z = pack_bf16(acc[4], acc[5]);
        o.w = pack_bf16(acc[6], acc[7]);
        for (uint32_t j = 0; j < ranks; ++j) {  // this rank last: its own copy is the cheapest
            const uint32_t q = (rank + 1 + j) % ranks;
            reinterpret_cast<uint4 *>(static_cast<__nv_bfloat16 *>(outs.p[q]) + own)[v] = o;
        }
    }
}

}  // namespace

bool find_peers(Context *ctx, const void *local, uint32_t ranks, PeerSet &out) {
    const auto it = ctx->peers.find(reinterpret_cast<uintptr_t>(local));
    if (it == ctx->peers.end() || it->second.size() != ranks) return false;
    for (uint32_t q = 0; q < kMaxPeerRanks; ++q) out.p[q] = q < ranks ? it->second[q] : nullptr;
    return true;
}

PeerSet peer_set(Context *ctx, const void *local, uint32_t ranks) {
    PeerSet s{};
    if (!find_peers(ctx, local, ranks, s)) throw IrError("buffer is not attached to peer memory for this number of ranks");
    return s;
}

void peer_detach(Context *ctx, const void *local) {
    const auto it = ctx->peers.find(reinterpret_cast<uintptr_t>(local));
    if (it == ctx->peers.end()) return;
    for (void *p : it->second)
        if (p && p != local) cudaIpcCloseMemHandle(p);
    ctx->peers.erase(it);
}

cudaError_t launch_peer_signal(cudaStream_t st, const PeerSet &flags, uint32_t ranks, uint32_t rank, int phase) {
    peer_signal_kernel<<<1, 32, 0, st>>>(flags, ranks, rank, phase);
    return cudaGetLastError();
}

LaunchFn make_shard_op(Context *ctx, const Spec &s, std::string &impl) {
    const uint32_t ranks = s.ranks, rank = s.rank, rows_per = s.rows / s.ranks, cols = s.cols;
    int *err = ctx->err_dev;
    if (s.op == Op::ShardGather) {
        impl = "shard_gather_wait_x" + std::to_string(ranks);
        return [=](cudaStream_t st, void **b) {
            PeerSet flags{};
            if (!find_peers(ctx, b[1], ranks, flags)) return cudaErrorInvalidResourceHandle;
            shard_wait_kernel<<<1, 32, 0, st>>>(flags, ranks, rank, 1, err);
            return cudaGetLastError();
        };
    }
    const bool res = s.residual;
    const uint64_t nvec = (uint64_t)rows_per * cols / 8;
    const int grid = (int)std::max<uint64_t>(1, std::min<uint64_t>((nvec + 255) / 256, (uint64_t)ctx->sm_count * 4));
    impl = std::string("shard_reduce_bf16_x") + std::to_string(ranks) + (res ? "_residual" : "");
    return [=](cudaStream_t st, void **b) {
        const int out_idx = res ? 2 : 1;
        PeerSet outs{}, flags{};
        if (!find_peers(ctx, b[out_idx], ranks, outs) || !find_peers(ctx, b[out_idx + 1], ranks, flags))
            return cudaErrorInvalidResourceHandle;
        // every rank's partial rows have arrived (phase 0), then the reduction
        shard_wait_kernel<<<1, 32, 0, st>>>(flags, ranks, rank, 0, err);
        shard_reduce_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16 *>(b[0]),
                                                  res ? static_cast<const __nv_bfloat16 *>(b[1]) : nullptr, outs, ranks, rank, rows_per, cols);
        const cudaError_t e = cudaGetLastError();
        return e != cudaSuccess ? e : launch_peer_signal(st, flags, ranks, rank, 1);
    };
}

}  // namespace jade

using jade::Context;

extern "C" int jr_peer_handle(void *handle, const void *ptr, unsigned char out[64], char *err, size_t cap) {
    return jade::c_entry(err, cap, [&] {
        auto *ctx = static_cast<Context *>(handle);
        jade::require(ctx && ptr && out, "null context, buffer or handle output");
        const auto it = ctx->allocations.find(reinterpret_cast<uintptr_t>(ptr));
        jade::require(it != ctx->allocations.end() && !it->second.host, "buffer is not a device buffer of this context");
        jade::check_cuda(cudaSetDevice(ctx->device), "cudaSetDevice");
        cudaIpcMemHandle_t h;
        static_assert(sizeof(h) == 64, "cudaIpcMemHandle_t is 64 bytes");
        jade::check_cuda(cudaIpcGetMemHandle(&h, const_cast<void *>(ptr)), "cudaIpcGetMemHandle");
        memcpy(out, &h, 64);
    });
}

extern "C" int jr_peer_attach(void *handle, const void *ptr, const unsigned char *handles, int nranks, int rank, char *err, size_t cap) {
    return jade::c_entry(err, cap, [&] {
        auto *ctx = static_cast<Context *>(handle);
        jade::require(ctx && ptr && (handles || nranks == 1), "null context, buffer or handles");
        if (nranks < 1 || nranks > (int)jade::kMaxPeerRanks || rank < 0 || rank >= nranks)
            jade::raise(JR_EINVAL, "rank %d of %d outside 1..%u ranks", rank, nranks, jade::kMaxPeerRanks);
        const auto it = ctx->allocations.find(reinterpret_cast<uintptr_t>(ptr));
        jade::require(it != ctx->allocations.end() && !it->second.host, "buffer is not a device buffer of this context");
        jade::require(!ctx->peers.count(reinterpret_cast<uintptr_t>(ptr)), "buffer is already attached");
        jade::check_cuda(cudaSetDevice(ctx->device), "cudaSetDevice");
        std::vector<void *> ptrs(nranks, nullptr);
        ptrs[rank] = const_cast<void *>(ptr);
        for (int q = 0; q < nranks; ++q) {
            if (q == rank) continue;
            cudaIpcMemHandle_t h;
            memcpy(&h, handles + 64 * q, 64);
            void *p = nullptr;
            const cudaError_t st = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
            if (st != cudaSuccess) {
                for (void *o : ptrs)
                    if (o && o != ptr) cudaIpcCloseMemHandle(o);
                jade::check_cuda(st, "cudaIpcOpenMemHandle");
            }
            ptrs[q] = p;
        }
        ctx->peers[reinterpret_cast<uintptr_t>(ptr)] = std::move(ptrs);
    });
}
