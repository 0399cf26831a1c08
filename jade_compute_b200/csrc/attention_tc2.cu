// Forward attention for head dim 128 on tcgen05 pairs of SMs (cta_group::2).
//
// Semantics are those of attention_tc.cu (the reference's online attention,
// src/runtime/metal_attention.rs:44-137, oracle src/runtime/metal_lab.rs:33-73,
// extended to [batch, heads, seq, dim] and a causal mask): O = softmax(Q K^T /
// sqrt(D)) V with FP32 softmax statistics, P rounded to the input type for P.V
// and O accumulated in FP32 in TMEM.
//
// A cluster of two CTAs (one per SM) owns 256 query rows of one (batch, head):
// CTA r holds rows [128 r, 128 r + 128) and each tensor-core instruction of the
// pair is an M=256 MMA issued by CTA 0. The B operand of every MMA is split by
// N between the two CTAs' shared memory, so each SM streams half of every K
// tile (64 keys x 128 dims) and half of every V tile (128 keys x 64 dims):
// the K/V bytes per SM per key step are those of a 256-row tile on one SM.
//
// TMEM per CTA: S0 | S1 | S2 | O (128 columns each). S is triple-buffered: S(j+3)
// is issued right behind P(j).V(j) into the buffer P(j) came from (same issuing
// thread, so in order), and S(j+1), S(j+2) are already computed when the softmax
// of S(j) ends, so the tensor core never sits on the softmax's critical path.
//
//   warp 0     TMA producer (both CTAs): own Q rows once; own K/V halves into
//              four-stage rings; completion is counted on CTA 0's barriers.
//   warp 1     CTA 0: MMA issuer  S(0) S(1) S(2) | P(j).V(j) S(j+3) ... (the whole
//              warp runs the loop, one elected lane issues); CTA 1: relays its
//              softmax warps' "P(j) written" to CTA 0 in one remote arrival.
//   warps 2-9  softmax: warps w and w+4 share TMEM lane quarter w%4 and take the
//              even and the odd key steps, one thread per query row. The running
//              maximum is handed from step to step through shared memory; P(j) is
//              computed speculatively with the last maximum seen and redone only
//              if step j-1 moved it or row j's maximum grows by more than 2^8
//              (then O is rescaled in place after P(j-1).V(j-1) has landed).
//              P(j) (16-bit pairs) is written over the first 64 columns of S(j).
// Every exponential runs on the MUFU unit: moving a share of them to the FMA-pipe
// polynomial (as the two-tile kernel does) measured 0.6-1% slower here.
// Short waits poll (mbarrier.test_wait) instead of suspending: a suspended
// waiter resumes a few hundred cycles after the phase completes.
// Every wait is bounded (the error word records where it gave up); every thread
// of both CTAs reaches the final cluster barrier, after which TMEM is released.
#include <cuda.h>

#include <climits>
#include <mutex>
#include <type_traits>

#include "attention_softmax.cuh"
#include "common.cuh"
#include "internal.hpp"

namespace jade {
namespace {

constexpr int kRows = 128;     // query rows per CTA
constexpr int kKeys = 128;     // keys per step
constexpr int kDim = 128;      // head dim
constexpr int kStages = 3;     // K and V ring depth (V loads trail K by one step)
// two softmax warps per TMEM lane quarter: one takes the even key steps, the
// other the odd ones, each thread a whole row (128 scores) of its steps
constexpr int kCols = kKeys;
constexpr int kThreads = 10 * 32;
constexpr long long kGroupBytes = 64ll << 20;  // L2 share for a head group's K/V (32 MB measured 10% slower)
constexpr int kMaxItems = 512;   // work items per CTA pair (the host checks the bound)
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct Layout {
    static constexpr uint32_t kQBuf = 32768;          // 2 chunks x 16 KB (128 rows x 64 dims, SW128)
    static constexpr uint32_t kKStage = 16384;        // 2 chunks x 8 KB (64 keys x 64 dims)
    static constexpr uint32_t kVStage = 16384;        // 128 keys x 64 dims
    static constexpr uint32_t kQ = 0;                 // two Q buffers: the next work item's Q loads early
    static constexpr uint32_t kK = kQ + 2 * kQBuf;
    static constexpr uint32_t kV = kK + kStages * kKStage;
    // O staging for the TMA store of 16-bit outputs: two halves of 64 columns
    // (128 rows x 128 B, 128-byte swizzle), one per softmax warp parity
    static constexpr uint32_t kO = kV + kStages * kVStage;
    static constexpr uint32_t kBar = kO + 2 * 16384;
    // floats: running-maximum tokens [2][128]; per work item (double-buffered)
    // final maxima [2][2][128] and row sums [2][2][128]
    static constexpr uint32_t kRed = kBar + 512;
    // this pair's work items (computed once at start; every role reads them here)
    static constexpr uint32_t kItems = kRed + (256 + 512 + 512) * 4;
    static constexpr uint32_t kSmem = kItems + kMaxItems * 4 + 1024;
};

struct Args {
    void *out;
    int seq, nq_tiles, npairs, nkv_tiles, causal;
    int bh_total;     // batch * heads
    int clusters;     // CTA pairs launched (persistent)
    int group_heads;  // heads per L2 group of the work order
    float scale_log2;
    int *err;
};

// ---------------------------------------------------------------- cluster helpers
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the same shared variable in CTA `rank`
__device__ __forceinline__ uint32_t map_rank(uint32_t smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Arrival on an mbarrier of either CTA. P reaches the tensor core through TMEM,
// ordered by tcgen05.wait::st and tcgen05.fence before this arrive, so the arrive
// needs no cluster-scope release (which costs about a microsecond per step).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA tile load into this CTA's shared memory whose completion is counted on an
// mbarrier of this CTA or of its peer (CTA 0 counts both CTAs' bytes).
__device__ __forceinline__ void tma_load_3d_pair(void *dst, const CUtensorMap *map, uint32_t bar_cluster_addr, int32_t c0, int32_t c1,
                                                 int32_t c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// The issuing helpers below are executed by a whole converged warp and issue
// from one elected lane: issuing from a single divergent thread starves the
// tensor core when the SM sub-partition is shared with busy softmax warps.
// Eight M=256 MMAs into one accumulator under a single election (whole warp):
// D (+)= A_0 B_0, then D += A_i B_i. `accumulate` applies to the first only; fewer
// instructions per MMA keep the issue ahead of the tensor core (each executes in 64
// cycles per SM) when this warp shares its sub-partition with softmax warps.
#define JADE_PAIR_HEAD "{\n\t.reg .pred p, q, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %2, 0;\n\tsetp.ne.b32 q, 1, 0;\n\t"
#define JADE_PAIR_SS(a, b, pr) "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %" #a ", %" #b ", %1, " #pr ";\n\t"
#define JADE_PAIR_TS(a, b, pr) "@e tcgen05.mma.cta_group::2.kind::f16 [%0], [%" #a "], %" #b ", %1, " #pr ";\n\t"
__device__ __forceinline__ void umma_pair_ss8(uint32_t d_tmem, const uint64_t (&a)[8], const uint64_t (&b)[8], uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(JADE_PAIR_HEAD JADE_PAIR_SS(3, 11, p) JADE_PAIR_SS(4, 12, q) JADE_PAIR_SS(5, 13, q) JADE_PAIR_SS(6, 14, q)
                     JADE_PAIR_SS(7, 15, q) JADE_PAIR_SS(8, 16, q) JADE_PAIR_SS(9, 17, q) JADE_PAIR_SS(10, 18, q) "}" ::"r"(d_tmem),
                 "r"(idesc), "r"(accumulate), "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]),
                 "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7])
                 : "memory");
}
// A from TMEM at a_tmem + 8 i (16-bit pairs), B from shared-memory descriptors
__device__ __forceinline__ void umma_pair_ts8(uint32_t d_tmem, uint32_t a_tmem, const uint64_t (&b)[8], uint32_t idesc, uint32_t accumulate) {
    asm volatile(JADE_PAIR_HEAD JADE_PAIR_TS(3, 11, p) JADE_PAIR_TS(4, 12, q) JADE_PAIR_TS(5, 13, q) JADE_PAIR_TS(6, 14, q)
                     JADE_PAIR_TS(7, 15, q) JADE_PAIR_TS(8, 16, q) JADE_PAIR_TS(9, 17, q) JADE_PAIR_TS(10, 18, q) "}" ::"r"(d_tmem),
                 "r"(idesc), "r"(accumulate), "r"(a_tmem), "r"(a_tmem + 8), "r"(a_tmem + 16), "r"(a_tmem + 24), "r"(a_tmem + 32),
                 "r"(a_tmem + 40), "r"(a_tmem + 48), "r"(a_tmem + 56), "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]),
                 "l"(b[5]), "l"(b[6]), "l"(b[7])
                 : "memory");
}
#undef JADE_PAIR_HEAD
#undef JADE_PAIR_SS
#undef JADE_PAIR_TS
// One arrival on the mbarrier at `bar_cluster_addr` (either CTA) once every
// tcgen05 operation issued so far by the elected thread has completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster_addr) {
    asm volatile(
        "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar_cluster_addr)
        : "memory");
}

// This thread's row of an S tile (keys k0..k0+127) from TMEM into sv, causal and
// tail masks applied as -inf; returns the row maximum times c.
__device__ __forceinline__ float load_row_max(float (&sv)[kCols], uint32_t ts, int k0, int q0, int q, int seq, int causal, float c) {
    tc_fence_after();
#pragma unroll
    for (int cc = 0; cc < kCols; cc += 32) tmem_ld32f(ts + cc, sv + cc);
    tmem_wait_ld();
    reg_fence(sv);
    if ((causal && k0 + kKeys - 1 > q0) || (k0 + kKeys > seq)) {  // keys k0 + i with i > lim are invisible
        const int lim = min(seq - 1, causal ? q : INT_MAX) - k0;
#pragma unroll
        for (int i = 0; i < kCols; ++i) sv[i] = i <= lim ? sv[i] : -INFINITY;
    }
    float mx[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) mx[e] = max3(sv[e], sv[e + 8], sv[e + 16]);
#pragma unroll
    for (int i = 24; i < kCols - 8; i += 16)
#pragma unroll
        for (int e = 0; e < 8; ++e) mx[e] = max3(mx[e], sv[i + e], sv[i + 8 + e]);
#pragma unroll
    for (int e = 0; e < 8; ++e) mx[e] = fmaxf(mx[e], sv[kCols - 8 + e]);
    return max3(max3(mx[0], mx[1], mx[2]), max3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7])) * c;
}

// kGrouped: heads in L2-sized groups (the work items' K/V exceed the L2 budget);
// otherwise the single heavy-first order, computed inline.
template <typename TIn, typename TOut, bool kGrouped>
__global__ void __launch_bounds__(kThreads, 1)
    attention_pair_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, const Args args) {
    using L = Layout;
    constexpr uint32_t kFmt = std::is_same<TIn, __nv_bfloat16>::value ? 1u : 0u;
    constexpr uint32_t kIdescS = idesc_f32acc(kFmt, kFmt, false, false, 2 * kRows, kKeys);
    constexpr uint32_t kIdescO = idesc_f32acc(kFmt, kFmt, false, true, 2 * kRows, kDim);

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBar);
    uint64_t *q_full = bars + 0, *q_empty = bars + 2;                                        // [Q buffer]
    uint64_t *k_full = bars + 4, *k_empty = bars + 8, *v_full = bars + 12, *v_empty = bars + 16;  // [stage]
    uint64_t *s_full = bars + 20, *p_full = bars + 23;                                       // [S buffer]
    // P(g).V(g) done, for the O rescale: S(g+3) in general (issued right behind
    // it); o_tail[0], o_tail[1] for this pair's last two key steps
    uint64_t *o_tail = bars + 26;
    uint64_t *o_last = bars + 28;  // per work item: its last P.V done (O complete)
    uint64_t *o_free = bars + 29;  // per work item: O read out by both CTAs (next item may overwrite)
    uint64_t *pub = bars + 30;     // [lane quarter][step parity]: running maximum after a step published
    uint64_t *fin = bars + 38;     // [lane quarter]: both warps' final maxima and sums posted
    uint64_t *mma_done = bars + 42;
    uint64_t *stg_empty = bars + 43, *stg_full = bars + 45;  // [warp parity]: O staging free / written
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 47);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    float *tok = reinterpret_cast<float *>(smem + L::kRed);  // [2][128]
    float *fin_m = tok + 256, *fin_l = tok + 768;             // [2 items][2 warps][128]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int cluster = blockIdx.x >> 1;
    const int total_items = args.bh_total * args.npairs;
    // work item it: heaviest causal pairs first, all heads of a pair index together
    auto item_bh = [&](int it) { return it % args.bh_total; };
    auto item_pair = [&](int it) { return args.npairs - 1 - it / args.bh_total; };
    auto item_steps = [&](int it) {
        const int p = item_pair(it);
        return args.causal ? min(2 * p + 2, args.nkv_tiles) : args.nkv_tiles;
    };
    // This pair's k-th work item, -1 past the last. Heads are taken in groups of
    // group_heads whose K/V fit in L2 together, so concurrently running items share
    // cached K/V; within a group the items go heaviest pair index first, dealt out
    // boustrophedon (round r forward for even r, backward for odd r), which
    // balances the causal triangle to within a few percent. Items are numbered
    // it = pair_order * bh_total + head.
    auto item_order = [&](int k) {
        const int C = args.clusters;
        for (int h0 = 0; h0 < args.bh_total; h0 += args.group_heads) {
            const int hg = min(args.group_heads, args.bh_total - h0), G = hg * args.npairs;
            const int full = G / C, rem = G % C, slot_last = (full & 1) ? C - 1 - cluster : cluster;
            const int mine = full + (rem > 0 && slot_last < rem ? 1 : 0);
            if (k < mine) {
                const int i = k * C + ((k & 1) ? C - 1 - cluster : cluster);
                return (i / hg) * args.bh_total + h0 + i % hg;
            }
            k -= mine;
        }
        return -1;
    };
    int *items = reinterpret_cast<int *>(smem + L::kItems);  // this pair's items, -1 terminated (grouped order)
    auto item_of = [&](int k) {
        if constexpr (kGrouped) {
            return items[k];
        } else {
            const int it = k * args.clusters + ((k & 1) ? args.clusters - 1 - cluster : cluster);
            return it < total_items ? it : -1;
        }
    };
    int total_steps = 0;  // key steps over all of this pair's work items
    if constexpr (!kGrouped)
        for (int k = 0, it; (it = item_of(k)) >= 0; ++k) total_steps += item_steps(it);
    int *err = args.err;

    if (threadIdx.x == 0) {
        if constexpr (kGrouped) {
            int k = 0;
            for (int it; k < kMaxItems - 1 && (it = item_order(k)) >= 0; ++k) items[k] = it;
            items[k] = -1;
        }
        for (int b = 0; b < 2; ++b) { mbar_init(&q_full[b], 1); mbar_init(&q_empty[b], 1); }
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&k_full[s], 1); mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1); mbar_init(&v_empty[s], 1);
        }
        for (int b = 0; b < 3; ++b) {
            mbar_init(&s_full[b], 1);
            // CTA 0: its 4 step-owning softmax warps + one relayed arrival for CTA 1's
            mbar_init(&p_full[b], 4 + (leader ? 1 : 0));
        }
        mbar_init(&o_tail[0], 1);
        mbar_init(&o_tail[1], 1);
        mbar_init(o_last, 1);
        mbar_init(o_free, 8 + (leader ? 1 : 0));
        for (int q = 0; q < 8; ++q) mbar_init(&pub[q], 32);
        for (int q = 0; q < 4; ++q) mbar_init(&fin[q], 64);
        mbar_init(mma_done, 1);
        for (int p = 0; p < 2; ++p) { mbar_init(&stg_empty[p], 1); mbar_init(&stg_full[p], 128); }
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc_pair(tmem_slot, 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // barriers and TMEM of both CTAs exist before any cross-CTA use
    tc_fence_after();
    if constexpr (kGrouped)  // the list in shared memory is complete now
        for (int k = 0, it; (it = item_of(k)) >= 0; ++k) total_steps += item_steps(it);
    const uint32_t tmem = *tmem_slot;
    const uint32_t tmem_o = tmem + 384;

    if (warp == 0) {
        if (lane == 0) {  // ------------------------------------- TMA producer (both CTAs)
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            int g = 0, k = 0, q_issued = 0, k_issued = 0, v_issued = 0;
            bool ok = true;
            for (int it; ok && (it = item_of(k)) >= 0; ++k) {
                const int bh = item_bh(it), n = item_steps(it), q0 = (2 * item_pair(it) + (int)rank) * kRows, qb = k & 1;
                if (!(ok = mbar_wait(&q_empty[qb], ((k >> 1) & 1) ^ 1, abort_flag, err, kErrWaitSmemEmpty))) break;
                if (leader) mbar_arrive_expect_tx(&q_full[qb], 2 * L::kQBuf);
                const uint32_t qf = map_rank(smem_u32(&q_full[qb]), 0);
                for (int c = 0; c < 2; ++c) tma_load_3d_pair(smem + L::kQ + qb * L::kQBuf + c * 16384, &tmQ, qf, c * 64, q0, bh);
                q_issued = k + 1;
                // K(g) then V(g-1): a K load never queues behind a V stage that P.V still reads
                for (int j = 0; j <= n && ok; ++j) {
                    if (j < n) {
                        const int gk = g + j, st = gk % kStages;
                        if (!(ok = mbar_wait(&k_empty[st], ((gk / kStages) & 1) ^ 1, abort_flag, err, kErrWaitSmemEmpty))) break;
                        if (leader) mbar_arrive_expect_tx(&k_full[st], 2 * L::kKStage);
                        const uint32_t kf = map_rank(smem_u32(&k_full[st]), 0);
                        for (int c = 0; c < 2; ++c)
                            tma_load_3d_pair(smem + L::kK + st * L::kKStage + c * 8192, &tmK, kf, c * 64, j * kKeys + (int)rank * 64, bh);
                        k_issued = gk + 1;
                    }
                    if (j > 0) {
                        const int gv = g + j - 1, st = gv % kStages;
                        if (!(ok = mbar_wait(&v_empty[st], ((gv / kStages) & 1) ^ 1, abort_flag, err, kErrWaitSmemEmpty))) break;
                        if (leader) mbar_arrive_expect_tx(&v_full[st], 2 * L::kVStage);
                        tma_load_3d_pair(smem + L::kV + st * L::kVStage, &tmV, map_rank(smem_u32(&v_full[st]), 0), (int)rank * 64,
                                         (j - 1) * kKeys, bh);
                        v_issued = gv + 1;
                    }
                }
                g += n;
            }
            if (*abort_flag && leader) {  // CTA 0 counts both CTAs' copies: wait for those still in flight
                for (int kk = max(0, q_issued - 2); kk < q_issued; ++kk) mbar_wait_drain(&q_full[kk & 1], (kk >> 1) & 1, err);
                for (int gg = max(0, k_issued - kStages); gg < k_issued; ++gg) mbar_wait_drain(&k_full[gg % kStages], (gg / kStages) & 1, err);
                for (int gg = max(0, v_issued - kStages); gg < v_issued; ++gg) mbar_wait_drain(&v_full[gg % kStages], (gg / kStages) & 1, err);
            }
        }
    } else if (warp == 1) {
        if (leader) {  // ------------------------------- MMA issuer (CTA 0, whole warp, one elected lane issues)
            auto commit_both = [&](uint64_t *bar) {
                umma_commit_pair(smem_u32(bar));
                umma_commit_pair(map_rank(smem_u32(bar), 1));
            };
            // polling waits: a suspended waiter resumes a few hundred cycles after
            // the phase completes, and this warp waits several times per key step
            auto wait = [&](uint64_t *bar, uint32_t parity, int code) {
                return __all_sync(0xffffffffu, mbar_spin(bar, parity, abort_flag, err, code));
            };
            // Descriptors are built once and advanced by the 16-byte address units of each
            // operand (the start address is the low 14 bits; shared memory stays below
            // 256 KB, so the additions never carry out of the field).
            const uint64_t dq0 = sdesc_sw128(smem_u32(smem + L::kQ), 16, 1024);
            const uint64_t dk0 = sdesc_sw128(smem_u32(smem + L::kK), 16, 1024);
            const uint64_t dv0 = sdesc_sw128(smem_u32(smem + L::kV), 16384, 1024);
            // S issue cursor: work item (index it, sequence number k, n steps), local step j
            int s_k = 0, s_j = 0, s_n = item_of(0) >= 0 ? item_steps(item_of(0)) : 0;
            auto issue_s = [&](int gs, bool wait_inputs) {  // S(gs) = Q K^T into buffer gs % 3
                const int st = gs % kStages, qb = s_k & 1;
                if (wait_inputs) {
                    if (s_j == 0 && !wait(&q_full[qb], (s_k >> 1) & 1, kErrWaitTmaFull)) return false;
                    if (!wait(&k_full[st], (gs / kStages) & 1, kErrWaitTmaFull)) return false;
                }
                tc_fence_after();
                const uint64_t dq = dq0 + ((qb * L::kQBuf) >> 4), dk = dk0 + ((st * L::kKStage) >> 4);
                uint64_t a[kDim / 16], b[kDim / 16];
#pragma unroll
                for (int k = 0; k < kDim / 16; ++k) {
                    a[k] = dq + (((k >> 2) * 16384 + (k & 3) * 32) >> 4);
                    b[k] = dk + (((k >> 2) * 8192 + (k & 3) * 32) >> 4);
                }
                umma_pair_ss8(tmem + (gs % 3) * 128, a, b, kIdescS, 0);
                commit_both(&s_full[gs % 3]);
                commit_both(&k_empty[st]);
                if (s_j == s_n - 1) commit_both(&q_empty[qb]);  // the item's last S: its Q buffer is free
                if (++s_j == s_n) {
                    s_j = 0;
                    ++s_k;
                    const int nx = item_of(s_k);
                    s_n = nx >= 0 ? item_steps(nx) : 0;
                }
                return true;
            };
            bool ok = true;
            for (int gs = 0; ok && gs < 3 && gs < total_steps; ++gs) ok = issue_s(gs, true);
            int p_k = 0, p_j = 0, p_n = item_of(0) >= 0 ? item_steps(item_of(0)) : 0;
            for (int g = 0; ok && g < total_steps; ++g) {
                const int st = g % kStages;
                const bool more = g + 3 < total_steps;
                const bool first = p_j == 0 && p_k > 0;  // O still holds the previous item until it is read out
                // this step's inputs (P(g), V(g), K(g+3), Q of S(g+3)'s item, O free)
                // are tested together so the barrier latencies overlap; the bounded
                // waits run only if one is missing
                bool r = mbar_test_wait(&p_full[g % 3], (g / 3) & 1);
                r &= mbar_test_wait(&v_full[st], (g / kStages) & 1);
                if (more) r &= mbar_test_wait(&k_full[(g + 3) % kStages], ((g + 3) / kStages) & 1);
                if (more && s_j == 0) r &= mbar_test_wait(&q_full[s_k & 1], (s_k >> 1) & 1);
                if (first) r &= mbar_test_wait(o_free, (p_k - 1) & 1);
                if (!__all_sync(0xffffffffu, r)) {
                    if (!(ok = wait(&p_full[g % 3], (g / 3) & 1, kErrWaitProb))) break;
                    if (!(ok = wait(&v_full[st], (g / kStages) & 1, kErrWaitTmaFull))) break;
                    if (more && !(ok = wait(&k_full[(g + 3) % kStages], ((g + 3) / kStages) & 1, kErrWaitTmaFull))) break;
                    if (more && s_j == 0 && !(ok = wait(&q_full[s_k & 1], (s_k >> 1) & 1, kErrWaitTmaFull))) break;
                    if (first && !(ok = wait(o_free, (p_k - 1) & 1, kErrWaitPv))) break;
                }
                tc_fence_after();
                const uint64_t dv = dv0 + ((st * L::kVStage) >> 4);
                uint64_t b[kKeys / 16];
#pragma unroll
                for (int k = 0; k < kKeys / 16; ++k) b[k] = dv + ((k * 2048) >> 4);  // keys 16k..16k+15: P columns 8k..8k+7
                umma_pair_ts8(tmem_o, tmem + (g % 3) * 128, b, kIdescO, p_j != 0);
                commit_both(&v_empty[st]);
                if (g == total_steps - 3) commit_both(&o_tail[0]);
                if (g == total_steps - 2) commit_both(&o_tail[1]);
                if (p_j == p_n - 1) commit_both(o_last);
                if (more) issue_s(g + 3, false);  // reuses P(g)'s buffer: after P(g).V(g) in issue order
                if (++p_j == p_n) {
                    p_j = 0;
                    ++p_k;
                    const int nx = item_of(p_k);
                    p_n = nx >= 0 ? item_steps(nx) : 0;
                }
            }
            umma_commit_pair(smem_u32(mma_done));
            mbar_wait_drain(mma_done, 0, err);
        } else if (lane == 0) {  // --------------------------- relay (CTA 1)
            // One remote arrival per event instead of one per softmax warp: the
            // softmax warps arrive locally and this thread relays, in the order the
            // events happen: P(g) for the steps of a work item, then O read out.
            int g = 0, k = 0;
            bool ok = true;
            for (int it; ok && (it = item_of(k)) >= 0; ++k) {
                const int n = item_steps(it);
                for (int j = 0; j < n; ++j, ++g) {
                    if (!(ok = mbar_spin(&p_full[g % 3], (g / 3) & 1, abort_flag, err, kErrWaitProb))) break;
                    tc_fence_after();
                    tc_fence_before();
                    mbar_arrive_remote(map_rank(smem_u32(&p_full[g % 3]), 0));
                }
                if (ok && (ok = mbar_wait(o_free, k & 1, abort_flag, err, kErrWaitPv))) {
                    tc_fence_after();
                    tc_fence_before();
                    mbar_arrive_remote(map_rank(smem_u32(o_free), 0));
                }
            }
        }
    } else {
        // ----------------------------------------------------- softmax (warps 2-9, both CTAs)
        // Warp pair (w, w + 4) shares lane quarter w % 4: warp parity p = (w - 2) / 4
        // takes the key steps g = p, p + 2, ... (counted over all work items), one
        // thread per row. Within a work item the running maximum m is passed along
        // the steps through shared memory: step g's owner computes P(g) with the
        // maximum it last saw, then reads step g-1's published maximum; if that moved
        // it redoes P(g) (and rescales its row sum). If the row maximum grows by more
        // than 2^8 it raises m, redoes P(g) and rescales O after P(g-1).V(g-1) has
        // landed. Consecutive steps of the two warps overlap, so one computes while
        // the other waits. After an item's steps both warps combine their row sums,
        // normalise and store half of O each, and release O for the next item.
        const int quarter = warp & 3;
        const int par = (warp - 2) >> 2;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        const float c = args.scale_log2;
        bool ok = true;
        int g0 = 0, k = 0;
        for (int it; ok && (it = item_of(k)) >= 0; ++k) {
            const int bh = item_bh(it), n = item_steps(it), q0 = (2 * item_pair(it) + (int)rank) * kRows, q = q0 + row;
            float m_view = -INFINITY, l_own = 0.0f;  // l_own is in the scale of m_view
            for (int j = (par + g0) & 1; ok && j < n; j += 2) {
                const int g = g0 + j, b = g % 3;
                const uint32_t ts = tmem + b * 128 + lane_off;
                // the item's first two steps start from the maximum over both of their
                // tiles, computed by both warps alike, so neither waits for the other
                float sv[kCols];
                float m_pre = -INFINITY;
                if (j <= 1 && n >= 2) {
                    const int go = g0 + (j ^ 1);
                    if (!(ok = __all_sync(0xffffffffu, mbar_spin(&s_full[go % 3], (go / 3) & 1, abort_flag, err, kErrWaitScore))))
                        break;
                    m_pre = load_row_max(sv, tmem + (go % 3) * 128 + lane_off, (j ^ 1) * kKeys, q0, q, args.seq, args.causal, c);
                }
                if (!(ok = __all_sync(0xffffffffu, mbar_spin(&s_full[b], (g / 3) & 1, abort_flag, err, kErrWaitScore)))) break;
                const float m_tile = load_row_max(sv, ts, j * kKeys, q0, q, args.seq, args.causal, c);
                // the maximum published by step g-1 of this item (the other warp's)
                auto read_prev = [&]() {
                    if (!__all_sync(0xffffffffu, mbar_spin(&pub[quarter * 2 + (par ^ 1)], ((g - 1) >> 1) & 1, abort_flag, err, kErrWaitScore)))
                        return false;
                    const float m_prev = tok[(par ^ 1) * 128 + row];
                    if (m_prev != m_view) {  // the other warp raised m since this warp's last step
                        l_own *= m_view == -INFINITY ? 0.0f : mufu_exp2(m_view - m_prev);
                        m_view = m_prev;
                    }
                    return true;
                };
                float psum = 0.0f;
                bool fresh = false;  // P(g) in TMEM was computed with the current m_view
                if (j == 0) {
                    m_view = fmaxf(m_tile, m_pre);
                } else {
                    if (j == 1) m_view = fmaxf(m_tile, m_pre);  // equals what step 0 publishes
                    const float m_spec = m_view;
                    psum = store_p<kFmt, false, kCols>(sv, c, m_spec, ts);  // all exponentials on MUFU (measured best here)
                    if (!(ok = read_prev())) break;
                    fresh = __all_sync(0xffffffffu, m_view == m_spec);
                }
                float alpha = 1.0f;
                if (j > 0 && __any_sync(0xffffffffu, m_tile > m_view + kRescaleThreshold)) {
                    if (m_tile > m_view + kRescaleThreshold) {
                        alpha = mufu_exp2(m_view - m_tile);
                        m_view = m_tile;
                    }
                    fresh = false;
                    // O (in TMEM) to the new maxima once P(g-1).V(g-1) has landed: S(g+2)
                    // was issued right behind it (its next phase needs P(g+2) from this
                    // warp, so the wait cannot alias); the last two steps have o_tail.
                    if (g + 2 < total_steps)
                        ok = __all_sync(0xffffffffu, mbar_wait(&s_full[(g + 2) % 3], ((g + 2) / 3) & 1, abort_flag, err, kErrWaitPv));
                    else
                        ok = __all_sync(0xffffffffu, mbar_wait(&o_tail[g + 2 - total_steps], 0, abort_flag, err, kErrWaitPv));
                    if (!ok) break;
                    tc_fence_after();
#pragma unroll 1
                    for (int oc = 0; oc < kDim; oc += 32) {
                        float ov[32];
                        tmem_ld32f(tmem_o + lane_off + oc, ov);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) ov[i] *= alpha;
                        tmem_st32f(tmem_o + lane_off + oc, ov);
                    }
                    l_own *= alpha;
                }
                if (!fresh) psum = store_p<kFmt, false, kCols>(sv, c, m_view, ts);
                l_own += psum;
                // publish the running maximum after step g for the owner of step g+1
                tok[par * 128 + row] = m_view;
                mbar_arrive(&pub[quarter * 2 + par]);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[b]);
            }
            if (!ok) break;
            // row sum: both warps' sums brought to the final (largest) maximum
            float *fm = fin_m + (k & 1) * 256, *fl = fin_l + (k & 1) * 256;
            fm[par * 128 + row] = m_view;
            fl[par * 128 + row] = l_own;
            mbar_arrive(&fin[quarter]);
            ok = __all_sync(0xffffffffu, mbar_spin(&fin[quarter], k & 1, abort_flag, err, kErrWaitScore));
            if (ok) ok = __all_sync(0xffffffffu, mbar_wait(o_last, k & 1, abort_flag, err, kErrWaitPv));
            if (!ok) break;
            const float m_other = fm[(par ^ 1) * 128 + row], l_other = fl[(par ^ 1) * 128 + row];
            const float m_final = fmaxf(m_view, m_other);
            const float l_row = (l_own > 0.0f ? l_own * mufu_exp2(m_view - m_final) : 0.0f) +
                                (l_other > 0.0f ? l_other * mufu_exp2(m_other - m_final) : 0.0f);
            const float inv = 1.0f / l_row;
            tc_fence_after();
            // this warp's half of the row's output columns, then O is free for the next item
            float r[64];
            tmem_ld32f(tmem_o + lane_off + par * 64, r);
            tmem_ld32f(tmem_o + lane_off + par * 64 + 32, r + 32);
            tmem_wait_ld();
            reg_fence(r);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_free);
            if constexpr (std::is_same<TOut, float>::value) {
                float *o = static_cast<float *>(args.out) + ((size_t)bh * args.seq + q) * kDim + par * 64;
                if (q < args.seq)
#pragma unroll
                    for (int e = 0; e < 64; e += 4) *reinterpret_cast<float4 *>(o + e) = make_float4(r[e] * inv, r[e + 1] * inv, r[e + 2] * inv, r[e + 3] * inv);
            } else {
                // staged in shared memory (128-byte swizzle, the tensor map's layout) and
                // written by one TMA store per half: coalesced, and rows past seq are clipped
                const bool issuer = warp == 2 + 4 * par && lane == 0;
                uint8_t *stg = smem + L::kO + par * 16384;
                if (issuer) {  // the previous item's store has finished reading the staging buffer
                    bulk_wait_read_all();
                    mbar_arrive(&stg_empty[par]);
                }
                ok = __all_sync(0xffffffffu, mbar_spin(&stg_empty[par], k & 1, abort_flag, err, kErrWaitPv));
                if (!ok) break;
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) {
                    uint4 u;
                    u.x = pack16<kFmt>(r[8 * ch] * inv, r[8 * ch + 1] * inv);
                    u.y = pack16<kFmt>(r[8 * ch + 2] * inv, r[8 * ch + 3] * inv);
                    u.z = pack16<kFmt>(r[8 * ch + 4] * inv, r[8 * ch + 5] * inv);
                    u.w = pack16<kFmt>(r[8 * ch + 6] * inv, r[8 * ch + 7] * inv);
                    *reinterpret_cast<uint4 *>(stg + row * 128 + ((ch ^ (row & 7)) << 4)) = u;
                }
                fence_proxy_async();
                mbar_arrive(&stg_full[par]);
                if (issuer) {
                    if (!(ok = mbar_spin(&stg_full[par], k & 1, abort_flag, err, kErrWaitPv))) break;
                    if (q0 < args.seq) tma_store_3d(&tmO, stg, par * 64, q0, bh);
                    bulk_commit_group();
                }
            }
            g0 += n;
        }
    }
    if (warp >= 2 && (warp - 2) % 4 == 0 && lane == 0) bulk_wait_all();  // output stores complete
    // every thread of both CTAs: the pair's MMAs and TMEM reads are over
    tc_fence_before();
    __syncwarp();
    cluster_sync();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, 512);
    }
}

// ------------------------------------------------------------------ host side
using EncodeFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *, const cuuint64_t *,
                              const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                              CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encoder() {
    static EncodeFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] { fn = reinterpret_cast<EncodeFn>(driver_entry("cuTensorMapEncodeTiled")); });
    return fn;
}

// [bh, seq, 128] tensor, box {64, rows, 1}, 128-byte swizzle.
bool make_map(CUtensorMap *map, CUtensorMapDataType dt, const void *ptr, uint64_t bh, uint64_t seq, uint32_t rows) {
    EncodeFn enc = encoder();
    if (!enc) return false;
    const cuuint64_t dims[3] = {kDim, seq, bh};
    const cuuint64_t strides[2] = {kDim * 2, seq * kDim * 2};
    const cuuint32_t box[3] = {64, rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, dt, 3, const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename TIn, typename TOut>
LaunchFn pair_launch(Context *ctx, const Spec &s) {
    const long long heads_all = (long long)s.batch * s.heads;
    // heads whose K and V fit in about 64 MB of the 126 MB L2, in even groups
    const int group_heads = attention_group_heads(heads_all, s.seq, kDim, kGroupBytes);
    const bool grouped = group_heads < heads_all;
    auto kernel = grouped ? attention_pair_kernel<TIn, TOut, true> : attention_pair_kernel<TIn, TOut, false>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Layout::kSmem) != cudaSuccess)
        throw IrError("cannot reserve shared memory for the tcgen05 pair attention");
    const CUtensorMapDataType dt = std::is_same<TIn, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    Args base{};
    base.seq = (int)s.seq;
    const int heads_total = (int)(s.batch * s.heads);
    base.nq_tiles = (int)((s.seq + kRows - 1) / kRows);
    base.npairs = (base.nq_tiles + 1) / 2;
    base.nkv_tiles = (int)((s.seq + kKeys - 1) / kKeys);
    base.causal = s.causal ? 1 : 0;
    base.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)kDim));
    base.err = ctx->err_dev;
    base.bh_total = heads_total;
    const long long items = (long long)heads_total * base.npairs;
    if (items > INT_MAX / 2) throw IrError("attention too large for the pair kernel's work-item index");
    // persistent: as many CTA pairs as can be resident, each looping over work items
    int resident = 0;
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * 148);
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = Layout::kSmem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&resident, kernel, &cfg) != cudaSuccess || resident <= 0)
            throw IrError("cannot size the persistent pair attention grid");
    }
    base.clusters = (int)std::min<long long>(items, resident);
    base.group_heads = group_heads;
    if (grouped) {  // items per pair: at most ceil(group items / pairs) per head group
        long long bound = 0;
        for (long long h0 = 0; h0 < heads_total; h0 += base.group_heads)
            bound += (std::min<long long>(base.group_heads, heads_total - h0) * base.npairs + base.clusters - 1) / base.clusters;
        if (bound > kMaxItems - 1) throw IrError("attention has too many work items per SM pair for the pair kernel");
    }
    const dim3 grid(2 * base.clusters);
    const uint64_t bh = heads_total, seq = s.seq;
    const bool out16 = !std::is_same<TOut, float>::value;
    return [=](cudaStream_t st, void **b) {
        CUtensorMap mq, mk, mv, mo;
        if (!make_map(&mq, dt, b[0], bh, seq, 128) || !make_map(&mk, dt, b[1], bh, seq, 64) || !make_map(&mv, dt, b[2], bh, seq, 128))
            return cudaErrorInvalidValue;
        // 16-bit outputs leave through TMA stores (same element type as the inputs)
        if (out16 ? !make_map(&mo, dt, b[3], bh, seq, 128) : !make_map(&mo, dt, b[0], bh, seq, 128)) return cudaErrorInvalidValue;
        Args a = base;
        a.out = b[3];
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = grid;
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = Layout::kSmem;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, kernel, mq, mk, mv, mo, a);
    };
}

}  // namespace

// Head dim 128, BF16/FP16 inputs: the CTA-pair kernel above.
LaunchFn make_attention_pair(Context *ctx, const Spec &s, std::string &impl) {
    if (s.op != Op::AttentionOnline || s.dim != 128) throw IrError("the pair attention kernel covers attention_online with dim 128");
    if (!encoder()) throw IrError("cuTensorMapEncodeTiled unavailable");
    impl = std::string("attention_tcgen05_fa_pair_q256_kv128_d128_") + dtype_name(s.dtype) + "_out_" + dtype_name(s.out_dtype) +
           (s.causal ? "_causal" : "");
    const bool f32out = s.out_dtype == DType::F32;
    if (s.dtype == DType::BF16)
        return f32out ? pair_launch<__nv_bfloat16, float>(ctx, s) : pair_launch<__nv_bfloat16, __nv_bfloat16>(ctx, s);
    return f32out ? pair_launch<__half, float>(ctx, s) : pair_launch<__half, __half>(ctx, s);
}

}  // namespace jade
