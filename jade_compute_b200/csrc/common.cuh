// Device helpers for sm_100a: bf16/fp16 conversion, mbarrier waits with a time
// limit, TMA tile loads, and the tcgen05 (5th-generation tensor core) PTX used by
// the GEMM and attention kernels. Every spin on an mbarrier is bounded: after
// JADE_WAIT_LIMIT_NS the waiter records an error code in the context's mapped
// error word and the kernel leaves through its normal exit path (TMEM freed).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef JADE_WAIT_LIMIT_NS
#define JADE_WAIT_LIMIT_NS 2000000000ull  // 2 s
#endif

namespace jade {

// Error codes written to the device error word (first writer wins).
enum DeviceError : int {
    kErrNone = 0,
    kErrWaitTmaFull = 1,    // MMA warp waiting for a TMA stage
    kErrWaitSmemEmpty = 2,  // producer waiting for a free stage
    kErrWaitAccFull = 3,    // epilogue waiting for an accumulator
    kErrWaitAccEmpty = 4,   // MMA waiting for the epilogue to drain TMEM
    kErrWaitScore = 5,      // attention softmax waiting for S
    kErrWaitProb = 6,       // attention MMA waiting for P
    kErrWaitPv = 7,         // attention correction waiting for PV
    kErrWaitDrain = 8,      // exit path waiting for copies in flight
    kErrBadLaunch = 9,      // launch geometry mismatch detected on device
    kErrWaitProbe = 10,     // wait_probe: a wait that nothing satisfies, expired as designed
};

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait. Returns false when the CTA already aborted or the limit expired
// (the error word then holds `code`). `abort_flag` is a CTA-shared word so that
// one expired wait ends every role of the CTA promptly.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *err, int code) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
#pragma unroll 1
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (globaltimer() - t0 > JADE_WAIT_LIMIT_NS) {
            if (err) atomicCAS(err, 0, code);
            *abort_flag = 1;
            return false;
        }
    }
}
// mbar_wait with a time limit given at run time (the wait_probe op).
__device__ __forceinline__ bool mbar_wait_for(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *err, int code,
                                              uint64_t limit_ns) {
    const uint64_t t0 = globaltimer();
#pragma unroll 1
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (globaltimer() - t0 > limit_ns) {
            if (err) atomicCAS(err, 0, code);
            *abort_flag = 1;
            return false;
        }
    }
}
// try_wait that lets the thread sleep up to `ns` nanoseconds (it wakes when the
// phase completes): for waits that may last many microseconds, so that the waiting
// warp does not loop on its sub-partition beside busy warps.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}
// Bounded wait built on mbar_try_wait_sleep (same contract as mbar_wait).
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *err, int code,
                                                uint32_t ns = 20000) {
    if (mbar_try_wait_sleep(bar, parity, ns)) return true;
    const uint64_t t0 = globaltimer();
#pragma unroll 1
    while (true) {
        if (mbar_try_wait_sleep(bar, parity, ns)) return true;
        if (*abort_flag) return false;
        if (globaltimer() - t0 > JADE_WAIT_LIMIT_NS) {
            if (err) atomicCAS(err, 0, code);
            *abort_flag = 1;
            return false;
        }
    }
}
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded polling wait (no suspension: the phases waited on here complete within
// a few hundred cycles, and a suspended waiter can resume much later than that).
__device__ __forceinline__ bool mbar_spin(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *err, int code) {
    if (mbar_test_wait(bar, parity)) return true;  // usual case: no timer read
    const uint64_t t0 = globaltimer();
#pragma unroll 1
    while (true) {
        if (mbar_test_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (globaltimer() - t0 > JADE_WAIT_LIMIT_NS) {
            if (err) atomicCAS(err, 0, code);
            *abort_flag = 1;
            return false;
        }
    }
}
// Wait used on exit paths for copies still in flight: ignores the abort flag and
// only gives up at the time limit.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t *bar, uint32_t parity, int *err) {
    const uint64_t t0 = globaltimer();
#pragma unroll 1
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - t0 > JADE_WAIT_LIMIT_NS) {
            if (err) atomicCAS(err, 0, kErrWaitDrain);
            return false;
        }
    }
    return true;
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int32_t c0, int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int32_t c0, int32_t c1, int32_t c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

// Contiguous bulk copy global -> this CTA's shared memory, completion counted on
// an mbarrier (addresses 16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
                 "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
// TMA tile store from this CTA's shared memory (rows beyond the tensor are clipped).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int32_t c0, int32_t c1, int32_t c2) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}
// Contiguous bulk copy this CTA's shared memory -> global, tracked by bulk groups
// (addresses 16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_store(void *dst, const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(reinterpret_cast<uint64_t>(dst)),
                 "r"(smem_u32(src)), "r"(bytes)
                 : "memory");
}
// all but this thread's newest bulk group have finished reading shared memory
__device__ __forceinline__ void bulk_wait_read_but_one() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// this thread's bulk stores have finished reading shared memory
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// this thread's bulk stores are complete
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Warp-group register reallocation (all four warps of the group execute it).
template <int N>
__device__ __forceinline__ void reg_alloc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }
template <int N>
__device__ __forceinline__ void reg_dealloc() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// The MMA issuing helpers below are executed by a whole converged warp and issue
// from one elected lane. A single divergent lane issuing MMAs gets starved of
// issue slots by busy warps on the same SM sub-partition (measured on B200: the
// tensor pipe fell to 37% of its rate beside FFMA-bound warps; the elected form
// keeps it at 100%).
// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16/fp16 inputs) or kind::tf32.
template <bool kTf32>
__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    if constexpr (kTf32) {
        asm volatile(
            "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    }
}
// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16 (whole warp, one elected lane issues).
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Groups of kind::f16 MMAs into one accumulator, issued with a single election
// (whole warp): D (+)= A_0 B_0, then D += A_i B_i for i >= 1. `accumulate`
// applies to the first MMA only. The fewer instructions per MMA keep the issue
// ahead of the tensor core when the issuing warp shares its sub-partition with
// busy warps (a 128x128x16 MMA executes in 64 cycles).
#define JADE_UMMA_HEAD "{\n\t.reg .pred p, q, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %2, 0;\n\tsetp.ne.b32 q, 1, 0;\n\t"
#define JADE_UMMA_SS(a, b, pr) "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %" #a ", %" #b ", %1, " #pr ";\n\t"
#define JADE_UMMA_TS(a, b, pr) "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%" #a "], %" #b ", %1, " #pr ";\n\t"
// N = 4 or 8: A and B from shared-memory descriptors
template <int N>
__device__ __forceinline__ void umma_ss_group(uint32_t d_tmem, const uint64_t (&a)[N], const uint64_t (&b)[N], uint32_t idesc,
                                              uint32_t accumulate) {
    static_assert(N == 4 || N == 8, "groups of 4 or 8 MMAs");
    if constexpr (N == 4) {
        asm volatile(JADE_UMMA_HEAD JADE_UMMA_SS(3, 7, p) JADE_UMMA_SS(4, 8, q) JADE_UMMA_SS(5, 9, q) JADE_UMMA_SS(6, 10, q) "}" ::"r"(d_tmem),
                     "r"(idesc), "r"(accumulate), "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3])
                     : "memory");
    } else {
        asm volatile(JADE_UMMA_HEAD JADE_UMMA_SS(3, 11, p) JADE_UMMA_SS(4, 12, q) JADE_UMMA_SS(5, 13, q) JADE_UMMA_SS(6, 14, q)
                         JADE_UMMA_SS(7, 15, q) JADE_UMMA_SS(8, 16, q) JADE_UMMA_SS(9, 17, q) JADE_UMMA_SS(10, 18, q) "}" ::"r"(d_tmem),
                     "r"(idesc), "r"(accumulate), "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]),
                     "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7])
                     : "memory");
    }
}
// 8 MMAs with A read from TMEM (a_tmem + 8 i: 16 columns of 16-bit pairs each) and
// B from shared-memory descriptors
__device__ __forceinline__ void umma_ts_group8(uint32_t d_tmem, uint32_t a_tmem, const uint64_t (&b)[8], uint32_t idesc,
                                               uint32_t accumulate) {
    asm volatile(JADE_UMMA_HEAD JADE_UMMA_TS(3, 11, p) JADE_UMMA_TS(4, 12, q) JADE_UMMA_TS(5, 13, q) JADE_UMMA_TS(6, 14, q)
                     JADE_UMMA_TS(7, 15, q) JADE_UMMA_TS(8, 16, q) JADE_UMMA_TS(9, 17, q) JADE_UMMA_TS(10, 18, q) "}" ::"r"(d_tmem),
                 "r"(idesc), "r"(accumulate), "r"(a_tmem), "r"(a_tmem + 8), "r"(a_tmem + 16), "r"(a_tmem + 24), "r"(a_tmem + 32),
                 "r"(a_tmem + 40), "r"(a_tmem + 48), "r"(a_tmem + 56), "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "l"(b[4]),
                 "l"(b[5]), "l"(b[6]), "l"(b[7])
                 : "memory");
}
#undef JADE_UMMA_HEAD
#undef JADE_UMMA_SS
#undef JADE_UMMA_TS

// Arrive once on `bar` when every tcgen05 operation issued so far by the elected
// lane completes (whole warp; the same lane is elected each time in a converged warp).
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
        : "memory");
}
// Bounded wait taken by a whole warp with a warp-uniform result.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *err, int code) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, err, code));
}

// Shared-memory matrix descriptor (tcgen05 format, version 1), 128-byte swizzle.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= 1ull << 46;  // descriptor version for tcgen05
    d |= 2ull << 61;  // SWIZZLE_128B
    return d;
}

// Instruction descriptor: FP32 accumulate, dense, A/B format codes (f16 0, bf16 1, tf32 2).
__host__ __device__ constexpr uint32_t idesc_f32acc(uint32_t a_fmt, uint32_t b_fmt, bool a_mn_major, bool b_mn_major, uint32_t m, uint32_t n) {
    return (1u << 4) | (a_fmt << 7) | (b_fmt << 10) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
           ((n >> 3) << 17) | ((m >> 4) << 24);
}

// 32 lanes x 32 columns of 32-bit TMEM values: thread t of the warp receives
// columns [col, col+32) of lane (lane_base + t).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
// Same load, straight into FP32 registers (no integer temporaries to keep alive).
__device__ __forceinline__ void tmem_ld32f(uint32_t taddr, float *r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3]), "=f"(r[4]), "=f"(r[5]), "=f"(r[6]), "=f"(r[7]), "=f"(r[8]),
          "=f"(r[9]), "=f"(r[10]), "=f"(r[11]), "=f"(r[12]), "=f"(r[13]), "=f"(r[14]), "=f"(r[15]), "=f"(r[16]),
          "=f"(r[17]), "=f"(r[18]), "=f"(r[19]), "=f"(r[20]), "=f"(r[21]), "=f"(r[22]), "=f"(r[23]), "=f"(r[24]),
          "=f"(r[25]), "=f"(r[26]), "=f"(r[27]), "=f"(r[28]), "=f"(r[29]), "=f"(r[30]), "=f"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32f(uint32_t taddr, const float *r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "f"(r[0]), "f"(r[1]), "f"(r[2]), "f"(r[3]), "f"(r[4]), "f"(r[5]), "f"(r[6]), "f"(r[7]), "f"(r[8]), "f"(r[9]),
        "f"(r[10]), "f"(r[11]), "f"(r[12]), "f"(r[13]), "f"(r[14]), "f"(r[15]), "f"(r[16]), "f"(r[17]), "f"(r[18]),
        "f"(r[19]), "f"(r[20]), "f"(r[21]), "f"(r[22]), "f"(r[23]), "f"(r[24]), "f"(r[25]), "f"(r[26]), "f"(r[27]),
        "f"(r[28]), "f"(r[29]), "f"(r[30]), "f"(r[31])
        : "memory");
}
// 32 lanes x 8 columns of 32-bit values from registers into TMEM.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t *r) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]),
                 "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- conversions
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}
__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// Stable logistic function in the reference's branch form (src/runtime/ir.rs:487).
__device__ __forceinline__ float stable_sigmoid(float v) {
    const float e = expf(-fabsf(v));
    return v >= 0.0f ? 1.0f / (1.0f + e) : e / (1.0f + e);
}

}  // namespace jade
