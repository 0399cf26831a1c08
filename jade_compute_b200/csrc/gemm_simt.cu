// FP32 FFMA GEMM (the faithful path) and the SIMT fallback for tensor-core
// dtypes on shapes whose strides TMA cannot describe.
//
// Reference: src/runtime/ir.rs:524-557 (gemm_naive / gemm_register32) and
// src/runtime/metal_simd.rs:24-110 (FP32 SIMD-group GEMM). Each output is
// accumulated as acc = fmaf(a[row,p], b[p,col], acc) for p = 0..K-1 in order,
// starting from 0, which is exactly what the reference kernels compute, so FP32
// results are bit-identical to them (and to the CPU restatement
// or_gemm_fp32_sequential). Tiling: BM x BN block tile, K-step 8, each thread
// holding TM x TN outputs in registers, shared-memory double buffering. Two
// shapes: 128x128 tiles of 8x8 per thread (256 threads) when the output has at
// least one tile per SM, else 32x64 tiles of 4x4 per thread (128 threads), which
// spread a small GEMM (512^3: 128 blocks instead of 16) over the SMs; the k
// order of every sum is the same in both.
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "internal.hpp"

namespace jade {
namespace {

constexpr int BK = 8;

template <typename TA> __device__ __forceinline__ float load_op(const TA *p, bool tf32);
template <> __device__ __forceinline__ float load_op<float>(const float *p, bool tf32) {
    float v = __ldg(p);
    if (tf32) {
        uint32_t r;
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
        v = __uint_as_float(r);
    }
    return v;
}
template <> __device__ __forceinline__ float load_op<__nv_bfloat16>(const __nv_bfloat16 *p, bool) { return __bfloat162float(*p); }
template <> __device__ __forceinline__ float load_op<__half>(const __half *p, bool) { return __half2float(*p); }

// C[M,N] = A[M,K] * B   (B is [K,N] row-major, or [N,K] when kBnk). Thread
// (tx, ty) owns TM/4 groups of 4 rows, group g at row ty*4 + g*BM/(TM/4), and
// likewise TN/4 groups of 4 columns, so each k step reads its operands from
// shared memory as conflict-free float4s.
template <typename TA, typename TO, bool kBnk, int BM, int BN, int TM, int TN>
__global__ void __launch_bounds__((BM / TM) * (BN / TN))
    gemm_ffma_kernel(const TA *__restrict__ A, const TA *__restrict__ B, TO *__restrict__ C, int M, int N, int K, bool tf32,
                     const float *__restrict__ row_scale, const TO *__restrict__ residual) {
    constexpr int kThreads = (BM / TM) * (BN / TN);
    constexpr int kLoadsA = BM * BK / kThreads, kLoadsB = BN * BK / kThreads;
    constexpr int kGroupsM = TM / 4, kGroupsN = TN / 4;
    constexpr int kRowStride = BM / kGroupsM, kColStride = BN / kGroupsN;
    static_assert(kLoadsA * kThreads == BM * BK && kLoadsB * kThreads == BN * BK, "tile loads must divide evenly");
    __shared__ __align__(16) float As[2][BK][BM];
    __shared__ __align__(16) float Bs[2][BK][BN];
    const int t = threadIdx.x;
    const int tx = t % (BN / TN), ty = t / (BN / TN);
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

    float ra[kLoadsA], rb[kLoadsB];
    auto gload = [&](int k0) {
#pragma unroll
        for (int i = 0; i < kLoadsA; ++i) {  // A element (r, kk): consecutive threads walk k within a row
            const int idx = t + kThreads * i;
            const int r = idx / BK, kk = idx % BK;
            const int gr = m0 + r, gk = k0 + kk;
            ra[i] = (gr < M && gk < K) ? load_op(A + (size_t)gr * K + gk, tf32) : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < kLoadsB; ++i) {
            const int idx = t + kThreads * i;
            if (!kBnk) {  // B element (kk, c): consecutive threads walk columns
                const int kk = idx / BN, c = idx % BN;
                const int gk = k0 + kk, gc = n0 + c;
                rb[i] = (gk < K && gc < N) ? load_op(B + (size_t)gk * N + gc, tf32) : 0.0f;
            } else {
                const int c = idx / BK, kk = idx % BK;
                const int gk = k0 + kk, gc = n0 + c;
                rb[i] = (gk < K && gc < N) ? load_op(B + (size_t)gc * K + gk, tf32) : 0.0f;
            }
        }
    };
    auto sstore = [&](int buf) {
#pragma unroll
        for (int i = 0; i < kLoadsA; ++i) {
            const int idx = t + kThreads * i;
            As[buf][idx % BK][idx / BK] = ra[i];
        }
#pragma unroll
        for (int i = 0; i < kLoadsB; ++i) {
            const int idx = t + kThreads * i;
            if (!kBnk) Bs[buf][idx / BN][idx % BN] = rb[i];
            else Bs[buf][idx % BK][idx / BK] = rb[i];
        }
    };

    const int ktiles = (K + BK - 1) / BK;
    gload(0);
    sstore(0);
    __syncthreads();
    for (int kt = 0; kt < ktiles; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < ktiles) gload((kt + 1) * BK);
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float a[TM], b[TN];
#pragma unroll
            for (int g = 0; g < kGroupsM; ++g) {
                const float4 v = *reinterpret_cast<const float4 *>(&As[buf][kk][g * kRowStride + ty * 4]);
                a[4 * g] = v.x; a[4 * g + 1] = v.y; a[4 * g + 2] = v.z; a[4 * g + 3] = v.w;
            }
#pragma unroll
            for (int g = 0; g < kGroupsN; ++g) {
                const float4 v = *reinterpret_cast<const float4 *>(&Bs[buf][kk][g * kColStride + tx * 4]);
                b[4 * g] = v.x; b[4 * g + 1] = v.y; b[4 * g + 2] = v.z; b[4 * g + 3] = v.w;
            }
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (kt + 1 < ktiles) {
            sstore(buf ^ 1);
            __syncthreads();
        }
    }
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int r = m0 + (i / 4) * kRowStride + ty * 4 + (i % 4);
        if (r >= M) continue;
        const float sc = row_scale ? row_scale[r] : 1.0f;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            const int c = n0 + (j / 4) * kColStride + tx * 4 + (j % 4);
            if (c >= N) continue;
            float v = row_scale ? acc[i][j] * sc : acc[i][j];
            if (residual) v += to_f32(residual[(size_t)r * N + c]);
            C[(size_t)r * N + c] = from_f32<TO>(v);
        }
    }
}

template <typename TA, typename TO, int BM, int BN, int TM, int TN>
LaunchFn ffma_launch_tiles(const Spec &s, bool tf32) {
    const int M = (int)s.m, N = (int)s.n, K = (int)s.k;
    const dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    constexpr int threads = (BM / TM) * (BN / TN);
    const bool bnk = s.b_nk, rs = s.row_scale, res = s.epilogue == "residual";
    return [=](cudaStream_t st, void **b) {
        int idx = 2;
        const float *row_scale = rs ? static_cast<const float *>(b[idx++]) : nullptr;
        const TO *residual = res ? static_cast<const TO *>(b[idx++]) : nullptr;
        TO *out = static_cast<TO *>(b[idx]);
        if (bnk)
            gemm_ffma_kernel<TA, TO, true, BM, BN, TM, TN>
                <<<grid, threads, 0, st>>>((const TA *)b[0], (const TA *)b[1], out, M, N, K, tf32, row_scale, residual);
        else
            gemm_ffma_kernel<TA, TO, false, BM, BN, TM, TN>
                <<<grid, threads, 0, st>>>((const TA *)b[0], (const TA *)b[1], out, M, N, K, tf32, row_scale, residual);
        return cudaGetLastError();
    };
}

// ------------------------------------------------------------------ FP32, TMA-fed
// FP32 A [M,K] . B [K,N] with both strides multiples of 16 bytes: the operand
// tiles arrive by TMA (cp.async.bulk.tensor) into a STAGES-deep shared-memory
// ring, k tiles of 16, one mbarrier per stage, so that STAGES-1 tiles are in
// flight while one is multiplied (the register-staged kernel above keeps one
// 8-wide k tile in flight and measured latency-bound: 26 FFMA/clk/SM). A lands
// row-major [BM][16]: a thread reads a float4 of 4 consecutive k per row it owns;
// B lands [16][BN]. Each output still sums its k products in order with one fmaf
// each (the ring only changes when operands arrive), so the result is the same
// bits as the sequential FP32 sum. Out-of-range rows, columns and k are
// zero-filled by TMA and never stored.
constexpr int kTmaBK = 16;

template <int BM, int BN, int TM, int TN, int STAGES>
__global__ void __launch_bounds__((BM / TM) * (BN / TN))
    gemm_ffma_tma_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, float *__restrict__ C, int M,
                         int N, int K, int *err) {
    constexpr int kGroupsM = TM / 4, kGroupsN = TN / 4;
    constexpr int kRowStride = BM / kGroupsM, kColStride = BN / kGroupsN;
    constexpr uint32_t kStageA = BM * kTmaBK * 4, kStageB = kTmaBK * BN * 4;
    extern __shared__ uint8_t smem_raw[];
    float *ring = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    __shared__ uint64_t full[STAGES];
    __shared__ int abort_flag;
    const int t = threadIdx.x;
    const int tx = t % (BN / TN), ty = t / (BN / TN);
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int ktiles = (K + kTmaBK - 1) / kTmaBK;
    auto stage_a = [&](int s) { return ring + s * ((kStageA + kStageB) / 4); };
    auto stage_b = [&](int s) { return ring + s * ((kStageA + kStageB) / 4) + kStageA / 4; };
    auto issue = [&](int kt) {
        const int s = kt % STAGES;
        mbar_arrive_expect_tx(&full[s], kStageA + kStageB);
        tma_load_2d(stage_a(s), &tmA, &full[s], kt * kTmaBK, m0);
        tma_load_2d(stage_b(s), &tmB, &full[s], n0, kt * kTmaBK);
    };
    if (t == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1);
        abort_flag = 0;
        fence_barrier_init();
        fence_proxy_async();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        for (int kt = 0; kt < STAGES - 1 && kt < ktiles; ++kt) issue(kt);
    }
    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;
    int issued = min(STAGES - 1, ktiles);
    bool failed = false;
    for (int kt = 0; kt < ktiles; ++kt) {
        // every thread is done with tile kt-1, so its slot takes tile kt+STAGES-1;
        // the vote also ends the loop in every thread at once after an expired wait
        if (__syncthreads_or(failed)) break;
        if (t == 0 && issued < ktiles) issue(issued);
        ++issued;
        const int s = kt % STAGES;
        if (!mbar_wait(&full[s], (kt / STAGES) & 1, &abort_flag, err, kErrWaitTmaFull)) {
            failed = true;
            continue;
        }
        const float *as = stage_a(s), *bs = stage_b(s);
#pragma unroll
        for (int k4 = 0; k4 < kTmaBK; k4 += 4) {
            float a[TM][4], b[4][TN];
#pragma unroll
            for (int i = 0; i < TM; ++i) {
                const int r = (i / 4) * kRowStride + ty * 4 + (i % 4);
                const float4 v = *reinterpret_cast<const float4 *>(as + r * kTmaBK + k4);
                a[i][0] = v.x; a[i][1] = v.y; a[i][2] = v.z; a[i][3] = v.w;
            }
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int g = 0; g < kGroupsN; ++g) {
                    const float4 v = *reinterpret_cast<const float4 *>(bs + (k4 + q) * BN + g * kColStride + tx * 4);
                    b[q][4 * g] = v.x; b[q][4 * g + 1] = v.y; b[q][4 * g + 2] = v.z; b[q][4 * g + 3] = v.w;
                }
#pragma unroll
            for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int i = 0; i < TM; ++i)
#pragma unroll
                    for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i][q], b[q][j], acc[i][j]);
        }
    }
    if (__syncthreads_or(failed)) {
        // the last copy issued into each slot lands before the CTA's shared memory
        // is released (a copy that never lands ends the drain at the time limit)
        if (t == 0) {
            const int n_issued = min(issued, ktiles);
            for (int kt = max(0, n_issued - STAGES); kt < n_issued; ++kt) mbar_wait_drain(&full[kt % STAGES], (kt / STAGES) & 1, err);
        }
        return;
    }
    const bool vec = (N % 4) == 0;
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int r = m0 + (i / 4) * kRowStride + ty * 4 + (i % 4);
        if (r >= M) continue;
#pragma unroll
        for (int g = 0; g < kGroupsN; ++g) {
            const int c = n0 + g * kColStride + tx * 4;
            float *dst = C + (size_t)r * N + c;
            if (vec && c + 4 <= N) {
                *reinterpret_cast<float4 *>(dst) = make_float4(acc[i][4 * g], acc[i][4 * g + 1], acc[i][4 * g + 2], acc[i][4 * g + 3]);
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    if (c + e < N) dst[e] = acc[i][4 * g + e];
            }
        }
    }
}

using TiledEncodeFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *, const cuuint64_t *,
                                   const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Row-major FP32 [rows, cols] described to TMA without swizzle, box {box_cols, box_rows}.
bool fp32_map(CUtensorMap *map, const void *ptr, uint64_t rows, uint64_t cols, uint32_t box_cols, uint32_t box_rows) {
    static const auto enc = reinterpret_cast<TiledEncodeFn>(driver_entry("cuTensorMapEncodeTiled"));
    if (!enc) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 4};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BM, int BN, int TM, int TN, int STAGES>
LaunchFn ffma_tma_launch(Context *ctx, const Spec &s) {
    auto kernel = gemm_ffma_tma_kernel<BM, BN, TM, TN, STAGES>;
    constexpr int threads = (BM / TM) * (BN / TN);
    constexpr int smem = STAGES * (BM + BN) * kTmaBK * 4 + 128;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        throw IrError("cannot reserve shared memory for the FFMA GEMM");
    const int M = (int)s.m, N = (int)s.n, K = (int)s.k;
    const dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    int *err = ctx->err_dev;
    return [=](cudaStream_t st, void **b) {
        CUtensorMap ma, mb;
        if (!fp32_map(&ma, b[0], M, K, kTmaBK, BM) || !fp32_map(&mb, b[1], K, N, BN, kTmaBK)) return cudaErrorInvalidValue;
        kernel<<<grid, threads, smem, st>>>(ma, mb, static_cast<float *>(b[2]), M, N, K, err);
        return cudaGetLastError();
    };
}

// FP32 (no epilogue, B [K,N]) with 16-byte strides takes the TMA-fed kernel.
bool ffma_tma_fits(const Spec &s) {
    return s.dtype == DType::F32 && !s.b_nk && !s.row_scale && s.epilogue == "none" && s.k % 4 == 0 && s.n % 4 == 0;
}

// 128x128 tiles when there is at least one per SM, else 32x64 tiles;
// JADE_FFMA_TILE=128x128 or 32x64 forces one (read when a kernel is compiled).
template <typename TA, typename TO>
LaunchFn ffma_launch(const Spec &s, bool tf32, int sm_count, std::string &impl) {
    const long long big_tiles = (long long)((s.m + 127) / 128) * ((s.n + 127) / 128);
    bool big = big_tiles >= sm_count;
    if (const char *force = std::getenv("JADE_FFMA_TILE"); force && *force) {
        if (!std::strcmp(force, "128x128")) big = true;
        else if (!std::strcmp(force, "32x64")) big = false;
        else throw IrError("JADE_FFMA_TILE must be 128x128 or 32x64");
    }
    if (big) {
        impl += "_128x128";
        return ffma_launch_tiles<TA, TO, 128, 128, 8, 8>(s, tf32);
    }
    impl += "_32x64";
    return ffma_launch_tiles<TA, TO, 32, 64, 4, 4>(s, tf32);
}

}  // namespace

LaunchFn make_gemm_simt(Context *ctx, const Spec &s, std::string &impl) {
    if (s.epilogue == "swiglu") throw IrError("swiglu epilogue needs the tcgen05 path (K a multiple of 8)");
    impl = std::string("gemm_ffma_") + dtype_name(s.dtype) + (s.b_nk ? "_nk" : "_kn");
    const int sms = ctx->sm_count;
    const char *force = std::getenv("JADE_FFMA_TILE");
    if (ffma_tma_fits(s) && !(force && *force)) {
        // the largest tile that still gives every SM a block (128x128: 8x8 outputs
        // per thread), else 32x64 while that gives two blocks per SM, else 16x32
        // blocks of one warp (512^3: 512 blocks, ~3.5 warps per SM instead of one)
        const long long big_tiles = (long long)((s.m + 127) / 128) * ((s.n + 127) / 128);
        const long long mid_tiles = (long long)((s.m + 31) / 32) * ((s.n + 63) / 64);
        if (big_tiles >= sms) {
            impl += "_tma_128x128";
            return ffma_tma_launch<128, 128, 8, 8, 4>(ctx, s);
        }
        const char *small = std::getenv("JADE_FFMA_SMALL");  // 32x64 or 16x32: forces the small-shape tile
        const bool tiny = small && *small ? std::strcmp(small, "16x32") == 0 : mid_tiles < 2LL * sms;
        if (tiny) {
            impl += "_tma_16x32";
            return ffma_tma_launch<16, 32, 4, 4, 4>(ctx, s);
        }
        impl += "_tma_32x64";
        return ffma_tma_launch<32, 64, 4, 4, 4>(ctx, s);
    }
    switch (s.dtype) {
        case DType::F32: return ffma_launch<float, float>(s, false, sms, impl);
        case DType::TF32: return ffma_launch<float, float>(s, true, sms, impl);
        case DType::BF16:
            return s.out_dtype == DType::BF16 ? ffma_launch<__nv_bfloat16, __nv_bfloat16>(s, false, sms, impl)
                                              : ffma_launch<__nv_bfloat16, float>(s, false, sms, impl);
        case DType::F16:
            return s.out_dtype == DType::F16 ? ffma_launch<__half, __half>(s, false, sms, impl)
                                             : ffma_launch<__half, float>(s, false, sms, impl);
        default: throw IrError("unsupported GEMM dtype");
    }
}

}  // namespace jade
