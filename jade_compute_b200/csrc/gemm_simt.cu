// FP32 FFMA GEMM (the faithful path) and the SIMT fallback for tensor-core
// dtypes on shapes whose strides TMA cannot describe.
//
// Reference: src/runtime/ir.rs:524-557 (gemm_naive / gemm_register32) and
// src/runtime/metal_simd.rs:24-110 (FP32 SIMD-group GEMM). Each output is
// accumulated as acc = fmaf(a[row,p], b[p,col], acc) for p = 0..K-1 in order,
// starting from 0, which is exactly what the reference kernels compute, so FP32
// results are bit-identical to them (and to the CPU restatement
// or_gemm_fp32_sequential). Tiling: 128x128 block tile, K-step 8, 256 threads,
// 8x8 outputs per thread held in registers, shared-memory double buffering.
#include "common.cuh"
#include "internal.hpp"

namespace jade {
namespace {

constexpr int BM = 128, BN = 128, BK = 8, kThreads = 256;

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

// C[M,N] = A[M,K] * B   (B is [K,N] row-major, or [N,K] when kBnk)
template <typename TA, typename TO, bool kBnk>
__global__ void __launch_bounds__(kThreads) gemm_ffma_kernel(const TA *__restrict__ A, const TA *__restrict__ B, TO *__restrict__ C,
                                                             int M, int N, int K, bool tf32, const float *__restrict__ row_scale,
                                                             const TO *__restrict__ residual) {
    __shared__ __align__(16) float As[2][BK][BM];
    __shared__ __align__(16) float Bs[2][BK][BN];
    const int t = threadIdx.x;
    const int tx = t % 16, ty = t / 16;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

    float ra[4], rb[4];
    auto gload = [&](int k0) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int idx = t + kThreads * i;
            {  // A element (r, kk): consecutive threads walk k within a row
                const int r = idx / BK, kk = idx % BK;
                const int gr = m0 + r, gk = k0 + kk;
                ra[i] = (gr < M && gk < K) ? load_op(A + (size_t)gr * K + gk, tf32) : 0.0f;
            }
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
        for (int i = 0; i < 4; ++i) {
            const int idx = t + kThreads * i;
            As[buf][idx % BK][idx / BK] = ra[i];
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
            float a[8], b[8];
            const float4 a0 = *reinterpret_cast<const float4 *>(&As[buf][kk][ty * 4]);
            const float4 a1 = *reinterpret_cast<const float4 *>(&As[buf][kk][64 + ty * 4]);
            const float4 b0 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][64 + tx * 4]);
            a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w; a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
            b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w; b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        if (kt + 1 < ktiles) {
            sstore(buf ^ 1);
            __syncthreads();
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (r >= M) continue;
        const float sc = row_scale ? row_scale[r] : 1.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int c = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
            if (c >= N) continue;
            float v = row_scale ? acc[i][j] * sc : acc[i][j];
            if (residual) v += to_f32(residual[(size_t)r * N + c]);
            C[(size_t)r * N + c] = from_f32<TO>(v);
        }
    }
}

template <typename TA, typename TO>
LaunchFn ffma_launch(const Spec &s, bool tf32) {
    const int M = (int)s.m, N = (int)s.n, K = (int)s.k;
    const dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    const bool bnk = s.b_nk, rs = s.row_scale, res = s.epilogue == "residual";
    return [=](cudaStream_t st, void **b) {
        int idx = 2;
        const float *row_scale = rs ? static_cast<const float *>(b[idx++]) : nullptr;
        const TO *residual = res ? static_cast<const TO *>(b[idx++]) : nullptr;
        TO *out = static_cast<TO *>(b[idx]);
        if (bnk)
            gemm_ffma_kernel<TA, TO, true><<<grid, kThreads, 0, st>>>((const TA *)b[0], (const TA *)b[1], out, M, N, K, tf32, row_scale, residual);
        else
            gemm_ffma_kernel<TA, TO, false><<<grid, kThreads, 0, st>>>((const TA *)b[0], (const TA *)b[1], out, M, N, K, tf32, row_scale, residual);
        return cudaGetLastError();
    };
}

}  // namespace

LaunchFn make_gemm_simt(Context *, const Spec &s, std::string &impl) {
    if (s.epilogue == "swiglu") throw IrError("swiglu epilogue needs the tcgen05 path (K a multiple of 8)");
    impl = std::string("gemm_ffma_128x128_") + dtype_name(s.dtype) + (s.b_nk ? "_nk" : "_kn");
    switch (s.dtype) {
        case DType::F32: return ffma_launch<float, float>(s, false);
        case DType::TF32: return ffma_launch<float, float>(s, true);
        case DType::BF16:
            return s.out_dtype == DType::BF16 ? ffma_launch<__nv_bfloat16, __nv_bfloat16>(s, false) : ffma_launch<__nv_bfloat16, float>(s, false);
        case DType::F16:
            return s.out_dtype == DType::F16 ? ffma_launch<__half, __half>(s, false) : ffma_launch<__half, float>(s, false);
        default: throw IrError("unsupported GEMM dtype");
    }
}

}  // namespace jade
