// HBM-bound kernels: axpy, add, SwiGLU (elementwise), RMSNorm, softmax and the
// per-row inverse RMS used by the fused MLP (row kernels), plus fill and L2 flush.
//
// Reference semantics: src/runtime/ir.rs:485-523 (emitted bodies) and the FP64
// oracles src/runtime/workloads.rs:36-55,134-141. Design for B200: 128-bit
// loads/stores with streaming cache hints, grid sized to a multiple of the SM
// count, and single-pass row kernels that keep the row in registers so x is read
// from HBM exactly once (the reference reads it 2-3 times).
#include <algorithm>
#include <cfloat>

#include "common.cuh"
#include "internal.hpp"

namespace jade {
namespace {

constexpr int kThreads = 256;

int grid_for(const Context *ctx, uint64_t work, int per_block, int blocks_per_sm = 8) {
    uint64_t need = (work + per_block - 1) / per_block;
    uint64_t cap = (uint64_t)ctx->sm_count * blocks_per_sm;
    if (need < 1) need = 1;
    return (int)(need < cap ? need : cap);
}

// ------------------------------------------------------------------ axpy / add
// out = fmaf(alpha, a, b): one correctly rounded FMA, bit-identical to ir.rs:485.
__global__ void __launch_bounds__(kThreads) axpy_kernel(const float *__restrict__ a, const float *__restrict__ b,
                                                        float *__restrict__ out, float alpha, uint64_t n) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t nv = n >> 2;
    for (uint64_t v = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += stride) {
        const float4 x = __ldcs(reinterpret_cast<const float4 *>(a) + v);
        const float4 y = __ldcs(reinterpret_cast<const float4 *>(b) + v);
        float4 r;
        r.x = fmaf(alpha, x.x, y.x);
        r.y = fmaf(alpha, x.y, y.y);
        r.z = fmaf(alpha, x.z, y.z);
        r.w = fmaf(alpha, x.w, y.w);
        __stcs(reinterpret_cast<float4 *>(out) + v, r);
    }
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t < (n & 3)) {
        const uint64_t i = (nv << 2) + t;
        out[i] = fmaf(alpha, a[i], b[i]);
    }
}

__global__ void __launch_bounds__(kThreads) add_kernel(const float *__restrict__ a, const float *__restrict__ b,
                                                       float *__restrict__ out, uint64_t n) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t nv = n >> 2;
    for (uint64_t v = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += stride) {
        const float4 x = __ldcs(reinterpret_cast<const float4 *>(a) + v);
        const float4 y = __ldcs(reinterpret_cast<const float4 *>(b) + v);
        float4 r;
        r.x = __fadd_rn(x.x, y.x);
        r.y = __fadd_rn(x.y, y.y);
        r.z = __fadd_rn(x.z, y.z);
        r.w = __fadd_rn(x.w, y.w);
        __stcs(reinterpret_cast<float4 *>(out) + v, r);
    }
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t < (n & 3)) {
        const uint64_t i = (nv << 2) + t;
        out[i] = __fadd_rn(a[i], b[i]);
    }
}

// ------------------------------------------------------------------ SwiGLU
// out = (v * sigmoid(v)) * up with the stable branch of ir.rs:487, same operation
// order (expf, IEEE division), so FP32 results match the emitted reference kernel.
__device__ __forceinline__ float swiglu1(float v, float u) { return (v * stable_sigmoid(v)) * u; }

__global__ void __launch_bounds__(kThreads) swiglu_f32_kernel(const float *__restrict__ g, const float *__restrict__ up,
                                                              float *__restrict__ out, uint64_t n) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t nv = n >> 2;
    for (uint64_t v = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += stride) {
        const float4 x = __ldcs(reinterpret_cast<const float4 *>(g) + v);
        const float4 y = __ldcs(reinterpret_cast<const float4 *>(up) + v);
        float4 r;
        r.x = swiglu1(x.x, y.x);
        r.y = swiglu1(x.y, y.y);
        r.z = swiglu1(x.z, y.z);
        r.w = swiglu1(x.w, y.w);
        __stcs(reinterpret_cast<float4 *>(out) + v, r);
    }
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t < (n & 3)) {
        const uint64_t i = (nv << 2) + t;
        out[i] = swiglu1(g[i], up[i]);
    }
}

__global__ void __launch_bounds__(kThreads) swiglu_bf16_kernel(const __nv_bfloat16 *__restrict__ g, const __nv_bfloat16 *__restrict__ up,
                                                               __nv_bfloat16 *__restrict__ out, uint64_t n) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t nv = n >> 3;  // 8 bf16 per 16 B
    for (uint64_t v = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += stride) {
        const uint4 x = __ldcs(reinterpret_cast<const uint4 *>(g) + v);
        const uint4 y = __ldcs(reinterpret_cast<const uint4 *>(up) + v);
        const __nv_bfloat162 *xa = reinterpret_cast<const __nv_bfloat162 *>(&x);
        const __nv_bfloat162 *ya = reinterpret_cast<const __nv_bfloat162 *>(&y);
        uint4 r;
        uint32_t *ra = reinterpret_cast<uint32_t *>(&r);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float2 a2 = __bfloat1622float2(xa[q]), b2 = __bfloat1622float2(ya[q]);
            ra[q] = pack_bf16(swiglu1(a2.x, b2.x), swiglu1(a2.y, b2.y));
        }
        __stcs(reinterpret_cast<uint4 *>(out) + v, r);
    }
    const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t < (n & 7)) {
        const uint64_t i = (nv << 3) + t;
        out[i] = __float2bfloat16_rn(swiglu1(__bfloat162float(g[i]), __bfloat162float(up[i])));
    }
}

// ------------------------------------------------------------------ block reductions
template <bool kMax>
__device__ __forceinline__ float warp_reduce(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float w = __shfl_xor_sync(0xffffffffu, v, o);
        v = kMax ? fmaxf(v, w) : v + w;
    }
    return v;
}
template <bool kMax>
__device__ __forceinline__ float block_reduce(float v, float *scratch /* >= 32 floats */) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_reduce<kMax>(v);
    __syncthreads();  // scratch may still be read from a previous reduction
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float r = lane < nw ? scratch[lane] : (kMax ? -INFINITY : 0.0f);
    return warp_reduce<kMax>(r);
}

// e^d for d <= 0 from the MUFU base-2 exponential: d is formed exactly (x and the
// maximum are close) and scaled by log2(e) once, so the relative error stays near
// 1e-6 (a few units of the FP32 format), inside the FP32 softmax tolerance.
__device__ __forceinline__ float exp_neg(float d) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(d * 1.4426950408889634f));
    return y;
}
// Row (max, sum of e^(x - max)) from per-thread pairs in one block reduction: the
// maxima are reduced first, each sum is rescaled to the new maximum once, then the
// sums are reduced (per warp, then across the warps).
__device__ __forceinline__ void block_reduce_softmax(float &m, float &s, float *scratch /* >= 64 floats */) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    float mw = warp_reduce<true>(m);
    float sw = warp_reduce<false>(m == -INFINITY ? 0.0f : s * exp_neg(m - mw));
    __syncthreads();  // scratch may still be read from a previous reduction
    if (lane == 0) { scratch[warp] = mw; scratch[32 + warp] = sw; }
    __syncthreads();
    const float mi = lane < nw ? scratch[lane] : -INFINITY, si = lane < nw ? scratch[32 + lane] : 0.0f;
    m = warp_reduce<true>(mi);
    s = warp_reduce<false>(mi == -INFINITY ? 0.0f : si * exp_neg(mi - m));
}

// Loads/stores of 16-byte vectors of T (4 fp32 or 8 bf16) as float arrays.
template <typename T> struct Vec;
template <> struct Vec<float> {
    static constexpr int N = 4;
    __device__ static void load(const float *p, float *d) {
        const float4 v = __ldcs(reinterpret_cast<const float4 *>(p));
        d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
    }
    __device__ static void load_keep(const float *p, float *d) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(p));
        d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
    }
    __device__ static void load_shared(const float *p, float *d) {
        const float4 v = *reinterpret_cast<const float4 *>(p);
        d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
    }
    __device__ static void store_shared(float *p, const float *d) { *reinterpret_cast<float4 *>(p) = make_float4(d[0], d[1], d[2], d[3]); }
    __device__ static void store(float *p, const float *d) {
        __stcs(reinterpret_cast<float4 *>(p), make_float4(d[0], d[1], d[2], d[3]));
    }
};
template <> struct Vec<__nv_bfloat16> {
    static constexpr int N = 8;
    __device__ static void unpack(uint4 v, float *d) {
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&v);
#pragma unroll
        for (int q = 0; q < 4; ++q) { const float2 f = __bfloat1622float2(h[q]); d[2 * q] = f.x; d[2 * q + 1] = f.y; }
    }
    __device__ static void load(const __nv_bfloat16 *p, float *d) { unpack(__ldcs(reinterpret_cast<const uint4 *>(p)), d); }
    __device__ static void load_keep(const __nv_bfloat16 *p, float *d) { unpack(__ldg(reinterpret_cast<const uint4 *>(p)), d); }
    __device__ static void load_shared(const __nv_bfloat16 *p, float *d) { unpack(*reinterpret_cast<const uint4 *>(p), d); }
    __device__ static uint4 pack(const float *d) {
        uint4 v;
        uint32_t *a = reinterpret_cast<uint32_t *>(&v);
#pragma unroll
        for (int q = 0; q < 4; ++q) a[q] = pack_bf16(d[2 * q], d[2 * q + 1]);
        return v;
    }
    __device__ static void store(__nv_bfloat16 *p, const float *d) { __stcs(reinterpret_cast<uint4 *>(p), pack(d)); }
    __device__ static void store_shared(__nv_bfloat16 *p, const float *d) { *reinterpret_cast<uint4 *>(p) = pack(d); }
};

// Row kernels, register-resident: one block per row (grid-stride over rows),
// each thread holds NV vectors. Requires cols % Vec::N == 0 and cols <= NV*N*blockDim.
enum class RowOp { RmsNorm, Softmax, RmsInv };

// The arithmetic of one row held in registers (thread t has vectors t + j*THREADS):
// softmax = each thread's max and sum of exp(x - its max), one block reduction of
// those pairs, then exp(x - own max) * exp(own max - row max) / row sum (one more
// rounding than exp(x - row max) / sum, for one block reduction instead of two;
// exponentials on the MUFU unit, exp_neg);
// RMSNorm = sum of squares, scale by inv*w; RmsInv = the per-row inverse RMS only.
// SINK: results go to `sink` (the row's shared-memory stage, written back by bulk
// copies) instead of global memory.
template <typename T, int NV, RowOp OP, int THREADS, bool SINK = false>
__device__ __forceinline__ void row_compute(float (&v)[NV][Vec<T>::N], uint32_t row, uint32_t nvec, uint32_t cols, const T *__restrict__ w,
                                            void *__restrict__ out_, float eps, float *scratch, T *sink = nullptr) {
    constexpr int N = Vec<T>::N;
    auto put = [&](uint32_t c, const float *d) {
        if constexpr (SINK) Vec<T>::store_shared(sink + (uint64_t)c * N, d);
        else Vec<T>::store(static_cast<T *>(out_) + (uint64_t)row * cols + (uint64_t)c * N, d);
    };
    if constexpr (OP == RowOp::Softmax) {
        float m = -INFINITY;
#pragma unroll
        for (int j = 0; j < NV; ++j)
            if (threadIdx.x + j * THREADS < nvec)
#pragma unroll
                for (int e = 0; e < N; ++e) m = fmaxf(m, v[j][e]);
        // a thread whose elements are all -inf (masked scores) shifts by 0 instead of
        // its own maximum, so that its exponentials are e^-inf = 0, not e^(-inf + inf)
        const float shift = m == -INFINITY ? 0.0f : m;
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < NV; ++j)
            if (threadIdx.x + j * THREADS < nvec)
#pragma unroll
                for (int e = 0; e < N; ++e) { v[j][e] = exp_neg(v[j][e] - shift); s += v[j][e]; }
        float mr = m, sr = s;
        block_reduce_softmax(mr, sr, scratch);
        const float inv = m == -INFINITY ? 0.0f : exp_neg(m - mr) / sr;  // a thread without elements stores nothing
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const uint32_t c = threadIdx.x + j * THREADS;
            if (c < nvec) {
#pragma unroll
                for (int e = 0; e < N; ++e) v[j][e] *= inv;
                put(c, v[j]);
            }
        }
    } else {
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < NV; ++j)
            if (threadIdx.x + j * THREADS < nvec)
#pragma unroll
                for (int e = 0; e < N; ++e) ss = fmaf(v[j][e], v[j][e], ss);
        ss = block_reduce<false>(ss, scratch);
        const float inv = 1.0f / sqrtf(ss / (float)cols + eps);
        if constexpr (OP == RowOp::RmsInv) {
            if (threadIdx.x == 0) static_cast<float *>(out_)[row] = inv;
        } else {
#pragma unroll
            for (int j = 0; j < NV; ++j) {
                const uint32_t c = threadIdx.x + j * THREADS;
                if (c < nvec) {
                    float wv[N];
                    Vec<T>::load_keep(w + (uint64_t)c * N, wv);
#pragma unroll
                    for (int e = 0; e < N; ++e) v[j][e] = v[j][e] * inv * wv[e];
                    put(c, v[j]);
                }
            }
        }
    }
}

template <typename T, int NV, RowOp OP, int THREADS>
__global__ void __launch_bounds__(THREADS) row_kernel(const T *__restrict__ x, const T *__restrict__ w, void *__restrict__ out_,
                                                      uint32_t rows, uint32_t cols, float eps) {
    __shared__ float scratch[64];
    constexpr int N = Vec<T>::N;
    const uint32_t nvec = cols / N;
    for (uint32_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const T *xr = x + (uint64_t)row * cols;
        float v[NV][N];
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const uint32_t c = threadIdx.x + j * THREADS;
            if (c < nvec) Vec<T>::load(xr + (uint64_t)c * N, v[j]);
        }
        row_compute<T, NV, OP, THREADS>(v, row, nvec, cols, w, out_, eps, scratch);
    }
}

// Row kernels with the rows staged in shared memory: thread 0 streams whole rows
// (bulk copies counted on an mbarrier) into a ring of STAGES buffers, running up
// to STAGES rows ahead of the arithmetic, so each SM keeps reads of several rows in
// flight through the reductions and stores of the current row (the register
// kernel has reads in flight only between its row loads and first reduction).
// Persistent: as many CTAs as fit, rows dealt round-robin.
//
// BULK: the results are written back into the row's own stage and leave by bulk
// copies (one thread issues them; the copy engine writes whole lines), instead of
// 16-byte stores from every thread. A stage is then refilled one iteration later,
// once its store has read it out, so STAGES - 1 rows are in flight ahead of the
// arithmetic.
constexpr uint32_t kRowChunk = 8192;  // bytes per bulk copy

template <typename T, int NV, RowOp OP, int STAGES, bool BULK>
__global__ void __launch_bounds__(kThreads) row_staged_kernel(const T *__restrict__ x, const T *__restrict__ w, void *__restrict__ out_,
                                                              uint32_t rows, uint32_t cols, float eps, uint32_t stage_bytes, int *err) {
    extern __shared__ __align__(128) uint8_t stage[];
    __shared__ float scratch[64];
    __shared__ uint64_t full[STAGES];
    __shared__ int abort_flag;
    constexpr int N = Vec<T>::N;
    static_assert(!BULK || OP != RowOp::RmsInv, "RmsInv writes one value per row");
    const uint32_t nvec = cols / N, row_bytes = cols * (uint32_t)sizeof(T);
    int issued[STAGES] = {};  // thread 0: rows loaded into each stage
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&full[s], 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    auto issue = [&](uint32_t row, int s) {  // thread 0
        mbar_arrive_expect_tx(&full[s], row_bytes);
        const uint8_t *src = reinterpret_cast<const uint8_t *>(x + (uint64_t)row * cols);
        for (uint32_t o = 0; o < row_bytes; o += kRowChunk)
            bulk_load(stage + s * stage_bytes + o, src + o, min(kRowChunk, row_bytes - o), &full[s]);
        ++issued[s];
    };
    if (threadIdx.x == 0)
        for (int s = 0; s < STAGES; ++s) {
            const uint64_t row = blockIdx.x + (uint64_t)s * gridDim.x;
            if (row < rows) issue((uint32_t)row, s);
        }
    uint32_t k = 0;
    for (uint32_t row = blockIdx.x; row < rows; row += gridDim.x, ++k) {
        const int s = k % STAGES;
        bool ok = true;
        if (threadIdx.x == 0) ok = mbar_wait(&full[s], (k / STAGES) & 1, &abort_flag, err, kErrWaitTmaFull);
        if (__syncthreads_or(!ok)) break;  // a uniform exit; also publishes the staged row to every thread
        T *xr = reinterpret_cast<T *>(stage + s * stage_bytes);
        float v[NV][N];
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const uint32_t c = threadIdx.x + j * kThreads;
            if (c < nvec) Vec<T>::load_shared(xr + (uint64_t)c * N, v[j]);
        }
        if constexpr (!BULK) {
            __syncthreads();  // the stage is read out: it takes the row STAGES ahead
            if (threadIdx.x == 0) {
                const uint64_t next = row + (uint64_t)STAGES * gridDim.x;
                if (next < rows) issue((uint32_t)next, s);
            }
            row_compute<T, NV, OP, kThreads, false>(v, row, nvec, cols, w, out_, eps, scratch);
        } else {
            // every thread overwrites only the vectors it read, so no barrier is
            // needed between the loads above and these stores
            row_compute<T, NV, OP, kThreads, true>(v, row, nvec, cols, w, out_, eps, scratch, xr);
            fence_proxy_async();  // this thread's shared stores, visible to the bulk copies
            __syncthreads();
            if (threadIdx.x == 0) {
                uint8_t *dst = reinterpret_cast<uint8_t *>(static_cast<T *>(out_) + (uint64_t)row * cols);
                for (uint32_t o = 0; o < row_bytes; o += kRowChunk)
                    bulk_store(dst + o, reinterpret_cast<uint8_t *>(xr) + o, min(kRowChunk, row_bytes - o));
                bulk_commit_group();
                if (k > 0) {  // the previous iteration's stage, once its store has read it out
                    const uint64_t next = row + (uint64_t)(STAGES - 1) * gridDim.x;
                    if (next < rows) {
                        bulk_wait_read_but_one();
                        issue((uint32_t)next, (k - 1) % STAGES);
                    }
                }
            }
        }
    }
    if (threadIdx.x == 0) {
        if (abort_flag)  // copies still in flight land before the CTA exits
            for (int s = 0; s < STAGES; ++s)
                if (issued[s]) mbar_wait_drain(&full[s], (issued[s] - 1) & 1, err);
        if constexpr (BULK) bulk_wait_all();
    }
}

// General fallback for any cols (ragged or very wide rows): three passes over the
// row through L2, one block per row, scalar accesses.
template <typename T, RowOp OP>
__global__ void __launch_bounds__(kThreads) row_kernel_general(const T *__restrict__ x, const T *__restrict__ w, void *__restrict__ out_,
                                                               uint32_t rows, uint32_t cols, float eps) {
    __shared__ float scratch[64];
    for (uint32_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const T *xr = x + (uint64_t)row * cols;
        if constexpr (OP == RowOp::Softmax) {
            float m = -INFINITY;
            for (uint32_t c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, to_f32(xr[c]));
            m = block_reduce<true>(m, scratch);
            float s = 0.0f;
            for (uint32_t c = threadIdx.x; c < cols; c += blockDim.x) s += expf(to_f32(xr[c]) - m);
            s = block_reduce<false>(s, scratch);
            const float inv = 1.0f / s;
            T *o = static_cast<T *>(out_) + (uint64_t)row * cols;
            for (uint32_t c = threadIdx.x; c < cols; c += blockDim.x) o[c] = from_f32<T>(expf(to_f32(xr[c]) - m) * inv);
        } else {
            float ss = 0.0f;
            for (uint32_t c = threadIdx.x; c < cols; c += blockDim.x) { const float v = to_f32(xr[c]); ss = fmaf(v, v, ss); }
            ss = block_reduce<false>(ss, scratch);
            const float inv = 1.0f / sqrtf(ss / (float)cols + eps);
            if constexpr (OP == RowOp::RmsInv) {
                if (threadIdx.x == 0) static_cast<float *>(out_)[row] = inv;
            } else {
                T *o = static_cast<T *>(out_) + (uint64_t)row * cols;
                for (uint32_t c = threadIdx.x; c < cols; c += blockDim.x) o[c] = from_f32<T>(to_f32(xr[c]) * inv * to_f32(w[c]));
            }
        }
    }
}

template <typename T, RowOp OP>
LaunchFn row_launch(Context *ctx, const Spec &s, std::string &impl) {
    constexpr int N = Vec<T>::N;
    const uint32_t rows = s.rows, cols = s.cols;
    const float eps = s.epsilon;
    const int grid = grid_for(ctx, rows, 1, 16);
    const bool vec = cols % N == 0;
    // Rows of up to 8 vectors per thread at 128 threads run 128-thread blocks (up
    // to 16 rows in flight per SM); wider rows use 256 threads.
    const uint32_t nv = cols / N;
    const int threads = (vec && nv <= 128 * 8) ? 128 : kThreads;
    const uint32_t per_thread = (nv + threads - 1) / threads;  // vectors per thread
    using KFn = void (*)(const T *, const T *, void *, uint32_t, uint32_t, float);
    KFn fn = nullptr;
    if (threads == 128) {
        if (per_thread <= 1) fn = row_kernel<T, 1, OP, 128>;
        else if (per_thread <= 2) fn = row_kernel<T, 2, OP, 128>;
        else if (per_thread <= 4) fn = row_kernel<T, 4, OP, 128>;
        else fn = row_kernel<T, 8, OP, 128>;
    } else if (vec && per_thread <= 8) fn = row_kernel<T, 8, OP, 256>;
    else if (vec && per_thread <= 16) fn = row_kernel<T, 16, OP, 256>;
    else fn = row_kernel_general<T, OP>;
    const int grid2 = threads == 128 ? grid_for(ctx, rows, 1, 32) : grid;
    impl = std::string(fn == (KFn)row_kernel_general<T, OP> ? "row_general_" : "row_register_") + dtype_name(s.dtype) + "_t" +
           std::to_string(threads);
    // Staged variant (whole rows of at least one vector per thread whose stages fit
    // in shared memory) for 16-bit rows and FP32 softmax rows. Measured on B200 at
    // 16384 x 8192 with per-thread stores, before the bulk-copy stores: BF16 RMSNorm
    // 5.23 vs 4.75 TB/s and softmax 5.23 vs 4.92 TB/s for the staged kernel; FP32
    // rows (twice the bytes per element) then ran faster on the register kernel
    // (6.18 vs 6.02 and 5.76 vs 5.29 TB/s).
    using SFn = void (*)(const T *, const T *, void *, uint32_t, uint32_t, float, uint32_t, int *);
    SFn sfn = nullptr;
    const uint32_t stage_bytes = (uint32_t)(((uint64_t)cols * sizeof(T) + 127) / 128 * 128);
    const uint32_t spt = (nv + kThreads - 1) / kThreads;
    // Results leave by bulk copies (RMSNorm, softmax) from a ring of 2 (RMSNorm) or
    // 3 (softmax) stages; measured on B200 at 16384 x 8192 BF16 (fraction of the
    // copy bandwidth, RMSNorm / softmax): per-thread stores from 3 stages 0.79 /
    // 0.79-0.82, from 2 stages 0.80 / 0.77, from 4 stages 0.72 / 0.78; bulk stores
    // from 2 stages 0.84 / 0.80, from 3 stages 0.78 / 0.85, from 4 stages 0.82 / 0.82.
    // FP32 rows (16384 x 8192) stay on the register kernel for RMSNorm (0.91-0.92 vs
    // 0.86-0.87 staged) and are staged for softmax (0.87 vs 0.85), with rows of up to
    // 32 KB (at least two CTAs per SM)
    constexpr bool kBulk = OP != RowOp::RmsInv;
    constexpr int kStages = OP == RowOp::RmsNorm ? 2 : 3;
    const bool staged = sizeof(T) == 2 || (OP == RowOp::Softmax && stage_bytes <= 32 * 1024);
    if (staged && vec && nv >= (uint32_t)kThreads && (uint64_t)kStages * stage_bytes <= 200 * 1024) {
        if (spt <= 1) sfn = row_staged_kernel<T, 1, OP, kStages, kBulk>;
        else if (spt <= 2) sfn = row_staged_kernel<T, 2, OP, kStages, kBulk>;
        else if (spt <= 4) sfn = row_staged_kernel<T, 4, OP, kStages, kBulk>;
        else if (spt <= 8) sfn = row_staged_kernel<T, 8, OP, kStages, kBulk>;
        else if (spt <= 16) sfn = row_staged_kernel<T, 16, OP, kStages, kBulk>;
    }
    const int used_stages = kStages;
    int sgrid = 0;
    const int smem = used_stages * (int)stage_bytes;
    if (sfn) {
        int per_sm = 0;
        if (cudaFuncSetAttribute(sfn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, sfn, kThreads, smem) != cudaSuccess || per_sm < 1)
            sfn = nullptr;
        else
            sgrid = (int)std::min<uint64_t>(rows, (uint64_t)per_sm * ctx->sm_count);
    }
    if (sfn)
        impl = std::string("row_staged_") + dtype_name(s.dtype) + "_t" + std::to_string(kThreads) + "_s" + std::to_string(used_stages) +
               (kBulk ? "_bulk" : "");
    int *err = ctx->err_dev;
    return [=](cudaStream_t st, void **b) {
        const T *x = static_cast<const T *>(b[0]);
        const T *w = OP == RowOp::RmsNorm ? static_cast<const T *>(b[1]) : nullptr;
        void *out = OP == RowOp::RmsNorm ? b[2] : b[1];
        if (sfn && reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0)  // bulk copies: 16-byte aligned rows
            sfn<<<sgrid, kThreads, smem, st>>>(x, w, out, rows, cols, eps, stage_bytes, err);
        else
            fn<<<grid2, threads, 0, st>>>(x, w, out, rows, cols, eps);
        return cudaGetLastError();
    };
}

// ------------------------------------------------------------------ fill / flush
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
// Counter-based synthetic inputs: element i of stream s from seed is
// splitmix64(seed ^ s*C ^ (offset + i)) (offset: this buffer is a slice of a
// larger generated tensor); uniform in [lo, hi) or normal (Box-Muller) with
// mean lo and standard deviation hi; rounded once to the output type.
template <typename T>
__global__ void fill_kernel(T *__restrict__ out, uint64_t n, uint64_t seed, uint32_t stream, int normal, float lo, float hi,
                            uint64_t offset) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t key = splitmix64(seed ^ (0xD1B54A32D192ED03ull * (uint64_t)(stream + 1)));
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint64_t h = splitmix64(key + offset + i);
        float v;
        if (normal) {
            const float u1 = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);            // (0,1)
            const float u2 = (float)((h >> 16) & 0xFFFFFFull) * (1.0f / 16777216.0f);     // [0,1)
            v = lo + hi * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
        } else {
            const float u = (float)(h >> 40) * (1.0f / 16777216.0f);
            v = lo + (hi - lo) * u;
        }
        out[i] = from_f32<T>(v);
    }
}

// Bounded-wait probe: thread 0 waits on an mbarrier that nothing arrives on,
// through the same bounded wait as the tcgen05 kernels but with the spec's time
// limit; on expiry it records kErrWaitProbe in the context's error word (which
// the batch reports as JR_ETIMEOUT), stores how long it waited and returns. It
// lets a test drive the expiry path on the GPU without a fault or a hang.
__global__ void wait_probe_kernel(float *__restrict__ out, int *err, uint64_t limit_ns) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint64_t t0 = globaltimer();
        const bool satisfied = mbar_wait_for(&bar, 0, &abort_flag, err, kErrWaitProbe, limit_ns);
        out[0] = (float)(globaltimer() - t0);
        out[1] = satisfied ? 1.0f : 0.0f;
    }
}

__global__ void flush_kernel(uint4 *__restrict__ p, uint64_t n16, uint32_t salt) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride)
        p[i] = make_uint4((uint32_t)i, salt, (uint32_t)(i >> 32), ~salt);
}

}  // namespace

LaunchFn make_row_kernel(Context *ctx, const Spec &s, std::string &impl) {
    const uint64_t n = s.len;
    switch (s.op) {
        case Op::Axpy: {
            const int grid = grid_for(ctx, (n + 3) / 4, kThreads);
            const float alpha = s.alpha;
            impl = "axpy_f32_v4";
            return [=](cudaStream_t st, void **b) {
                axpy_kernel<<<grid, kThreads, 0, st>>>((const float *)b[0], (const float *)b[1], (float *)b[2], alpha, n);
                return cudaGetLastError();
            };
        }
        case Op::Add: {
            const int grid = grid_for(ctx, (n + 3) / 4, kThreads);
            impl = "add_f32_v4";
            return [=](cudaStream_t st, void **b) {
                add_kernel<<<grid, kThreads, 0, st>>>((const float *)b[0], (const float *)b[1], (float *)b[2], n);
                return cudaGetLastError();
            };
        }
        case Op::SwiGlu: {
            if (s.dtype == DType::BF16) {
                const int grid = grid_for(ctx, (n + 7) / 8, kThreads);
                impl = "swiglu_bf16_v8";
                return [=](cudaStream_t st, void **b) {
                    swiglu_bf16_kernel<<<grid, kThreads, 0, st>>>((const __nv_bfloat16 *)b[0], (const __nv_bfloat16 *)b[1], (__nv_bfloat16 *)b[2], n);
                    return cudaGetLastError();
                };
            }
            const int grid = grid_for(ctx, (n + 3) / 4, kThreads);
            impl = "swiglu_f32_v4";
            return [=](cudaStream_t st, void **b) {
                swiglu_f32_kernel<<<grid, kThreads, 0, st>>>((const float *)b[0], (const float *)b[1], (float *)b[2], n);
                return cudaGetLastError();
            };
        }
        case Op::RmsNorm:
            return s.dtype == DType::BF16 ? row_launch<__nv_bfloat16, RowOp::RmsNorm>(ctx, s, impl) : row_launch<float, RowOp::RmsNorm>(ctx, s, impl);
        case Op::Softmax:
            return s.dtype == DType::BF16 ? row_launch<__nv_bfloat16, RowOp::Softmax>(ctx, s, impl) : row_launch<float, RowOp::Softmax>(ctx, s, impl);
        case Op::RmsInv:
            return s.dtype == DType::BF16 ? row_launch<__nv_bfloat16, RowOp::RmsInv>(ctx, s, impl) : row_launch<float, RowOp::RmsInv>(ctx, s, impl);
        default: throw IrError("not a row kernel");
    }
}

LaunchFn make_misc_kernel(Context *ctx, const Spec &s, std::string &impl) {
    if (s.op == Op::Fill) {
        const uint64_t n = s.len, seed = s.seed, offset = s.offset;
        const uint32_t stream = s.stream_id;
        const int normal = s.dist == "normal";
        const float lo = s.lo, hi = s.hi;
        const int grid = grid_for(ctx, n, kThreads);
        impl = std::string("fill_") + s.dist + "_" + dtype_name(s.dtype);
        const DType d = s.dtype;
        return [=](cudaStream_t st, void **b) {
            if (d == DType::BF16) fill_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>((__nv_bfloat16 *)b[0], n, seed, stream, normal, lo, hi, offset);
            else if (d == DType::F16) fill_kernel<__half><<<grid, kThreads, 0, st>>>((__half *)b[0], n, seed, stream, normal, lo, hi, offset);
            else fill_kernel<float><<<grid, kThreads, 0, st>>>((float *)b[0], n, seed, stream, normal, lo, hi, offset);
            return cudaGetLastError();
        };
    }
    if (s.op == Op::WaitProbe) {
        const uint64_t limit = s.limit_ns;
        int *err = ctx->err_dev;
        impl = "wait_probe";
        return [=](cudaStream_t st, void **b) {
            wait_probe_kernel<<<1, 32, 0, st>>>((float *)b[0], err, limit);
            return cudaGetLastError();
        };
    }
    if (s.op == Op::L2Flush) {
        const uint64_t n16 = s.bytes / 16;
        const int grid = grid_for(ctx, n16, kThreads, 4);
        impl = "l2_flush";
        auto salt = std::make_shared<uint32_t>(1);
        return [=](cudaStream_t st, void **b) {
            flush_kernel<<<grid, kThreads, 0, st>>>((uint4 *)b[0], n16, (*salt)++);
            return cudaGetLastError();
        };
    }
    throw IrError("not a utility kernel");
}

}  // namespace jade
