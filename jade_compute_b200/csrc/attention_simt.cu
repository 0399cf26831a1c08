// FP32 attention on CUDA cores: the faithful path for the reference's FP32
// attention specs (src/runtime/metal_attention.rs:44-197; oracle
// src/runtime/metal_lab.rs:33-73). Layout [batch*heads, seq, dim], scale
// 1/sqrt(dim), a causal query sees keys 0..query.
//
// Online kernel: a block of 4 warps owns 32 queries of one (batch, head); K and V
// tiles of 32 keys are staged in shared memory and reused by all 32 queries (the
// reference re-reads K/V per query). Lane j of a warp scores key j of the tile;
// the running max / normaliser follow FlashAttention's online recurrence; the
// output accumulator is split across lanes by channel.
#include "common.cuh"
#include "internal.hpp"

namespace jade {
namespace {

constexpr int kQ = 32, kKeys = 32, kWarps = 4, kMaxD = 128;
constexpr size_t kSmemBytes = sizeof(float) * (kKeys * (kMaxD + 1) + kKeys * kMaxD + kQ * kMaxD);

__global__ void __launch_bounds__(kWarps * 32) attention_online_f32(const float *__restrict__ q, const float *__restrict__ k,
                                                                    const float *__restrict__ v, float *__restrict__ out,
                                                                    int seq, int dim, int causal, float scale) {
    extern __shared__ float smem_f[];
    float (*Ks)[kMaxD + 1] = reinterpret_cast<float (*)[kMaxD + 1]>(smem_f);
    float (*Vs)[kMaxD] = reinterpret_cast<float (*)[kMaxD]>(smem_f + kKeys * (kMaxD + 1));
    float (*Qs)[kMaxD] = reinterpret_cast<float (*)[kMaxD]>(smem_f + kKeys * (kMaxD + 1) + kKeys * kMaxD);
    const int bh = blockIdx.y, q0 = blockIdx.x * kQ;
    const size_t base = (size_t)bh * seq * dim;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < kQ * dim; i += blockDim.x) {
        const int r = i / dim, c = i % dim;
        Qs[r][c] = (q0 + r < seq) ? q[base + (size_t)(q0 + r) * dim + c] : 0.0f;
    }
    constexpr int kPerWarp = kQ / kWarps;
    float m[kPerWarp], l[kPerWarp], o[kPerWarp][kMaxD / 32];
#pragma unroll
    for (int i = 0; i < kPerWarp; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int c = 0; c < kMaxD / 32; ++c) o[i][c] = 0.0f;
    }
    const int q_last = min(seq, q0 + kQ) - 1;
    const int key_end = causal ? q_last + 1 : seq;
    for (int k0 = 0; k0 < key_end; k0 += kKeys) {
        __syncthreads();
        for (int i = threadIdx.x; i < kKeys * dim; i += blockDim.x) {
            const int r = i / dim, c = i % dim;
            const bool ok = k0 + r < seq;
            Ks[r][c] = ok ? k[base + (size_t)(k0 + r) * dim + c] : 0.0f;
            Vs[r][c] = ok ? v[base + (size_t)(k0 + r) * dim + c] : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < kPerWarp; ++i) {
            const int qi = warp * kPerWarp + i, qrow = q0 + qi;
            if (qrow >= seq) continue;  // warp-uniform
            const int key = k0 + lane;
            const bool valid = key < seq && (!causal || key <= qrow);
            float s = 0.0f;
            for (int c = 0; c < dim; ++c) s = fmaf(Qs[qi][c], Ks[lane][c], s);
            s = valid ? s * scale : -INFINITY;
            float tile_max = s;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) tile_max = fmaxf(tile_max, __shfl_xor_sync(0xffffffffu, tile_max, off));
            if (tile_max == -INFINITY) continue;  // no visible key in this tile (warp-uniform)
            const float m_new = fmaxf(m[i], tile_max);
            const float corr = expf(m[i] - m_new);
            const float p = valid ? expf(s - m_new) : 0.0f;
            float psum = p;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
            l[i] = fmaf(l[i], corr, psum);
            m[i] = m_new;
#pragma unroll
            for (int c = 0; c < kMaxD / 32; ++c) {
                const int ch = lane + 32 * c;
                float acc = o[i][c] * corr;
                if (ch < dim) {
                    for (int j = 0; j < kKeys; ++j) acc = fmaf(__shfl_sync(0xffffffffu, p, j), Vs[j][ch], acc);
                } else {
                    for (int j = 0; j < kKeys; ++j) (void)__shfl_sync(0xffffffffu, p, j);
                }
                o[i][c] = acc;
            }
        }
    }
#pragma unroll
    for (int i = 0; i < kPerWarp; ++i) {
        const int qrow = q0 + warp * kPerWarp + i;
        if (qrow >= seq) continue;
        const float inv = 1.0f / l[i];
#pragma unroll
        for (int c = 0; c < kMaxD / 32; ++c) {
            const int ch = lane + 32 * c;
            if (ch < dim) out[base + (size_t)qrow * dim + ch] = o[i][c] * inv;
        }
    }
}

// Materialized comparator (metal_attention.rs:139-197): scaled QK^T with -inf
// above the diagonal when causal, then P.V after a row softmax.
__global__ void attention_scores_f32(const float *__restrict__ q, const float *__restrict__ k, float *__restrict__ scores,
                                     int seq, int dim, int causal, float scale) {
    const int col = blockIdx.x * blockDim.x + threadIdx.x, row = blockIdx.y * blockDim.y + threadIdx.y, h = blockIdx.z;
    if (row >= seq || col >= seq) return;
    const size_t base = (size_t)h * seq * dim;
    float s = 0.0f;
    for (int d = 0; d < dim; ++d) s = fmaf(q[base + (size_t)row * dim + d], k[base + (size_t)col * dim + d], s);
    scores[((size_t)h * seq + row) * seq + col] = (causal && col > row) ? -INFINITY : s * scale;
}
__global__ void attention_apply_f32(const float *__restrict__ p, const float *__restrict__ v, float *__restrict__ out, int seq, int dim) {
    const int d = blockIdx.x * blockDim.x + threadIdx.x, row = blockIdx.y * blockDim.y + threadIdx.y, h = blockIdx.z;
    if (row >= seq || d >= dim) return;
    const size_t base = (size_t)h * seq * dim;
    float acc = 0.0f;
    for (int j = 0; j < seq; ++j) acc = fmaf(p[((size_t)h * seq + row) * seq + j], v[base + (size_t)j * dim + d], acc);
    out[base + (size_t)row * dim + d] = acc;
}

}  // namespace

LaunchFn make_attention_simt(Context *, const Spec &s, std::string &impl) {
    const int seq = (int)s.seq, dim = (int)s.dim, causal = s.causal ? 1 : 0;
    const int bh = (int)(s.batch * s.heads);
    const float scale = 1.0f / sqrtf((float)dim);
    if (s.op == Op::AttentionOnline) {
        impl = "attention_online_f32_simt";
        const dim3 grid((seq + kQ - 1) / kQ, bh);
        cudaFuncSetAttribute(attention_online_f32, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
        return [=](cudaStream_t st, void **b) {
            attention_online_f32<<<grid, kWarps * 32, kSmemBytes, st>>>((const float *)b[0], (const float *)b[1], (const float *)b[2], (float *)b[3], seq,
                                                               dim, causal, scale);
            return cudaGetLastError();
        };
    }
    if (s.op == Op::AttentionScores) {
        impl = "attention_scores_f32";
        const dim3 grid((seq + 15) / 16, (seq + 15) / 16, bh), block(16, 16);
        return [=](cudaStream_t st, void **b) {
            attention_scores_f32<<<grid, block, 0, st>>>((const float *)b[0], (const float *)b[1], (float *)b[2], seq, dim, causal, scale);
            return cudaGetLastError();
        };
    }
    impl = "attention_apply_f32";
    const dim3 grid((dim + 15) / 16, (seq + 15) / 16, bh), block(16, 16);
    return [=](cudaStream_t st, void **b) {
        attention_apply_f32<<<grid, block, 0, st>>>((const float *)b[0], (const float *)b[1], (float *)b[2], seq, dim);
        return cudaGetLastError();
    };
}

}  // namespace jade
