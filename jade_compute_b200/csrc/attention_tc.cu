// FlashAttention-style forward attention on tcgen05 for BF16/FP16 inputs.
//
// Semantics: O = softmax(Q K^T / sqrt(D) [causal: key <= query]) V, the
// reference's online attention (src/runtime/metal_attention.rs:44-137, oracle
// src/runtime/metal_lab.rs:33-73) extended to a batch dimension: Q/K/V/O are
// [batch, heads, seq, dim] row-major, dim 64 or 128. Softmax statistics are
// FP32; P is rounded to the input type for the P.V product; O accumulates in FP32.
//
// One CTA owns 128 queries of one (batch, head):
//   warp 0      TMA producer: Q once, then K_j / V_j into two-stage rings with
//               separate K and V barriers (K_j's slot refills once S_j is done)
//   warp 1      MMA issuer: S_{j+1} = Q K_{j+1}^T is issued before O_j = P_j V_j, so
//               the tensor core computes the next scores while softmax runs
//   warps 2-9   softmax + correction + epilogue. Two warps share each 32-lane TMEM
//               quarter (= 32 query rows) and split the 128 score columns and the
//               D output columns; the pair exchanges row maxima through shared
//               memory (named barrier per pair).
// TMEM: S double buffer (2 x 128 columns) + P.V tile (D columns). The running
// output stays in registers (64 FP32 per thread), rescaled by exp2(m_old-m_new).
// Causal: key tiles above the diagonal are skipped; q-tiles are scheduled
// heaviest first. Every wait is bounded and the abort decision is made
// uniformly per warp pair so no thread is left at a barrier.
#include <cuda.h>

#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "internal.hpp"

namespace jade {
namespace {

constexpr int kBQ = 128, kBK = 128, kSoftWarps = 8, kThreads = (2 + kSoftWarps) * 32, kFirstSoftWarp = 2;

template <int D>
struct AttnLayout {
    static constexpr uint32_t kChunk = 128 * 128;              // 128 rows x 128 B (64 elements)
    static constexpr uint32_t kTile = (D / 64) * kChunk;       // Q / K / V tile bytes
    static constexpr uint32_t kQ = 0;
    static constexpr uint32_t kK = kQ + kTile;                  // 2 stages
    static constexpr uint32_t kV = kK + 2 * kTile;              // 2 stages
    static constexpr uint32_t kP = kV + 2 * kTile;              // 128 x 128 (2 chunks)
    static constexpr uint32_t kBar = kP + 2 * kChunk;
    static constexpr uint32_t kXch = kBar + 256;                // pair exchange buffers
    static constexpr uint32_t kEnd = kXch + 4 * 2 * 128 * 8;    // [slot 4][half 2][row 128] x (float, int)
    static constexpr uint32_t kSmem = kEnd + 1024;
};

struct AttnArgs {
    void *out;
    int seq, heads_total, nq_tiles, nkv_tiles, causal;
    float scale_log2;
    int *err;
};

__device__ __forceinline__ void named_bar_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int D, typename TIn, typename TOut>
__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const AttnArgs args) {
    using L = AttnLayout<D>;
    constexpr uint32_t kFmt = std::is_same<TIn, __nv_bfloat16>::value ? 1u : 0u;
    constexpr uint32_t kIdescS = idesc_f32acc(kFmt, kFmt, false, false, kBQ, kBK);
    constexpr uint32_t kIdescO = idesc_f32acc(kFmt, kFmt, false, true, kBQ, D);
    constexpr int kDChunks = D / 64;
    constexpr int kHalfCols = D / 2;  // output columns per softmax thread

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBar);
    uint64_t *q_full = bars + 0;
    uint64_t *k_full = bars + 1, *k_empty = bars + 3, *v_full = bars + 5, *v_empty = bars + 7;
    uint64_t *s_full = bars + 9, *s_empty = bars + 11, *p_full = bars + 13, *o_full = bars + 14, *o_empty = bars + 15;
    uint64_t *mma_done = bars + 16;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 17);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    float *xch_v = reinterpret_cast<float *>(smem + L::kXch);
    int *xch_ok = reinterpret_cast<int *>(smem + L::kXch + 4 * 2 * 128 * 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int bh = blockIdx.x;
    const int qt = args.nq_tiles - 1 - (int)blockIdx.y;  // heaviest causal tiles first
    const int q0 = qt * kBQ;
    const int n_kv = args.causal ? min(qt + 1, args.nkv_tiles) : args.nkv_tiles;
    int *err = args.err;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&k_full[s], 1); mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1); mbar_init(&v_empty[s], 1);
            mbar_init(&s_full[s], 1); mbar_init(&s_empty[s], kSoftWarps * 32);
        }
        mbar_init(p_full, kSoftWarps * 32);
        mbar_init(o_full, 1);
        mbar_init(o_empty, kSoftWarps * 32);
        mbar_init(mma_done, 1);
        *abort_flag = 0;
        fence_barrier_init();
        fence_proxy_async();
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tmem_s[2] = {tmem, tmem + 128};
    const uint32_t tmem_o = tmem + 256;

    if (warp == 0) {
        if (lane == 0) {  // ------------------------------------- TMA producer
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            bool k_issued[2] = {false, false}, v_issued[2] = {false, false}, q_issued = false;
            uint32_t k_last[2] = {0, 0}, v_last[2] = {0, 0};
            mbar_arrive_expect_tx(q_full, L::kTile);
            for (int c = 0; c < kDChunks; ++c) tma_load_3d(smem + L::kQ + c * L::kChunk, &tmQ, q_full, c * 64, q0, bh);
            q_issued = true;
            for (int j = 0; j < n_kv && !*abort_flag; ++j) {
                const int st = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                if (!mbar_wait(&k_empty[st], ph ^ 1, abort_flag, err, kErrWaitSmemEmpty)) break;
                mbar_arrive_expect_tx(&k_full[st], L::kTile);
                for (int c = 0; c < kDChunks; ++c)
                    tma_load_3d(smem + L::kK + st * L::kTile + c * L::kChunk, &tmK, &k_full[st], c * 64, j * kBK, bh);
                k_issued[st] = true;
                k_last[st] = ph;
                if (!mbar_wait(&v_empty[st], ph ^ 1, abort_flag, err, kErrWaitSmemEmpty)) break;
                mbar_arrive_expect_tx(&v_full[st], L::kTile);
                for (int c = 0; c < kDChunks; ++c)
                    tma_load_3d(smem + L::kV + st * L::kTile + c * L::kChunk, &tmV, &v_full[st], c * 64, j * kBK, bh);
                v_issued[st] = true;
                v_last[st] = ph;
            }
            if (*abort_flag) {
                if (q_issued) mbar_wait_drain(q_full, 0, err);
                for (int s = 0; s < 2; ++s) {
                    if (k_issued[s]) mbar_wait_drain(&k_full[s], k_last[s], err);
                    if (v_issued[s]) mbar_wait_drain(&v_full[s], v_last[s], err);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ------------------------------------- MMA issuer
            const uint32_t sq = smem_u32(smem + L::kQ), sp = smem_u32(smem + L::kP);
            auto issue_s = [&](int j) -> bool {
                const int st = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                if (!mbar_wait(&k_full[st], ph, abort_flag, err, kErrWaitTmaFull)) return false;
                if (!mbar_wait(&s_empty[st], ph ^ 1, abort_flag, err, kErrWaitScore)) return false;
                tc_fence_after();
                const uint32_t sk = smem_u32(smem + L::kK + st * L::kTile);
#pragma unroll
                for (int t = 0; t < D / 16; ++t) {
                    const uint32_t off = (t >> 2) * L::kChunk + (t & 3) * 32;
                    umma<false>(tmem_s[st], sdesc_sw128(sq + off, 16, 1024), sdesc_sw128(sk + off, 16, 1024), kIdescS, t != 0);
                }
                umma_commit(&k_empty[st]);
                umma_commit(&s_full[st]);
                return true;
            };
            bool ok = mbar_wait(q_full, 0, abort_flag, err, kErrWaitTmaFull);
            if (ok) ok = issue_s(0);
            for (int j = 0; ok && j < n_kv; ++j) {
                if (j + 1 < n_kv && !(ok = issue_s(j + 1))) break;
                const int st = j & 1;
                if (!mbar_wait(&v_full[st], (j >> 1) & 1, abort_flag, err, kErrWaitTmaFull)) break;
                // P_j is in shared memory and O has been rescaled to the new row
                // maxima by the softmax warps before they arrive on p_full.
                if (!mbar_wait(p_full, j & 1, abort_flag, err, kErrWaitProb)) break;
                tc_fence_after();
                const uint32_t sv = smem_u32(smem + L::kV + st * L::kTile);
#pragma unroll
                for (int t = 0; t < kBK / 16; ++t) {
                    const uint64_t a = sdesc_sw128(sp + (t >> 2) * L::kChunk + (t & 3) * 32, 16, 1024);
                    const uint64_t b = sdesc_sw128(sv + t * 16 * 128, L::kChunk, 1024);
                    umma<false>(tmem_o, a, b, kIdescO, (j | t) != 0);
                }
                umma_commit(&v_empty[st]);
                umma_commit(o_full);
            }
            umma_commit(mma_done);
            mbar_wait_drain(mma_done, 0, err);
        }
    } else if (warp >= kFirstSoftWarp) {
        // ----------------------------------------------------- softmax warps
        const int sw = warp - kFirstSoftWarp;  // 0..7
        const int quarter = warp & 3;          // TMEM lane quarter
        const int half = sw >> 2;              // column half
        const int row = quarter * 32 + lane;   // query row within the tile
        const int q = q0 + row;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        TIn *pbuf = reinterpret_cast<TIn *>(smem + L::kP + half * L::kChunk);

        // exchange with the partner thread (same row, other half); returns the
        // partner's value; `ok` becomes the pair-uniform conjunction of votes.
        int xslot = 0;
        auto exchange = [&](float v, bool &ok) -> float {
            const int vote = __all_sync(0xffffffffu, ok) ? 1 : 0;
            const int base = xslot * 256;
            xch_v[base + half * 128 + row] = v;
            xch_ok[base + half * 128 + row] = vote;
            named_bar_sync(1 + quarter, 64);
            const float other = xch_v[base + (half ^ 1) * 128 + row];
            const int other_ok = xch_ok[base + (half ^ 1) * 128 + row];
            ok = vote && other_ok;
            xslot = (xslot + 1) & 3;
            return other;
        };

        float m_run = -INFINITY, l_run = 0.0f;
        bool ok = true;
        int j = 0;
        for (; j < n_kv; ++j) {
            const int st = j & 1;
            // ---- scores S_j (this thread's 64 columns of its row)
            ok = mbar_wait(&s_full[st], (j >> 1) & 1, abort_flag, err, kErrWaitScore);
            ok = __all_sync(0xffffffffu, ok);
            float s[64];
            float pmax = -INFINITY;
            if (ok) {
                tc_fence_after();
                tmem_ld32f(tmem_s[st] + lane_off + half * 64, s);
                tmem_ld32f(tmem_s[st] + lane_off + half * 64 + 32, s + 32);
                tmem_wait_ld();
                tc_fence_before();
                mbar_arrive(&s_empty[st]);
                const int k0 = j * kBK + half * 64;
                const bool need_mask = (args.causal && j == qt) || (j * kBK + kBK > args.seq);
#pragma unroll
                for (int i = 0; i < 64; ++i) s[i] *= args.scale_log2;
                if (need_mask) {
#pragma unroll
                    for (int i = 0; i < 64; ++i) {
                        const int key = k0 + i;
                        if (key >= args.seq || (args.causal && key > q)) s[i] = -INFINITY;
                    }
                }
#pragma unroll
                for (int i = 0; i < 64; ++i) pmax = fmaxf(pmax, s[i]);
            }
            const float other_max = exchange(pmax, ok);
            if (!ok) break;
            const float m_new = fmaxf(m_run, fmaxf(pmax, other_max));
            const float alpha = fast_exp2(m_run - m_new);
            m_run = m_new;
            float psum = 0.0f;
#pragma unroll
            for (int i = 0; i < 64; ++i) {
                s[i] = fast_exp2(s[i] - m_new);
                psum += s[i];
            }
            l_run = l_run * alpha + psum;
            // ---- P_{j-1} V_{j-1} must be done before P and O are touched
            if (j > 0) {
                ok = mbar_wait(o_full, (j - 1) & 1, abort_flag, err, kErrWaitPv);
                (void)exchange(0.0f, ok);
                if (!ok) break;
            }
#pragma unroll
            for (int g = 0; g < 8; ++g) {
                uint4 u;
                if constexpr (kFmt == 1) {
                    u.x = pack_bf16(s[8 * g + 0], s[8 * g + 1]); u.y = pack_bf16(s[8 * g + 2], s[8 * g + 3]);
                    u.z = pack_bf16(s[8 * g + 4], s[8 * g + 5]); u.w = pack_bf16(s[8 * g + 6], s[8 * g + 7]);
                } else {
                    u.x = pack_f16(s[8 * g + 0], s[8 * g + 1]); u.y = pack_f16(s[8 * g + 2], s[8 * g + 3]);
                    u.z = pack_f16(s[8 * g + 4], s[8 * g + 5]); u.w = pack_f16(s[8 * g + 6], s[8 * g + 7]);
                }
                *reinterpret_cast<uint4 *>(reinterpret_cast<uint8_t *>(pbuf) + row * 128 + ((g ^ (row & 7)) << 4)) = u;
            }
            fence_proxy_async();
            // ---- rescale the running output O (in TMEM) to the new maxima; skipped
            // when no row of this warp changed its maximum (alpha == 1 exactly)
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
                tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < kHalfCols; c += 32) {
                    float r[32];
                    const uint32_t ta = tmem_o + lane_off + half * kHalfCols + c;
                    tmem_ld32f(ta, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) r[i] *= alpha;
                    tmem_st32f(ta, r);
                }
                tmem_wait_st();
            }
            tc_fence_before();
            mbar_arrive(p_full);
        }
        if (ok && j == n_kv) {
            ok = mbar_wait(o_full, (n_kv - 1) & 1, abort_flag, err, kErrWaitPv);
            ok = __all_sync(0xffffffffu, ok);
            const float other_l = exchange(l_run, ok);
            if (ok) {
                tc_fence_after();
                const float inv = 1.0f / (l_run + other_l);
                TOut *o = static_cast<TOut *>(args.out) + ((size_t)bh * args.seq + q) * D + half * kHalfCols;
#pragma unroll 1
                for (int c = 0; c < kHalfCols; c += 32) {
                    float r[32];
                    tmem_ld32f(tmem_o + lane_off + half * kHalfCols + c, r);
                    tmem_wait_ld();
                    if (q < args.seq) {
#pragma unroll
                        for (int e = 0; e < 32; e += 8) {
                            if constexpr (std::is_same<TOut, float>::value) {
                                *reinterpret_cast<float4 *>(o + c + e) = make_float4(r[e] * inv, r[e + 1] * inv, r[e + 2] * inv, r[e + 3] * inv);
                                *reinterpret_cast<float4 *>(o + c + e + 4) =
                                    make_float4(r[e + 4] * inv, r[e + 5] * inv, r[e + 6] * inv, r[e + 7] * inv);
                            } else {
                                uint4 u;
                                if constexpr (std::is_same<TOut, __nv_bfloat16>::value) {
                                    u.x = pack_bf16(r[e] * inv, r[e + 1] * inv); u.y = pack_bf16(r[e + 2] * inv, r[e + 3] * inv);
                                    u.z = pack_bf16(r[e + 4] * inv, r[e + 5] * inv); u.w = pack_bf16(r[e + 6] * inv, r[e + 7] * inv);
                                } else {
                                    u.x = pack_f16(r[e] * inv, r[e + 1] * inv); u.y = pack_f16(r[e + 2] * inv, r[e + 3] * inv);
                                    u.z = pack_f16(r[e + 4] * inv, r[e + 5] * inv); u.w = pack_f16(r[e + 6] * inv, r[e + 7] * inv);
                                }
                                *reinterpret_cast<uint4 *>(o + c + e) = u;
                            }
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
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

// [bh, seq, D] tensor, box {64, 128, 1}, 128-byte swizzle.
bool make_map3(CUtensorMap *map, CUtensorMapDataType dt, const void *ptr, uint64_t bh, uint64_t seq, uint64_t d) {
    EncodeFn enc = encoder();
    if (!enc) return false;
    const cuuint64_t dims[3] = {d, seq, bh};
    const cuuint64_t strides[2] = {d * 2, seq * d * 2};
    const cuuint32_t box[3] = {64, 128, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, dt, 3, const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D, typename TIn, typename TOut>
LaunchFn attn_launch(Context *ctx, const Spec &s) {
    using L = AttnLayout<D>;
    auto kernel = attention_tc_kernel<D, TIn, TOut>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kSmem) != cudaSuccess)
        throw IrError("cannot reserve shared memory for the tcgen05 attention");

    const CUtensorMapDataType dt = std::is_same<TIn, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    AttnArgs base{};
    base.seq = (int)s.seq;
    base.heads_total = (int)(s.batch * s.heads);
    base.nq_tiles = (int)((s.seq + kBQ - 1) / kBQ);
    base.nkv_tiles = (int)((s.seq + kBK - 1) / kBK);
    base.causal = s.causal ? 1 : 0;
    base.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)D));
    base.err = ctx->err_dev;
    const dim3 grid(base.heads_total, base.nq_tiles);
    const uint64_t bh = base.heads_total, seq = s.seq;
    return [=](cudaStream_t st, void **b) {
        CUtensorMap mq, mk, mv;
        if (!make_map3(&mq, dt, b[0], bh, seq, D) || !make_map3(&mk, dt, b[1], bh, seq, D) || !make_map3(&mv, dt, b[2], bh, seq, D))
            return cudaErrorInvalidValue;
        AttnArgs a = base;
        a.out = b[3];
        kernel<<<grid, kThreads, L::kSmem, st>>>(mq, mk, mv, a);
        return cudaGetLastError();
    };
}

}  // namespace

LaunchFn make_attention_tc(Context *ctx, const Spec &s, std::string &impl) {
    if (s.op != Op::AttentionOnline) throw IrError("only attention_online has a tensor-core path");
    if (!encoder()) throw IrError("cuTensorMapEncodeTiled unavailable");
    impl = std::string("attention_tcgen05_fa_q128_kv128_d") + std::to_string(s.dim) + "_" + dtype_name(s.dtype) + "_out_" +
           dtype_name(s.out_dtype) + (s.causal ? "_causal" : "");
    const bool f32out = s.out_dtype == DType::F32;
    if (s.dtype == DType::BF16) {
        if (s.dim == 128) return f32out ? attn_launch<128, __nv_bfloat16, float>(ctx, s) : attn_launch<128, __nv_bfloat16, __nv_bfloat16>(ctx, s);
        return f32out ? attn_launch<64, __nv_bfloat16, float>(ctx, s) : attn_launch<64, __nv_bfloat16, __nv_bfloat16>(ctx, s);
    }
    if (s.dim == 128) return f32out ? attn_launch<128, __half, float>(ctx, s) : attn_launch<128, __half, __half>(ctx, s);
    return f32out ? attn_launch<64, __half, float>(ctx, s) : attn_launch<64, __half, __half>(ctx, s);
}

}  // namespace jade
