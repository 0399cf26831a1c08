// FlashAttention-style forward attention on tcgen05 for BF16/FP16 inputs.
//
// Semantics: O = softmax(Q K^T / sqrt(D) [causal: key <= query]) V, the
// reference's online attention (src/runtime/metal_attention.rs:44-137, oracle
// src/runtime/metal_lab.rs:33-73) extended to a batch dimension: Q/K/V/O are
// [batch, heads, seq, dim] row-major, dim 64 or 128. Softmax statistics are
// FP32; P is rounded to the input type for P.V; O accumulates in FP32 in TMEM.
//
// One CTA owns two 128-query tiles (A, B) of one (batch, head) and streams the
// shared K/V tiles of 128 keys once for both:
//   warp 0     TMA: Q_A, Q_B once; K_j, V_j into two-stage rings (separate K and
//              V barriers: K_j's slot refills as soon as both S_A(j), S_B(j) are done)
//   warp 1     MMA, in the order  S_A(0) S_B(0) | PV_A(j) S_A(j+1) PV_B(j) S_B(j+1) ...
//              so the tensor core works on one tile while the other tile's
//              softmax runs (ping-pong). P_t(j) is read from TMEM (A operand).
//   warps 2-5  softmax of tile A, warps 6-9 softmax of tile B: one thread per
//              query row (TMEM lane) reads the row of S_t(j) in one round trip and
//              writes P = exp2(S*scale - m) (attention_softmax.cuh) as 16-bit pairs
//              over the first 64 columns of the same TMEM buffer.
// TMEM: S_A | S_B | O_A | O_B (128 columns each). O is rescaled in place only
// when a row maximum grows by more than 2^8 (until then P <= 256 is exact
// enough in FP32 accumulation), so steady-state iterations never touch O.
// When S_t(j) lands, P_t(j-1).V(j-1) has completed (both come from the MMA lane
// in that order), so the rescale needs no extra wait.
// Causal: tiles above the diagonal are skipped; the heaviest pairs go first.
// Every wait is bounded; an abort makes each warp leave at a warp-uniform point.
#include <cuda.h>

#include <climits>
#include <mutex>
#include <type_traits>

#include "attention_softmax.cuh"
#include "common.cuh"
#include "internal.hpp"

namespace jade {
namespace {

constexpr int kBQ = 128, kBK = 128, kThreads = 10 * 32;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O when a row max grows by more than 2^8

template <int D>
struct AttnLayout {
    static constexpr uint32_t kChunk = 128 * 128;          // 128 rows x 128 B (64 elements)
    static constexpr uint32_t kTile = (D / 64) * kChunk;   // Q / K / V tile bytes
    static constexpr uint32_t kQ = 0;                       // Q_A, Q_B
    static constexpr uint32_t kK = kQ + 2 * kTile;          // 2 stages
    static constexpr uint32_t kV = kK + 2 * kTile;          // 2 stages
    static constexpr uint32_t kBar = kV + 2 * kTile;
    static constexpr uint32_t kSmem = kBar + 256 + 1024;
};

struct AttnArgs {
    void *out;
    int seq, nq_tiles, npairs, nkv_tiles, causal;
    int bh_total, group_heads;  // block order: heads in L2-sized groups, heaviest pairs first
    float scale_log2;
    int *err;
};

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
template <int D, typename TIn, typename TOut>
__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, const AttnArgs args) {
    using L = AttnLayout<D>;
    constexpr uint32_t kFmt = std::is_same<TIn, __nv_bfloat16>::value ? 1u : 0u;
    constexpr uint32_t kIdescS = idesc_f32acc(kFmt, kFmt, false, false, kBQ, kBK);
    constexpr uint32_t kIdescO = idesc_f32acc(kFmt, kFmt, false, true, kBQ, D);
    constexpr int kDChunks = D / 64;

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBar);
    uint64_t *q_full = bars + 0;
    uint64_t *k_full = bars + 1, *k_empty = bars + 3, *v_full = bars + 5, *v_empty = bars + 7;
    uint64_t *s_full = bars + 9, *p_full = bars + 11, *o_full = bars + 13;  // [tile]
    uint64_t *mma_done = bars + 15;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 16);
    uint64_t *o_staged = bars + 17;  // [tile]: 16-bit O rows written to the tile's Q buffer
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Block b covers head group g (group_heads heads whose K/V fit in L2 together, so
    // the blocks resident at one time share cached K/V) and, inside it, the heaviest
    // causal q-tile pairs first.
    int bh, pair;
    {
        const int b = blockIdx.x, per_group = args.group_heads * args.npairs, g = b / per_group;
        const int h0 = g * args.group_heads, hg = min(args.group_heads, args.bh_total - h0), i = b - g * per_group;
        bh = h0 + i % hg;
        pair = args.npairs - 1 - i / hg;
    }
    int qt[2], nkv[2];
    for (int t = 0; t < 2; ++t) {
        qt[t] = 2 * pair + t;
        nkv[t] = qt[t] >= args.nq_tiles ? 0 : (args.causal ? min(qt[t] + 1, args.nkv_tiles) : args.nkv_tiles);
    }
    const int nkv_max = max(nkv[0], nkv[1]);
    int *err = args.err;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&k_full[s], 1); mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1); mbar_init(&v_empty[s], 1);
            mbar_init(&s_full[s], 1); mbar_init(&p_full[s], 128); mbar_init(&o_full[s], 1);
        }
        mbar_init(mma_done, 1);
        mbar_init(&o_staged[0], 128);
        mbar_init(&o_staged[1], 128);
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
    const uint32_t tmem_o[2] = {tmem + 256, tmem + 384};

    if (warp == 0) {
        if (lane == 0) {  // ------------------------------------- TMA producer
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            bool k_issued[2] = {false, false}, v_issued[2] = {false, false};
            uint32_t k_last[2] = {0, 0}, v_last[2] = {0, 0};
            const int ntiles = (nkv[0] > 0) + (nkv[1] > 0);
            mbar_arrive_expect_tx(q_full, ntiles * L::kTile);
            for (int t = 0; t < 2; ++t)
                if (nkv[t] > 0)
                    for (int c = 0; c < kDChunks; ++c)
                        tma_load_3d(smem + L::kQ + t * L::kTile + c * L::kChunk, &tmQ, q_full, c * 64, qt[t] * kBQ, bh);
            for (int j = 0; j < nkv_max && !*abort_flag; ++j) {
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
                if (ntiles) mbar_wait_drain(q_full, 0, err);
                for (int s = 0; s < 2; ++s) {
                    if (k_issued[s]) mbar_wait_drain(&k_full[s], k_last[s], err);
                    if (v_issued[s]) mbar_wait_drain(&v_full[s], v_last[s], err);
                }
            }
        }
    } else if (warp == 1) {
        {  // ------------------------------------- MMA issuer (whole warp, one elected lane issues)
            const uint32_t sq0 = smem_u32(smem + L::kQ);
            // suspending waits: in this kernel the softmax warps sharing the SM
            // sub-partition are busy while this warp waits, and polling would take
            // their issue slots (measured slower than try_wait on B200)
            auto wait = [&](uint64_t *bar, uint32_t parity, int code) {
                return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, err, code));
            };
            auto issue_s = [&](int t, int j) {
                const uint32_t sq = sq0 + t * L::kTile, sk = smem_u32(smem + L::kK + (j & 1) * L::kTile);
#pragma unroll
                for (int k = 0; k < D / 16; ++k) {
                    const uint32_t off = (k >> 2) * L::kChunk + (k & 3) * 32;
                    umma<false>(tmem_s[t], sdesc_sw128(sq + off, 16, 1024), sdesc_sw128(sk + off, 16, 1024), kIdescS, k != 0);
                }
                umma_commit(&s_full[t]);
            };
            auto issue_pv = [&](int t, int j) {
                const uint32_t sv = smem_u32(smem + L::kV + (j & 1) * L::kTile);
#pragma unroll
                for (int k = 0; k < kBK / 16; ++k)
                    umma_ts(tmem_o[t], tmem_s[t] + k * 8, sdesc_sw128(sv + k * 16 * 128, L::kChunk, 1024), kIdescO, (j | k) != 0);
                umma_commit(&o_full[t]);
            };
            bool ok = nkv_max > 0 && mbar_wait_warp(q_full, 0, abort_flag, err, kErrWaitTmaFull);
            if (ok) ok = mbar_wait_warp(&k_full[0], 0, abort_flag, err, kErrWaitTmaFull);
            if (ok) {
                tc_fence_after();
                for (int t = 0; t < 2; ++t)
                    if (nkv[t] > 0) issue_s(t, 0);
                umma_commit(&k_empty[0]);
            }
            for (int j = 0; ok && j < nkv_max; ++j) {
                const bool more = j + 1 < nkv_max;
                bool k_ready = false;
                if (!(ok = wait(&v_full[j & 1], (j >> 1) & 1, kErrWaitTmaFull))) break;
                for (int t = 0; t < 2 && ok; ++t) {
                    if (j >= nkv[t]) continue;
                    if (!(ok = wait(&p_full[t], j & 1, kErrWaitProb))) break;
                    tc_fence_after();
                    issue_pv(t, j);  // reads P_t(j) from TMEM: must precede S_t(j+1)
                    if (j + 1 < nkv[t]) {
                        if (!k_ready && !(ok = wait(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, kErrWaitTmaFull))) break;
                        k_ready = true;
                        tc_fence_after();
                        issue_s(t, j + 1);  // overwrites S_t / P_t
                    }
                }
                if (!ok) break;
                umma_commit(&v_empty[j & 1]);
                if (more) umma_commit(&k_empty[(j + 1) & 1]);
            }
            umma_commit(mma_done);
            mbar_wait_drain(mma_done, 0, err);
        }
    } else {
        // ----------------------------------------------------- softmax (warps 2-5: tile A, 6-9: tile B)
        const int t = (warp - 2) >> 2;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const int q = qt[t] * kBQ + row;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        const uint32_t ts = tmem_s[t] + lane_off, to = tmem_o[t] + lane_off;
        const float c = args.scale_log2;
        float m_used = -INFINITY, l_run = 0.0f;
        bool ok = true;
        int j = 0;
        for (; j < nkv[t]; ++j) {
            ok = __all_sync(0xffffffffu, mbar_wait(&s_full[t], j & 1, abort_flag, err, kErrWaitScore));
            if (!ok) break;
            tc_fence_after();
            const bool need_mask = (args.causal && j == qt[t]) || (j * kBK + kBK > args.seq);
            const int k0 = j * kBK;
            // the whole row of S_t(j) in one round trip (one wait for four loads)
            float sv[128];
            tmem_ld32f(ts, sv);
            tmem_ld32f(ts + 32, sv + 32);
            tmem_ld32f(ts + 64, sv + 64);
            tmem_ld32f(ts + 96, sv + 96);
            tmem_wait_ld();
            if (need_mask) {  // keys k0 + i with i > lim are invisible to this row
                const int lim = min(args.seq - 1, args.causal ? q : INT_MAX) - k0;
#pragma unroll
                for (int i = 0; i < 128; ++i) sv[i] = i <= lim ? sv[i] : -INFINITY;
            }
            float mx[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) mx[e] = max3(sv[e], sv[e + 8], sv[e + 16]);
#pragma unroll
            for (int i = 24; i < 120; i += 16)
#pragma unroll
                for (int e = 0; e < 8; ++e) mx[e] = max3(mx[e], sv[i + e], sv[i + 8 + e]);
#pragma unroll
            for (int e = 0; e < 8; ++e) mx[e] = fmaxf(mx[e], sv[120 + e]);
            const float mraw = max3(max3(mx[0], mx[1], mx[2]), max3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
            const float m_tile = mraw * c;
            // lazy rescale: keep the old maximum unless it grew by more than 2^8
            float m_new = m_used, alpha = 1.0f;
            if (j == 0) m_new = m_tile;
            else if (m_tile > m_used + kRescaleThreshold) {
                m_new = m_tile;
                alpha = fast_exp2(m_used - m_new);
            }
            m_used = m_new;
            // P = exp2(S*c - m) as 16-bit pairs over S's first 64 columns; masked
            // scores are -inf and go through MUFU, which gives exact zeros.
            const float psum = need_mask ? store_p<kFmt, false, 128>(sv, c, m_used, ts) : store_p<kFmt, kFmt == 1, 128>(sv, c, m_used, ts);
            // O (in TMEM) to the new maxima, after P so the scores' registers are free
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
                for (int oc = 0; oc < D; oc += 32) {
                    float ov[32];
                    tmem_ld32f(to + oc, ov);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) ov[i] *= alpha;
                    tmem_st32f(to + oc, ov);
                }
            }
            l_run = l_run * alpha + psum;
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&p_full[t]);
        }
        if (ok && nkv[t] > 0) {
            ok = __all_sync(0xffffffffu, mbar_wait(&o_full[t], (nkv[t] - 1) & 1, abort_flag, err, kErrWaitPv));
            if (ok) {
                tc_fence_after();
                const float inv = 1.0f / l_run;
                if constexpr (std::is_same<TOut, float>::value) {
                    float *o = static_cast<float *>(args.out) + ((size_t)bh * args.seq + q) * D;
#pragma unroll 1
                    for (int oc = 0; oc < D; oc += 32) {
                        float r[32];
                        tmem_ld32f(to + oc, r);
                        tmem_wait_ld();
                        if (q < args.seq)
#pragma unroll
                            for (int e = 0; e < 32; e += 4)
                                *reinterpret_cast<float4 *>(o + oc + e) = make_float4(r[e] * inv, r[e + 1] * inv, r[e + 2] * inv, r[e + 3] * inv);
                    }
                } else {
                    // The tile's Q buffer is free (every S_t MMA completed before the last
                    // P_t.V did): stage O there in the Q tensor map's layout (64-column
                    // chunks, 128-byte swizzle) and write it with TMA stores - coalesced,
                    // clipped at seq, and off the warps' memory pipe.
                    uint8_t *stg = smem + L::kQ + t * L::kTile;
#pragma unroll 1
                    for (int oc = 0; oc < D; oc += 32) {
                        float r[32];
                        tmem_ld32f(to + oc, r);
                        tmem_wait_ld();
                        uint8_t *rowp = stg + (oc / 64) * L::kChunk + row * 128;
#pragma unroll
                        for (int e = 0; e < 32; e += 8) {
                            uint4 u;
                            u.x = pack16<kFmt>(r[e] * inv, r[e + 1] * inv);
                            u.y = pack16<kFmt>(r[e + 2] * inv, r[e + 3] * inv);
                            u.z = pack16<kFmt>(r[e + 4] * inv, r[e + 5] * inv);
                            u.w = pack16<kFmt>(r[e + 6] * inv, r[e + 7] * inv);
                            const int unit = ((oc % 64) + e) / 8;  // 16-byte unit within the 128-byte row
                            *reinterpret_cast<uint4 *>(rowp + ((unit ^ (row & 7)) << 4)) = u;
                        }
                    }
                    fence_proxy_async();
                    mbar_arrive(&o_staged[t]);
                    if (quarter == 2 && lane == 0) {  // one issuer per tile
                        if (mbar_wait(&o_staged[t], 0, abort_flag, err, kErrWaitPv) && qt[t] * kBQ < args.seq) {
                            for (int c = 0; c < kDChunks; ++c) tma_store_3d(&tmO, stg + c * L::kChunk, c * 64, qt[t] * kBQ, bh);
                            bulk_commit_group();
                        }
                        bulk_wait_all();  // the stores have read shared memory before the CTA exits
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
    const int heads_total = (int)(s.batch * s.heads);
    base.nq_tiles = (int)((s.seq + kBQ - 1) / kBQ);
    base.npairs = (base.nq_tiles + 1) / 2;
    base.nkv_tiles = (int)((s.seq + kBK - 1) / kBK);
    base.causal = s.causal ? 1 : 0;
    base.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)D));
    base.err = ctx->err_dev;
    base.bh_total = heads_total;
    base.group_heads = (int)std::max<long long>(1, std::min<long long>(heads_total, (64ll << 20) / (4ll * (long long)s.seq * D)));
    if ((long long)heads_total * base.npairs > INT_MAX) throw IrError("attention too large for one launch");
    const dim3 grid(heads_total * base.npairs);
    const uint64_t bh = heads_total, seq = s.seq;
    return [=](cudaStream_t st, void **b) {
        CUtensorMap mq, mk, mv;
        if (!make_map3(&mq, dt, b[0], bh, seq, D) || !make_map3(&mk, dt, b[1], bh, seq, D) || !make_map3(&mv, dt, b[2], bh, seq, D))
            return cudaErrorInvalidValue;
        // 16-bit outputs (same element type as the inputs) leave through TMA stores
        CUtensorMap mo;
        if (!make_map3(&mo, dt, std::is_same<TOut, float>::value ? b[0] : b[3], bh, seq, D)) return cudaErrorInvalidValue;
        AttnArgs a = base;
        a.out = b[3];
        kernel<<<grid, kThreads, L::kSmem, st>>>(mq, mk, mv, mo, a);
        return cudaGetLastError();
    };
}

}  // namespace

LaunchFn make_attention_tc(Context *ctx, const Spec &s, std::string &impl) {
    if (s.op != Op::AttentionOnline) throw IrError("only attention_online has a tensor-core path");
    if (!encoder()) throw IrError("cuTensorMapEncodeTiled unavailable");
    impl = std::string("attention_tcgen05_fa_2xq128_kv128_d") + std::to_string(s.dim) + "_" + dtype_name(s.dtype) + "_out_" +
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
