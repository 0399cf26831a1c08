// FlashAttention-style forward attention on tcgen05 for BF16/FP16 inputs.
//
// Semantics: O = softmax(Q K^T / sqrt(D) [causal: key <= query]) V, the
// reference's online attention (src/runtime/metal_attention.rs:44-137, oracle
// src/runtime/metal_lab.rs:33-73) extended to a batch dimension: Q/K/V/O are
// [batch, heads, seq, dim] row-major, dim 64 or 128. Softmax statistics are
// FP32; P is rounded to the input type for P.V; O accumulates in FP32 in TMEM.
//
// Persistent: one CTA per SM loops over work items. An item is two 128-query
// tiles (A, B) of one (batch, head) that share the stream of K/V tiles of 128 keys:
//   warp 0     TMA: Q_A, Q_B of each item (a tile's Q buffer refills for the next
//              item as soon as its last S MMA has read it); K_j, V_j into
//              two-stage rings that run on across items
//   warp 1     MMA, in the order  S_A(0) S_B(0) | PV_A(j) S_A(j+1) PV_B(j) S_B(j+1) ...
//              so the tensor core works on one tile while the other tile's
//              softmax runs (ping-pong). P_t(j) is read from TMEM (A operand).
//              The next item's first S MMAs follow the last P.V of this one.
//   warps 2-5  softmax of tile A, warps 6-9 softmax of tile B: one thread per
//              query row (TMEM lane) reads the row of S_t(j) in one round trip and
//              writes P = exp2(S*scale - m) (attention_softmax.cuh) as 16-bit pairs
//              over the first 64 columns of the same TMEM buffer. At the end of an
//              item they read O_t out of TMEM (releasing it to the next item's
//              P.V) and write it: FP32 directly, 16-bit through a staging buffer
//              and TMA stores, while the tensor core already works on the next item.
// TMEM: S_A | S_B | O_A | O_B (128 columns each). O is rescaled in place only
// when a row maximum grows by more than 2^8 (until then P <= 256 is exact
// enough in FP32 accumulation), so steady-state iterations never touch O.
// When S_t(j) lands, P_t(j-1).V(j-1) has completed (both come from the MMA warp
// in that order), so the rescale needs no extra wait.
// Causal: tiles above the diagonal are skipped. Work order: heads in groups
// whose K/V fit in L2 together; inside a group the heaviest pairs first, dealt to
// the CTAs boustrophedon (balanced to a few percent on the causal triangle).
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
    static constexpr uint32_t kTile = (D / 64) * kChunk;   // Q / K / V / O tile bytes
    static constexpr uint32_t kQ = 0;                       // Q_A, Q_B
    static constexpr uint32_t kK = kQ + 2 * kTile;          // 2 stages
    static constexpr uint32_t kV = kK + 2 * kTile;          // 2 stages
    static constexpr uint32_t kO = kV + 2 * kTile;          // 16-bit O staging (TMA store source)
    static constexpr uint32_t kBar = kO + kTile;
    static constexpr uint32_t kSmem = kBar + 256 + 1024;
};

struct AttnArgs {
    void *out;
    int seq, nq_tiles, npairs, nkv_tiles, causal;
    int bh_total, group_heads;  // heads per group of the work order (K/V of a group fit in L2)
    int ctas;                   // persistent CTAs launched
    float scale_log2;
    int *err;
};

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// The work items of one persistent CTA, in order: item (bh, pair) covers query
// tiles 2*pair and 2*pair+1 of head bh. Heads go in groups of group_heads; inside
// a group the items are numbered heaviest pair index first (all heads of a pair
// index together) and dealt to the CTAs boustrophedon: round r gives item
// r*C + s to the CTA in slot s for even r and to slot C-1-s for odd r. The slot
// of a CTA rotates from group to group by the previous groups' remainders, so
// the partial last rounds do not fall on the same CTAs every time. Every role of
// the CTA walks the same sequence.
struct WorkItems {
    int h0 = 0, hg = 0, k = 0, mine = 0, slot = 0, rot = 0;
    __device__ __forceinline__ void open(const AttnArgs &a, int cta) {  // the group that starts at head h0
        hg = min(a.group_heads, a.bh_total - h0);
        const int count = hg * a.npairs, full = count / a.ctas, rem = count % a.ctas;
        slot = (cta - rot + a.ctas) % a.ctas;
        mine = full + (((full & 1) ? a.ctas - 1 - slot : slot) < rem ? 1 : 0);
        rot = (rot + rem) % a.ctas;
        k = 0;
    }
    __device__ __forceinline__ WorkItems(const AttnArgs &a, int cta) { open(a, cta); }
    __device__ __forceinline__ bool next(const AttnArgs &a, int cta, int &bh, int &pair) {
        while (k >= mine) {
            h0 += a.group_heads;
            if (h0 >= a.bh_total) return false;
            open(a, cta);
        }
        const int i = k * a.ctas + ((k & 1) ? a.ctas - 1 - slot : slot);
        ++k;
        bh = h0 + i % hg;
        pair = a.npairs - 1 - i / hg;
        return true;
    }
};

template <int D, typename TIn, typename TOut>
__global__ void __launch_bounds__(kThreads, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, const AttnArgs args) {
    using L = AttnLayout<D>;
    constexpr uint32_t kFmt = std::is_same<TIn, __nv_bfloat16>::value ? 1u : 0u;
    constexpr uint32_t kIdescS = idesc_f32acc(kFmt, kFmt, false, false, kBQ, kBK);
    constexpr uint32_t kIdescO = idesc_f32acc(kFmt, kFmt, false, true, kBQ, D);
    constexpr int kDChunks = D / 64;
    constexpr bool kStaged = !std::is_same<TOut, float>::value;  // 16-bit O leaves through TMA stores

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::kBar);
    uint64_t *q_full = bars + 0, *q_empty = bars + 2;                                            // [tile]
    uint64_t *k_full = bars + 4, *k_empty = bars + 6, *v_full = bars + 8, *v_empty = bars + 10;  // [stage]
    uint64_t *s_full = bars + 12, *p_full = bars + 14;                                           // [tile], per key step
    uint64_t *o_full = bars + 16, *o_free = bars + 18;                                           // [tile], per item
    uint64_t *stg_full = bars + 20, *stg_empty = bars + 21;                                      // O staging
    uint64_t *mma_done = bars + 22;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 23);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int *err = args.err;
    // query tiles of an item and the key tiles each of them attends to
    auto tiles_of = [&](int pair, int (&qt)[2], int (&nkv)[2]) {
        for (int t = 0; t < 2; ++t) {
            qt[t] = 2 * pair + t;
            nkv[t] = qt[t] >= args.nq_tiles ? 0 : (args.causal ? min(qt[t] + 1, args.nkv_tiles) : args.nkv_tiles);
        }
    };
    // TMA loads issued by the producer (read on the abort path, after every role ended)
    int q_armed[2] = {0, 0}, k_last[2] = {-1, -1}, v_last[2] = {-1, -1};

    if (threadIdx.x == 0) {
        for (int t = 0; t < 2; ++t) {
            mbar_init(&q_full[t], 1); mbar_init(&q_empty[t], 1);
            mbar_init(&s_full[t], 1); mbar_init(&p_full[t], 128);
            mbar_init(&o_full[t], 1); mbar_init(&o_free[t], 128);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&k_full[s], 1); mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1); mbar_init(&v_empty[s], 1);
        }
        mbar_init(stg_full, 128);
        mbar_init(stg_empty, 1);
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
    const uint32_t tmem_o[2] = {tmem + 256, tmem + 384};

    if (warp == 0) {
        if (lane == 0) {  // ------------------------------------- TMA producer
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            WorkItems items(args, blockIdx.x);
            int g = 0, bh, pair;  // g: key step over all of this CTA's items (ring position)
            bool ok = true;
            while (ok && items.next(args, blockIdx.x, bh, pair)) {
                int qt[2], nkv[2];
                tiles_of(pair, qt, nkv);
                const int nmax = max(nkv[0], nkv[1]);
                for (int t = 0; t < 2 && ok; ++t) {
                    if (!nkv[t]) continue;
                    if (!(ok = mbar_wait(&q_empty[t], (q_armed[t] & 1) ^ 1, abort_flag, err, kErrWaitSmemEmpty))) break;
                    mbar_arrive_expect_tx(&q_full[t], L::kTile);
                    for (int c = 0; c < kDChunks; ++c)
                        tma_load_3d(smem + L::kQ + t * L::kTile + c * L::kChunk, &tmQ, &q_full[t], c * 64, qt[t] * kBQ, bh);
                    ++q_armed[t];
                }
                for (int j = 0; j < nmax && ok; ++j) {
                    const int gj = g + j, st = gj & 1;
                    const uint32_t ph = (gj >> 1) & 1;
                    if (!(ok = mbar_wait(&k_empty[st], ph ^ 1, abort_flag, err, kErrWaitSmemEmpty))) break;
                    mbar_arrive_expect_tx(&k_full[st], L::kTile);
                    for (int c = 0; c < kDChunks; ++c)
                        tma_load_3d(smem + L::kK + st * L::kTile + c * L::kChunk, &tmK, &k_full[st], c * 64, j * kBK, bh);
                    k_last[st] = gj;
                    if (!(ok = mbar_wait(&v_empty[st], ph ^ 1, abort_flag, err, kErrWaitSmemEmpty))) break;
                    mbar_arrive_expect_tx(&v_full[st], L::kTile);
                    for (int c = 0; c < kDChunks; ++c)
                        tma_load_3d(smem + L::kV + st * L::kTile + c * L::kChunk, &tmV, &v_full[st], c * 64, j * kBK, bh);
                    v_last[st] = gj;
                }
                g += nmax;
            }
        }
    } else if (warp == 1) {
        // ------------------------------------- MMA issuer (whole warp, one elected lane issues)
        // suspending waits: the softmax warps sharing the SM sub-partition are busy
        // while this warp waits, and polling would take their issue slots (measured
        // slower than try_wait on B200)
        auto wait = [&](uint64_t *bar, uint32_t parity, int code) {
            return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag, err, code));
        };
        // Descriptors are built once per tile and advanced by the 16-byte address
        // units of each K step (the start address field is the low 14 bits and
        // shared memory stays below 256 KB, so the addition never carries out):
        // this warp shares its sub-partition with two softmax warps, and fewer
        // instructions per MMA keep the issue ahead of the tensor core.
        const uint64_t dq0 = sdesc_sw128(smem_u32(smem + L::kQ), 16, 1024);
        const uint64_t dk0 = sdesc_sw128(smem_u32(smem + L::kK), 16, 1024);
        const uint64_t dv0 = sdesc_sw128(smem_u32(smem + L::kV), L::kChunk, 1024);
        auto issue_s = [&](int t, int stage) {
            const uint64_t dq = dq0 + ((t * L::kTile) >> 4), dk = dk0 + ((stage * L::kTile) >> 4);
            uint64_t a[D / 16], b[D / 16];
#pragma unroll
            for (int k = 0; k < D / 16; ++k) {
                const uint32_t off = ((k >> 2) * L::kChunk + (k & 3) * 32) >> 4;
                a[k] = dq + off;
                b[k] = dk + off;
            }
            umma_ss_group<D / 16>(tmem_s[t], a, b, kIdescS, 0);
            umma_commit(&s_full[t]);
        };
        auto issue_pv = [&](int t, int stage, bool accumulate) {
            const uint64_t dv = dv0 + ((stage * L::kTile) >> 4);
            uint64_t b[kBK / 16];
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) b[k] = dv + ((k * 16 * 128) >> 4);
            umma_ts_group8(tmem_o[t], tmem_s[t], b, kIdescO, accumulate);
        };
        WorkItems items(args, blockIdx.x);
        // g: ring position; qa: Q loads consumed; cp: P steps consumed; oi: items finished [tile]
        int g = 0, qa[2] = {0, 0}, cp[2] = {0, 0}, oi[2] = {0, 0}, bh, pair;
        bool ok = true;
        while (ok && items.next(args, blockIdx.x, bh, pair)) {
            int qt[2], nkv[2];
            tiles_of(pair, qt, nkv);
            const int nmax = max(nkv[0], nkv[1]);
            for (int t = 0; t < 2 && ok; ++t)
                if (nkv[t]) ok = wait(&q_full[t], qa[t]++ & 1, kErrWaitTmaFull);
            if (ok) ok = wait(&k_full[g & 1], (g >> 1) & 1, kErrWaitTmaFull);
            if (!ok) break;
            tc_fence_after();
            // S_t(0) overwrites S_t / P_t of the previous item: its last P_t.V was issued
            // before, and the tensor core runs one thread's MMAs in order
            for (int t = 0; t < 2; ++t)
                if (nkv[t]) {
                    issue_s(t, g & 1);
                    if (nkv[t] == 1) umma_commit(&q_empty[t]);
                }
            umma_commit(&k_empty[g & 1]);
            for (int j = 0; ok && j < nmax; ++j) {
                const int gj = g + j;
                bool k_ready = false;
                if (!(ok = wait(&v_full[gj & 1], (gj >> 1) & 1, kErrWaitTmaFull))) break;
                for (int t = 0; t < 2 && ok; ++t) {
                    if (j >= nkv[t]) continue;
                    if (!(ok = wait(&p_full[t], cp[t]++ & 1, kErrWaitProb))) break;
                    // the first P.V of an item overwrites O_t: the previous item's O must be read out
                    if (j == 0 && oi[t] > 0 && !(ok = wait(&o_free[t], (oi[t] - 1) & 1, kErrWaitAccEmpty))) break;
                    tc_fence_after();
                    issue_pv(t, gj & 1, j > 0);  // reads P_t(j) from TMEM: must precede S_t(j+1)
                    if (j + 1 < nkv[t]) {
                        if (!k_ready && !(ok = wait(&k_full[(gj + 1) & 1], ((gj + 1) >> 1) & 1, kErrWaitTmaFull))) break;
                        k_ready = true;
                        tc_fence_after();
                        issue_s(t, (gj + 1) & 1);  // overwrites S_t / P_t
                        if (j + 2 == nkv[t]) umma_commit(&q_empty[t]);  // last S of the tile: Q_t may refill
                    } else {
                        umma_commit(&o_full[t]);
                        ++oi[t];
                    }
                }
                if (!ok) break;
                umma_commit(&v_empty[gj & 1]);
                if (j + 1 < nmax) umma_commit(&k_empty[(gj + 1) & 1]);
            }
            g += nmax;
        }
        umma_commit(mma_done);
        mbar_wait_drain(mma_done, 0, err);
    } else {
        // ----------------------------------------------------- softmax (warps 2-5: tile A, 6-9: tile B)
        const int t = (warp - 2) >> 2;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        const uint32_t ts = tmem_s[t] + lane_off, to = tmem_o[t] + lane_off;
        const float c = args.scale_log2;
        WorkItems items(args, blockIdx.x);
        // cs: S steps consumed; oi: items finished; stg_uses: O staging uses so far (both tiles)
        int cs = 0, oi = 0, stg_uses = 0, bh, pair;
        bool ok = true;
        while (ok && items.next(args, blockIdx.x, bh, pair)) {
            int qt[2], nkv[2];
            tiles_of(pair, qt, nkv);
            // the staging buffer serves A then B of each item
            const int use = stg_uses + (t == 1 && nkv[0] > 0 ? 1 : 0);
            stg_uses += (nkv[0] > 0) + (nkv[1] > 0);
            if (nkv[t] == 0) continue;
            const int q = qt[t] * kBQ + row;
            float m_used = -INFINITY, l_run = 0.0f;
            for (int j = 0; j < nkv[t]; ++j) {
                ok = __all_sync(0xffffffffu, mbar_wait(&s_full[t], cs++ & 1, abort_flag, err, kErrWaitScore));
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
                // scores are -inf and go through MUFU, which gives exact zeros. On unmasked
                // tiles 2 of every 8 pairs use the FMA-pipe polynomial (measured best here).
                const float psum =
                    need_mask ? store_p<kFmt, false, 128>(sv, c, m_used, ts) : store_p<kFmt, kFmt == 1, 128, 2>(sv, c, m_used, ts);
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
            if (!ok) break;
            // ------------------------------------------------- epilogue of tile t
            ok = __all_sync(0xffffffffu, mbar_wait(&o_full[t], oi++ & 1, abort_flag, err, kErrWaitPv));
            if (!ok) break;
            tc_fence_after();
            float r[D];
#pragma unroll
            for (int oc = 0; oc < D; oc += 32) tmem_ld32f(to + oc, r + oc);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(&o_free[t]);  // O_t may take the next item's first P.V
            const float inv = 1.0f / l_run;
            if constexpr (!kStaged) {
                if (q < args.seq) {
                    float *o = static_cast<float *>(args.out) + ((size_t)bh * args.seq + q) * D;
#pragma unroll
                    for (int e = 0; e < D; e += 4)
                        *reinterpret_cast<float4 *>(o + e) = make_float4(r[e] * inv, r[e + 1] * inv, r[e + 2] * inv, r[e + 3] * inv);
                }
            } else {
                // stage O in the Q tensor map's layout (64-column chunks, 128-byte
                // swizzle) and write it with TMA stores: coalesced, clipped at seq
                ok = __all_sync(0xffffffffu, mbar_wait(stg_empty, (use & 1) ^ 1, abort_flag, err, kErrWaitAccEmpty));
                if (!ok) break;
                uint8_t *stg = smem + L::kO;
#pragma unroll
                for (int oc = 0; oc < D; oc += 8) {
                    uint4 u;
                    u.x = pack16<kFmt>(r[oc] * inv, r[oc + 1] * inv);
                    u.y = pack16<kFmt>(r[oc + 2] * inv, r[oc + 3] * inv);
                    u.z = pack16<kFmt>(r[oc + 4] * inv, r[oc + 5] * inv);
                    u.w = pack16<kFmt>(r[oc + 6] * inv, r[oc + 7] * inv);
                    const int unit = (oc % 64) / 8;  // 16-byte unit within the 128-byte row
                    *reinterpret_cast<uint4 *>(stg + (oc / 64) * L::kChunk + row * 128 + ((unit ^ (row & 7)) << 4)) = u;
                }
                fence_proxy_async();
                mbar_arrive(stg_full);
                if (quarter == 2 && lane == 0) {  // one issuer per tile
                    if (mbar_wait(stg_full, use & 1, abort_flag, err, kErrWaitPv)) {
                        for (int cc = 0; cc < kDChunks; ++cc) tma_store_3d(&tmO, stg + cc * L::kChunk, cc * 64, qt[t] * kBQ, bh);
                        bulk_commit_group();
                        bulk_wait_read_all();  // the staging buffer is free again
                    }
                    mbar_arrive(stg_empty);
                }
                __syncwarp();
            }
        }
        if (kStaged && quarter == 2 && lane == 0) bulk_wait_all();  // the stores are done before the CTA exits
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        if (lane == 0 && *abort_flag) {  // TMA loads still in flight land before the CTA exits
            for (int t = 0; t < 2; ++t)
                if (q_armed[t]) mbar_wait_drain(&q_full[t], (q_armed[t] - 1) & 1, err);
            for (int s = 0; s < 2; ++s) {
                if (k_last[s] >= 0) mbar_wait_drain(&k_full[s], (k_last[s] >> 1) & 1, err);
                if (v_last[s] >= 0) mbar_wait_drain(&v_full[s], (v_last[s] >> 1) & 1, err);
            }
        }
        __syncwarp();
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
    // K/V of a head group in 32 MB of L2 (measured against 16, 48 and 64 MB: the
    // persistent CTAs drift apart and work on two groups at once near a boundary)
    base.group_heads = attention_group_heads(heads_total, s.seq, D, 32ll << 20);
    if ((long long)heads_total * base.npairs > INT_MAX) throw IrError("attention too large for one launch");
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, L::kSmem) != cudaSuccess || per_sm < 1)
        throw IrError("the tcgen05 attention does not fit on an SM");
    base.ctas = std::min(heads_total * base.npairs, per_sm * ctx->sm_count);  // persistent
    const dim3 grid(base.ctas);
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
