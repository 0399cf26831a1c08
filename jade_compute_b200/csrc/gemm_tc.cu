// tcgen05 GEMM for BF16 / FP16 / TF32 inputs with FP32 accumulation in tensor
// memory (TMEM), fed by TMA, persistent and warp-specialised.
//
// Reference semantics: C = A.B row-major, A [M,K], B [K,N] (src/runtime/ir.rs:298-303,
// 524-557); the reference computes it with SIMT FP32 FMAs only. Extensions for
// the residual MLP (src/runtime/workloads.rs:422-465): B may be stored [N,K]
// (pre-transposed weights), each output row may be scaled by a per-row FP32
// factor (RMSNorm folded in as diag(inv_rms) . x . (diag(w) W)), and the epilogue
// may apply SwiGLU to a gate/up column pair or add a residual.
//
// Design:
//   * CTA tile 128 x 256 (one tcgen05.mma.cta_group::1 M=128,N=256), K step of
//     128 bytes per row (64 BF16/FP16 or 32 TF32 elements), 4-stage TMA ring of
//     48 KB stages in 128-byte-swizzled shared memory, one CTA per SM.
//   * warp 0: TMA producer; warp 1: MMA issuer (one elected lane); warps 2-5:
//     epilogue (each owns one 32-lane quarter of TMEM = 32 output rows).
//   * two 256-column FP32 accumulators in TMEM (all 512 columns), so the epilogue
//     of tile i overlaps the MMAs of tile i+1.
//   * grouped tile raster (8 M-blocks per group) for L2 reuse of A and B.
//   * every mbarrier wait is bounded (common.cuh); the MMA lane drains its own
//     tcgen05 work and the producer its TMA copies before TMEM is freed.
#include <cuda.h>

#include <climits>
#include <cstdlib>
#include <cstdio>
#include <mutex>
#include <type_traits>

#include "../../include/jade_runtime.h"
#include "common.cuh"
#include "internal.hpp"

namespace jade {
namespace {

constexpr int BM = 128, BN = 256, kStages = 4, kThreads = 192;
constexpr uint32_t kStageA = BM * 128, kStageB = BN * 128, kStageBytes = kStageA + kStageB;
// per epilogue warp: a 32 x 32 FP32 block padded to 33 columns (transposes its stores)
constexpr uint32_t kEpiBlock = 32 * 33 * 4, kEpiBytes = 4 * kEpiBlock;
constexpr uint32_t kSmemBytes = kStages * kStageBytes + 256 /*barriers*/ + kEpiBytes + 1024 /*align*/;

enum Epi { kEpiNone = 0, kEpiSwiglu = 1, kEpiResidual = 2, kEpiScatter = 3 };

struct GemmArgs {
    void *out;
    const float *row_scale;
    const void *residual;
    int M, N, K;  // N = output columns
    int tiles_m, tiles_n, num_tiles, kblocks;
    // split-K: work unit u is tile u % num_tiles over K-blocks [s * kb_per, (s + 1) * kb_per)
    // of split s = u / num_tiles, written to out + s * split_stride elements (FP32
    // partials that a second kernel sums in split order); ksplit = 1 otherwise
    int ksplit, kb_per, num_units;
    long long split_stride;
    int group_m;  // M-blocks per raster group (tile_coords)
    int *err;
    // scatter epilogue: every rank's receive buffer; the rows of rank r are
    // [r * rows_per_rank, (r + 1) * rows_per_rank), this GEMM's rank is my_rank
    void *scatter[kMaxPeerRanks];
    int rows_per_rank, my_rank;
    // M-blocks the raster is rotated by: the scatter GEMM starts with the next
    // rank's rows and ends with its own, so the tiles computed last are written to
    // local memory and no NVLink transfer trails the last MMA
    int m_rotate;
};

// M-blocks per raster group: as many as keep the group's A rows (group x 128 x K
// elements) within 48 MB of L2, between 8 and 32 (the MLP gate/up GEMM, K = 4096,
// measured 10% faster at 24-32 than at 8; 64 was slower again), at most all of
// them; JADE_GEMM_GROUP_M overrides (read when a kernel is compiled).
int raster_group(int tiles_m, uint64_t k, int eb) {
    if (const char *force = std::getenv("JADE_GEMM_GROUP_M"); force && *force) return std::max(1, std::min(tiles_m, std::atoi(force)));
    const uint64_t fit = (48ull << 20) / ((uint64_t)BM * k * eb);
    return (int)std::max<uint64_t>(1, std::min<uint64_t>((uint64_t)tiles_m, std::min<uint64_t>(32, std::max<uint64_t>(8, fit))));
}

// Tile t of the grouped raster: M-blocks in groups of `group` rows, every N-block
// of a group before the next group, M fastest inside a group. A group's A rows
// stay in L2 while its N-blocks stream past, so B is read from DRAM about
// tiles_m / group times and A about once.
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int group, int rotate, int &tm, int &tn) {
    const int per_group = group * tiles_n;
    const int g = t / per_group, first_m = g * group;
    const int gm = min(tiles_m - first_m, group);
    const int r = t % per_group;
    tm = first_m + r % gm;
    tn = r / gm;
    if (rotate) tm = (tm + rotate) % tiles_m;
}

template <typename TOut>
__device__ __forceinline__ void store32(TOut *dst, const float (&v)[32], int valid, bool vec_ok);
template <>
__device__ __forceinline__ void store32<float>(float *dst, const float (&v)[32], int valid, bool vec_ok) {
    if (valid >= 32 && vec_ok) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4 *>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (j < valid) dst[j] = v[j];
    }
}
template <typename T16>
__device__ __forceinline__ void store32_16(T16 *dst, const float (&v)[32], int valid, bool vec_ok) {
    if (valid >= 32 && vec_ok) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
            uint4 u;
            if constexpr (std::is_same<T16, __nv_bfloat16>::value) {
                u.x = pack_bf16(v[j], v[j + 1]); u.y = pack_bf16(v[j + 2], v[j + 3]);
                u.z = pack_bf16(v[j + 4], v[j + 5]); u.w = pack_bf16(v[j + 6], v[j + 7]);
            } else {
                u.x = pack_f16(v[j], v[j + 1]); u.y = pack_f16(v[j + 2], v[j + 3]);
                u.z = pack_f16(v[j + 4], v[j + 5]); u.w = pack_f16(v[j + 6], v[j + 7]);
            }
            *reinterpret_cast<uint4 *>(dst + j) = u;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (j < valid) dst[j] = from_f32<T16>(v[j]);
    }
}
template <>
__device__ __forceinline__ void store32<__nv_bfloat16>(__nv_bfloat16 *dst, const float (&v)[32], int valid, bool vec_ok) {
    store32_16(dst, v, valid, vec_ok);
}
// Two values rounded to a 16-bit type, packed low | high << 16.
template <typename T16>
__device__ __forceinline__ uint32_t pack16_out(float lo, float hi) {
    if constexpr (std::is_same<T16, __nv_bfloat16>::value) return pack_bf16(lo, hi);
    else return pack_f16(lo, hi);
}
// Four consecutive values of a row (16 B of FP32, 8 B of 16-bit types).
template <typename TOut>
__device__ __forceinline__ void store4(TOut *dst, const float (&v)[4], int valid, bool vec_ok) {
    if (valid >= 4 && vec_ok) {
        if constexpr (std::is_same<TOut, float>::value) {
            *reinterpret_cast<float4 *>(dst) = make_float4(v[0], v[1], v[2], v[3]);
        } else if constexpr (std::is_same<TOut, __nv_bfloat16>::value) {
            *reinterpret_cast<uint2 *>(dst) = make_uint2(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]));
        } else {
            *reinterpret_cast<uint2 *>(dst) = make_uint2(pack_f16(v[0], v[1]), pack_f16(v[2], v[3]));
        }
    } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
            if (e < valid) dst[e] = from_f32<TOut>(v[e]);
    }
}
template <>
__device__ __forceinline__ void store32<__half>(__half *dst, const float (&v)[32], int valid, bool vec_ok) {
    store32_16(dst, v, valid, vec_ok);
}

// One epilogue lane's share of a 32-column chunk of the residual: rows
// row0 + 4 i + r_sub (i = 0..7), four consecutive columns each, kept as raw words
// (two 16-bit values or one FP32 value per word) until they are added, so the
// loads of a chunk are all in flight while the previous chunk is stored.
template <typename TOut>
struct ResidualChunk {
    static constexpr int kWords = sizeof(TOut);  // 4 values of TOut
    uint32_t w[8][kWords];
};

template <typename TOut>
__device__ __forceinline__ void load_residual(ResidualChunk<TOut> &r, const TOut *__restrict__ res, int row0, int r_sub, int gcol, int M,
                                              int N, bool vec_ok) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int grow = row0 + 4 * i + r_sub;
#pragma unroll
        for (int q = 0; q < ResidualChunk<TOut>::kWords; ++q) r.w[i][q] = 0;
        if (grow >= M || gcol >= N) continue;
        const TOut *p = res + (size_t)grow * N + gcol;
        if (vec_ok && gcol + 4 <= N) {
            if constexpr (sizeof(TOut) == 4) {
                const uint4 v = __ldg(reinterpret_cast<const uint4 *>(p));
                r.w[i][0] = v.x; r.w[i][1] = v.y; r.w[i][2] = v.z; r.w[i][3] = v.w;
            } else {
                const uint2 v = __ldg(reinterpret_cast<const uint2 *>(p));
                r.w[i][0] = v.x; r.w[i][1] = v.y;
            }
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (gcol + e >= N) break;
                if constexpr (sizeof(TOut) == 4) {
                    r.w[i][e] = __ldg(reinterpret_cast<const uint32_t *>(p) + e);
                } else {
                    const uint32_t h = __ldg(reinterpret_cast<const unsigned short *>(p) + e);
                    r.w[i][e >> 1] |= h << ((e & 1) * 16);
                }
            }
        }
    }
}

template <typename TOut>
__device__ __forceinline__ float residual_value(const ResidualChunk<TOut> &r, int i, int e) {
    if constexpr (sizeof(TOut) == 4) {
        return __uint_as_float(r.w[i][e]);
    } else {
        const uint32_t h = (r.w[i][e >> 1] >> ((e & 1) * 16)) & 0xffffu;
        if constexpr (std::is_same<TOut, __nv_bfloat16>::value) return __uint_as_float(h << 16);
        else return __half2float(__ushort_as_half((unsigned short)h));
    }
}

template <int kEB, uint32_t kFmt, bool kBmn, typename TOut, int kEpi, bool kRowScale>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmArgs args) {
    constexpr int BK = 128 / kEB;          // elements per 128-byte row
    constexpr int UK = 32 / kEB;           // K per tcgen05.mma (32 bytes)
    constexpr int kSteps = BK / UK;        // 4
    constexpr uint32_t kIdesc = idesc_f32acc(kFmt, kFmt, false, kBmn, BM, BN);
    constexpr int kBoxMN = 128 / kEB;      // MN-major B: elements per box row
    constexpr int kBoxesB = BN / kBoxMN;   // MN-major B: boxes per stage
    constexpr uint32_t kBoxBytesB = kBoxMN * kEB * BK;  // MN-major B: bytes per box (= BK rows x 128 B)

    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStages * kStageBytes);
    uint64_t *empty = full + kStages;
    uint64_t *acc_full = empty + kStages;
    uint64_t *acc_empty = acc_full + 2;
    uint64_t *mma_done = acc_empty + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(mma_done + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int a = 0; a < 2; ++a) { mbar_init(&acc_full[a], 1); mbar_init(&acc_empty[a], 128); }
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
    const uint32_t tmem_base = *tmem_slot;
    int *err = args.err;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            tma_prefetch_desc(&tmA);
            tma_prefetch_desc(&tmB);
            int stage = 0;
            uint32_t phase = 0;
            bool issued[kStages] = {};
            uint32_t last_phase[kStages] = {};
            for (int u = blockIdx.x; u < args.num_units && !*abort_flag; u += gridDim.x) {
                const int t = u % args.num_tiles, kb0 = (u / args.num_tiles) * args.kb_per;
                int tm, tn;
                tile_coords(t, args.tiles_m, args.tiles_n, args.group_m, args.m_rotate, tm, tn);
                const int m0 = tm * BM, nb0 = tn * BN;  // B rows (nk) or columns (kn) of this tile
                for (int kb = kb0; kb < min(args.kblocks, kb0 + args.kb_per); ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, err, kErrWaitSmemEmpty)) break;
                    uint8_t *sa = smem + stage * kStageBytes;
                    uint8_t *sb = sa + kStageA;
                    mbar_arrive_expect_tx(&full[stage], kStageBytes);
                    tma_load_2d(sa, &tmA, &full[stage], kb * BK, m0);
                    if constexpr (kBmn) {
#pragma unroll
                        for (int j = 0; j < kBoxesB; ++j) tma_load_2d(sb + j * kBoxBytesB, &tmB, &full[stage], nb0 + j * kBoxMN, kb * BK);
                    } else {
                        tma_load_2d(sb, &tmB, &full[stage], kb * BK, nb0);
                    }
                    issued[stage] = true;
                    last_phase[stage] = phase;
                    if (++stage == kStages) { stage = 0; phase ^= 1; }
                }
            }
            if (*abort_flag)
                for (int s = 0; s < kStages; ++s)
                    if (issued[s]) mbar_wait_drain(&full[s], last_phase[s], err);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer (whole warp, one elected lane issues)
        {
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            for (int u = blockIdx.x; u < args.num_units && !__any_sync(0xffffffffu, *abort_flag); u += gridDim.x) {
                const int kb0 = (u / args.num_tiles) * args.kb_per;
                if (!mbar_wait_warp(&acc_empty[acc], acc_phase ^ 1, abort_flag, err, kErrWaitAccEmpty)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                bool ok = true;
                for (int kb = kb0; kb < min(args.kblocks, kb0 + args.kb_per); ++kb) {
                    if (!mbar_wait_warp(&full[stage], phase, abort_flag, err, kErrWaitTmaFull)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + stage * kStageBytes);
                    const uint32_t sb = sa + kStageA;
#pragma unroll
                    for (int k = 0; k < kSteps; ++k) {
                        const uint64_t adesc = sdesc_sw128(sa + k * 32, 16, 1024);
                        uint64_t bdesc;
                        if constexpr (kBmn) bdesc = sdesc_sw128(sb + k * UK * 128, kBoxBytesB, 1024);
                        else bdesc = sdesc_sw128(sb + k * 32, 16, 1024);
                        umma<kFmt == 2>(d_tmem, adesc, bdesc, kIdesc, (kb != kb0) | (k != 0));
                    }
                    umma_commit(&empty[stage]);  // frees the stage when these MMAs finish reading it
                    if (++stage == kStages) { stage = 0; phase ^= 1; }
                }
                if (!ok) break;
                umma_commit(&acc_full[acc]);
                if (++acc == 2) { acc = 0; acc_phase ^= 1; }
            }
            umma_commit(mma_done);  // all tcgen05 work of this thread, done or aborted
            mbar_wait_drain(mma_done, 0, err);
        }
    } else {
        // ------------------------------------------------ epilogue (warps 2..5)
        const int quarter = warp & 3;  // TMEM lanes this warp may access
        const int row_in_tile = quarter * 32 + lane;
        int acc = 0;
        uint32_t acc_phase = 0;
        const int r_sub = lane >> 3, c_sub = (lane & 7) * 4;  // this lane's row in each group of 4, its columns
        ResidualChunk<TOut> res_next;
        for (int u = blockIdx.x; u < args.num_units && !*abort_flag; u += gridDim.x) {
            const int t = u % args.num_tiles;
            int tm, tn;
            tile_coords(t, args.tiles_m, args.tiles_n, args.group_m, args.m_rotate, tm, tn);
            if constexpr (kEpi == kEpiResidual)  // the residual does not wait for the MMAs: fetch chunk 0 now
                load_residual(res_next, static_cast<const TOut *>(args.residual), tm * BM + quarter * 32, r_sub, tn * BN + c_sub,
                              args.M, args.N, (args.N % 4) == 0);
            if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag, err, kErrWaitAccFull)) break;
            tc_fence_after();
            const int row = tm * BM + row_in_tile;
            const uint32_t tbase = tmem_base + ((uint32_t)(quarter * 32) << 16) + acc * BN;
            const float scale = (kRowScale && row < args.M) ? args.row_scale[row] : 1.0f;
            TOut *out = static_cast<TOut *>(args.out) + (u / args.num_tiles) * args.split_stride;
            if constexpr (kEpi == kEpiScatter) {
                // the tile's rows belong to one rank: its receive buffer, this rank's slot
                const int owner = (tm * BM) / args.rows_per_rank;
                out = static_cast<TOut *>(args.scatter[owner]) + (ptrdiff_t)(args.my_rank - owner) * args.rows_per_rank * args.N;
            }
            if constexpr (kEpi == kEpiSwiglu) {
                const int c0 = tn * 128;
#pragma unroll 1
                for (int c = 0; c < 128; c += 32) {
                    uint32_t g[32], u[32];
                    tmem_ld32(tbase + c, g);
                    tmem_ld32(tbase + 128 + c, u);
                    tmem_wait_ld();
                    float h[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float gv = __uint_as_float(g[j]) * scale, uv = __uint_as_float(u[j]) * scale;
                        h[j] = (gv * stable_sigmoid(gv)) * uv;
                    }
                    const int col = c0 + c;
                    if (row < args.M && col < args.N)
                        store32<TOut>(out + (size_t)row * args.N + col, h, args.N - col, (args.N % 8) == 0);
                }
            } else if constexpr (sizeof(TOut) == 2 && (kEpi == kEpiNone || kEpi == kEpiScatter)) {
                // 16-bit output: the warp's 32 rows x 64 columns are rounded first and
                // go through its padded shared-memory block as packed pairs, so that each
                // lane stores 16 bytes and each row segment of a store instruction is one
                // whole 128-byte line (local or, for the scatter, a peer's memory)
                uint32_t *blk = reinterpret_cast<uint32_t *>(smem + kStages * kStageBytes + 256) + (warp - 2) * (32 * 33);
                const int c0 = tn * BN, row0 = tm * BM + quarter * 32;
                const int c8 = (lane & 7) * 8;  // this lane's 8 columns; its row in each group of 4 is r_sub
                const bool vec_ok = (args.N % 8) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
#pragma unroll 1
                for (int c = 0; c < BN; c += 64) {
                    const int col = c0 + c;
                    if (col >= args.N) break;  // uniform across the warp
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        uint32_t r[32];
                        tmem_ld32(tbase + c + 32 * h, r);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            blk[lane * 33 + 16 * h + j] = pack16_out<TOut>(__uint_as_float(r[2 * j]) * scale, __uint_as_float(r[2 * j + 1]) * scale);
                    }
                    __syncwarp();
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int rl = i * 4 + r_sub, grow = row0 + rl, gcol = col + c8;
                        if (grow < args.M && gcol < args.N) {
                            const uint32_t *src = blk + rl * 33 + (c8 >> 1);
                            const uint4 u = make_uint4(src[0], src[1], src[2], src[3]);
                            TOut *dst = out + (size_t)grow * args.N + gcol;
                            if (vec_ok) {
                                *reinterpret_cast<uint4 *>(dst) = u;
                            } else {
                                const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                                for (int e = 0; e < 8; ++e)
                                    if (gcol + e < args.N) reinterpret_cast<uint16_t *>(dst)[e] = (uint16_t)(w[e >> 1] >> (16 * (e & 1)));
                            }
                        }
                    }
                    __syncwarp();  // the block is read before the next chunk overwrites it
                }
            } else {
                // The warp's 32 rows x 32 columns go through its padded shared-memory
                // block, so that each store instruction writes 4 rows x 32 columns
                // (row-contiguous) instead of 32 rows x 4 columns: a thread-per-row
                // store touches 32 cache lines per instruction and made the epilogue
                // of a 128 x 256 FP32 tile take ~5 us.
                float *blk = reinterpret_cast<float *>(smem + kStages * kStageBytes + 256) + (warp - 2) * (32 * 33);
                const int c0 = tn * BN, row0 = tm * BM + quarter * 32;
                const bool vec_ok = (args.N % 4) == 0;
#pragma unroll 1
                for (int c = 0; c < BN; c += 32) {
                    const int col = c0 + c;
                    if (col >= args.N) break;  // uniform across the warp
                    ResidualChunk<TOut> res_cur;
                    if constexpr (kEpi == kEpiResidual) {
                        res_cur = res_next;
                        if (c + 32 < BN)  // next chunk's residual in flight during this chunk's stores
                            load_residual(res_next, static_cast<const TOut *>(args.residual), row0, r_sub, col + 32 + c_sub, args.M, args.N,
                                          vec_ok);
                    }
                    uint32_t r[32];
                    tmem_ld32(tbase + c, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; ++j) blk[lane * 33 + j] = __uint_as_float(r[j]) * scale;
                    __syncwarp();
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int rl = i * 4 + r_sub, grow = row0 + rl, gcol = col + c_sub;
                        if (grow < args.M && gcol < args.N) {
                            float v[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) v[e] = blk[rl * 33 + c_sub + e];
                            if constexpr (kEpi == kEpiResidual) {
#pragma unroll
                                for (int e = 0; e < 4; ++e) v[e] += residual_value(res_cur, i, e);
                            }
                            store4<TOut>(out + (size_t)grow * args.N + gcol, v, args.N - gcol, vec_ok);
                        }
                    }
                    __syncwarp();  // the block is read before the next chunk overwrites it
                }
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[acc]);
            if (++acc == 2) { acc = 0; acc_phase ^= 1; }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 512);
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

// 2-D row-major tensor [rows, cols], box {box_cols, box_rows}, 128-byte swizzle.
bool make_map(CUtensorMap *map, CUtensorMapDataType dt, int eb, const void *ptr, uint64_t rows, uint64_t cols, uint32_t box_cols,
              uint32_t box_rows) {
    EncodeFn enc = encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * (uint64_t)eb};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, dt, 2, const_cast<void *>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int kEB, uint32_t kFmt, bool kBmn, typename TOut, int kEpi, bool kRowScale>
LaunchFn tc_launch(Context *ctx, const Spec &s, int ksplit = 1) {
    auto kernel = gemm_tc_kernel<kEB, kFmt, kBmn, TOut, kEpi, kRowScale>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) != cudaSuccess)
        throw IrError("cannot reserve shared memory for the tcgen05 GEMM");
    const CUtensorMapDataType dt = kFmt == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : kFmt == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                                           : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    GemmArgs base{};
    base.M = (int)s.m;
    base.N = (int)s.n;
    base.K = (int)s.k;
    const bool swiglu = kEpi == kEpiSwiglu;
    const uint64_t brows = swiglu ? 2ull * s.n : s.n;  // rows of B in nk layout / cols in kn layout
    base.tiles_m = (int)((s.m + BM - 1) / BM);
    base.tiles_n = swiglu ? (int)(s.n / 128) : (int)((s.n + BN - 1) / BN);
    base.num_tiles = base.tiles_m * base.tiles_n;
    base.kblocks = (int)((s.k + (128 / kEB) - 1) / (128 / kEB));
    base.group_m = raster_group(base.tiles_m, s.k, kEB);
    base.err = ctx->err_dev;
    base.ksplit = ksplit;
    base.kb_per = (base.kblocks + ksplit - 1) / ksplit;
    base.num_units = base.num_tiles * ksplit;
    base.split_stride = ksplit > 1 ? (long long)s.m * s.n : 0;
    const int grid = std::min(base.num_units, s.sm_limit ? std::min<int>((int)s.sm_limit, ctx->sm_count) : ctx->sm_count);
    const uint32_t ranks = s.ranks, rank = s.rank;
    if (kEpi == kEpiScatter) {
        base.rows_per_rank = (int)(s.m / s.ranks);
        base.my_rank = (int)s.rank;
        base.m_rotate = (int)(((s.rank + 1) % s.ranks) * (s.m / s.ranks) / BM);
    }
    const uint64_t M = s.m, K = s.k;
    return [=](cudaStream_t st, void **b) {
        CUtensorMap ma, mb;
        if (!make_map(&ma, dt, kEB, b[0], M, K, 128 / kEB, BM)) return cudaErrorInvalidValue;
        const bool okb = kBmn ? make_map(&mb, dt, kEB, b[1], K, brows, 128 / kEB, 128 / kEB)
                              : make_map(&mb, dt, kEB, b[1], brows, K, 128 / kEB, BN);
        if (!okb) return cudaErrorInvalidValue;
        GemmArgs a = base;
        int idx = 2;
        a.row_scale = kRowScale ? static_cast<const float *>(b[idx++]) : nullptr;
        a.residual = kEpi == kEpiResidual ? b[idx++] : nullptr;
        a.out = b[idx];
        PeerSet flags{};
        if constexpr (kEpi == kEpiScatter) {
            PeerSet recv{};
            if (!find_peers(ctx, b[idx], ranks, recv) || !find_peers(ctx, b[idx + 1], ranks, flags)) return cudaErrorInvalidResourceHandle;
            for (uint32_t q = 0; q < kMaxPeerRanks; ++q) a.scatter[q] = recv.p[q];
        }
        kernel<<<grid, kThreads, kSmemBytes, st>>>(ma, mb, a);
        cudaError_t e = cudaGetLastError();
        if constexpr (kEpi == kEpiScatter)  // phase 0: this rank's partial rows are in their owners' buffers
            if (e == cudaSuccess) e = launch_peer_signal(st, flags, ranks, rank, 0);
        return e;
    };
}

// Device workspace owned by a compiled kernel, released with it.
struct Workspace {
    void *ptr = nullptr;
    int device = 0;
    ~Workspace() {
        if (ptr) {
            cudaSetDevice(device);
            cudaFree(ptr);
        }
    }
};

// out = sum over s of part[s] (in split order, FP32), rounded once to TOut.
template <typename TOut>
__global__ void splitk_reduce(const float *__restrict__ part, TOut *__restrict__ out, long long n, int ksplit, long long stride, bool vec) {
    const long long step = (long long)gridDim.x * blockDim.x;
    long long i0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {  // n % 4 == 0 and out aligned: 16-byte partial loads
        for (long long i = i0; i < n / 4; i += step) {
            float4 acc = reinterpret_cast<const float4 *>(part)[i];
#pragma unroll 4
            for (int k = 1; k < ksplit; ++k) {
                const float4 v = reinterpret_cast<const float4 *>(part + k * stride)[i];
                acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
            }
            const float r[4] = {acc.x, acc.y, acc.z, acc.w};
            store4<TOut>(out + 4 * i, r, 4, true);
        }
        return;
    }
    for (long long i = i0; i < n; i += step) {
        float acc = part[i];
        for (int k = 1; k < ksplit; ++k) acc += part[k * stride + i];
        out[i] = from_f32<TOut>(acc);
    }
}

// Split-K for GEMMs with at most half as many output tiles as SMs and a long K
// (each tile alone on an SM leaves most SMs idle while it runs its K loop): the
// K-blocks are cut into `ksplit` ranges of at least 32 blocks, every (tile, range)
// unit writes an FP32 partial tile into a workspace owned by the compiled kernel,
// and a second kernel sums the partials in range order (the result is
// deterministic) and rounds once to the output type. Shorter ranges do not pay:
// a unit's fixed cost (pipeline fill, the 128 KB FP32 partial tile it writes, its
// share of the reduction) outweighs its MMAs (1024^3 BF16 with 4 ranges of 4
// blocks: 19.3 us against 17.5 us unsplit; TF32 with 2 ranges of 16 blocks: 1.4%
// slower). 1 = no split. JADE_GEMM_SPLIT_K
// overrides the choice (read when a kernel is compiled).
int splitk_factor(Context *ctx, const Spec &s, int kEB) {
    const int sms = s.sm_limit ? std::min<int>((int)s.sm_limit, ctx->sm_count) : ctx->sm_count;
    const long long tiles = (long long)((s.m + BM - 1) / BM) * (long long)((s.n + BN - 1) / BN);
    const int kblocks = (int)((s.k + (128 / kEB) - 1) / (128 / kEB));
    int ks = 1;
    if (const char *force = std::getenv("JADE_GEMM_SPLIT_K"); force && *force) ks = std::atoi(force);
    else if (tiles * 2 <= sms) ks = (int)std::min<long long>(std::min<long long>(sms / tiles, kblocks / 32), 16);
    ks = std::max(1, std::min(ks, kblocks));
    const int per = (kblocks + ks - 1) / ks;
    return (kblocks + per - 1) / per;  // every range non-empty
}

template <int kEB, uint32_t kFmt, bool kBmn, typename TOut>
LaunchFn splitk_launch(Context *ctx, const Spec &s, int ksplit) {
    LaunchFn gemm = tc_launch<kEB, kFmt, kBmn, float, kEpiNone, false>(ctx, s, ksplit);
    auto ws = std::make_shared<Workspace>();
    ws->device = ctx->device;
    const long long n = (long long)s.m * s.n;
    if (cudaMalloc(&ws->ptr, (size_t)ksplit * n * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        throw IrError("cannot allocate the split-K workspace");
    }
    const int blocks = (int)std::max<long long>(1, std::min<long long>((n / 4 + 255) / 256, 8ll * ctx->sm_count));
    return [=](cudaStream_t st, void **b) {
        void *nb[3] = {b[0], b[1], ws->ptr};
        cudaError_t e = gemm(st, nb);
        if (e != cudaSuccess) return e;
        const bool vec = n % 4 == 0 && reinterpret_cast<uintptr_t>(b[2]) % (4 * sizeof(TOut)) == 0;
        splitk_reduce<TOut><<<blocks, 256, 0, st>>>(static_cast<const float *>(ws->ptr), static_cast<TOut *>(b[2]), n, ksplit, n, vec);
        return cudaGetLastError();
    };
}

template <int kEB, uint32_t kFmt, typename TOut, typename T16>
LaunchFn pick_epilogue(Context *ctx, const Spec &s) {
    if (s.epilogue == "scatter") {
        if constexpr (!std::is_same<TOut, float>::value) return tc_launch<kEB, kFmt, false, TOut, kEpiScatter, false>(ctx, s);
        throw IrError("scatter epilogue needs a 16-bit output");
    }
    if (s.epilogue == "swiglu") {
        if (s.row_scale) return tc_launch<kEB, kFmt, false, TOut, kEpiSwiglu, true>(ctx, s);
        return tc_launch<kEB, kFmt, false, TOut, kEpiSwiglu, false>(ctx, s);
    }
    if (s.epilogue == "residual") {
        if (s.b_nk) {
            if (s.row_scale) return tc_launch<kEB, kFmt, false, TOut, kEpiResidual, true>(ctx, s);
            return tc_launch<kEB, kFmt, false, TOut, kEpiResidual, false>(ctx, s);
        }
        return tc_launch<kEB, kFmt, true, TOut, kEpiResidual, false>(ctx, s);
    }
    if (!s.row_scale) {
        if (const int ks = splitk_factor(ctx, s, kEB); ks > 1)
            return s.b_nk ? splitk_launch<kEB, kFmt, false, TOut>(ctx, s, ks) : splitk_launch<kEB, kFmt, true, TOut>(ctx, s, ks);
    }
    if (s.b_nk) {
        if (s.row_scale) return tc_launch<kEB, kFmt, false, TOut, kEpiNone, true>(ctx, s);
        return tc_launch<kEB, kFmt, false, TOut, kEpiNone, false>(ctx, s);
    }
    if (s.row_scale) return tc_launch<kEB, kFmt, true, TOut, kEpiNone, true>(ctx, s);
    return tc_launch<kEB, kFmt, true, TOut, kEpiNone, false>(ctx, s);
}

// FP32 [rows, cols] -> [cols, rows] through 32x32 shared-memory tiles.
// out[c][r] = in[r][c] for a rows x cols FP32 matrix, through 32 x 33 shared
// tiles. Row blocks are grid-strided, so any row count fits the 65535 limit of
// gridDim.y (launch with transpose_grid).
__global__ void transpose_f32(const float *__restrict__ in, float *__restrict__ out, int rows, int cols) {
    __shared__ float tile[32][33];
    const int c0 = blockIdx.x * 32;
    for (int r0 = blockIdx.y * 32; r0 < rows; r0 += gridDim.y * 32) {
        for (int i = threadIdx.y; i < 32; i += blockDim.y) {
            const int r = r0 + i, c = c0 + threadIdx.x;
            if (r < rows && c < cols) tile[i][threadIdx.x] = in[(size_t)r * cols + c];
        }
        __syncthreads();
        for (int i = threadIdx.y; i < 32; i += blockDim.y) {
            const int c = c0 + i, r = r0 + threadIdx.x;
            if (r < rows && c < cols) out[(size_t)c * rows + r] = tile[threadIdx.x][i];
        }
        __syncthreads();
    }
}
inline dim3 transpose_grid(int rows, int cols) { return dim3((cols + 31) / 32, std::min((rows + 31) / 32, 65535)); }

}  // namespace

bool gemm_tc_supports(const Spec &s, std::string &why) {
    const uint64_t eb = dtype_size(s.dtype);
    if (s.op != Op::Gemm || s.dtype == DType::F32) { why = "not a tensor-core dtype"; return false; }
    if ((s.k * eb) % 16) { why = "TMA needs K * element size to be a multiple of 16 bytes"; return false; }
    if (!s.b_nk && (s.n * eb) % 16) { why = "TMA needs N * element size to be a multiple of 16 bytes for B [K,N]"; return false; }
    if (!encoder()) { why = "cuTensorMapEncodeTiled unavailable"; return false; }
    return true;
}

LaunchFn make_gemm_tc(Context *ctx, const Spec &s, std::string &impl) {
    std::string why;
    if (!gemm_tc_supports(s, why)) throw IrError(why);
    impl = std::string("gemm_tcgen05_128x256_") + dtype_name(s.dtype) + (s.b_nk ? "_nk" : "_kn") + "_out_" + dtype_name(s.out_dtype) +
           (s.epilogue != "none" ? "_" + s.epilogue : std::string()) + (s.row_scale ? "_rowscale" : "");
    if (s.epilogue == "none" && !s.row_scale)
        if (const int ks = splitk_factor(ctx, s, (int)dtype_size(s.dtype)); ks > 1) impl += "_splitk" + std::to_string(ks);
    switch (s.dtype) {
        case DType::TF32:
            if (!s.b_nk) {
                // MN-major TF32 operands need the 32-byte-atom swizzle; B [K,N] is
                // instead transposed once per launch into a [N,K] workspace (K-major),
                // a 2*K*N*4-byte pass that is part of every launch.
                Spec t = s;
                t.b_nk = true;
                LaunchFn inner = pick_epilogue<4, 2, float, float>(ctx, t);
                auto ws = std::make_shared<Workspace>();
                ws->device = ctx->device;
                if (cudaMalloc(&ws->ptr, (size_t)s.k * s.n * 4) != cudaSuccess) {
                    cudaGetLastError();
                    throw IrError("cannot allocate the TF32 B-transpose workspace");
                }
                impl += "_transposeB";
                const int K = (int)s.k, N = (int)s.n;
                const bool extra = s.row_scale || s.epilogue == "residual";
                return [=](cudaStream_t st, void **b) {
                    transpose_f32<<<transpose_grid(K, N), dim3(32, 8), 0, st>>>((const float *)b[0 + 1], (float *)ws->ptr, K, N);
                    void *nb[5] = {b[0], ws->ptr, b[2], extra ? b[3] : nullptr, extra ? b[4] : nullptr};
                    return inner(st, nb);
                };
            }
            return pick_epilogue<4, 2, float, float>(ctx, s);
        case DType::BF16:
            if (s.out_dtype == DType::BF16) return pick_epilogue<2, 1, __nv_bfloat16, __nv_bfloat16>(ctx, s);
            return pick_epilogue<2, 1, float, __nv_bfloat16>(ctx, s);
        case DType::F16:
            if (s.out_dtype == DType::F16) return pick_epilogue<2, 0, __half, __half>(ctx, s);
            return pick_epilogue<2, 0, float, __half>(ctx, s);
        default: throw IrError("unsupported tensor-core dtype");
    }
}

}  // namespace jade

// ---------------------------------------------------------------------------
// Allocation-free TF32 GEMM with B stored [K,N] (jr_gemm_tf32_kn_noalloc).
//
// The compiled path above transposes B into a workspace that jr_compile obtains
// with cudaMalloc. Callers that must not allocate device memory at call time
// (a plugin running inside a host framework that owns every device allocation
// through its own pool, or a latency-critical loop where cudaMalloc's implicit
// device synchronisation is unacceptable) use this entry point instead: its
// scratch is a fixed, file-scope device array that every GPU loading this
// library holds until process exit.
namespace jade {
namespace {

constexpr size_t kNoAllocScratchFloats = size_t(4) << 20;  // 16 MiB: K*N <= 4,194,304
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];
static __device__ int g_noalloc_error;  // bounded-wait expiry code of the last call

struct NoAllocDevice {
    bool ready = false;
    float *scratch = nullptr;  // device address of g_noalloc_scratch on this device
    int *err = nullptr;        // device address of g_noalloc_error on this device
    int sm_count = 0;
};
std::mutex g_noalloc_mutex;
NoAllocDevice g_noalloc_devices[64];

int noalloc_fail(int code, char *err, size_t cap, const char *msg) {
    if (err && cap) {
        snprintf(err, cap, "%s", msg);
        err[cap - 1] = '\0';
    }
    return code;
}

}  // namespace
}  // namespace jade

extern "C" JR_API int jr_gemm_tf32_kn_noalloc(const float *a, const float *b, float *out, uint32_t m, uint32_t n, uint32_t k,
                                              void *stream, char *err, size_t cap) {
    using namespace jade;
    if (err && cap) err[0] = '\0';
    if (!a || !b || !out) return noalloc_fail(1, err, cap, "null operand pointer");
    if (!m || !n || !k || m > INT_MAX || n > INT_MAX || k > INT_MAX || (uint64_t)m * k > INT_MAX || (uint64_t)m * n > INT_MAX)
        return noalloc_fail(1, err, cap, "dimension must be in 1..=INT_MAX with products within 31-bit indexing");
    if ((uint64_t)k * n > kNoAllocScratchFloats) {
        char msg[160];
        snprintf(msg, sizeof msg, "K*N = %llu exceeds the %llu-element (16 MiB) static scratch of this entry point",
                 (unsigned long long)k * n, (unsigned long long)kNoAllocScratchFloats);
        return noalloc_fail(1, err, cap, msg);
    }
    if (k % 4 || (reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b)) % 16)
        return noalloc_fail(1, err, cap, "TMA needs K to be a multiple of 4 and 16-byte aligned A and B");
    if (reinterpret_cast<uintptr_t>(out) % 16)  // the epilogue stores 16-byte vectors of a row
        return noalloc_fail(1, err, cap, "out must be 16-byte aligned");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return noalloc_fail(2, err, cap, "cudaGetDevice failed");
    auto kernel = gemm_tc_kernel<4, 2, false, float, kEpiNone, false>;
    NoAllocDevice *d = &g_noalloc_devices[dev];
    {
        // One-time set-up for this device (the current device): resolve the device
        // addresses of the static arrays; host code never passes the symbols themselves.
        std::lock_guard<std::mutex> lock(g_noalloc_mutex);
        if (!d->ready) {
            if (cudaGetSymbolAddress(reinterpret_cast<void **>(&d->scratch), g_noalloc_scratch) != cudaSuccess ||
                cudaGetSymbolAddress(reinterpret_cast<void **>(&d->err), g_noalloc_error) != cudaSuccess) {
                cudaGetLastError();
                return noalloc_fail(2, err, cap, "cudaGetSymbolAddress failed for the static scratch");
            }
            if (cudaMemset(d->err, 0, sizeof(int)) != cudaSuccess ||
                cudaDeviceGetAttribute(&d->sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
                cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) != cudaSuccess) {
                cudaGetLastError();
                return noalloc_fail(2, err, cap, "static scratch set-up failed");
            }
            d->ready = true;
        }
    }
    CUtensorMap ma, mb;
    if (!make_map(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a, m, k, 32, BM) ||
        !make_map(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, d->scratch, n, k, 32, BN))
        return noalloc_fail(2, err, cap, "cuTensorMapEncodeTiled failed");
    GemmArgs args{};
    args.out = out;
    args.M = (int)m;
    args.N = (int)n;
    args.K = (int)k;
    args.tiles_m = (int)((m + BM - 1) / BM);
    args.tiles_n = (int)((n + BN - 1) / BN);
    args.num_tiles = args.tiles_m * args.tiles_n;
    args.kblocks = (int)((k + 31) / 32);
    args.ksplit = 1;
    args.kb_per = args.kblocks;
    args.num_units = args.num_tiles;
    args.group_m = 8;
    args.err = d->err;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // B [K,N] -> scratch [N,K]: the whole K*N region is rewritten, nothing needs clearing.
    transpose_f32<<<transpose_grid((int)k, (int)n), dim3(32, 8), 0, st>>>(b, d->scratch, (int)k, (int)n);
    kernel<<<std::min(args.num_tiles, d->sm_count), kThreads, kSmemBytes, st>>>(ma, mb, args);
    cudaError_t status = cudaGetLastError();
    if (status == cudaSuccess) status = cudaStreamSynchronize(st);
    if (status != cudaSuccess) return noalloc_fail(2, err, cap, cudaGetErrorString(status));
    // The error word is read on the caller's stream (no legacy-stream copy, so no
    // implicit synchronisation with other streams of the device).
    int code = 0;
    status = cudaMemcpyAsync(&code, d->err, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (status == cudaSuccess) status = cudaStreamSynchronize(st);
    if (status != cudaSuccess) return noalloc_fail(2, err, cap, "error word read failed");
    if (code) {
        // the word must start at zero for the next call
        if (cudaMemsetAsync(d->err, 0, sizeof(int), st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess)
            return noalloc_fail(2, err, cap, "error word reset failed");
        return noalloc_fail(4, err, cap, "device-side bounded wait expired in the TF32 GEMM");
    }
    return 0;
}
