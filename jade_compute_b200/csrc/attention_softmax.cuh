// Softmax arithmetic shared by the tcgen05 attention kernels: packed FP32x2
// arithmetic, 3-input maxima, MUFU exp2, a cubic-polynomial exp2 on the FMA pipe
// (to take part of the exponentials off the MUFU unit), and the P = exp2(S*c - m)
// row writer that stores 16-bit P pairs into TMEM for the P.V MMA.
#pragma once
#include "common.cuh"

namespace jade {

// exponentials per 16-element group evaluated by the polynomial (unmasked tiles)
constexpr int kPolyPairs = 1;

__device__ __forceinline__ uint64_t pack2f(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void unpack2f(uint64_t v, float &a, float &b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v)); }
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}
__device__ __forceinline__ float mufu_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
template <uint32_t kFmt>
__device__ __forceinline__ uint32_t pack16(float lo, float hi) {
    return kFmt == 1 ? pack_bf16(lo, hi) : pack_f16(lo, hi);
}
// 2^x for two finite x on the FMA pipe: x = n + f with n = round(x), |f| <= 1/2,
// 2^f by a cubic (relative-error least-squares fit on [-1/2, 1/2], max relative
// error 7.5e-5, below the 16-bit rounding of P), 2^n added to the exponent field.
// x is clamped to -125 so the exponent stays in the normal range (results below
// 2^-125 are returned as about 2^-125 instead of smaller values).
__device__ __forceinline__ uint64_t poly_exp2_pair(uint64_t x) {
    float x0, x1;
    unpack2f(x, x0, x1);
    const uint64_t xc = pack2f(fmaxf(x0, -125.0f), fmaxf(x1, -125.0f));
    const uint64_t shifter = pack2f(12582912.0f, 12582912.0f);  // 1.5 * 2^23: adding it rounds to an integer
    const uint64_t t = add2(xc, shifter);
    const uint64_t f = sub2(xc, sub2(t, shifter));
    uint64_t p = fma2(pack2f(0.055171635f, 0.055171635f), f, pack2f(0.24261113f, 0.24261113f));
    p = fma2(p, f, pack2f(0.69326097f, 0.69326097f));
    p = fma2(p, f, pack2f(0.99992806f, 0.99992806f));
    float t0, t1, p0, p1;
    unpack2f(t, t0, t1);
    unpack2f(p, p0, p1);
    // the low mantissa bits of t hold n (two's complement); shifting by 23 moves n
    // into the exponent field and drops the shifter's own bits
    const float r0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
    const float r1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
    return pack2f(r0, r1);
}

// Makes the compiler treat v as written here: uses of registers filled by an
// asynchronous tcgen05.ld stay behind the tcgen05.wait::ld that precedes this.
template <int N>
__device__ __forceinline__ void reg_fence(float (&v)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) asm volatile("" : "+f"(v[i]));
}
// P = exp2(s * c - m) for a row of scores, written as 16-bit pairs to TMEM
// columns [ts, ts + kCols/2) eight at a time; returns the row sum.
// kPoly: evaluate kPolyN of every 8 pairs with the FMA-pipe polynomial.
template <uint32_t kFmt, bool kPoly, int kCols, int kPolyN = kPolyPairs>
__device__ __forceinline__ float store_p(const float (&sv)[kCols], float c, float m, uint32_t ts) {
    const uint64_t c2 = pack2f(c, c), nm2 = pack2f(-m, -m);
    uint64_t acc[2] = {pack2f(0.0f, 0.0f), pack2f(0.0f, 0.0f)};
#pragma unroll
    for (int g = 0; g < kCols / 16; ++g) {
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint64_t xv = fma2(pack2f(sv[16 * g + 2 * i], sv[16 * g + 2 * i + 1]), c2, nm2);
            uint64_t p;
            if (kPoly && i < kPolyN) {
                p = poly_exp2_pair(xv);
            } else {
                float x0, x1;
                unpack2f(xv, x0, x1);
                p = pack2f(mufu_exp2(x0), mufu_exp2(x1));
            }
            acc[i & 1] = add2(acc[i & 1], p);
            float p0, p1;
            unpack2f(p, p0, p1);
            pk[i] = pack16<kFmt>(p0, p1);
        }
        tmem_st8(ts + g * 8, pk);
    }
    float a0, a1, b0, b1;
    unpack2f(acc[0], a0, a1);
    unpack2f(acc[1], b0, b1);
    return (a0 + a1) + (b0 + b1);
}


}  // namespace jade
