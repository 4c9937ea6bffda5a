// tsrc_numerics.cuh -- the Tesseract f32 rules and integer-exact helpers on sm_100a.
//
// The reference defines every f32 operation of the hot path as one IEEE binary32 operation with
// round-to-nearest-even and gradual underflow, on DAZ'd inputs, whose result is flushed to a signed
// zero when it is subnormal, with NaN results made canonical (0x7FC00000)
// (jwkim04/tesseract-npu sw/sim/include/tsr_ref.h:47-70, sw/sim/tsr_ref.c:54-104).
// On the GPU: __fadd_rn / __fmul_rn / __fdiv_rn / __frcp_rn compiled with -ftz=false give exactly
// that native operation (no FMA contraction: the library is built with -fmad=false and these
// intrinsics are never fused); the flush is an explicit bit test. Values produced by these
// operations are never subnormal, so DAZ is applied only where outside data enters (activations,
// addends, queries). NaN canonicalisation is applied where a value leaves a kernel: every
// operation on a NaN gives a NaN, so only the payload differs before that point.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "tsrc_exp_tables.h"

namespace tsrc {

constexpr uint32_t kSign = 0x80000000u;
constexpr uint32_t kExp = 0x7F800000u;
constexpr uint32_t kMant = 0x007FFFFFu;
constexpr uint32_t kCanonNaN = 0x7FC00000u;

__device__ __forceinline__ uint32_t fbits(float f) { return __float_as_uint(f); }
__device__ __forceinline__ float ffrom(uint32_t u) { return __uint_as_float(u); }

// Input rule: a zero exponent field reads as a signed zero.
__device__ __forceinline__ float daz(float x) {
    const uint32_t u = fbits(x);
    return (u & kExp) ? x : ffrom(u & kSign);
}
// Result rule, subnormal part: a subnormal result becomes a signed zero.
__device__ __forceinline__ float flush(float r) {
    const uint32_t u = fbits(r);
    return (u & kExp) ? r : ffrom(u & kSign);
}
// Result rule, NaN part.
__device__ __forceinline__ float canon(float r) {
    return ((fbits(r) & ~kSign) > kExp) ? ffrom(kCanonNaN) : r;
}

// Operations on values that are already normal-or-zero (results of these operations, fp16
// scales, int32 conversions).
__device__ __forceinline__ float fadd(float a, float b) { return flush(__fadd_rn(a, b)); }
__device__ __forceinline__ float fsub(float a, float b) { return flush(__fsub_rn(a, b)); }
__device__ __forceinline__ float fmul(float a, float b) { return flush(__fmul_rn(a, b)); }
__device__ __forceinline__ float fdiv(float a, float b) { return flush(__fdiv_rn(a, b)); }
__device__ __forceinline__ float frecip(float a) { return flush(__frcp_rn(a)); }
__device__ __forceinline__ float i2f(int32_t v) { return __int2float_rn(v); }
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// two signed 16-bit values of a times unsigned bytes 0,1 (lo) or 2,3 (hi) of b, plus c
__device__ __forceinline__ int32_t dp2a_lo(uint32_t a, uint32_t b, int32_t c) {
    int32_t d;
    asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int32_t dp2a_hi(uint32_t a, uint32_t b, int32_t c) {
    int32_t d;
    asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// QACT's f32 -> int8 conversion (sw/sim/tsr_ref.c:202-229): NaN -> 0, the rounded value
// saturated to [-128, 127]; half_even: ties to even (A256), else ties away from zero (A32).
__device__ __forceinline__ int32_t round_sat8(float v, bool half_even) {
    const uint32_t u = fbits(v), a = u & ~kSign;
    if (a > kExp) return 0;
    const bool neg = (u >> 31) != 0;
    if (a >= 0x43800000u) return neg ? -128 : 127;       // |v| >= 256 (or Inf)
    if (a < 0x3F000000u) return 0;                        // |v| < 0.5
    const uint32_t sig = 0x00800000u | (a & kMant);
    const uint32_t sh = 150u - (a >> 23);                 // 16 .. 24
    const uint32_t rem = sig & ((1u << sh) - 1u), half = 1u << (sh - 1u);
    int32_t ip = (int32_t)(sig >> sh);
    if (half_even ? (rem > half || (rem == half && (ip & 1))) : (rem >= half)) ip += 1;
    if (neg) ip = -ip;
    return ip < -128 ? -128 : (ip > 127 ? 127 : ip);
}

// The same conversions on the hardware's float-to-integer instructions (a NaN converts to 0 and an
// out-of-range value saturates): half-even is one round-to-nearest-even conversion; half-away is a
// truncation plus one step away from zero when the exact remainder is at least one half.
__device__ __forceinline__ int32_t round_even_sat8(float v) {
    int32_t r;
    asm("cvt.rni.s32.f32 %0, %1;" : "=r"(r) : "f"(v));
    return max(-128, min(127, r));
}
__device__ __forceinline__ int32_t round_away_sat8(float v) {
    int32_t r;
    asm("cvt.rzi.s32.f32 %0, %1;" : "=r"(r) : "f"(v));
    r = max(-1024, min(1024, r));
    const float f = __fsub_rn(v, __int2float_rn(r));      // the exact remainder for |v| < 2^24; NaN stays NaN
    r += (fabsf(f) >= 0.5f) ? (v < 0.0f ? -1 : 1) : 0;
    return max(-128, min(127, r));
}

// The amax key of QACT: |DAZ(x)| as bits for a non-NaN x (comparable as unsigned), 0 for NaN
// (a NaN does not take part; 0 never wins a strict > against a real candidate).
__device__ __forceinline__ uint32_t amax_key(float x) {
    const uint32_t a = fbits(daz(x)) & ~kSign;
    return a <= kExp ? a : 0u;
}

// ---- EXPK (VU §6.3; sw/sim/tsr_ref_math.c:78-161): an integer algorithm, exact on any device ----
// tabs: the constants (any memory space; the caller stages them where divergent indexing is cheap).
// Straight-line form: the special cases (NaN, zero, saturation) are chosen by selects after the
// main path instead of early returns, so that a thread's independent evaluations interleave (the
// same results as the early-return form for every f32 input and every kappa, checked over all
// 2^32 bit patterns on the GPU).
__device__ __forceinline__ float expk(float v, unsigned kappa, const uint32_t* __restrict__ t64,
                                      const uint64_t* __restrict__ lk) {
    uint32_t u = fbits(v);
    u = (u & kExp) ? u : (u & kSign);
    const uint32_t a = u & ~kSign;
    const bool neg = ((u >> 31) ^ (kappa != 0u)) != 0;
    const uint32_t ev = a >> 23;
    const uint32_t sh = 156u - (ev > 156u ? 156u : ev);
    const uint64_t prod = (uint64_t)(0x00800000u | (a & kMant)) * lk[kappa];
    const uint64_t t = sh >= 64u ? 0ull : (prod >> sh);
    const bool sat = ev > 156u || t >= (1ull << 40);       // also every infinite input
    const uint64_t tc = t & ((1ull << 40) - 1u);             // t itself whenever the result is used
    int32_t n = neg ? -(int32_t)((tc + 0xFFFFFFFFull) >> 32) : (int32_t)(tc >> 32);
    const uint32_t frac = neg ? 0u - (uint32_t)tc : (uint32_t)tc;
    const uint32_t j = frac >> 26;
    const uint64_t g = frac & 0x03FFFFFFu;
    const uint64_t s2 = TSRC_EXPK_P2F + ((g * TSRC_EXPK_P3F) >> 32);
    const uint64_t s1 = TSRC_EXPK_P1F + ((g * s2) >> 32);
    const uint64_t pf = (g * s1) >> 32;
    const uint64_t tj = t64[j];
    const uint64_t m = tj + ((tj * pf) >> 32);
    const bool hi = m >= (1ull << 31);
    const uint32_t drop = hi ? 8u : 7u;
    n += hi ? 1 : 0;
    uint64_t sig = m >> drop;
    const uint64_t rem = m & ((1ull << drop) - 1u), half = 1ull << (drop - 1u);
    sig += (rem > half || (rem == half && (sig & 1u))) ? 1u : 0u;
    const bool carry = sig == (1ull << 24);
    sig = carry ? (1ull << 23) : sig;
    n += carry ? 1 : 0;
    const int32_t be = n + 127;
    float r = ffrom(((uint32_t)be << 23) | (uint32_t)(sig & kMant));
    r = be >= 255 ? ffrom(kExp) : r;
    r = be <= 0 ? 0.0f : r;
    r = sat ? (neg ? 0.0f : ffrom(kExp)) : r;
    r = a == 0u ? 1.0f : r;
    r = a > kExp ? ffrom(kCanonNaN) : r;
    return r;
}

// TANH (VU §6.5; sw/sim/tsr_ref_math.c:206-229) on top of EXPK(., N2).
__device__ __forceinline__ float tanh_vu(float x, const uint32_t* __restrict__ t64, const uint64_t* __restrict__ lk) {
    const uint32_t u = fbits(x);
    if ((u & ~kSign) > kExp) return ffrom(kCanonNaN);
    const float ax = ffrom(fbits(daz(x)) & ~kSign);
    float t;
    if (fbits(ax) < 0x3C800000u) {
        const float w = fsub(3.0f, fmul(ax, ax));
        t = fmul(fmul(w, ax), ffrom(0x3EAAAAABu));
    } else {
        const float e = expk(ax, 2u, t64, lk);
        t = fmul(fsub(1.0f, e), frecip(fadd(1.0f, e)));
    }
    return (u & kSign) ? ffrom(fbits(t) ^ kSign) : t;
}

// Device-global copies of the EXPK constants (one per translation unit; 288 bytes).
static __device__ const uint32_t g_expk_t64[64] = TSRC_EXPK_T64_INIT;
static __device__ const uint64_t g_expk_lk[4] = TSRC_EXPK_LK_INIT;

}  // namespace tsrc
