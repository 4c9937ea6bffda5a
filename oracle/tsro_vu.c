// tsro_vu.c — CPU restatement of the decoder layer's vector kinds (TEST INFRASTRUCTURE ONLY; see
// tsro.h). RMS_NORM + MUL, ROPE (recurrence form), the VOPs ADD / MUL / SILU / SWIGLU, SIN / COS
// and the dequantization of a ggml row, each following the reference's vector-unit definition
// (jwkim04/tesseract-npu sw/sim/tsr_ref_vu.c, tsr_ref_math.c, tsr_ref.c) in plain C11.
#include <math.h>
#include <string.h>

#include "tsro.h"

#define SIGN_BIT 0x80000000u
#define EXP_MASK 0x7F800000u
#define MANT_MASK 0x007FFFFFu
#define CANON_NAN 0x7FC00000u

static inline uint32_t bits_of(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float float_of(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline float daz(float x) { const uint32_t u = bits_of(x); return (u & EXP_MASK) ? x : float_of(u & SIGN_BIT); }
static inline float neg(float x) { return float_of(bits_of(x) ^ SIGN_BIT); }

#define FA tsro_fadd
#define FS tsro_fsub
#define FM tsro_fmul
#define RC tsro_frecip

// SQ (tsr_ref.c:54-71 rules around the IEEE square root)
float tsro_fsqrt(float a) {
    const float r = sqrtf(daz(a));
    const uint32_t u = bits_of(r), e = u & EXP_MASK;
    if (e == EXP_MASK) return (u & MANT_MASK) ? float_of(CANON_NAN) : r;
    if (e == 0) return float_of(u & SIGN_BIT);
    return r;
}

// RED.SUMSQ post RMS (tsr_ref_vu.c:171-263): 128 partials in element order, the 7-level pairwise
// tree, RC(SQ(FA(FM(y, inv_n), eps))); then VOP.MULCB FM(FM(x, s), w) (rmsnorm_ref.cpp:59-78).
void tsro_rms_norm(const float * x, float * y, const float * w, uint32_t n, uint32_t rows, float eps, float inv_n) {
    for (uint32_t r = 0; r < rows; ++r) {
        const float * xr = x + (size_t)r * n;
        float * yr = y + (size_t)r * n;
        float p[128];
        for (int i = 0; i < 128; ++i) p[i] = 0.0f;
        for (uint32_t i = 0; i < n; ++i) p[i % 128u] = FA(p[i % 128u], FM(xr[i], xr[i]));
        for (uint32_t m = 128; m > 1u; m >>= 1)
            for (uint32_t k = 0; k < m / 2u; ++k) p[k] = FA(p[2u * k], p[2u * k + 1u]);
        const float s = RC(tsro_fsqrt(FA(FM(p[0], inv_n), eps)));
        for (uint32_t j = 0; j < n; ++j) yr[j] = w ? FM(FM(xr[j], s), w[j]) : FM(xr[j], s);
    }
}

// ---- SIN / COS (tsr_ref_math.c:336-412) ------------------------------------------------------
typedef unsigned __int128 u128;

static float r_to_f32(u128 R, int negative) {             // nearest-even f32 of R * 2^-124
    int b = 127;
    while (!((R >> b) & 1u)) --b;
    const unsigned shift = (unsigned)(b - 23);
    uint64_t sig = (uint64_t)(R >> shift);
    const int guard = (int)((R >> (shift - 1u)) & 1u);
    const int sticky = (R & (((u128)1 << (shift - 1u)) - 1u)) != 0;
    uint32_t be = (uint32_t)(b + 3);
    if (guard && (sticky || (sig & 1u))) {
        sig += 1u;
        if (sig == (1ull << 24)) {
            sig >>= 1;
            be += 1u;
        }
    }
    return float_of((negative ? SIGN_BIT : 0u) | (be << 23) | ((uint32_t)sig & MANT_MASK));
}

void tsro_sincos(float t, float * s_out, float * c_out) {
    const uint32_t u = bits_of(daz(t)), a = u & ~SIGN_BIT;
    if (a >= EXP_MASK) {
        *s_out = float_of(CANON_NAN);
        *c_out = float_of(CANON_NAN);
        return;
    }
    const uint32_t E = a >> 23;
    if (E < 115u) {                                        // |t| < 2^-12
        *s_out = float_of(u);
        *c_out = 1.0f;
        return;
    }
    const uint64_t M = 0x00800000u | (a & MANT_MASK);
    const u128 P = (u128)M * 0xA2F9836E4E44152Aull;        // t * 2/pi, scaled
    const int sh = 214 - (int)E;
    const uint64_t mask62 = (1ull << 62) - 1u;
    uint32_t k4;
    uint64_t F;
    if (sh >= 62) {
        k4 = (uint32_t)((sh >= 128 ? (u128)0 : P >> sh) & 3u);
        F = (uint64_t)(P >> (sh - 62)) & mask62;
    } else if (sh >= 0) {
        k4 = (uint32_t)((P >> sh) & 3u);
        F = (uint64_t)(P << (62 - sh)) & mask62;
    } else {
        k4 = (uint32_t)((P << (-sh)) & 3u);
        F = 0;
    }
    int rneg = 0;
    uint64_t Fm = F;
    if (F >= (1ull << 61)) {
        k4 = (k4 + 1u) & 3u;
        rneg = 1;
        Fm = (1ull << 62) - F;
    }
    const float r = Fm == 0 ? 0.0f : r_to_f32((u128)Fm * 0x6487ED5110B4611Aull, rneg);
    const float z = FM(r, r);
    float p = FM(float_of(0xB94CA1F9u), z);               // Cephes sinf coefficients
    p = FA(p, float_of(0x3C08839Eu));
    p = FM(p, z);
    p = FA(p, float_of(0xBE2AAAA3u));
    p = FM(p, z);
    p = FM(p, r);
    const float sn = FA(p, r);
    p = FM(float_of(0x37CCF5CEu), z);                     // Cephes cosf coefficients
    p = FA(p, float_of(0xBAB6061Au));
    p = FM(p, z);
    p = FA(p, float_of(0x3D2AAAA5u));
    p = FM(p, z);
    p = FM(p, z);
    const float cs = FA(FS(p, FM(0.5f, z)), 1.0f);
    float S, C;
    switch (k4) {
        case 0: S = sn; C = cs; break;
        case 1: S = cs; C = neg(sn); break;
        case 2: S = neg(sn); C = neg(cs); break;
        default: S = neg(cs); C = sn; break;
    }
    *s_out = (u & SIGN_BIT) ? neg(S) : S;
    *c_out = C;
}

// ROPE recurrence form (tsr_ref_vu.c:308-376) on T tokens of n_heads * hd values.
void tsro_rope(const float * x, float * y, const int32_t * pos, uint32_t T, uint32_t n_heads, uint32_t hd, uint32_t nd,
               uint32_t mode, float ts, float m) {
    const uint32_t half = nd / 2u;
    float c[512], s[512];
    for (uint32_t t = 0; t < T; ++t) {
        float theta = tsro_i32_to_f32(pos[t]);
        for (uint32_t i = 0; i < half; ++i) {
            float sn, cs;
            tsro_sincos(theta, &sn, &cs);
            c[i] = FM(m, cs);
            s[i] = FM(m, sn);
            theta = FM(theta, ts);
        }
        const float * xt = x + (size_t)t * n_heads * hd;
        float * yt = y + (size_t)t * n_heads * hd;
        for (uint32_t h = 0; h < n_heads; ++h) {
            for (uint32_t i = 0; i < half; ++i) {
                const uint32_t j0 = h * hd + (mode ? i : 2u * i), j1 = h * hd + (mode ? i + half : 2u * i + 1u);
                const float x0 = xt[j0], x1 = xt[j1];
                yt[j0] = FS(FM(x0, c[i]), FM(x1, s[i]));
                yt[j1] = FA(FM(x0, s[i]), FM(x1, c[i]));
            }
            for (uint32_t j = nd; j < hd; ++j) yt[h * hd + j] = xt[h * hd + j];
        }
    }
}

// VOP functions (tsr_ref_vu.c:104-130; SIG / SILU tsr_ref_math.c:165-171)
static float silu(float a) { return FM(a, RC(FA(1.0f, tsro_expk(a, 1u)))); }

void tsro_vop(uint32_t func, const float * a, const float * b, float * y, size_t n) {
    for (size_t j = 0; j < n; ++j) {
        switch (func) {
            case 0u: y[j] = FA(a[j], b[j]); break;
            case 2u: y[j] = FM(a[j], b[j]); break;
            case 6u: y[j] = silu(a[j]); break;
            default: y[j] = FM(silu(a[j]), b[j]); break;
        }
    }
}

// Dequantization of one ggml row (tsr_dequant_row, tsr_ref.c:369-401).
void tsro_dequant_row(uint32_t fmt, const uint8_t * row, uint32_t K, float * y) {
    if (fmt == TSRO_FMT_Q8_0) {
        for (uint32_t b = 0; b < K / 32u; ++b) {
            const uint8_t * blk = row + 34u * b;
            const float d = tsro_fp16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
            for (uint32_t l = 0; l < 32u; ++l) y[32u * b + l] = FM(d, tsro_i32_to_f32((int8_t)blk[2 + l]));
        }
        return;
    }
    for (uint32_t b = 0; b < K / 256u; ++b) {
        const uint8_t * blk = row + 144u * b;
        const float d = tsro_fp16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        const float dmin = tsro_fp16_to_f32((uint16_t)(blk[2] | (blk[3] << 8)));
        const uint8_t * sc12 = blk + 4, * qs = blk + 16;
        for (int j = 0; j < 8; ++j) {
            int sc, mn;
            if (j < 4) {
                sc = sc12[j] & 63;
                mn = sc12[j + 4] & 63;
            } else {
                sc = (sc12[j + 4] & 0x0F) | ((sc12[j - 4] >> 6) << 4);
                mn = (sc12[j + 4] >> 4) | ((sc12[j] >> 6) << 4);
            }
            const float d1 = FM(d, tsro_i32_to_f32(sc)), m1 = FM(dmin, tsro_i32_to_f32(mn));
            for (int l = 0; l < 32; ++l) {
                const int qv = (qs[32 * (j / 2) + l] >> (4 * (j % 2))) & 0xF;
                y[256u * b + 32u * (uint32_t)j + (uint32_t)l] = FS(FM(d1, tsro_i32_to_f32(qv)), m1);
            }
        }
    }
}
