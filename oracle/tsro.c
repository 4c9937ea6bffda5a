// tsro.c — CPU restatement of the matvec numerics (TEST INFRASTRUCTURE ONLY; see tsro.h).
//
// Every function names the reference definition it restates (jwkim04/tesseract-npu, paths inside
// that project). Built with -ffp-contract=off -fno-fast-math: each f32 expression below is one
// IEEE binary32 operation in the default environment (round to nearest even, gradual underflow),
// which the helpers then post-process with explicit bit tests, exactly as the reference states its
// rules.
#include "tsro.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#if defined(__FAST_MATH__)
#error "tsro.c must not be compiled with -ffast-math"
#endif

#define SIGN_BIT 0x80000000u
#define EXP_MASK 0x7F800000u
#define MANT_MASK 0x007FFFFFu
#define CANON_NAN 0x7FC00000u

static inline uint32_t bits_of(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float float_of(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

// Input rule (tsr_ref.h:47-49): an encoding with a zero exponent field is read as a signed zero.
static inline float in_rule(float x) {
    const uint32_t u = bits_of(x);
    return (u & EXP_MASK) ? x : float_of(u & SIGN_BIT);
}
// Result rule (tsr_ref.h:49-57, tsr_ref.c:58-71): the native RNE result with gradual underflow is
// kept unless it is subnormal (-> signed zero) or a NaN (-> 0x7FC00000).
static inline float out_rule(float r) {
    const uint32_t u = bits_of(r);
    const uint32_t e = u & EXP_MASK;
    if (e == EXP_MASK) return (u & MANT_MASK) ? float_of(CANON_NAN) : r;
    if (e == 0) return float_of(u & SIGN_BIT);
    return r;
}

float tsro_fadd(float a, float b) { return out_rule(in_rule(a) + in_rule(b)); }
float tsro_fsub(float a, float b) { return out_rule(in_rule(a) - in_rule(b)); }
float tsro_fmul(float a, float b) { return out_rule(in_rule(a) * in_rule(b)); }
float tsro_fdiv(float a, float b) { return out_rule(in_rule(a) / in_rule(b)); }
float tsro_frecip(float a) { return out_rule(1.0f / in_rule(a)); }

// int32 -> f32 with round to nearest even (tsr_ref.c:107-132). The C conversion rounds with the
// current mode, which is the default RNE here.
float tsro_i32_to_f32(int32_t v) { return (float)v; }

// fp16 -> f32, exact (tsr_ref.c:136-158): a NaN keeps sign and payload with the quiet bit set.
float tsro_fp16_to_f32(uint16_t h) {
    const uint32_t s = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    if (e == 0x1Fu) return float_of(s | EXP_MASK | (m ? (0x00400000u | (m << 13)) : 0u));
    if (e != 0) return float_of(s | ((e + 112u) << 23) | (m << 13));
    // zero or subnormal: m * 2^-24 is exact in f32
    const float mag = (float)m * 0x1p-24f;
    return float_of(s | bits_of(mag));
}

// f32 -> fp16 with RNE, overflow to Inf, NaN -> sign | 0x7E00 (tsr_ref.c:162-198).
uint16_t tsro_f32_to_fp16(float f) {
    const uint32_t u = bits_of(f);
    const uint16_t s = (uint16_t)((u >> 16) & 0x8000u);
    const uint32_t a = u & ~SIGN_BIT;
    if (a > EXP_MASK) return (uint16_t)(s | 0x7E00u);
    if (a == EXP_MASK) return (uint16_t)(s | 0x7C00u);
    const int e = (int)(a >> 23) - 127;
    if ((a >> 23) == 0 || e < -25) return s;
    if (e > 15) return (uint16_t)(s | 0x7C00u);
    const uint32_t sig = 0x00800000u | (a & MANT_MASK);
    // keep `keep` significant bits: normal fp16 has 11, a subnormal fewer
    const uint32_t drop = (e >= -14) ? 13u : (uint32_t)(13 + (-14 - e));
    uint32_t q = sig >> drop;
    const uint32_t rem = sig & ((1u << drop) - 1u), half = 1u << (drop - 1u);
    if (rem > half || (rem == half && (q & 1u))) q += 1u;
    uint32_t out;
    if (e >= -14) out = ((uint32_t)(e + 15) << 10) + (q - 0x400u);   // q in [2^10, 2^11]: carry is fine
    else out = q;                                                        // subnormal units of 2^-24
    return (uint16_t)(s | out);
}

// 16 partials reduced pairwise by levels (tsr_ref.c:592-598).
float tsro_tree16(const float p[16]) {
    float v[16];
    memcpy(v, p, sizeof v);
    for (int n = 16; n > 1; n /= 2)
        for (int k = 0; k < n / 2; ++k) v[k] = tsro_fadd(v[2 * k], v[2 * k + 1]);
    return v[0];
}

// ---------------------------------------------------------------------------------------------
// EXPK (tsr_ref_math.c:78-161, VU design doc §6.3 and Appendix A). The constants are derived here
// from their defining formulas (long double), not tabulated: LK = round(|K|·log2(e)·2^38) (LK(N2) =
// 2·LK(P1) by definition), P1F/P2F/P3F = round(ln2^i/i!·2^32), T64[j] = round(2^(j/64)·2^30).
// ---------------------------------------------------------------------------------------------
static uint64_t g_lk[4];
static uint64_t g_pf[3];
static uint32_t g_t64[64];
static pthread_once_t g_tables_once = PTHREAD_ONCE_INIT;

static uint64_t round_ld(long double v) { return (uint64_t)llroundl(v); }

static void tables_init(void) {
    const long double ln2 = logl(2.0L), log2e = 1.0L / ln2;
    const long double two38 = ldexpl(1.0L, 38), two32 = ldexpl(1.0L, 32);
    const long double c2g = 2.0L * sqrtl(2.0L / acosl(-1.0L)) * 0.044715L;
    g_lk[0] = round_ld(log2e * two38);
    g_lk[1] = g_lk[0];
    g_lk[2] = 2u * g_lk[0];
    g_lk[3] = round_ld(c2g * log2e * two38);
    g_pf[0] = round_ld(ln2 * two32);
    g_pf[1] = round_ld(ln2 * ln2 / 2.0L * two32);
    g_pf[2] = round_ld(ln2 * ln2 * ln2 / 6.0L * two32);
    for (int j = 0; j < 64; ++j) g_t64[j] = (uint32_t)round_ld(exp2l((long double)j / 64.0L) * ldexpl(1.0L, 30));
}

float tsro_expk(float v, unsigned kappa) {
    pthread_once(&g_tables_once, tables_init);
    if (kappa > 3u) return float_of(CANON_NAN);
    uint32_t u = bits_of(v);
    if ((u & EXP_MASK) == 0) u &= SIGN_BIT;                     // DAZ
    if ((u & ~SIGN_BIT) > EXP_MASK) return float_of(CANON_NAN);
    const int neg = (int)((u >> 31) ^ (kappa != 0u));           // sign of K·v (K < 0 unless P1)
    const uint32_t a = u & ~SIGN_BIT;
    if (a == EXP_MASK) return float_of(neg ? 0u : EXP_MASK);
    if (a == 0) return 1.0f;
    const uint32_t ev = a >> 23;
    if (ev > 156u) return float_of(neg ? 0u : EXP_MASK);
    // |K·v·log2 e| in units of 2^-32
    const uint64_t prod = (uint64_t)(0x00800000u | (a & MANT_MASK)) * g_lk[kappa];
    const uint32_t sh = 156u - ev;
    const uint64_t t = sh >= 64u ? 0u : prod >> sh;
    if (t >= (1ull << 40)) return float_of(neg ? 0u : EXP_MASK);
    int32_t n;
    uint32_t frac;
    if (neg) { n = -(int32_t)((t + 0xFFFFFFFFull) >> 32); frac = (uint32_t)(0u - (uint32_t)t); }
    else     { n = (int32_t)(t >> 32);                    frac = (uint32_t)t; }
    const uint32_t j = frac >> 26;
    const uint64_t g = frac & 0x03FFFFFFu;
    // 2^(g·2^-32) - 1 by a Horner scheme on truncated fixed-point products
    const uint64_t s2 = g_pf[1] + ((g * g_pf[2]) >> 32);
    const uint64_t s1 = g_pf[0] + ((g * s2) >> 32);
    const uint64_t pf = (g * s1) >> 32;
    const uint64_t m = (uint64_t)g_t64[j] + (((uint64_t)g_t64[j] * pf) >> 32);   // Q1.30
    uint32_t drop = 7u;
    if (m >= (1ull << 31)) { drop = 8u; n += 1; }
    uint64_t sig = m >> drop;
    const uint64_t rem = m & ((1ull << drop) - 1u), half = 1ull << (drop - 1u);
    if (rem > half || (rem == half && (sig & 1u))) sig += 1u;
    if (sig == (1ull << 24)) { sig = 1ull << 23; n += 1; }
    const int32_t be = n + 127;
    if (be >= 255) return float_of(EXP_MASK);
    if (be <= 0) return 0.0f;
    return float_of(((uint32_t)be << 23) | (uint32_t)(sig & MANT_MASK));
}

float tsro_exp(float x) { return tsro_expk(x, 0u); }

// TANH (tsr_ref_math.c:206-229, VU §6.5).
float tsro_tanh(float x) {
    const uint32_t u = bits_of(x);
    if ((u & ~SIGN_BIT) > EXP_MASK) return float_of(CANON_NAN);
    const float ax = float_of(bits_of(in_rule(x)) & ~SIGN_BIT);
    float t;
    if (bits_of(ax) < 0x3C800000u) {            // |x| < 2^-6: x·(3 - x^2)·f32(1/3)
        const float w = tsro_fsub(3.0f, tsro_fmul(ax, ax));
        t = tsro_fmul(tsro_fmul(w, ax), float_of(0x3EAAAAABu));
    } else {
        const float e = tsro_expk(ax, 2u);      // exp(-2|x|)
        t = tsro_fmul(tsro_fsub(1.0f, e), tsro_frecip(tsro_fadd(1.0f, e)));
    }
    return (u & SIGN_BIT) ? float_of(bits_of(t) ^ SIGN_BIT) : t;
}

// ---------------------------------------------------------------------------------------------
// QACT (tsr_ref.c:202-229 rounding, :456-518 the two kinds)
// ---------------------------------------------------------------------------------------------
// NaN -> 0; otherwise the rounded value saturated to [-128, 127].
static int8_t round_sat8(float v, int half_even) {
    if (isnan(v)) return 0;
    const float r = half_even ? nearbyintf(v) : roundf(v);
    if (r <= -128.0f) return -128;
    if (r >= 127.0f) return 127;
    return (int8_t)(int)r;
}

// |DAZ(x)| as bits when x takes part in the amax search (not a NaN), else UINT32_MAX.
static inline uint32_t amax_key(float x) {
    const uint32_t a = bits_of(in_rule(x)) & ~SIGN_BIT;
    return a <= EXP_MASK ? a : UINT32_MAX;
}

void tsro_qact_a32(const float * x, uint32_t K, int8_t * q, float * d) {
    for (uint32_t b = 0; b < K / 32u; ++b) {
        const float * xb = x + 32u * b;
        uint32_t amax = 0;
        for (int i = 0; i < 32; ++i) {
            const uint32_t k = amax_key(xb[i]);
            if (k != UINT32_MAX && k > amax) amax = k;
        }
        const float db = tsro_fdiv(float_of(amax), 127.0f);
        const float id = (bits_of(db) & ~SIGN_BIT) ? tsro_frecip(db) : 0.0f;
        for (int i = 0; i < 32; ++i) q[32u * b + i] = round_sat8(tsro_fmul(xb[i], id), 0);
        d[b] = tsro_fp16_to_f32(tsro_f32_to_fp16(db));
    }
}

void tsro_qact_a256(const float * x, uint32_t K, int8_t * q, float * d, int16_t * bs) {
    for (uint32_t b = 0; b < K / 256u; ++b) {
        const float * xb = x + 256u * b;
        int8_t * qb = q + 256u * b;
        uint32_t amax = 0;
        float mx = 0.0f;                          // signed value of the first largest |x|
        for (int i = 0; i < 256; ++i) {
            const uint32_t k = amax_key(xb[i]);
            if (k != UINT32_MAX && k > amax) { amax = k; mx = in_rule(xb[i]); }
        }
        float db = 0.0f;
        if (amax) {
            const float iscale = tsro_fdiv(-127.0f, mx);
            for (int i = 0; i < 256; ++i) qb[i] = round_sat8(tsro_fmul(iscale, xb[i]), 1);
            db = tsro_frecip(iscale);
        } else {
            memset(qb, 0, 256);
        }
        d[b] = db;
        for (int g = 0; g < 16; ++g) {
            int s = 0;
            for (int i = 0; i < 16; ++i) s += qb[16 * g + i];
            bs[16u * b + g] = (int16_t)s;
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Row dot products (tsr_ref.c:526-635)
// ---------------------------------------------------------------------------------------------
static inline uint16_t u16le(const uint8_t * p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// 6-bit scale and min of sub-block j (ggml get_scale_min_k4; tsr_ref.c:359-367).
static inline void q4k_sc_m(int j, const uint8_t * s, int * sc, int * m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

float tsro_dot_q8_0(const uint8_t * row, uint32_t K, const int8_t * q, const float * d, int32_t * isum) {
    float p[16] = { 0 };
    for (uint32_t b = 0; b < K / 32u; ++b) {
        const uint8_t * blk = row + 34u * b;
        const int8_t * qw = (const int8_t *)(blk + 2);
        int32_t s = 0;
        for (int i = 0; i < 32; ++i) s += (int32_t)qw[i] * (int32_t)q[32u * b + i];
        if (isum) isum[b] = s;
        const float t = tsro_fmul(tsro_fmul(tsro_fp16_to_f32(u16le(blk)), d[b]), tsro_i32_to_f32(s));
        p[b % 16u] = tsro_fadd(p[b % 16u], t);
    }
    return tsro_tree16(p);
}

float tsro_dot_q4_K(const uint8_t * row, uint32_t K, const int8_t * q, const float * d, const int16_t * bs,
                    int32_t * isum) {
    float p[16] = { 0 };
    for (uint32_t sb = 0; sb < K / 256u; ++sb) {
        const uint8_t * blk = row + 144u * sb;
        const uint8_t * qs = blk + 16;
        const int8_t * qx = q + 256u * sb;
        const int16_t * b16 = bs + 16u * sb;
        int32_t acc = 0, macc = 0;
        for (int j = 0; j < 8; ++j) {             // sub-block j: nibble (j & 1) of bytes 32·(j/2) ..
            const uint8_t * qq = qs + 32 * (j / 2);
            const int sh = 4 * (j & 1);
            int32_t s = 0;
            for (int i = 0; i < 32; ++i) s += (int32_t)((qq[i] >> sh) & 0x0F) * (int32_t)qx[32 * j + i];
            int sc, m;
            q4k_sc_m(j, blk + 4, &sc, &m);
            acc += sc * s;
            macc += m * ((int32_t)b16[2 * j] + (int32_t)b16[2 * j + 1]);
        }
        if (isum) { isum[2u * sb] = acc; isum[2u * sb + 1] = macc; }
        const float t1 = tsro_fmul(tsro_fmul(tsro_fp16_to_f32(u16le(blk)), d[sb]), tsro_i32_to_f32(acc));
        const float t2 = tsro_fmul(tsro_fmul(tsro_fp16_to_f32(u16le(blk + 2)), d[sb]), tsro_i32_to_f32(macc));
        p[sb % 16u] = tsro_fadd(p[sb % 16u], tsro_fsub(t1, t2));
    }
    return tsro_tree16(p);
}

// ---------------------------------------------------------------------------------------------
// MUL_MAT composite (sw/ctrl/ref/mulmat_ref.hpp:8-13; the MVM epilogues tsr_sim.c:1648-1670)
// ---------------------------------------------------------------------------------------------
typedef struct mv_job {
    uint32_t fmt, N, K, T, flags, add_stride;
    const uint8_t * w;
    const int8_t * q;
    const float * d;
    const int16_t * bs;
    const float * add;
    float s0, s1;
    float * y;
    uint32_t lo, hi;
} mv_job;

static void * mv_rows(void * arg) {
    const mv_job * j = (const mv_job *)arg;
    const size_t row_bytes = j->fmt == TSRO_FMT_Q8_0 ? (size_t)(j->K / 32u) * 34u : (size_t)(j->K / 256u) * 144u;
    const uint32_t nd = j->fmt == TSRO_FMT_Q8_0 ? j->K / 32u : j->K / 256u;
    for (uint32_t n = j->lo; n < j->hi; ++n) {
        const uint8_t * row = j->w + (size_t)n * row_bytes;
        for (uint32_t t = 0; t < j->T; ++t) {
            const int8_t * q = j->q + (size_t)t * j->K;
            const float * d = j->d + (size_t)t * nd;
            float v = j->fmt == TSRO_FMT_Q8_0 ? tsro_dot_q8_0(row, j->K, q, d, NULL)
                                               : tsro_dot_q4_K(row, j->K, q, d, j->bs + (size_t)t * (j->K / 16u), NULL);
            if (j->flags & TSRO_MM_ADD) v = tsro_fadd(j->add[(size_t)t * j->add_stride + n], v);
            if (j->flags & TSRO_MM_SOFTCAP) v = tsro_fmul(tsro_tanh(tsro_fmul(v, j->s0)), j->s1);
            else if (j->flags & TSRO_MM_SCALE) v = tsro_fmul(v, j->s1);
            j->y[(size_t)t * j->N + n] = v;
        }
    }
    return NULL;
}

int tsro_matvec(uint32_t fmt, const uint8_t * w, uint32_t N, uint32_t K, const float * x, uint32_t T,
                const float * add, uint32_t add_stride, uint32_t flags, float s0, float s1, float * y,
                int threads) {
    const uint32_t bsz = fmt == TSRO_FMT_Q8_0 ? 32u : fmt == TSRO_FMT_Q4_K ? 256u : 0u;
    if (!bsz || K == 0 || K % bsz || T == 0 || (flags & ~7u)) return -1;
    if ((flags & TSRO_MM_ADD) && (flags & (TSRO_MM_SCALE | TSRO_MM_SOFTCAP))) return -1;
    if ((flags & TSRO_MM_ADD) && !add) return -1;
    int8_t * q = (int8_t *)malloc((size_t)T * K);
    float * d = (float *)malloc((size_t)T * (K / 32u) * sizeof(float));
    int16_t * bs = (int16_t *)malloc((size_t)T * (K / 16u) * sizeof(int16_t));
    if (!q || !d || !bs) { free(q); free(d); free(bs); return -1; }
    for (uint32_t t = 0; t < T; ++t) {
        if (fmt == TSRO_FMT_Q8_0) tsro_qact_a32(x + (size_t)t * K, K, q + (size_t)t * K, d + (size_t)t * (K / 32u));
        else tsro_qact_a256(x + (size_t)t * K, K, q + (size_t)t * K, d + (size_t)t * (K / 256u), bs + (size_t)t * (K / 16u));
    }
    if (threads < 1) threads = 1;
    if ((uint32_t)threads > N) threads = (int)(N ? N : 1);
    mv_job * jobs = (mv_job *)calloc((size_t)threads, sizeof(mv_job));
    pthread_t * th = (pthread_t *)calloc((size_t)threads, sizeof(pthread_t));
    const uint32_t per = (N + (uint32_t)threads - 1u) / (uint32_t)threads;
    for (int i = 0; i < threads; ++i) {
        mv_job j = { fmt, N, K, T, flags, add_stride, w, q, d, bs, add, s0, s1, y, 0, 0 };
        j.lo = (uint32_t)i * per < N ? (uint32_t)i * per : N;
        j.hi = j.lo + per < N ? j.lo + per : N;
        jobs[i] = j;
        if (i > 0) pthread_create(&th[i], NULL, mv_rows, &jobs[i]);
    }
    mv_rows(&jobs[0]);
    for (int i = 1; i < threads; ++i) pthread_join(th[i], NULL);
    free(jobs); free(th); free(q); free(d); free(bs);
    return 0;
}

// ---------------------------------------------------------------------------------------------
// Synthetic weight encoders
// ---------------------------------------------------------------------------------------------
void tsro_quantize_q8_0(const float * x, uint32_t K, uint8_t * blocks) {
    int8_t q[32];
    float d;
    for (uint32_t b = 0; b < K / 32u; ++b) {
        tsro_qact_a32(x + 32u * b, 32u, q, &d);
        const uint16_t h = tsro_f32_to_fp16(d);
        blocks[34u * b] = (uint8_t)h;
        blocks[34u * b + 1] = (uint8_t)(h >> 8);
        memcpy(blocks + 34u * b + 2, q, 32);
    }
}

// The sub-block min/scale encoder of gen_tiny_models.py:91-130: per 32 values, lo = min(min, 0),
// step = (max - lo)/15; d, dmin = fp16(max step / 63), fp16(max(-lo) / 63); 6-bit sc, m by RNE.
void tsro_quantize_q4_K(const float * x, uint32_t K, uint8_t * blocks) {
    for (uint32_t sb = 0; sb < K / 256u; ++sb) {
        const float * xb = x + 256u * sb;
        uint8_t * blk = blocks + 144u * sb;
        float step[8], mins[8], smax = 0.0f, mmax = 0.0f;
        for (int j = 0; j < 8; ++j) {
            float lo = 0.0f, hi = xb[32 * j];
            for (int i = 0; i < 32; ++i) {
                const float v = xb[32 * j + i];
                if (v < lo) lo = v;
                if (v > hi) hi = v;
            }
            step[j] = (hi - lo) / 15.0f;
            mins[j] = -lo;
            if (step[j] > smax) smax = step[j];
            if (mins[j] > mmax) mmax = mins[j];
        }
        const uint16_t hd = tsro_f32_to_fp16(smax / 63.0f), hm = tsro_f32_to_fp16(mmax / 63.0f);
        const float d = tsro_fp16_to_f32(hd), dmin = tsro_fp16_to_f32(hm);
        uint8_t sc[8], m[8], qv[256];
        for (int j = 0; j < 8; ++j) {
            float a = d > 0.0f ? nearbyintf(step[j] / d) : 0.0f;
            float b = dmin > 0.0f ? nearbyintf(mins[j] / dmin) : 0.0f;
            sc[j] = (uint8_t)(a < 0.0f ? 0.0f : a > 63.0f ? 63.0f : a);
            m[j] = (uint8_t)(b < 0.0f ? 0.0f : b > 63.0f ? 63.0f : b);
            const float s = d * (float)sc[j], off = dmin * (float)m[j];
            for (int i = 0; i < 32; ++i) {
                float r = s > 0.0f ? nearbyintf((xb[32 * j + i] + off) / s) : 0.0f;
                qv[32 * j + i] = (uint8_t)(r < 0.0f ? 0.0f : r > 15.0f ? 15.0f : r);
            }
        }
        blk[0] = (uint8_t)hd; blk[1] = (uint8_t)(hd >> 8);
        blk[2] = (uint8_t)hm; blk[3] = (uint8_t)(hm >> 8);
        for (int j = 0; j < 4; ++j) {
            blk[4 + j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
            blk[8 + j] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
            blk[12 + j] = (uint8_t)((sc[j + 4] & 15) | ((m[j + 4] & 15) << 4));
        }
        for (int c = 0; c < 4; ++c)
            for (int i = 0; i < 32; ++i) blk[16 + 32 * c + i] = (uint8_t)(qv[64 * c + i] | (qv[64 * c + 32 + i] << 4));
    }
}
