// tsro_fa.c — CPU restatement of flash attention over a q8_0 KV cache (TEST INFRASTRUCTURE ONLY).
//
// Restates the composite FA of the reference (jwkim04/tesseract-npu sw/sim/tsr_ref_at.c:774-860,
// design doc AT §6.6) on a ggml-layout cache (row j = cell j, E/32 block_q8_0 per row). The FPGA's
// KV planes only decide where bytes live; the numerics depend on the cell groups (16 cells), the
// channel of a group (u mod C), the 64-cell segments of a channel (4 of its groups) and the chunk
// plan, which are all restated here:
//   - chunk planner: sw/sim/include/tsr_fa_plan.h rules 1-8 (this file keeps the whole cut list of
//     a sub-range, the "direct implementation" that header describes),
//   - ATTQK / SEG: tsr_ref_at.c:294-375, ASMAX: :558-568, AMASK: :570-586,
//   - ATTPV block floating point and LSUM: tsr_ref_at.c:380-553,
//   - CTREE / AMERGE / ANORM: tsr_ref_at.c:588-641,
//   - mask summary: tsr_ref_at.c:646-715.
#include "tsro.h"

#include <stdlib.h>
#include <string.h>

#define SIGN_BIT 0x80000000u
#define EXP_MASK 0x7F800000u
#define MANT_MASK 0x007FFFFFu
#define CANON_NAN 0x7FC00000u
#define NEG_INF 0xFF800000u
#define M_FLOOR 0xF1800000u          // -2^100 (tsr_tables.h:89)
#define L_FLOOR 0x00800000u          // 2^-126 (tsr_tables.h:90)

static inline uint32_t fbits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float ffrom(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t daz_u(uint32_t u) { return (u & EXP_MASK) ? u : (u & SIGN_BIT); }
static inline int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }
static inline int64_t imax64(int64_t a, int64_t b) { return a > b ? a : b; }

// MAXT (VU §6.8, tsr_ref_at.c:318-325): NaN -> canonical NaN; else the larger DAZ'd value, -0 < +0.
static float maxt(float a, float b) {
    const uint32_t ua = daz_u(fbits(a)), ub = daz_u(fbits(b));
    if ((ua & ~SIGN_BIT) > EXP_MASK || (ub & ~SIGN_BIT) > EXP_MASK) return ffrom(CANON_NAN);
    // order-preserving keys of sign-magnitude encodings
    const uint32_t ka = (ua & SIGN_BIT) ? ~ua : (ua | SIGN_BIT);
    const uint32_t kb = (ub & SIGN_BIT) ? ~ub : (ub | SIGN_BIT);
    return ffrom(ka >= kb ? ua : ub);
}

// CTREE (tsr_ref_at.c:588-598): pairwise by levels, an unpaired last element passes through.
static float ctree(const float * x, uint32_t n) {
    float v[16];
    memcpy(v, x, n * sizeof(float));
    while (n > 1) {
        for (uint32_t k = 0; 2 * k + 1 < n; ++k) v[k] = tsro_fadd(v[2 * k], v[2 * k + 1]);
        if (n & 1u) v[n / 2] = v[n - 1];
        n = (n + 1) / 2;
    }
    return v[0];
}

// ---------------------------------------------------------------------------------------------
// Block floating point of ATTPV (tsr_ref_at.c:380-430)
// ---------------------------------------------------------------------------------------------
// RNE_int(w·2^(23-es)) for a finite w with exponent <= es; a zero or subnormal w gives 0.
static int32_t bf_int(float w, int32_t es) {
    const uint32_t u = fbits(w), a = u & ~SIGN_BIT;
    if ((a >> 23) == 0) return 0;
    const int32_t ew = (int32_t)(a >> 23) - 127;
    const uint32_t m = 0x00800000u | (a & MANT_MASK);
    const int32_t sh = es - ew;                // >= 0
    uint32_t v;
    if (sh == 0) v = m;
    else if (sh >= 26) v = 0;
    else {
        v = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (v & 1u))) v++;
    }
    return (u & SIGN_BIT) ? -(int32_t)v : (int32_t)v;
}

// RNE to 24 significant bits of A, times 2^k; below 2^-126 -> signed zero; >= 2^128 -> inf.
static float bf_f(int64_t A, int32_t k) {
    if (A == 0) return 0.0f;
    const uint32_t s = A < 0 ? SIGN_BIT : 0u;
    uint64_t mag = A < 0 ? (uint64_t)0 - (uint64_t)A : (uint64_t)A;
    int msb = 63 - __builtin_clzll(mag);
    int64_t e;                                  // value = m·2^(e - 23)
    if (msb > 23) {
        int sh = msb - 23;
        uint64_t m = mag >> sh;
        const uint64_t rem = mag & ((1ull << sh) - 1u), half = 1ull << (sh - 1);
        if (rem > half || (rem == half && (m & 1u))) m++;
        if (m == (1ull << 24)) { m >>= 1; sh++; }
        mag = m;
        e = 23 + sh + (int64_t)k;
    } else {
        mag <<= (23 - msb);
        e = msb + (int64_t)k;
    }
    if (e < -126) return ffrom(s);
    if (e > 127) return ffrom(s | EXP_MASK);
    return ffrom(s | ((uint32_t)(e + 127) << 23) | ((uint32_t)mag & MANT_MASK));
}

static inline int nonfinite(uint32_t u) { return (u & EXP_MASK) == EXP_MASK; }
static inline int32_t ilog2_normal(uint32_t u) { return (int32_t)((u >> 23) & 0xFFu) - 127; }

// ---------------------------------------------------------------------------------------------
// Mask summary (tsr_ref_at.c:646-692): per row at most two runs of cells whose f16 mask is +-0;
// GENERAL when a row has a value other than +-0 / -inf or more than two runs.
// ---------------------------------------------------------------------------------------------
typedef struct msum_row { uint32_t lo0, hi0, lo1, hi1; } msum_row;

static int build_msum(const uint16_t * mask, size_t stride, uint32_t n_kv, uint32_t T, msum_row * rows) {
    int general = 0;
    for (uint32_t q = 0; q < T; ++q) {
        msum_row r = { 0, 0, 0, 0 };
        if (!mask) {
            r.lo0 = 0; r.hi0 = n_kv;
            if (n_kv == 0) r.hi0 = 0;
            rows[q] = r;
            continue;
        }
        const uint16_t * m = mask + (size_t)q * stride;
        uint32_t nrun = 0;
        uint32_t j = 0;
        while (j < n_kv) {
            if (m[j] == 0xFC00u) { j++; continue; }
            if (m[j] & 0x7FFFu) { general = 1; j++; continue; }
            uint32_t e = j;
            while (e < n_kv && (m[e] & 0x7FFFu) == 0) e++;
            if (nrun == 0) { r.lo0 = j; r.hi0 = e; }
            else if (nrun == 1) { r.lo1 = j; r.hi1 = e; }
            nrun++;
            j = e;
        }
        if (nrun > 2) general = 1;
        rows[q] = r;
    }
    return general;
}

// ---------------------------------------------------------------------------------------------
// Chunk planner (tsr_fa_plan.h rules 1-8)
// ---------------------------------------------------------------------------------------------
typedef struct chunk { uint32_t u0, n, c_lo, c_hi, flags, general; } chunk;
#define FL_CAUSAL 1u
#define FL_SLIDE 2u

typedef struct subr {
    uint32_t ulo, uhi, general, multi, flags;
    int64_t lo, hi;
} subr;

static uint32_t ncg_of(uint32_t C, uint32_t pcap, uint32_t E, uint32_t D, uint32_t n_total) {
    if (D == 0 || E % D || C == 0 || E / D == 0) return 0;
    const uint64_t pc = (uint64_t)C * (pcap / (16u * (E / D)));
    if (pc == 0) return 0;
    const uint64_t half = ((uint64_t)n_total + 1u) / 2u, c4 = 4u * (uint64_t)C;
    const uint64_t m = c4 >= half ? c4 : (half + c4 - 1u) / c4 * c4;
    uint64_t r = 128u;
    if (pc < r) r = pc;
    if (m < r) r = m;
    return (uint32_t)r;
}

static int cmp_u32(const void * a, const void * b) {
    const uint32_t x = *(const uint32_t *)a, y = *(const uint32_t *)b;
    return x < y ? -1 : x > y;
}

// Rule 6 for the chunk [a, b) of sub-range s (and its verification for FAST T > 1). 0 or -3.
static int encode_chunk(const subr * s, uint32_t T, const int64_t * L, const int64_t * H, uint32_t a, uint32_t b,
                        chunk * c) {
    c->u0 = a; c->n = b - a; c->flags = 0; c->general = 0;
    const int64_t A = 16 * (int64_t)a, A2 = 16 * (int64_t)b, n16 = A2 - A;
    if (s->general) { c->general = 1; c->c_lo = 0; c->c_hi = (uint32_t)n16; return 0; }
    if (!s->multi) {
        c->c_lo = (uint32_t)imax64(s->lo - A, 0);
        c->c_hi = (uint32_t)imin64(s->hi - A, n16);
        return 0;
    }
    int64_t clo = 0, chi = n16;
    uint32_t fl = 0;
    if (s->lo > A) { clo = s->lo - A; if (s->flags & FL_SLIDE) fl |= FL_SLIDE; }
    if (s->hi - ((s->flags & FL_CAUSAL) ? (int64_t)T - 1 : 0) < A2) { chi = s->hi - A; if (s->flags & FL_CAUSAL) fl |= FL_CAUSAL; }
    if (clo < 0 || clo > chi || chi > n16) return -3;
    for (uint32_t q = 0; q < T; ++q) {
        const int64_t dq = (int64_t)T - 1 - q;
        const int64_t lq = imax64(0, clo - ((fl & FL_SLIDE) ? dq : 0));
        const int64_t hq = imin64(chi - ((fl & FL_CAUSAL) ? dq : 0), n16);
        const int64_t el = imax64(L[q] - A, 0), eh = imin64(H[q] - A, n16);
        const int ea = hq <= lq, eb = eh <= el;
        if (ea != eb || (!ea && (lq != el || hq != eh))) return -3;
    }
    c->c_lo = (uint32_t)clo; c->c_hi = (uint32_t)chi; c->flags = fl;
    return 0;
}

// The tile's chunk list in execution order. Returns the count (out malloc'd), or -1 (NCG = 0),
// -2 (malformed MSUM row), -3 (an encoding that does not reproduce the rows' runs).
static long plan_tile(uint32_t C, uint32_t pcap, uint32_t E, uint32_t D, uint32_t n_kv, int general_msum,
                      const msum_row * rows, uint32_t T, uint32_t new_lo, uint32_t new_hi, chunk ** out) {
    subr sub[2];
    uint32_t nsub = 0;
    int64_t L[8] = { 0 }, H[8] = { 0 };
    *out = NULL;
    if (general_msum) {
        if (n_kv > 0) { sub[0] = (subr){ 0, (n_kv + 15) >> 4, 1, 0, 0, 0, 0 }; nsub = 1; }
    } else {
        int64_t rl[8][2], rh[8][2];
        uint32_t nr[8];
        int all_one = 1;
        int64_t hlo = INT64_MAX, hhi = -1;
        for (uint32_t q = 0; q < T; ++q) {
            const msum_row * w = &rows[q];
            if (w->lo0 > w->hi0 || w->lo1 > w->hi1 || w->hi0 > n_kv || w->hi1 > n_kv) return -2;
            if (w->hi0 > w->lo0 && w->hi1 > w->lo1 && !(w->hi0 <= w->lo1 || w->hi1 <= w->lo0)) return -2;
            uint32_t n = 0;
            if (w->hi0 > w->lo0) { rl[q][n] = w->lo0; rh[q][n] = w->hi0; n++; }
            if (w->hi1 > w->lo1) { rl[q][n] = w->lo1; rh[q][n] = w->hi1; n++; }
            if (n == 2 && rl[q][1] < rl[q][0]) {
                int64_t t0 = rl[q][0], t1 = rh[q][0];
                rl[q][0] = rl[q][1]; rh[q][0] = rh[q][1]; rl[q][1] = t0; rh[q][1] = t1;
            }
            nr[q] = n;
            if (n != 1) all_one = 0;
            for (uint32_t k = 0; k < n; ++k) { hlo = imin64(hlo, rl[q][k]); hhi = imax64(hhi, rh[q][k]); }
        }
        if (T == 1) {
            for (uint32_t k = 0; k < nr[0]; ++k)
                sub[nsub++] = (subr){ (uint32_t)(rl[0][k] / 16), (uint32_t)((rh[0][k] + 15) / 16), 0, 0, 0, rl[0][k], rh[0][k] };
        } else if (hhi >= 0) {
            int fit = all_one;
            uint32_t fl = 0;
            int64_t lo_abs = 0, hi_abs = 0;
            if (fit) {
                for (uint32_t q = 0; q < T; ++q) { L[q] = rl[q][0]; H[q] = rh[q][0]; }
                hi_abs = H[T - 1]; lo_abs = L[T - 1];
                int heq = 1, leq = 1, hca = 1, lsl = lo_abs > 0;
                for (uint32_t q = 0; q < T; ++q) {
                    const int64_t dq = (int64_t)T - 1 - q;
                    heq &= H[q] == hi_abs;
                    leq &= L[q] == lo_abs;
                    hca &= H[q] == hi_abs - dq;
                    lsl &= L[q] == imax64(0, lo_abs - dq);
                }
                if (!heq) { if (hca) fl |= FL_CAUSAL; else fit = 0; }
                if (!leq) { if (lsl) fl |= FL_SLIDE; else fit = 0; }
            }
            if (fit) {
                int64_t mnL = INT64_MAX, mxH = -1;
                for (uint32_t q = 0; q < T; ++q) { mnL = imin64(mnL, L[q]); mxH = imax64(mxH, H[q]); }
                sub[nsub++] = (subr){ (uint32_t)(mnL / 16), (uint32_t)((mxH + 15) / 16), 0, 1, fl, lo_abs, hi_abs };
            } else {
                sub[nsub++] = (subr){ (uint32_t)(hlo / 16), (uint32_t)((hhi + 15) / 16), 1, 0, 0, 0, 0 };
            }
        }
    }
    if (nsub == 0) {                              // rule 8: one empty chunk
        chunk * c = (chunk *)malloc(sizeof(chunk));
        if (!c) return -1;
        *c = (chunk){ 0, 1, 0, 0, 0, 0 };
        *out = c;
        return 1;
    }
    uint32_t n_total = 0;
    for (uint32_t k = 0; k < nsub; ++k) n_total += sub[k].uhi - sub[k].ulo;
    const uint32_t ncg = ncg_of(C, pcap, E, D, n_total);
    if (ncg == 0) return -1;
    // Generate every chunk (rules 4-6), then order them (rule 7).
    size_t cap = 16, cnt = 0;
    chunk * list = (chunk *)malloc(cap * sizeof(chunk));
    if (!list) return -1;
    for (uint32_t k = 0; k < nsub; ++k) {
        const subr * s = &sub[k];
        size_t ncut = 0, ccap = 16 + (s->uhi - s->ulo) / ncg;
        uint32_t * cuts = (uint32_t *)malloc((ccap + 64) * sizeof(uint32_t));
        if (!cuts) { free(list); return -1; }
        for (uint64_t x = (uint64_t)s->ulo + ncg; x < s->uhi; x += ncg) cuts[ncut++] = (uint32_t)x;
        if (s->multi && s->flags) {               // rule 5: no cut strictly inside a bound spread
            int64_t sp[2][2];
            uint32_t nsp = 0;
            if (s->flags & FL_CAUSAL) { sp[nsp][0] = s->hi - (int64_t)(T - 1); sp[nsp][1] = s->hi; nsp++; }
            if (s->flags & FL_SLIDE) { sp[nsp][0] = imax64(0, s->lo - (int64_t)(T - 1)); sp[nsp][1] = s->lo; nsp++; }
            for (int round = 0; round < 8; ++round) {
                int changed = 0;
                for (size_t i = 0; i < ncut; ++i) {
                    const int64_t X = 16 * (int64_t)cuts[i];
                    for (uint32_t t = 0; t < nsp; ++t) {
                        if (sp[t][0] < X && X < sp[t][1]) {
                            cuts[i] = (uint32_t)(sp[t][0] / 16);
                            cuts[ncut++] = (uint32_t)((sp[t][1] + 15) / 16);
                            changed = 1;
                            break;
                        }
                    }
                }
                qsort(cuts, ncut, sizeof(uint32_t), cmp_u32);
                size_t m = 0;
                for (size_t i = 0; i < ncut; ++i) {
                    if (cuts[i] <= s->ulo || cuts[i] >= s->uhi) continue;
                    if (m && cuts[m - 1] == cuts[i]) continue;
                    cuts[m++] = cuts[i];
                }
                ncut = m;
                if (!changed) break;
            }
        }
        uint32_t a = s->ulo;
        for (size_t i = 0; i <= ncut; ++i) {
            const uint32_t b = i < ncut ? cuts[i] : s->uhi;
            if (cnt == cap) {
                cap *= 2;
                chunk * nl = (chunk *)realloc(list, cap * sizeof(chunk));
                if (!nl) { free(cuts); free(list); return -1; }
                list = nl;
            }
            if (encode_chunk(s, T, L, H, a, b, &list[cnt]) != 0) { free(cuts); free(list); return -3; }
            cnt++;
            a = b;
        }
        free(cuts);
    }
    // rule 7: chunks holding a cell written in this launch go last, keeping their order
    chunk * ord = (chunk *)malloc(cnt * sizeof(chunk));
    if (!ord) { free(list); return -1; }
    size_t o = 0;
    for (int pass = 0; pass < 2; ++pass) {
        for (size_t i = 0; i < cnt; ++i) {
            const uint64_t A = 16u * (uint64_t)list[i].u0, B = 16u * ((uint64_t)list[i].u0 + list[i].n);
            const int nw = new_hi > new_lo && new_lo < B && new_hi > A;
            if (nw == pass) ord[o++] = list[i];
        }
    }
    free(list);
    *out = ord;
    return (long)cnt;
}

// ---------------------------------------------------------------------------------------------
// The composite (tsr_ref_at.c:774-860)
// ---------------------------------------------------------------------------------------------
static inline uint16_t u16le(const uint8_t * p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// SEG (tsr_ref_at.c:327-338): the Q8_0 row rule over one head's D values of cell row `krow`.
static float seg(uint32_t D, const uint8_t * kblk, const int8_t * qx, const float * dx, int32_t * isum) {
    float p[16] = { 0 };
    for (uint32_t k = 0; k < D / 32u; ++k) {
        const uint8_t * b = kblk + 34u * k;
        const int8_t * qk = (const int8_t *)(b + 2);
        int32_t s = 0;
        for (int i = 0; i < 32; ++i) s += (int32_t)qk[i] * (int32_t)qx[32u * k + i];
        if (isum) isum[k] = s;
        p[k] = tsro_fadd(0.0f, tsro_fmul(tsro_fmul(tsro_fp16_to_f32(u16le(b)), dx[k]), tsro_i32_to_f32(s)));
    }
    return tsro_tree16(p);
}

void tsro_fa_qk_isums(const tsro_fa_params * p, const float * q, const uint8_t * k_rows, int32_t * isum) {
    const uint32_t D = p->D, G = p->n_head / p->n_head_kv, K = p->n_head * D, E = p->n_head_kv * D;
    int8_t * qx = (int8_t *)malloc(K);
    float * dx = (float *)malloc((K / 32u) * sizeof(float));
    tsro_qact_a32(q, K, qx, dx);
    const size_t row_bytes = (size_t)(E / 32u) * 34u;
    for (uint32_t h = 0; h < p->n_head; ++h)
        for (uint32_t j = 0; j < p->n_kv; ++j)
            (void)seg(D, k_rows + (size_t)j * row_bytes + (size_t)(h / G) * (D / 32u) * 34u, qx + (size_t)h * D,
                      dx + (size_t)h * (D / 32u), isum + ((size_t)h * p->n_kv + j) * (D / 32u));
    free(qx); free(dx);
}

int tsro_fa(const tsro_fa_params * p, const float * q, const uint8_t * k_rows, const uint8_t * v_rows,
            const uint16_t * mask, size_t mask_stride, float * out) {
    const uint32_t C = p->C, D = p->D, T = p->T, n_head = p->n_head, nkvh = p->n_head_kv, n_kv = p->n_kv;
    if (C == 0 || C > 16 || p->t_max == 0 || p->t_max > 8 || T == 0) return TSRO_FA_E_SHAPE;
    if (!(D == 64 || D == 128 || D == 256 || D == 512) || nkvh == 0 || n_head % nkvh) return TSRO_FA_E_SHAPE;
    const uint32_t G = n_head / nkvh, E = nkvh * D, K = n_head * D;
    if (G == 0 || G > 64 || E / 64u > 511u) return TSRO_FA_E_SHAPE;
    const uint32_t sb = fbits(p->scale);
    if ((sb & SIGN_BIT) || (sb & EXP_MASK) == 0 || (sb & EXP_MASK) == EXP_MASK) return TSRO_FA_E_SHAPE;
    if ((uint64_t)G * E > 32768u) return TSRO_FA_E_SHAPE;          // K_MAX of the release image
    const uint32_t GS0 = G < p->t_max ? G : p->t_max, Tq0 = p->t_max / GS0;
    if (nkvh * GS0 * Tq0 > 128u || Tq0 * n_head > 1024u) return TSRO_FA_E_SHAPE;
    if (ncg_of(C, p->pcap, E, D, 1) == 0) return TSRO_FA_E_SHAPE;

    msum_row * rows = (msum_row *)calloc(T, sizeof(msum_row));
    if (!rows) return TSRO_FA_E_NOMEM;
    const int general_msum = build_msum(mask, mask_stride, n_kv, T, rows);
    const uint32_t ng_kv = (n_kv + 15u) / 16u;
    const size_t row_bytes = (size_t)(E / 32u) * 34u;
    const uint32_t R0 = Tq0 * n_head, nsl = D / 64u;
    int8_t * qx = (int8_t *)malloc((size_t)Tq0 * K);
    float * dx = (float *)malloc((size_t)Tq0 * (K / 32u) * sizeof(float));
    float * S = (float *)malloc((size_t)R0 * 128u * 16u * sizeof(float));
    float * mk = (float *)malloc(R0 * sizeof(float));
    float * Oc = (float *)malloc((size_t)C * R0 * D * sizeof(float));
    float * lc = (float *)malloc((size_t)C * R0 * sizeof(float));
    float * Orun = (float *)malloc((size_t)R0 * D * sizeof(float));
    float * mrun = (float *)malloc(R0 * sizeof(float));
    float * lrun = (float *)malloc(R0 * sizeof(float));
    float * mrow = (float *)malloc(((size_t)ng_kv * 16u + 16u) * sizeof(float));
    int rc = TSRO_FA_OK;
    chunk * ch = NULL;
    if (!qx || !dx || !S || !mk || !Oc || !lc || !Orun || !mrun || !lrun || !mrow) { rc = TSRO_FA_E_NOMEM; goto done; }

    for (uint32_t q0 = 0; q0 < T; q0 += Tq0) {
        const uint32_t Tq = T - q0 < Tq0 ? T - q0 : Tq0, R = Tq * n_head;
        for (uint32_t t = 0; t < Tq; ++t) tsro_qact_a32(q + (size_t)(q0 + t) * K, K, qx + (size_t)t * K, dx + (size_t)t * (K / 32u));
        free(ch);
        ch = NULL;
        const long nch = plan_tile(C, p->pcap, E, D, n_kv, general_msum, rows + q0, Tq, p->new_lo, p->new_hi, &ch);
        if (nch < 0) { rc = nch == -2 ? TSRO_FA_E_MSUM : TSRO_FA_E_SHAPE; goto done; }
        for (long k = 0; k < nch; ++k)
            if (ch[k].general && !mask) { rc = TSRO_FA_E_MASK; goto done; }
        for (long k = 0; k < nch; ++k) {
            const chunk * c = &ch[k];
            const uint32_t ncell = 16u * c->n;
            // ATTQK (+ AMASK for GENERAL): scores of row r = t·n_head + h, cell j of the chunk
            for (uint32_t t = 0; t < Tq; ++t) {
                const int64_t dq = (int64_t)Tq - 1 - t;
                const int64_t lo = imax64(0, (int64_t)c->c_lo - ((c->flags & FL_SLIDE) ? dq : 0));
                const int64_t hi = (int64_t)c->c_hi - ((c->flags & FL_CAUSAL) ? dq : 0);
                if (c->general) {                  // the f32 mask copy: fdiv(mask, scale), -inf past n_kv
                    const uint16_t * m = mask + (size_t)(q0 + t) * mask_stride;
                    for (uint32_t j = 0; j < ncell; ++j) {
                        const uint32_t cell = 16u * c->u0 + j;
                        mrow[j] = cell < n_kv ? tsro_fdiv(tsro_fp16_to_f32(m[cell]), p->scale) : ffrom(NEG_INF);
                    }
                }
                for (uint32_t h = 0; h < n_head; ++h) {
                    const uint32_t r = t * n_head + h, g = h / G;
                    float * srow = S + (size_t)r * ncell;
                    float mx = ffrom(M_FLOOR);
                    for (uint32_t j = 0; j < ncell; ++j) {
                        const uint32_t cell = 16u * c->u0 + j;
                        const int vis = c->general ? 1 : ((int64_t)j >= lo && (int64_t)j < hi);
                        float s = ffrom(NEG_INF);
                        if (vis && cell < n_kv)
                            s = seg(D, k_rows + (size_t)cell * row_bytes + (size_t)g * (D / 32u) * 34u,
                                    qx + (size_t)t * K + (size_t)h * D, dx + (size_t)t * (K / 32u) + (size_t)h * (D / 32u), NULL);
                        if (c->general) s = fbits(mrow[j]) == NEG_INF ? ffrom(NEG_INF) : tsro_fadd(s, mrow[j]);
                        srow[j] = s;
                        mx = maxt(mx, s);
                    }
                    mk[r] = mx;
                }
            }
            // ASMAX
            for (uint32_t r = 0; r < R; ++r)
                for (uint32_t j = 0; j < ncell; ++j)
                    S[(size_t)r * ncell + j] = tsro_exp(tsro_fmul(tsro_fsub(S[(size_t)r * ncell + j], mk[r]), p->scale));
            // ATTPV with LSUM, per channel: its groups u = ch (mod C) of the chunk, 4 per segment
            for (uint32_t cc = 0; cc < C; ++cc) {
                uint32_t U[128];
                uint32_t nu = 0;
                for (uint32_t u = c->u0; u < c->u0 + c->n; ++u) if (u % C == cc) U[nu++] = u;
                for (uint32_t r = 0; r < R; ++r) {
                    const uint32_t h = r % n_head, g = h / G;
                    const float * prow = S + (size_t)r * ncell;
                    float * orow = Oc + ((size_t)cc * R + r) * D;
                    for (uint32_t L = 0; L < D; ++L) orow[L] = 0.0f;
                    for (uint32_t sl = 0; sl < nsl; ++sl) {
                        const uint32_t s = g * nsl + sl;          // 64-value slice of the cell row
                        for (uint32_t k0 = 0; k0 < nu; k0 += 4u) {
                            // w = p (*) dV per cell and block of the slice
                            float w[64][2];
                            const int8_t * qv[64];
                            uint32_t n = 0;
                            for (uint32_t k = k0; k < nu && k < k0 + 4u; ++k)
                                for (uint32_t rr = 0; rr < 16u; ++rr) {
                                    const uint32_t cell = 16u * U[k] + rr;
                                    const float pj = prow[cell - 16u * c->u0];
                                    if ((daz_u(fbits(pj)) & ~SIGN_BIT) == 0) continue;
                                    const uint8_t * vb = v_rows + (size_t)cell * row_bytes + (size_t)(2u * s) * 34u;
                                    w[n][0] = tsro_fmul(pj, tsro_fp16_to_f32(u16le(vb)));
                                    w[n][1] = tsro_fmul(pj, tsro_fp16_to_f32(u16le(vb + 34)));
                                    qv[n] = (const int8_t *)vb;     // block 2s at +2, block 2s+1 at +36
                                    n++;
                                }
                            int bad[2] = { 0, 0 }, any = 0;
                            int32_t es = -1000;
                            for (uint32_t i = 0; i < n; ++i)
                                for (int e = 0; e < 2; ++e) {
                                    const uint32_t u = fbits(w[i][e]);
                                    if (nonfinite(u)) bad[e] = 1;
                                    else if (u & ~SIGN_BIT) { const int32_t le = ilog2_normal(u); if (le > es) es = le; any = 1; }
                                }
                            for (int e = 0; e < 2; ++e) {
                                int64_t A[32] = { 0 };
                                if (any && !bad[e])
                                    for (uint32_t i = 0; i < n; ++i) {
                                        const int64_t W = bf_int(w[i][e], es);
                                        if (!W) continue;
                                        const int8_t * qq = qv[i] + 2 + 34 * e;
                                        for (int l = 0; l < 32; ++l) A[l] += W * (int64_t)qq[l];
                                    }
                                for (int l = 0; l < 32; ++l) {
                                    const float cv = bad[e] ? ffrom(CANON_NAN) : !any ? 0.0f : bf_f(A[l], es - 23);
                                    float * o = &orow[64u * sl + 32u * (uint32_t)e + (uint32_t)l];
                                    *o = tsro_fadd(*o, cv);
                                }
                            }
                        }
                    }
                    // LSUM: per segment, block floating point over its cells' p values
                    float l = 0.0f;
                    for (uint32_t k0 = 0; k0 < nu; k0 += 4u) {
                        int bad = 0, any = 0;
                        int32_t ep = -1000;
                        uint32_t pu[64];
                        uint32_t n = 0;
                        for (uint32_t k = k0; k < nu && k < k0 + 4u; ++k)
                            for (uint32_t rr = 0; rr < 16u; ++rr) pu[n++] = daz_u(fbits(prow[16u * (U[k] - c->u0) + rr]));
                        for (uint32_t i = 0; i < n; ++i) {
                            if (nonfinite(pu[i])) bad = 1;
                            else if (pu[i] & ~SIGN_BIT) { const int32_t le = ilog2_normal(pu[i]); if (le > ep) ep = le; any = 1; }
                        }
                        float v;
                        if (bad) v = ffrom(CANON_NAN);
                        else if (!any) v = 0.0f;
                        else {
                            int64_t sum = 0;
                            for (uint32_t i = 0; i < n; ++i) sum += bf_int(ffrom(pu[i]), ep);
                            v = bf_f(sum, ep - 23);
                        }
                        l = tsro_fadd(l, v);
                    }
                    lc[(size_t)cc * R + r] = l;
                }
            }
            // AMERGE
            for (uint32_t r = 0; r < R; ++r) {
                float xv[16];
                for (uint32_t cc = 0; cc < C; ++cc) xv[cc] = lc[(size_t)cc * R + r];
                const float lk = ctree(xv, C);
                float a = 0.0f, b = 0.0f;
                if (k == 0) { lrun[r] = lk; mrun[r] = mk[r]; }
                else {
                    const float mn = maxt(mrun[r], mk[r]);
                    a = tsro_exp(tsro_fmul(tsro_fsub(mrun[r], mn), p->scale));
                    b = tsro_exp(tsro_fmul(tsro_fsub(mk[r], mn), p->scale));
                    lrun[r] = tsro_fadd(tsro_fmul(lrun[r], a), tsro_fmul(lk, b));
                    mrun[r] = mn;
                }
                for (uint32_t d = 0; d < D; ++d) {
                    for (uint32_t cc = 0; cc < C; ++cc) xv[cc] = Oc[((size_t)cc * R + r) * D + d];
                    const float ok = ctree(xv, C);
                    float * o = &Orun[(size_t)r * D + d];
                    *o = k == 0 ? ok : tsro_fadd(tsro_fmul(*o, a), tsro_fmul(ok, b));
                }
            }
        }
        // ANORM
        for (uint32_t r = 0; r < R; ++r) {
            const float rinv = tsro_frecip(maxt(lrun[r], ffrom(L_FLOOR)));
            for (uint32_t d = 0; d < D; ++d)
                out[((size_t)q0 * n_head + r) * D + d] = tsro_fmul(Orun[(size_t)r * D + d], rinv);
        }
    }
done:
    free(ch); free(rows); free(qx); free(dx); free(S); free(mk); free(Oc); free(lc); free(Orun); free(mrun); free(lrun); free(mrow);
    return rc;
}
