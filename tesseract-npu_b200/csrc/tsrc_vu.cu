// tsrc_vu.cu -- the decoder layer's vector kinds around MUL_MAT and FLASH_ATTN on sm_100a:
// RMS_NORM (+ the weight MUL), ROPE (NORM / NEOX), the elementwise VOPs a decode step needs (ADD,
// MUL, SILU, SWIGLU) and GET_ROWS of a quantized weight (the token embedding: DQROW).
//
// Numerics: the reference's vector unit bit for bit (jwkim04/tesseract-npu sw/sim/tsr_ref_vu.c and
// tsr_ref_math.c): every f32 operation is separately rounded with DAZ inputs, FTZ results and the
// canonical NaN (FA / FS / FM / SQ / RC), the reductions use the 128-partial tree, SILU is built on
// the integer EXPK algorithm, SIN / COS on an exact 2/pi reduction and the Cephes polynomials.
// These kinds are latency work on a decode step (kilobytes per call): one CTA per token row.
#include "tsrc_internal.h"
#include "tsrc_layout.cuh"
#include "tsrc_numerics.cuh"

namespace tsrc {

namespace {

__device__ unsigned int g_vu_error;                // 1: GET_ROWS met a token id outside the weight

// the reference's FA / FS / FM / SQ / RC on arbitrary inputs (DAZ in, FTZ out; NaN canonical at the store)
__device__ __forceinline__ float FA(float a, float b) { return fadd(daz(a), daz(b)); }
__device__ __forceinline__ float FS(float a, float b) { return fsub(daz(a), daz(b)); }
__device__ __forceinline__ float FM(float a, float b) { return fmul(daz(a), daz(b)); }
__device__ __forceinline__ float SQ(float a) { return flush(__fsqrt_rn(daz(a))); }
__device__ __forceinline__ float RC(float a) { return frecip(daz(a)); }

// ---- RMS_NORM: rmsnorm_ref_rows (sw/ctrl/ref/rmsnorm_ref.cpp:59-78) = RED.SUMSQ post RMS
// (tsr_ref_vu.c:171-263) then VOP.MULCB / MULC (tsr_ref_vu.c:104-130). The row is staged in shared
// memory by all threads (coalesced, many loads in flight); thread i < 128 then owns partial p_i
// (elements i, i + 128, ... in order), the 7-level pairwise tree runs over lanes and warps.
constexpr uint32_t kRedThreads = 512;
constexpr uint32_t kRedPartials = 128;

__global__ void __launch_bounds__(kRedThreads) rms_norm_kernel(const float* __restrict__ x, uint32_t xs, float* y, uint32_t ys,
                                                              const float* __restrict__ w, uint32_t n, float eps, float inv_n,
                                                              bool stage_w) {
    extern __shared__ float xrow[];                       // [n] the row, then (stage_w) [n] the weight
    __shared__ float part[4];
    __shared__ float scale;
    const float* xr = x + (size_t)blockIdx.x * xs;
    float* wrow = xrow + n;
    // every global load of the kernel is issued here, before the first barrier (the output loop
    // then only stores)
    for (uint32_t j = threadIdx.x; j < n; j += kRedThreads) {
        xrow[j] = daz(xr[j]);
        if (stage_w) wrow[j] = w[j];
    }
    __syncthreads();
    if (threadIdx.x < kRedPartials) {
        float p = 0.0f;
        for (uint32_t j = threadIdx.x; j < n; j += kRedPartials) p = fadd(p, fmul(xrow[j], xrow[j]));
#pragma unroll
        for (uint32_t off = 1; off < 32u; off <<= 1) {      // levels 1-5: lane 2^l k holds partials 2^l k ..
            const float o = __shfl_down_sync(0xFFFFFFFFu, p, off);
            p = fadd(p, o);
        }
        if ((threadIdx.x & 31u) == 0) part[threadIdx.x >> 5] = p;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const float s = fadd(fadd(part[0], part[1]), fadd(part[2], part[3]));   // levels 6-7
        scale = RC(SQ(FA(FM(s, inv_n), eps)));
    }
    __syncthreads();
    const float sc = scale;
    float* yr = y + (size_t)blockIdx.x * ys;
    for (uint32_t j = threadIdx.x; j < n; j += kRedThreads) {
        const float v = fmul(xrow[j], sc);
        yr[j] = canon(w ? FM(v, stage_w ? wrow[j] : w[j]) : v);
    }
}

// ---- SIN / COS: tsr_m_sincos (tsr_ref_math.c:336-412, VU §6.6). |t| < 2^-12: (t, 1). Otherwise
// t * 2/pi with a 64-bit constant gives the quadrant and a 62-bit fraction, rounded to the nearest
// quadrant; r = fraction * pi/2 rounded once to f32; the Cephes single-precision polynomials.
struct U128 {
    uint64_t hi, lo;
};
__device__ __forceinline__ U128 mul64(uint64_t a, uint64_t b) { return {__umul64hi(a, b), a * b}; }
__device__ __forceinline__ U128 shr128(U128 x, uint32_t n) {
    if (n >= 128u) return {0, 0};
    if (n >= 64u) return {0, x.hi >> (n - 64u)};
    if (n == 0u) return x;
    return {x.hi >> n, (x.lo >> n) | (x.hi << (64u - n))};
}
__device__ __forceinline__ U128 shl128(U128 x, uint32_t n) {
    if (n >= 128u) return {0, 0};
    if (n >= 64u) return {x.lo << (n - 64u), 0};
    if (n == 0u) return x;
    return {(x.hi << n) | (x.lo >> (64u - n)), x.lo << n};
}
__device__ __forceinline__ bool any_low_bits(U128 x, uint32_t n) {          // bits [0, n) of x, n <= 127
    if (n == 0u) return false;
    if (n >= 64u) return x.lo != 0 || (n > 64u && (x.hi & ((1ull << (n - 64u)) - 1u)) != 0);
    return (x.lo & ((1ull << n) - 1u)) != 0;
}
// nearest-even f32 of R * 2^-124 (R in (0, 2^124); the result is normal)
__device__ __forceinline__ float r_to_f32(U128 R, bool neg) {
    const int b = R.hi ? 127 - __clzll(R.hi) : 63 - __clzll(R.lo);
    const uint32_t shift = (uint32_t)(b - 23);
    uint64_t sig = shr128(R, shift).lo;
    const bool guard = (shr128(R, shift - 1u).lo & 1u) != 0;
    const bool sticky = any_low_bits(R, shift - 1u);
    uint32_t be = (uint32_t)(b + 3);
    if (guard && (sticky || (sig & 1u))) {
        sig += 1u;
        if (sig == (1ull << 24)) {
            sig >>= 1;
            be += 1u;
        }
    }
    return ffrom((neg ? kSign : 0u) | (be << 23) | ((uint32_t)sig & kMant));
}

constexpr uint64_t kTwoOverPi64 = 0xA2F9836E4E44152Aull;   // round(2/pi * 2^64)
constexpr uint64_t kPiOver2_62 = 0x6487ED5110B4611Aull;    // round(pi/2 * 2^62)
constexpr uint64_t kMask62 = (1ull << 62) - 1u;

__device__ void sincos_vu(float t, float* s_out, float* c_out) {
    const uint32_t u = fbits(daz(t)), a = u & ~kSign;
    if (a >= kExp) {
        *s_out = ffrom(kCanonNaN);
        *c_out = ffrom(kCanonNaN);
        return;
    }
    const uint32_t E = a >> 23;
    if (E < 115u) {
        *s_out = ffrom(u);
        *c_out = 1.0f;
        return;
    }
    const uint64_t M = 0x00800000u | (a & kMant);
    const U128 P = mul64(M, kTwoOverPi64);
    const int sh = 214 - (int)E;
    uint32_t k4;
    uint64_t F;
    if (sh >= 62) {
        k4 = (uint32_t)(shr128(P, (uint32_t)sh).lo & 3u);
        F = shr128(P, (uint32_t)(sh - 62)).lo & kMask62;
    } else if (sh >= 0) {
        k4 = (uint32_t)(shr128(P, (uint32_t)sh).lo & 3u);
        F = shl128(P, (uint32_t)(62 - sh)).lo & kMask62;
    } else {
        k4 = (uint32_t)(shl128(P, (uint32_t)(-sh)).lo & 3u);
        F = 0;
    }
    bool rneg = false;
    uint64_t Fmag = F;
    if (F >= (1ull << 61)) {
        k4 = (k4 + 1u) & 3u;
        rneg = true;
        Fmag = (1ull << 62) - F;
    }
    const float r = Fmag == 0 ? 0.0f : r_to_f32(mul64(Fmag, kPiOver2_62), rneg);
    const float z = fmul(r, r);
    float p = fmul(ffrom(0xB94CA1F9u), z);                     // Cephes sinf
    p = fadd(p, ffrom(0x3C08839Eu));
    p = fmul(p, z);
    p = fadd(p, ffrom(0xBE2AAAA3u));
    p = fmul(p, z);
    p = fmul(p, r);
    const float sn = fadd(p, r);
    p = fmul(ffrom(0x37CCF5CEu), z);                           // Cephes cosf
    p = fadd(p, ffrom(0xBAB6061Au));
    p = fmul(p, z);
    p = fadd(p, ffrom(0x3D2AAAA5u));
    p = fmul(p, z);
    p = fmul(p, z);
    const float cs = fadd(fsub(p, fmul(0.5f, z)), 1.0f);
    const float nsn = ffrom(fbits(sn) ^ kSign), ncs = ffrom(fbits(cs) ^ kSign);
    float S, C;
    switch (k4) {
        case 0: S = sn; C = cs; break;
        case 1: S = cs; C = nsn; break;
        case 2: S = nsn; C = ncs; break;
        default: S = ncs; C = sn; break;
    }
    *s_out = (u & kSign) ? ffrom(fbits(S) ^ kSign) : S;
    *c_out = C;
}

// ---- ROPE: tsr_ref_rope (tsr_ref_vu.c:308-376), recurrence form without frequency factors: per
// token theta_0 = f32(pos), theta_(i+1) = FM(theta_i, TS); c_i = FM(M, COS), s_i = FM(M, SIN);
// pair (j0, j1): y0 = FS(FM(x0, c), FM(x1, s)), y1 = FA(FM(x0, s), FM(x1, c)); dims >= n_dims raw.
constexpr uint32_t kMaxHalf = 512;

__global__ void __launch_bounds__(256) rope_kernel(const float* x, uint32_t xs, float* y, uint32_t ys,
                                                   const int32_t* __restrict__ pos, uint32_t n_heads, uint32_t hd,
                                                   uint32_t nd, uint32_t neox, float ts, float m) {
    __shared__ float cs_c[kMaxHalf], cs_s[kMaxHalf];
    const uint32_t t = blockIdx.x, half = nd / 2u;
    if (threadIdx.x == 0) {
        float theta = __int2float_rn(pos[t]);
        for (uint32_t i = 0; i < half; ++i) {
            cs_c[i] = theta;
            theta = FM(theta, ts);
        }
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < half; i += blockDim.x) {
        float sn, cs;
        sincos_vu(cs_c[i], &sn, &cs);
        cs_c[i] = FM(m, cs);
        cs_s[i] = FM(m, sn);
    }
    __syncthreads();
    const float* xt = x + (size_t)t * xs;
    float* yt = y + (size_t)t * ys;
    for (uint32_t idx = threadIdx.x; idx < n_heads * half; idx += blockDim.x) {
        const uint32_t h = idx / half, i = idx - h * half;
        const uint32_t j0 = h * hd + (neox ? i : 2u * i), j1 = h * hd + (neox ? i + half : 2u * i + 1u);
        const float x0 = xt[j0], x1 = xt[j1], c = cs_c[i], s = cs_s[i];
        yt[j0] = canon(FS(FM(x0, c), FM(x1, s)));
        yt[j1] = canon(FA(FM(x0, s), FM(x1, c)));
    }
    if (nd < hd)
        for (uint32_t idx = threadIdx.x; idx < n_heads * (hd - nd); idx += blockDim.x) {
            const uint32_t h = idx / (hd - nd), j = h * hd + nd + (idx - h * (hd - nd));
            yt[j] = xt[j];
        }
}

// ROPE with the per-position c_i, s_i precomputed (the same values rope_kernel computes): one CTA
// per position fills row p of the tables; then rope_apply_kernel rotates from the table rows.
__global__ void __launch_bounds__(256) rope_table_kernel(uint32_t nd, float ts, float m, float* cs_tab, float* sn_tab) {
    __shared__ float phi[kMaxHalf];
    const uint32_t p = blockIdx.x, half = nd / 2u;
    if (threadIdx.x == 0) {
        float theta = __int2float_rn((int32_t)p);
        for (uint32_t i = 0; i < half; ++i) {
            phi[i] = theta;
            theta = FM(theta, ts);
        }
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < half; i += blockDim.x) {
        float sn, cs;
        sincos_vu(phi[i], &sn, &cs);
        cs_tab[(size_t)p * half + i] = FM(m, cs);
        sn_tab[(size_t)p * half + i] = FM(m, sn);
    }
}

__global__ void __launch_bounds__(256) rope_apply_kernel(const float* x, uint32_t xs, float* y, uint32_t ys,
                                                         const int32_t* __restrict__ pos, uint32_t n_heads, uint32_t hd,
                                                         uint32_t nd, uint32_t neox, const float* __restrict__ cs_tab,
                                                         const float* __restrict__ sn_tab) {
    const uint32_t t = blockIdx.x, half = nd / 2u;
    const float* ct = cs_tab + (size_t)pos[t] * half;
    const float* st = sn_tab + (size_t)pos[t] * half;
    const float* xt = x + (size_t)t * xs;
    float* yt = y + (size_t)t * ys;
    for (uint32_t idx = threadIdx.x; idx < n_heads * half; idx += blockDim.x) {
        const uint32_t h = idx / half, i = idx - h * half;
        const uint32_t j0 = h * hd + (neox ? i : 2u * i), j1 = h * hd + (neox ? i + half : 2u * i + 1u);
        const float x0 = xt[j0], x1 = xt[j1], c = ct[i], s = st[i];
        yt[j0] = canon(FS(FM(x0, c), FM(x1, s)));
        yt[j1] = canon(FA(FM(x0, s), FM(x1, c)));
    }
    if (nd < hd)
        for (uint32_t idx = threadIdx.x; idx < n_heads * (hd - nd); idx += blockDim.x) {
            const uint32_t h = idx / (hd - nd), j = h * hd + nd + (idx - h * (hd - nd));
            yt[j] = xt[j];
        }
}

// ROPE of q and k, then KVST of k and v: one CTA of 512 threads per (token, KV head g), which
// rotates the g-th group of q heads and k head g, then stores k and v head g. The rotation is
// rope_apply_kernel's, item by item, with each thread's loads issued before its stores (the rows
// are rotated in place); after the barrier one warp per 32-value block of k or v runs KVST
// (QACT A32, tsr_ref_at.c:244-264) exactly as kv_store_kernel.
constexpr uint32_t kRkThreads = 512;
constexpr uint32_t kRkBatch = 4;

__global__ void __launch_bounds__(kRkThreads) rope_kvst_kernel(RopeKvst a) {
    // a programmatic dependent launch: the next kernel (attention) may start its prologue now;
    // this one reads the projections only after the kernel that wrote them has finished
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t t = blockIdx.x, g = blockIdx.y, half = a.nd / 2u, tid = threadIdx.x;
    const uint32_t nkv = a.n_head_kv, nq = a.n_rot_heads - nkv, G = nq / nkv;
    const float* ct = a.cs_tab + (size_t)a.pos[t] * half;
    const float* st = a.sn_tab + (size_t)a.pos[t] * half;
    float* xt = a.qkv + (size_t)t * a.stride;
    const uint32_t items = (G + 1u) * half;               // q heads g G .. g G + G - 1, then k head g
    for (uint32_t i0 = tid; i0 < items; i0 += kRkBatch * kRkThreads) {
        float x0[kRkBatch], x1[kRkBatch], c[kRkBatch], s[kRkBatch];
        uint32_t j0[kRkBatch], j1[kRkBatch];
#pragma unroll
        for (uint32_t b = 0; b < kRkBatch; ++b) {
            const uint32_t idx = i0 + b * kRkThreads;
            if (idx < items) {
                const uint32_t lh = idx / half, i = idx - lh * half;
                const uint32_t h = lh < G ? g * G + lh : nq + g;
                j0[b] = h * a.hd + (a.neox ? i : 2u * i);
                j1[b] = h * a.hd + (a.neox ? i + half : 2u * i + 1u);
                x0[b] = xt[j0[b]];
                x1[b] = xt[j1[b]];
                c[b] = ct[i];
                s[b] = st[i];
            }
        }
#pragma unroll
        for (uint32_t b = 0; b < kRkBatch; ++b) {
            if (i0 + b * kRkThreads < items) {
                xt[j0[b]] = canon(FS(FM(x0[b], c[b]), FM(x1[b], s[b])));
                xt[j1[b]] = canon(FA(FM(x0[b], s[b]), FM(x1[b], c[b])));
            }
        }
    }
    // (nd < hd: the values past nd stay as they are, in place)
    __syncthreads();
    const uint32_t D = a.hd, nb = D / 32u, warp = tid >> 5, lane = tid & 31u;
    const int64_t cell = a.cells ? a.cells[t] : (int64_t)a.cell0 + t;
    if (cell < 0 || cell >= (int64_t)a.n_cells) {
        if (tid == 0) atomicCAS(a.err, 0u, 1u);           // a row index outside the cache: not stored
        return;
    }
    for (uint32_t wi = warp; wi < 2u * nb; wi += kRkThreads / 32u) {
        const bool vt = wi >= nb;
        const uint32_t k = 32u * (vt ? wi - nb : wi);      // the block's first value inside head g
        const float v = xt[(vt ? a.v_off : a.k_off) + g * D + k + lane];
        const uint32_t amax = __reduce_max_sync(0xFFFFFFFFu, amax_key(v));
        const float db = fdiv(ffrom(amax), 127.0f);
        const float id = (fbits(db) & ~kSign) ? frecip(db) : 0.0f;
        const size_t hc = (size_t)g * a.n_cells + (size_t)cell;
        (vt ? a.vq : a.kq)[kv_qoff(vt, g, a.n_cells, D, (size_t)cell, k + lane)] = (int8_t)round_away_sat8(fmul(daz(v), id));
        if (lane == 0) (vt ? a.vd : a.kd)[hc * (D / 32u) + k / 32u] = f2h(db);
    }
}

// ---- VOP (tsr_ref_vu.c:104-130): ADD FA(a, b), MUL FM(a, b), SILU FM(a, SIG(a)), SWIGLU
// FM(SILU(a), b); SIG(a) = RC(FA(1, EXPK(a, N1))) (tsr_ref_math.c:165-171)
__device__ __forceinline__ float silu_vu(float a) {
    const float e = expk(a, 1u, g_expk_t64, g_expk_lk);
    return FM(a, RC(fadd(1.0f, e)));
}

__global__ void vop_kernel(uint32_t func, const float* a, uint32_t as, const float* b, uint32_t bs, float* y, uint32_t ys,
                           uint32_t n) {
    const uint32_t r = blockIdx.y;
    const float* ar = a + (size_t)r * as;
    const float* br = b ? b + (size_t)r * bs : nullptr;
    float* yr = y + (size_t)r * ys;
    for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) {
        float v;
        switch (func) {
            case 0u: v = FA(ar[j], br[j]); break;
            case 2u: v = FM(ar[j], br[j]); break;
            case 6u: v = silu_vu(ar[j]); break;
            case 8u: v = FM(silu_vu(ar[2u * j]), ar[2u * j + 1u]); break;     // SWIGLU of interleaved (gate, up) pairs
            default: v = FM(silu_vu(ar[j]), br[j]); break;
        }
        yr[j] = canon(v);
    }
}

// ---- GET_ROWS of a quantized weight: tsr_dequant_row (tsr_ref.c:369-401): Q8_0 FM(d, f32(q)),
// Q4_K FS(FM(FM(d, f32(sc_j)), f32(q)), FM(dmin, f32(m_j))) per value of sub-block j.
__global__ void get_rows_kernel(uint32_t fmt, const uint8_t* __restrict__ qs, const uint8_t* __restrict__ meta,
                                uint32_t n_rows, uint32_t K, const int32_t* __restrict__ ids, float* y, uint32_t ys) {
    const uint32_t t = blockIdx.y;
    const int32_t id = ids[t];
    if (id < 0 || (uint32_t)id >= n_rows) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicCAS(&g_vu_error, 0u, 1u);
        return;
    }
    const Layout L{fmt, K};
    const uint32_t row = (uint32_t)id;
    float* yr = y + (size_t)t * ys;
    for (uint32_t k = blockIdx.x * blockDim.x + threadIdx.x; k < K; k += gridDim.x * blockDim.x) {
        float v;
        if (fmt == 0u) {
            const uint32_t b = k >> 5, l = k & 31u;
            const int8_t q = (int8_t)qs[L.qs_off(row, b, l >> 4) + (l & 15u)];
            const float d = h2f(*reinterpret_cast<const uint16_t*>(meta + L.meta_off(row, b)));
            v = FM(d, (float)q);
        } else {
            const uint32_t sb = k >> 8, j = (k >> 5) & 7u, l = k & 31u;
            const uint8_t* m = meta + L.meta_off(row, sb);
            const uint8_t* sc12 = m + 4;
            uint32_t sc, mn;
            if (j < 4u) {
                sc = sc12[j] & 63u;
                mn = sc12[j + 4u] & 63u;
            } else {
                sc = (sc12[j + 4u] & 15u) | ((sc12[j - 4u] >> 6) << 4);
                mn = (sc12[j + 4u] >> 4) | ((sc12[j] >> 6) << 4);
            }
            const uint32_t byte = 32u * (j >> 1) + l;                   // qs byte of the value
            const uint8_t qb = qs[L.qs_off(row, sb, byte >> 4) + (byte & 15u)];
            const uint32_t qv = (qb >> (4u * (j & 1u))) & 15u;
            const float d = h2f(*reinterpret_cast<const uint16_t*>(m)), dmin = h2f(*reinterpret_cast<const uint16_t*>(m + 2));
            v = FS(FM(FM(d, (float)sc), (float)qv), FM(dmin, (float)mn));
        }
        yr[k] = canon(v);
    }
}

}  // namespace

cudaError_t launch_rms_norm(const float* x, uint32_t xs, float* y, uint32_t ys, const float* w, uint32_t n, uint32_t rows,
                            float eps, float inv_n, cudaStream_t st) {
    size_t smem = (size_t)n * sizeof(float);
    if (smem > 200u * 1024u) return cudaErrorInvalidValue;
    const bool stage_w = w && 2u * smem <= 200u * 1024u;
    if (stage_w) smem *= 2u;
    static int done_dev[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && done_dev[dev] != dev + 1) {
        e = cudaFuncSetAttribute(rms_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        done_dev[dev] = dev + 1;
    }
    rms_norm_kernel<<<rows, kRedThreads, smem, st>>>(x, xs, y, ys, w, n, eps, inv_n, stage_w);
    return cudaGetLastError();
}

cudaError_t launch_rope_table(uint32_t n_pos, uint32_t nd, float ts, float m, float* cs_tab, float* sn_tab, cudaStream_t st) {
    if (nd / 2u > kMaxHalf || n_pos == 0) return cudaErrorInvalidValue;
    rope_table_kernel<<<n_pos, 256, 0, st>>>(nd, ts, m, cs_tab, sn_tab);
    return cudaGetLastError();
}

cudaError_t launch_rope_apply(const float* x, uint32_t xs, float* y, uint32_t ys, const int32_t* pos, uint32_t T,
                              uint32_t n_heads, uint32_t hd, uint32_t nd, uint32_t neox, const float* cs_tab,
                              const float* sn_tab, cudaStream_t st) {
    rope_apply_kernel<<<T, 256, 0, st>>>(x, xs, y, ys, pos, n_heads, hd, nd, neox, cs_tab, sn_tab);
    return cudaGetLastError();
}

cudaError_t launch_rope(const float* x, uint32_t xs, float* y, uint32_t ys, const int32_t* pos, uint32_t T, uint32_t n_heads,
                        uint32_t hd, uint32_t nd, uint32_t neox, float ts, float m, cudaStream_t st) {
    if (nd / 2u > kMaxHalf) return cudaErrorInvalidValue;
    rope_kernel<<<T, 256, 0, st>>>(x, xs, y, ys, pos, n_heads, hd, nd, neox, ts, m);
    return cudaGetLastError();
}

cudaError_t launch_rope_kvst(const RopeKvst& a, uint32_t T, cudaStream_t st) {
    if (T == 0) return cudaSuccess;
    if (a.nd / 2u > kMaxHalf || a.nd > a.hd || a.hd % 32u) return cudaErrorInvalidValue;
    // q heads then k heads are rotated, the q heads in n_head_kv equal groups, k right after q
    if (a.n_head_kv == 0 || a.n_rot_heads <= a.n_head_kv || (a.n_rot_heads - a.n_head_kv) % a.n_head_kv ||
        a.k_off != (a.n_rot_heads - a.n_head_kv) * a.hd)
        return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(T, a.n_head_kv);
    cfg.blockDim = dim3(kRkThreads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, rope_kvst_kernel, a);
}

cudaError_t launch_vop(uint32_t func, const float* a, uint32_t as, const float* b, uint32_t bs, float* y, uint32_t ys,
                       uint32_t n, uint32_t rows, cudaStream_t st) {
    const uint32_t per = 256u, blocks = (n + per - 1u) / per;
    vop_kernel<<<dim3(blocks < 64u ? blocks : 64u, rows), per, 0, st>>>(func, a, as, b, bs, y, ys, n);
    return cudaGetLastError();
}

cudaError_t launch_get_rows(uint32_t fmt, const uint8_t* qs, const void* meta, uint32_t n_rows, uint32_t K, const int32_t* ids,
                            uint32_t T, float* y, uint32_t ys, cudaStream_t st) {
    const uint32_t blocks = (K + 255u) / 256u;
    get_rows_kernel<<<dim3(blocks < 32u ? blocks : 32u, T), 256, 0, st>>>(fmt, qs, static_cast<const uint8_t*>(meta), n_rows, K,
                                                                        ids, y, ys);
    return cudaGetLastError();
}

cudaError_t vu_error(uint32_t* code, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(code, g_vu_error, sizeof(uint32_t));
    if (e != cudaSuccess || !clear || *code == 0u) return e;
    const uint32_t zero = 0u;
    return cudaMemcpyToSymbol(g_vu_error, &zero, sizeof(uint32_t));
}

}  // namespace tsrc
