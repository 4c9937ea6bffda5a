// tsrc_matvec.cu -- decode (small-T) Q8_0 / Q4_K MUL_MAT on sm_100a.
//
// Numerics: the reference's MVM row rule bit for bit (jwkim04/tesseract-npu
// sw/sim/tsr_ref.c:533-635): per block i an exact int32 sum, the term
// t_i = (d_w (*) Dx_i) (*) f32(isum_i) [Q4_K: minus (dmin (*) Dx_i) (*) f32(msum_i)], term i
// added in order into partial p[i mod 16] (from +0), then the fixed tree ((p0+p1)+(p2+p3))+...,
// then the MVM epilogue (addend / scale / softcap, tsr_sim.c:1648-1670).
//
// Structure (an HBM stream; tsrc_layout.cuh has the tiled weight layout):
//   - one CTA per SM owns a contiguous range of rows; at entry one thread asks the memory system
//     to move that whole range from HBM into L2 (cp.async.bulk.prefetch.L2: HBM -> L2 only, no
//     shared memory and no SM ingress used), so HBM streams at full rate from the first
//     microsecond, independently of how far the warps have got;
//   - warps read the weights from L2 with 128-bit non-allocating loads into registers, the next
//     unit's loads issued before the current unit is computed;
//   - a warp owns a pair of rows; lane L serves row L/16 and block 16 t + (L % 16) of tile t, so
//     it owns its block's whole integer sum (no cross-lane sums) and accumulates exactly partial
//     p[L % 16] of its row, tile by tile (the reference's order); the 16-partial tree is four
//     xor-shuffle levels inside each half-warp;
//   - the quantized activation sits in shared memory in the same chunk-major tiles, so the 16
//     lanes of a half-warp read 256 contiguous bytes (conflict-free) at immediate offsets; for one
//     token the CTA quantizes x itself (QACT fused; its loads are issued in batches), otherwise it
//     copies a QA image;
//   - the kernel lets the next launch on the stream start early (programmatic dependent launch:
//     its L2 prefetch overlaps this launch's tail) and waits for the previous one before it
//     touches the activation;
//   - fast path: if every nonzero activation scale Dx is >= 2^-79, every term and partial is 0 or
//     a multiple of 2^-126 of magnitude >= 2^-126 (|d_w| >= 2^-24 for a nonzero fp16), so no
//     result can be subnormal and the flush tests are skipped (a CTA-uniform choice; the values
//     are the same either way).
#include <algorithm>
#include <cstdlib>
#include <type_traits>

#include "tsrc_internal.h"
#include "tsrc_layout.cuh"
#include "tsrc_numerics.cuh"

namespace tsrc {

#ifndef TSRC_MV_WARPS
#define TSRC_MV_WARPS 16
#endif
// Warps per CTA. 16 warps, one CTA per SM: the bytes a warp keeps in flight from L2 (one unit
// ahead) bound the stream rate, so more warps per SM beat co-residency of two launches (8 warps,
// two CTAs an SM, measured 1.37x slower on the Q4_K 14336 x 4096 launch).
constexpr uint32_t kCWarps = TSRC_MV_WARPS;
constexpr uint32_t kThreads = kCWarps * 32;
constexpr int kCtasPerSm = kCWarps <= 8 ? 2 : 1;
constexpr uint32_t kSafeDx = 0x18000000u;           // 2^-79
constexpr uint32_t kPrefetchChunk = 64u * 1024u;    // bytes per L2 prefetch instruction

__device__ unsigned int g_mv_error;                 // first error code of any launch (0 = none; reserved)

// ---- mbarrier and bulk-copy helpers -----------------------------------------------------------
__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kCWarps * 32) : "memory"); }

// ---- integer dot products -----------------------------------------------------------------------
__device__ __forceinline__ int32_t dot16s(const uint4 w, const uint4 x, int32_t acc) {
    acc = __dp4a((int)w.x, (int)x.x, acc);
    acc = __dp4a((int)w.y, (int)x.y, acc);
    acc = __dp4a((int)w.z, (int)x.z, acc);
    acc = __dp4a((int)w.w, (int)x.w, acc);
    return acc;
}
__device__ __forceinline__ int32_t dp4a_us(uint32_t a, uint32_t b, int32_t c) {   // unsigned a x signed b
    int32_t d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int32_t dot16us(const uint4 w, const uint4 x, int32_t acc) {
    acc = dp4a_us(w.x, x.x, acc);
    acc = dp4a_us(w.y, x.y, acc);
    acc = dp4a_us(w.z, x.z, acc);
    acc = dp4a_us(w.w, x.w, acc);
    return acc;
}
__device__ __forceinline__ int32_t ubyte(uint32_t w, uint32_t i) { return (int32_t)__byte_perm(w, 0u, 0x4440u | i); }

template <class T>
__device__ __forceinline__ T lds(const uint8_t* p) { return *reinterpret_cast<const T*>(p); }

// f32 rules with the flush test only off the fast path.
template <bool SAFE>
__device__ __forceinline__ float mul_(float a, float b) { return SAFE ? __fmul_rn(a, b) : fmul(a, b); }
template <bool SAFE>
__device__ __forceinline__ float sub_(float a, float b) { return SAFE ? __fsub_rn(a, b) : fsub(a, b); }
template <bool SAFE>
__device__ __forceinline__ float add_(float a, float b) { return SAFE ? __fadd_rn(a, b) : fadd(a, b); }

__device__ __forceinline__ float tree16_lanes(float v) {
    v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
    v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
    v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 4));
    v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 8));
    return v;
}

// SILU of the vector unit (tsr_ref_vu.c SILU, as tsrc_vu.cu): FM(a, RC(FA(1, EXPK(a, N1))))
__device__ __forceinline__ float silu_mv(float a) {
    const float e = expk(a, 1u, g_expk_t64, g_expk_lk);
    return fmul(daz(a), daz(frecip(daz(fadd(1.0f, e)))));
}

__device__ __forceinline__ float mm_epilogue(float v, const MvArgs& a, uint32_t t, uint32_t n) {
    if (a.flags & kMmAdd) v = fadd(daz(a.add[(size_t)t * a.add_stride + n]), v);
    if (a.flags & kMmSoftcap)
        v = fmul(tanh_vu(fmul(v, a.s0), g_expk_t64, g_expk_lk), a.s1);
    else if (a.flags & kMmScale)
        v = fmul(v, a.s1);
    return canon(v);
}

// ---- the activation image in shared memory --------------------------------------------------------
// per token: quants in chunk-major tiles (Q8_0 512 B / Q4_K 4096 B per tile of 16 blocks: chunk c
// of block 16 t + k at tile + 256 c + 16 k); scales d[blocks] f32; Q4_K sub-block sums as int16,
// 8 per superblock (16 B) at tile t: 256 t + 16 k.
struct Qa {
    uint8_t* q;
    float* d;
    uint8_t* bs;
    uint32_t q_tok, d_tok, bs_tok;     // bytes per token
};

__host__ __device__ constexpr size_t a16(size_t n) { return (n + 15u) & ~(size_t)15u; }

struct Plan {                          // shared-memory plan of one launch (host and device agree)
    uint32_t qa_q, qa_d, qa_bs;        // per-token bytes of the activation image
    __host__ __device__ size_t qa_bytes(uint32_t T) const { return (size_t)T * (qa_q + qa_d + qa_bs); }
    __host__ __device__ size_t total(uint32_t T) const { return a16(qa_bytes(T)) + 4u * kCWarps; }   // + a flag per warp
};

__host__ __device__ inline Plan make_plan(uint32_t fmt, uint32_t K) {
    const Layout L{fmt, K};
    Plan p{};
    p.qa_q = L.tiles() * (fmt == 0 ? 512u : 4096u);
    p.qa_d = (uint32_t)a16((size_t)L.blocks() * 4u);
    p.qa_bs = fmt == 0 ? 0u : L.tiles() * 256u;
    return p;
}

// QACT A32 of one block (tsr_ref.c:472-487), one warp; v = the lane's value.
// Returns (uniform over the warp) whether the stored scale is 0 or >= 2^-79.
__device__ __forceinline__ bool qact32_to_smem(float v, uint32_t b, uint32_t lane, uint8_t* q, float* d) {
    const uint32_t amax = __reduce_max_sync(0xFFFFFFFFu, amax_key(v));
    const float db = fdiv(ffrom(amax), 127.0f);
    const float id = (fbits(db) & ~kSign) ? frecip(db) : 0.0f;
    q[(b >> 4) * 512u + 256u * (lane >> 4) + 16u * (b & 15u) + (lane & 15u)] = (uint8_t)round_away_sat8(fmul(daz(v), id));
    const float ds = h2f(f2h(db));
    if (lane == 0) d[b] = ds;
    const uint32_t u = fbits(ds) & ~kSign;
    return u == 0u || u >= kSafeDx;
}

// QACT A256 of one superblock (tsr_ref.c:488-518), one warp; lane l holds values 8 l .. 8 l + 7.
// Returns (uniform over the warp) whether the stored scale is 0 or >= 2^-79.
__device__ __forceinline__ bool qact256_to_smem(const float (&v)[8], uint32_t s, uint32_t lane, uint8_t* q, float* d, uint8_t* bs) {
    uint32_t best = 0;
    float mine = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t kk = amax_key(v[i]);
        if (kk > best) { best = kk; mine = v[i]; }
    }
    const uint32_t amax = __reduce_max_sync(0xFFFFFFFFu, best);
    const uint32_t owner = __reduce_min_sync(0xFFFFFFFFu, (best == amax && amax != 0u) ? lane : 32u);
    const float mx = __shfl_sync(0xFFFFFFFFu, daz(mine), owner & 31u);
    int32_t qv[8];
    float db = 0.0f;
    if (amax != 0u) {
        const float iscale = fdiv(-127.0f, mx);
#pragma unroll
        for (int i = 0; i < 8; ++i) qv[i] = round_even_sat8(fmul(iscale, daz(v[i])));
        db = frecip(iscale);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) qv[i] = 0;
    }
    uint32_t lo = 0, hi = 0;
    int32_t sum = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        lo |= ((uint32_t)qv[i] & 0xFFu) << (8 * i);
        hi |= ((uint32_t)qv[i + 4] & 0xFFu) << (8 * i);
        sum += qv[i] + qv[i + 4];
    }
    *reinterpret_cast<uint2*>(q + (s >> 4) * 4096u + 256u * (lane >> 1) + 16u * (s & 15u) + 8u * (lane & 1u)) = make_uint2(lo, hi);
    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);     // lanes 4j .. 4j+3: sub-block j (32 values)
    if ((lane & 3u) == 0)
        *reinterpret_cast<int16_t*>(bs + (s >> 4) * 256u + 16u * (s & 15u) + 2u * (lane >> 2)) = (int16_t)sum;
    if (lane == 0) d[s] = db;
    const uint32_t u = fbits(db) & ~kSign;
    return u == 0u || u >= kSafeDx;
}

// RMS_NORM's scale of the token x[0 .. K), computed exactly as the RMS_NORM kind's kernel does
// (tsrc_vu.cu; sw/sim/tsr_ref_vu.c): 128 partials of x^2 in element order (partial p takes
// x_p, x_p+128, ...), the pairwise tree over the lanes of each of four warps (levels 1-5), then
// ((q0 + q1) + (q2 + q3)); scale = RC(SQ(FA(FM(s, inv_n), eps))). Every CTA computes it (a few
// microseconds of one kernel saved per norm on a decode step); ends with a barrier of the CTA.
template <uint32_t NBAR>      // threads of the named barrier 1 (the warps that call this)
__device__ __forceinline__ float rms_scale_n(const MvArgs& a) {
    __shared__ float part[4];
    const uint32_t tid = threadIdx.x;
    if (tid < 128u) {
        float p = 0.0f;
        for (uint32_t j = tid; j < a.K; j += 128u) {
            const float v = daz(a.x[j]);
            p = fadd(p, fmul(v, v));
        }
#pragma unroll
        for (uint32_t off = 1; off < 32u; off <<= 1) p = fadd(p, __shfl_down_sync(0xFFFFFFFFu, p, off));
        if ((tid & 31u) == 0) part[tid >> 5] = p;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(NBAR) : "memory");
    const float s = fadd(fadd(part[0], part[1]), fadd(part[2], part[3]));
    const float m = fadd(daz(fmul(daz(s), daz(a.rms_inv_n))), daz(a.rms_eps));     // FA(FM(s, inv_n), eps)
    return frecip(daz(flush(__fsqrt_rn(daz(m)))));                                    // RC(SQ(.))
}
__device__ __forceinline__ float rms_scale(const MvArgs& a) { return rms_scale_n<kCWarps * 32>(a); }
// the normalised activation value j (raw = x_j; w_j of the norm weight, if any)
__device__ __forceinline__ float rms_apply(float raw, float wj, bool has_w, float sc) {
    const float v = fmul(daz(raw), sc);
    return canon(has_w ? fmul(daz(v), daz(wj)) : v);
}

// Fills the activation image. Returns (uniform over the CTA) whether every nonzero scale is
// >= 2^-79: each warp writes its own verdict to flags[warp] before the one barrier, and every
// thread reads all of them after it.
template <int FMT>
__device__ __forceinline__ bool stage_qa(const MvArgs& a, const Qa& s, const Layout& L, uint32_t* flags) {
    const uint32_t K = a.K, T = a.T, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const uint32_t nb = L.blocks();
    bool ok = true;
    if (a.x) {
        // one token: RMS_NORM (+ MUL) fused in front (the scale first, then each value as it loads)
        const bool rms = a.rms != 0u, rms_w = a.rms_w != nullptr;
        const float sc = rms ? rms_scale(a) : 0.0f;
        // each warp takes blocks i = warp + kCWarps j; the loads of a batch are all issued before
        // any of them is used (one memory latency per batch, not per block)
        if (FMT == 0) {
            constexpr uint32_t B = 8;
            for (uint32_t i0 = warp; i0 < T * nb; i0 += B * kCWarps) {
                float v[B], wv[B];
#pragma unroll
                for (uint32_t j = 0; j < B; ++j) {
                    const uint32_t i = i0 + j * kCWarps;
                    const uint32_t t = i / nb, b = i - t * nb;
                    v[j] = i < T * nb ? a.x[(size_t)t * a.x_stride + 32u * b + lane] : 0.0f;
                    wv[j] = (rms_w && i < T * nb) ? a.rms_w[32u * b + lane] : 0.0f;
                }
                if (rms) {
#pragma unroll
                    for (uint32_t j = 0; j < B; ++j) v[j] = rms_apply(v[j], wv[j], rms_w, sc);
                }
#pragma unroll
                for (uint32_t j = 0; j < B; ++j) {
                    const uint32_t i = i0 + j * kCWarps;
                    if (i < T * nb) {
                        const uint32_t t = i / nb, b = i - t * nb;
                        ok &= qact32_to_smem(v[j], b, lane, s.q + (size_t)t * s.q_tok,
                                             reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(s.d) + (size_t)t * s.d_tok));
                    }
                }
            }
        } else {
            constexpr uint32_t B = 2;
            for (uint32_t i0 = warp; i0 < T * nb; i0 += B * kCWarps) {
                float v[B][8];
#pragma unroll
                for (uint32_t j = 0; j < B; ++j) {
                    const uint32_t i = i0 + j * kCWarps;
                    const uint32_t t = i / nb, b = i - t * nb;
                    const float* src = a.x + (size_t)t * a.x_stride + 256u * b + 8u * lane;
                    if (i < T * nb && ((reinterpret_cast<uintptr_t>(src) & 15u) == 0)) {
                        const float4 f0 = reinterpret_cast<const float4*>(src)[0], f1 = reinterpret_cast<const float4*>(src)[1];
                        v[j][0] = f0.x; v[j][1] = f0.y; v[j][2] = f0.z; v[j][3] = f0.w;
                        v[j][4] = f1.x; v[j][5] = f1.y; v[j][6] = f1.z; v[j][7] = f1.w;
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; ++e) v[j][e] = i < T * nb ? src[e] : 0.0f;
                    }
                }
                if (rms) {
#pragma unroll
                    for (uint32_t j = 0; j < B; ++j) {
                        const uint32_t i = i0 + j * kCWarps;
                        if (i < T * nb) {
                            const uint32_t b = i % nb;
#pragma unroll
                            for (int e = 0; e < 8; ++e)
                                v[j][e] = rms_apply(v[j][e], rms_w ? a.rms_w[256u * b + 8u * lane + e] : 0.0f, rms_w, sc);
                        }
                    }
                }
#pragma unroll
                for (uint32_t j = 0; j < B; ++j) {
                    const uint32_t i = i0 + j * kCWarps;
                    if (i < T * nb) {
                        const uint32_t t = i / nb, b = i - t * nb;
                        ok &= qact256_to_smem(v[j], b, lane, s.q + (size_t)t * s.q_tok,
                                              reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(s.d) + (size_t)t * s.d_tok),
                                              s.bs + (size_t)t * s.bs_tok);
                    }
                }
            }
        }
    } else {
        // first batch: up to 4 chunks of q per thread, loaded before the arrive
        constexpr uint32_t B = 4;
        uint4 first[B];
#pragma unroll
        for (uint32_t j = 0; j < B; ++j) {
            const uint32_t i = tid + j * kCWarps * 32u;
            const uint32_t t = i / (K / 16u), c = i - t * (K / 16u);
            first[j] = i < T * (K / 16u) ? reinterpret_cast<const uint4*>(a.qx + (size_t)t * K)[c] : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (uint32_t j = 0; j < B; ++j) {
            const uint32_t i = tid + j * kCWarps * 32u;
            if (i < T * (K / 16u)) {
                const uint32_t t = i / (K / 16u), c = i - t * (K / 16u);
                uint32_t off;
                if (FMT == 0) {
                    const uint32_t b = c >> 1;
                    off = (b >> 4) * 512u + 256u * (c & 1u) + 16u * (b & 15u);
                } else {
                    const uint32_t sb = c >> 4;
                    off = (sb >> 4) * 4096u + 256u * (c & 15u) + 16u * (sb & 15u);
                }
                *reinterpret_cast<uint4*>(s.q + (size_t)t * s.q_tok + off) = first[j];
            }
        }
        for (uint32_t i = tid + B * kCWarps * 32u; i < T * (K / 16u); i += kCWarps * 32u) {    // the rest
            const uint32_t t = i / (K / 16u), c = i - t * (K / 16u);
            const uint4 v = reinterpret_cast<const uint4*>(a.qx + (size_t)t * K)[c];
            uint32_t off;
            if (FMT == 0) {
                const uint32_t b = c >> 1;
                off = (b >> 4) * 512u + 256u * (c & 1u) + 16u * (b & 15u);
            } else {
                const uint32_t sb = c >> 4;
                off = (sb >> 4) * 4096u + 256u * (c & 15u) + 16u * (sb & 15u);
            }
            *reinterpret_cast<uint4*>(s.q + (size_t)t * s.q_tok + off) = v;
        }
        for (uint32_t i = tid; i < T * nb; i += kCWarps * 32u) {
            const uint32_t t = i / nb, b = i - t * nb;
            const float dv = a.dx[i];
            reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(s.d) + (size_t)t * s.d_tok)[b] = dv;
            const uint32_t u = fbits(dv) & ~kSign;
            ok = ok && (u == 0u || u >= kSafeDx);
        }
        if (FMT == 1) {
            for (uint32_t i = tid; i < T * nb * 8u; i += kCWarps * 32u) {
                const uint32_t t = i / (nb * 8u), r = i - t * nb * 8u, sb = r >> 3, j = r & 7u;
                const int16_t* b16 = a.bsx + (size_t)t * (K / 16u) + 16u * sb + 2u * j;
                *reinterpret_cast<int16_t*>(s.bs + (size_t)t * s.bs_tok + (sb >> 4) * 256u + 16u * (sb & 15u) + 2u * j) =
                    (int16_t)((int32_t)b16[0] + (int32_t)b16[1]);
            }
        }
    }
    const uint32_t bad = __any_sync(0xFFFFFFFFu, !ok);
    if (lane == 0) flags[warp] = bad;
    consumer_sync();
    uint32_t any = 0;
#pragma unroll
    for (uint32_t w = 0; w < kCWarps; w += 4) {
        const uint4 f = *reinterpret_cast<const uint4*>(flags + w);
        any |= f.x | f.y | f.z | f.w;
    }
    return any == 0u;
}

// ---- per-lane units: loads into registers, then the math ----------------------------------------
// Q8_0: a unit is up to 4 tiles of one row pair; per lane 2 x 16 B of quants and one fp16 scale
// per tile. Q4_K: a unit is one tile; per lane its superblock's 8 x 16 B of quants and 16 B meta.
// A lane's pointers qp / mp address its block k of tile 0 of its row (row base + 16 k, + 2 k or
// 16 k in the meta row); tile t adds t x the tile's bytes, and a full tile's chunks are 256 B apart.
constexpr uint32_t kQ8Tiles = 4;

struct Q8Unit {
    uint4 w[kQ8Tiles][2];
    uint32_t d[kQ8Tiles];
};
struct Q4Unit {
    uint4 w[8];
    uint4 m;
};

__device__ __forceinline__ void load_unit(const uint8_t* qp, const uint8_t* mp, uint32_t nb, uint32_t t0, uint32_t k, Q8Unit& u) {
#pragma unroll
    for (uint32_t i = 0; i < kQ8Tiles; ++i) {
        const uint32_t t = t0 + i, b = 16u * t + k;
        if (b < nb) {
            const uint8_t* q = qp + (size_t)t * 512u;
            const uint32_t rest = nb - 16u * t;
            u.w[i][0] = ld_stream(q);
            u.w[i][1] = ld_stream(q + (rest >= 16u ? 256u : 16u * rest));
            u.d[i] = __ldg(reinterpret_cast<const uint16_t*>(mp + (size_t)t * 32u));
        }
    }
}

__device__ __forceinline__ void load_unit(const uint8_t* qp, const uint8_t* mp, uint32_t nsb, uint32_t t, uint32_t k, Q4Unit& u) {
    const uint32_t sb = 16u * t + k;
    if (sb < nsb) {
        const uint8_t* q = qp + (size_t)t * 2048u;
        const uint32_t rest = nsb - 16u * t;
        if (rest >= 16u) {
#pragma unroll
            for (uint32_t j = 0; j < 8; ++j) u.w[j] = ld_stream(q + 256u * j);
        } else {
            const uint32_t cs = 16u * rest;
#pragma unroll
            for (uint32_t j = 0; j < 8; ++j) u.w[j] = ld_stream(q + j * cs);
        }
        u.m = __ldg(reinterpret_cast<const uint4*>(mp + (size_t)t * 256u));
    }
}

template <bool SAFE, int MAXT>
__device__ __forceinline__ void compute_unit(const Q8Unit& u, const Qa& s, uint32_t nb, uint32_t T, uint32_t t0, uint32_t k,
                                             float (&p)[MAXT], int32_t* isum_out) {
#pragma unroll
    for (uint32_t i = 0; i < kQ8Tiles; ++i) {
        const uint32_t t = t0 + i, b = 16u * t + k;
        if (b >= nb) break;
        const float dw = h2f((uint16_t)u.d[i]);
#pragma unroll
        for (int tok = 0; tok < MAXT; ++tok) {
            if (tok < (int)T) {
                const uint8_t* xq = s.q + (size_t)tok * s.q_tok + (size_t)t * 512u + 16u * k;
                const int32_t isum = dot16s(u.w[i][1], lds<uint4>(xq + 256u), dot16s(u.w[i][0], lds<uint4>(xq), 0));
                if (isum_out && tok == 0) isum_out[b] = isum;
                const float Dx = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(s.d) + (size_t)tok * s.d_tok)[b];
                p[tok] = add_<SAFE>(p[tok], mul_<SAFE>(mul_<SAFE>(dw, Dx), i2f(isum)));
            }
        }
    }
}

template <bool SAFE, int MAXT>
__device__ __forceinline__ void compute_unit(const Q4Unit& u, const Qa& s, uint32_t nsb, uint32_t T, uint32_t t, uint32_t k,
                                             float (&p)[MAXT], int32_t* isum_out) {
    const uint32_t sb = 16u * t + k;
    if (sb >= nsb) return;
    const uint32_t sc_lo = u.m.y & 0x3F3F3F3Fu, mn_lo = u.m.z & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (u.m.w & 0x0F0F0F0Fu) | ((u.m.y >> 2) & 0x30303030u);
    const uint32_t mn_hi = ((u.m.w >> 4) & 0x0F0F0F0Fu) | ((u.m.z >> 2) & 0x30303030u);
    const float dw = h2f((uint16_t)(u.m.x & 0xFFFFu)), dmw = h2f((uint16_t)(u.m.x >> 16));
#pragma unroll
    for (int tok = 0; tok < MAXT; ++tok) {
        if (tok < (int)T) {
            const uint8_t* xq = s.q + (size_t)tok * s.q_tok + (size_t)t * 4096u + 16u * k;
            int32_t S[8];
#pragma unroll
            for (int c = 0; c < 4; ++c) {          // qs bytes 32c .. 32c+31 = chunks 2c, 2c+1
                const uint4 a0 = u.w[2 * c], a1 = u.w[2 * c + 1];
                const uint4 l0 = make_uint4(a0.x & 0x0F0F0F0Fu, a0.y & 0x0F0F0F0Fu, a0.z & 0x0F0F0F0Fu, a0.w & 0x0F0F0F0Fu);
                const uint4 l1 = make_uint4(a1.x & 0x0F0F0F0Fu, a1.y & 0x0F0F0F0Fu, a1.z & 0x0F0F0F0Fu, a1.w & 0x0F0F0F0Fu);
                const uint4 h0 = make_uint4(a0.x & 0xF0F0F0F0u, a0.y & 0xF0F0F0F0u, a0.z & 0xF0F0F0F0u, a0.w & 0xF0F0F0F0u);
                const uint4 h1 = make_uint4(a1.x & 0xF0F0F0F0u, a1.y & 0xF0F0F0F0u, a1.z & 0xF0F0F0F0u, a1.w & 0xF0F0F0F0u);
                S[2 * c] = dot16s(l1, lds<uint4>(xq + 256u * (4 * c + 1)), dot16s(l0, lds<uint4>(xq + 256u * (4 * c)), 0));
                S[2 * c + 1] =
                    dot16us(h1, lds<uint4>(xq + 256u * (4 * c + 3)), dot16us(h0, lds<uint4>(xq + 256u * (4 * c + 2)), 0)) >> 4;
            }
            int32_t isum = 0;
#pragma unroll
            for (uint32_t j = 0; j < 4; ++j) isum += ubyte(sc_lo, j) * S[j] + ubyte(sc_hi, j) * S[4 + j];
            const uint4 B = lds<uint4>(s.bs + (size_t)tok * s.bs_tok + (size_t)t * 256u + 16u * k);
            const int32_t msum = dp2a_hi(B.w, mn_hi, dp2a_lo(B.z, mn_hi, dp2a_hi(B.y, mn_lo, dp2a_lo(B.x, mn_lo, 0))));
            if (isum_out && tok == 0) {
                isum_out[2u * sb] = isum;
                isum_out[2u * sb + 1u] = msum;
            }
            const float Dx = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(s.d) + (size_t)tok * s.d_tok)[sb];
            const float t1v = mul_<SAFE>(mul_<SAFE>(dw, Dx), i2f(isum));
            const float t2v = mul_<SAFE>(mul_<SAFE>(dmw, Dx), i2f(msum));
            p[tok] = add_<SAFE>(p[tok], sub_<SAFE>(t1v, t2v));
        }
    }
}

// The row pairs of one warp: pair = warp, warp + kCWarps, ...; per pair the units in order, each
// unit's loads issued one unit ahead. Two unit buffers alternate roles (no register copies).
template <int FMT, int MAXT, bool SAFE>
__device__ __forceinline__ void stream_rows(const MvArgs& a, const Qa& qa, uint32_t r_begin, uint32_t r_end, uint32_t warp,
                                            uint32_t lane, float* team_rows) {
    using Unit = typename std::conditional<FMT == 0, Q8Unit, Q4Unit>::type;
    const Layout L{(uint32_t)FMT, a.K};
    constexpr uint32_t TPU = FMT == 0 ? kQ8Tiles : 1u;      // tiles per unit
    const uint32_t nb = L.blocks(), units = (L.tiles() + TPU - 1u) / TPU;
    const uint32_t k = lane & 15u, half = lane >> 4;
    const uint32_t n_pairs = (r_end - r_begin + 1u) / 2u;
    const size_t qrow = L.qs_row_bytes(), mrow = L.meta_row_bytes();
    const uint8_t* qbase = a.qs + 16u * k;
    const uint8_t* mbase = static_cast<const uint8_t*>(a.meta) + (FMT == 0 ? 2u : 16u) * k;
    const uint32_t isum_row = FMT == 0 ? nb : 2u * nb;

    uint32_t pair = warp, ui = 0;
    if (pair >= n_pairs) return;
    float p[MAXT];
#pragma unroll
    for (int t = 0; t < MAXT; ++t) p[t] = 0.0f;

    // loads unit ui of pair pr into u (nothing for a padding row)
    auto load = [&](Unit& u, uint32_t pr, uint32_t uix) {
        const uint32_t row = r_begin + 2u * pr + half;
        if (row < r_end) load_unit(qbase + (size_t)row * qrow, mbase + (size_t)row * mrow, nb, uix * TPU, k, u);
    };
    // computes cur (unit ui of pair) and loads the next unit into nxt; false when the warp is done
    auto step = [&](const Unit& cur, Unit& nxt) -> bool {
        const uint32_t row = r_begin + 2u * pair + half;
        const bool rv = row < r_end;
        uint32_t npair = pair, nui = ui + 1u;
        if (nui == units) { npair = pair + kCWarps; nui = 0; }
        if (npair < n_pairs) load(nxt, npair, nui);
        if (rv) compute_unit<SAFE, MAXT>(cur, qa, nb, a.T, ui * TPU, k, p, a.isum_out ? a.isum_out + (size_t)row * isum_row : nullptr);
        if (nui == 0) {                // the pair is complete: tree, epilogue, store
#pragma unroll
            for (int t = 0; t < MAXT; ++t) {
                if (t < (int)a.T) {
                    const float v = tree16_lanes(p[t]);
                    if (MAXT == 1 && a.swiglu_pairs) {            // gate (half 0) and up (half 1) rows
                        const float up = __shfl_sync(0xFFFFFFFFu, v, 16);
                        if (lane == 0 && rv) {
                            const float yv = canon(fmul(daz(silu_mv(canon(v))), daz(canon(up))));
                            if (a.team_world) team_rows[(row - r_begin) >> 1] = yv;
                            else a.y[row >> 1] = yv;
                        }
                    } else if (k == 0 && rv) {
                        const float yv = mm_epilogue(v, a, (uint32_t)t, row);
                        if (a.team_world) {                 // collected per CTA, sent in team_finish
                            team_rows[row - r_begin] = yv;
                        } else {
                            a.y[(size_t)t * a.y_stride + row] = yv;
                        }
                    }
                }
                p[t] = 0.0f;
            }
        }
        pair = npair;
        ui = nui;
        return pair < n_pairs;
    };
    Unit A, B;
    load(A, pair, 0);
    while (step(A, B) && step(B, A)) {
    }
}

// ---- fused all-gather: the end of a team launch ----------------------------------------------------
// Every CTA stores each of its rows into every rank's staging half (step parity) as ONE 64-bit
// word {value bits, step + 1}: a naturally aligned 8-byte store is single-copy atomic, so a reader
// that sees the tag sees the value with it, and no fence, flag or counter is needed between ranks.
// Every CTA of every rank then copies its share of the vector out, polling each word of the share
// (bounded) until it carries this step's tag. Double buffering by step parity keeps a rank that
// runs one step ahead from overwriting a half that a slower rank still reads: it cannot finish
// step s + 1 (and so start writing step s + 2 into half s & 1) before every rank has stored its
// rows of step s + 1, which a rank does only after its launch of step s has completed. The step
// count advances when the launch's last CTA counts itself done (every CTA reads it at entry).
// A word that never arrives records error code 2 (tsrc_sync reports it) and the launch ends.
constexpr uint32_t kTeamSpin = 1u << 22;             // x ~100 ns: a peer absent for ~0.4 s is an error

__device__ __forceinline__ void st_relaxed_sys64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// step: the team step this launch read after its wait for the previous kernel; or, with step_smem,
// the shared-memory word where one thread stored it (read after the barrier)
__device__ __forceinline__ void team_finish(const MvArgs& a, uint32_t step, const uint32_t* step_smem, const float* rows,
                                            uint32_t r_begin, uint32_t r_end) {
    __syncthreads();                                     // the CTA's rows (and step_smem) are in shared memory
    if (step_smem) step = *step_smem;
    const unsigned long long tag = (unsigned long long)(step + 1u) << 32;
    const size_t o = (size_t)(step & 1u) * a.team_half + a.team_row0 + r_begin;
    for (uint32_t r = 0; r < a.team_world; ++r)
        for (uint32_t i = threadIdx.x; i < r_end - r_begin; i += blockDim.x)
            st_relaxed_sys64(a.team_y[r] + o + i, tag | __float_as_uint(rows[i]));
    // this CTA's share of the gathered vector
    const unsigned long long* src = a.team_y[a.team_rank] + (size_t)(step & 1u) * a.team_half;
    const uint32_t n = a.team_n, share = (n + gridDim.x - 1u) / gridDim.x, i0 = blockIdx.x * share;
    const uint32_t i1 = min(n, i0 + share);
    bool gave_up = false;
    for (uint32_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        unsigned long long w = ld_relaxed_sys64(src + i);
        uint32_t it = 0;
        while ((w & 0xFFFFFFFF00000000ull) != tag && !gave_up) {
            if (++it >= kTeamSpin) {
                gave_up = true;
                atomicCAS(&g_mv_error, 0u, 2u);
            }
            __nanosleep(64);
            w = ld_relaxed_sys64(src + i);
        }
        a.y[i] = __uint_as_float((uint32_t)w);
    }
    // the step count: every CTA has read it at entry before the last one counts itself done
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(a.team_state + 1, 1u) + 1u == gridDim.x) {
        a.team_state[1] = 0u;
        a.team_state[0] = step + 1u;
    }
}

// The same exchange for plain vectors: T token rows, each of n values of which this rank holds
// [offset, offset + n_local). Token t's row sits at words [t n, t n + n) of the staging half. Every
// CTA stores its share of this rank's values into every rank's staging half as tagged words, then
// copies its share of all T n words out.
__global__ void __launch_bounds__(256) team_gather_kernel(TeamGather g) {
    const uint32_t step = *reinterpret_cast<volatile uint32_t*>(g.team_state);
    const unsigned long long tag = (unsigned long long)(step + 1u) << 32;
    const size_t half = (size_t)(step & 1u) * g.half;
    const uint32_t nl = g.T * g.n_local;
    const uint32_t ls = (nl + gridDim.x - 1u) / gridDim.x, l0 = blockIdx.x * ls, l1 = min(nl, l0 + ls);
    for (uint32_t r = 0; r < g.world; ++r)
        for (uint32_t k = l0 + threadIdx.x; k < l1; k += blockDim.x) {
            const uint32_t t = k / g.n_local, i = k - t * g.n_local;
            st_relaxed_sys64(g.team_y[r] + half + (size_t)t * g.n + g.offset + i,
                             tag | __float_as_uint(g.src[(size_t)t * g.src_stride + i]));
        }
    const unsigned long long* src = g.team_y[g.rank] + half;
    const uint32_t na = g.T * g.n;
    const uint32_t share = (na + gridDim.x - 1u) / gridDim.x, i0 = blockIdx.x * share, i1 = min(na, i0 + share);
    bool gave_up = false;
    for (uint32_t k = i0 + threadIdx.x; k < i1; k += blockDim.x) {
        unsigned long long w = ld_relaxed_sys64(src + k);
        uint32_t it = 0;
        while ((w & 0xFFFFFFFF00000000ull) != tag && !gave_up) {
            if (++it >= kTeamSpin) {
                gave_up = true;
                atomicCAS(&g_mv_error, 0u, 2u);
            }
            __nanosleep(64);
            w = ld_relaxed_sys64(src + k);
        }
        const uint32_t t = k / g.n, j = k - t * g.n;
        g.dst[(size_t)t * g.dst_stride + j] = __uint_as_float((uint32_t)w);
    }
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(g.team_state + 1, 1u) + 1u == gridDim.x) {
        g.team_state[1] = 0u;
        g.team_state[0] = step + 1u;
    }
}

cudaError_t launch_team_gather(const TeamGather& g, cudaStream_t st) {
    const uint32_t na = g.T * g.n;
    if (na == 0) return cudaSuccess;
    uint32_t blocks = (na + 1023u) / 1024u;
    blocks = blocks < 1u ? 1u : (blocks > 148u ? 148u : blocks);
    team_gather_kernel<<<blocks, 256, 0, st>>>(g);
    return cudaGetLastError();
}

// ---- the kernel ---------------------------------------------------------------------------------
template <int FMT, int MAXT>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) matvec_kernel(MvArgs a, Plan P, uint32_t rows_per_cta) {
    extern __shared__ __align__(128) uint8_t smem[];
    const Layout L{(uint32_t)FMT, a.K};
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const uint32_t r_begin = blockIdx.x * rows_per_cta;
    const uint32_t r_end = min(a.n_rows, r_begin + rows_per_cta);
    if (r_begin >= r_end) return;

    // weights of this CTA: HBM -> L2 now (read-only data: safe before the previous kernel ends);
    // the lanes of warp 0 issue the chunks in parallel, quants then meta
    if (warp == 0) {
        const uint8_t* q0 = a.qs + (size_t)r_begin * L.qs_row_bytes();
        const uint8_t* m0 = static_cast<const uint8_t*>(a.meta) + (size_t)r_begin * L.meta_row_bytes();
        const size_t qb = (size_t)(r_end - r_begin) * L.qs_row_bytes(), mb = (size_t)(r_end - r_begin) * L.meta_row_bytes();
        const size_t nq = (qb + kPrefetchChunk - 1u) / kPrefetchChunk, nm = (mb + kPrefetchChunk - 1u) / kPrefetchChunk;
        for (size_t c = lane; c < nq + nm; c += 32u) {
            const bool isq = c < nq;
            const size_t off = (isq ? c : c - nq) * kPrefetchChunk, tot = isq ? qb : mb;
            prefetch_l2((isq ? q0 : m0) + off, (uint32_t)(tot - off < kPrefetchChunk ? tot - off : kPrefetchChunk));
        }
    }
    asm volatile("griddepcontrol.launch_dependents;");

    // the activation (after the previous kernel on the stream has completed); no weight load is
    // issued before it, so the activation's loads do not queue behind them
    asm volatile("griddepcontrol.wait;" ::: "memory");
    Qa qa;
    qa.q = smem;
    qa.q_tok = P.qa_q;
    qa.d = reinterpret_cast<float*>(smem + (size_t)a.T * P.qa_q);
    qa.d_tok = P.qa_d;
    qa.bs = reinterpret_cast<uint8_t*>(qa.d) + (size_t)a.T * P.qa_d;
    qa.bs_tok = P.qa_bs;
    uint32_t* flags = reinterpret_cast<uint32_t*>(smem + a16(P.qa_bytes(a.T)));
    const uint32_t team_step = a.team_world ? *reinterpret_cast<volatile uint32_t*>(a.team_state) : 0u;
    float* team_rows = reinterpret_cast<float*>(smem + a16(P.qa_bytes(a.T)) + 4u * kCWarps);   // [rows_per_cta]
    if (stage_qa<FMT>(a, qa, L, flags)) stream_rows<FMT, MAXT, true>(a, qa, r_begin, r_end, warp, lane, team_rows);
    else stream_rows<FMT, MAXT, false>(a, qa, r_begin, r_end, warp, lane, team_rows);
    if (a.team_world)
        team_finish(a, team_step, nullptr, team_rows,
                    a.swiglu_pairs ? r_begin / 2u : r_begin, a.swiglu_pairs ? r_end / 2u : r_end);
}

// ---- one-token decode kernel: QACT fused, weights staged in shared memory by TMA ----------------
// The MUL_MAT of one token (the decode step) is the hot path. Its structure (measured on B200):
//   - a producer warp issues bulk copies (cp.async.bulk, the TMA engine; no multicast) of the
//     CTA's rows into shared memory before the kernel waits for the previous one on the stream
//     (weights are read-only): 32 rows per chunk, one mbarrier per chunk. When the CTA's share fits
//     (a Q4_K 14336 x 4096 matrix: 98 rows x 2304 B per SM) every chunk has its own place, else the
//     chunks (32 rows x one unit of tiles) cycle through a ring and are refilled as the consumers
//     release them. Bulk copies leave the SM's load/store path free: per-thread cp.async copies of
//     the same bytes slowed QACT's shuffles and shared-memory stores by 8x (7.3k against 0.9k
//     cycles for one superblock);
//   - 16 consumer warps run QACT (optionally after RMS_NORM) into the chunk-major image, then take
//     one row pair per chunk (lane L: row L / 16 of the pair, block / superblock L % 16 of each
//     tile, so a lane owns whole block sums and exactly partial p[L % 16] of its row, the
//     reference's term order); a lane keeps the activation of a one-unit row in registers;
//   - every consumer warp waits on every chunk in order (an mbarrier parity never aliases), and
//     every wait is bounded (about a second of SM clock; then error code 3, which tsrc_sync
//     reports, and the producer waits for its copies before the CTA ends);
//   - the 16-partial tree is four xor-shuffle levels inside each half-warp.
namespace dec {

// NW consumer warps + one producer warp; rows per chunk at most 2 NW (one pair per consumer warp).
// NW = 16 (x of a one-unit row in registers) or 24 (x read from shared memory); either uses a
// whole SM.
template <int NW>
struct Shape {
    static constexpr uint32_t kThreads = (NW + 1u) * 32u;
    static constexpr uint32_t kRowGroup = 2u * NW;
    static constexpr int kMinBlocks = NW <= 8 ? 2 : 1;
};
constexpr uint32_t kTpuQ8 = 4;                        // Q8_0 tiles per unit (Q4_K: 1)
constexpr long long kWaitCycles = 2000000000ll;       // ~1 s of SM clock

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
                 : "=r"(ok)
                 : "r"(su32(b)), "r"(parity)
                 : "memory");
    return ok != 0;
}
// false when about a second of SM clock passed without the phase completing
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity) {
    if (mbar_try(b, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try(b, parity))
        if (clock64() - t0 > kWaitCycles) return false;
    return true;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(su32(dst)),
                 "l"(src), "r"(bytes), "r"(su32(bar))
                 : "memory");
}

struct Geo {
    uint32_t nb, tiles, tpu, upp, qt, mt, qrow, mrow, bpb;
    Geo() = default;
    __host__ __device__ Geo(uint32_t fmt, uint32_t K) {
        nb = fmt == 0 ? K / 32u : K / 256u;
        tiles = (nb + 15u) / 16u;
        tpu = fmt == 0 ? kTpuQ8 : 1u;
        upp = (tiles + tpu - 1u) / tpu;
        qt = fmt == 0 ? 512u : 2048u;        // quant bytes of a full tile of one row
        mt = fmt == 0 ? 32u : 256u;          // meta bytes of a full tile of one row
        bpb = fmt == 0 ? 32u : 128u;         // quant bytes per block / superblock
        qrow = nb * bpb;
        mrow = fmt == 0 ? (nb * 2u + 15u) & ~15u : nb * 16u;
    }
};

// Shared-memory plan and geometry of one launch (computed on the host: no divisions on the device).
struct Plan {
    Geo g;
    uint32_t rpc;                 // rows per CTA (even)
    uint32_t ring;                // 0: the CTA's rows all resident; else chunk slots in the ring
    uint32_t R;                   // rows per chunk (even, <= 32: at most one pair per consumer warp)
    uint32_t tt;                  // tiles per chunk: every tile (whole rows, one contiguous copy) or one unit
    uint32_t kchunks;             // chunks per row group (1 for whole rows)
    uint32_t qstride, mstride;    // shared-memory bytes per row of a chunk
    uint32_t slot_bytes;          // ring: bytes of a slot (R rows)
    uint32_t qa_q, qa_d;          // QA image: quant bytes, scale bytes (Q4_K sums follow)
    uint32_t flags_off, team_off, slots_off, bars_off, nbars;
};

// QACT A256 of one superblock into the image (tsr_ref.c:488-518), one warp, lane l holds values
// 8 l .. 8 l + 7. When the largest |value| is at least 2^-100, DAZ of a value and the flush of its
// product cannot change the rounded result (|iscale * v| < 2^-19 for any subnormal v), so they are
// skipped. Returns (uniform over the warp) whether the stored scale is 0 or >= 2^-79.
__device__ __forceinline__ bool qact256_img(const float (&v)[8], uint32_t s, uint32_t lane, uint8_t* q, float* d, uint8_t* bs) {
    uint32_t best = 0;
    float mine = v[0];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t a = fbits(v[i]) & ~kSign;
        const uint32_t key = (a - 0x00800000u <= 0x7F000000u) ? a : 0u;   // |DAZ(v)| of a non-NaN v, else 0
        if (key > best) {
            best = key;
            mine = v[i];
        }
    }
    const uint32_t amax = __reduce_max_sync(0xFFFFFFFFu, best);
    const uint32_t owner = __reduce_min_sync(0xFFFFFFFFu, (best == amax && amax != 0u) ? lane : 32u);
    const float mx = __shfl_sync(0xFFFFFFFFu, mine, owner & 31u);       // normal or infinite when amax != 0
    int32_t qv[8];
    float db = 0.0f;
    if (amax != 0u) {
        const float iscale = fdiv(-127.0f, mx);
        if (amax >= 0x0D800000u) {
#pragma unroll
            for (int i = 0; i < 8; ++i) qv[i] = round_even_sat8(__fmul_rn(iscale, v[i]));
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) qv[i] = round_even_sat8(fmul(iscale, daz(v[i])));
        }
        db = frecip(iscale);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) qv[i] = 0;
    }
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        lo |= ((uint32_t)qv[i] & 0xFFu) << (8 * i);
        hi |= ((uint32_t)qv[i + 4] & 0xFFu) << (8 * i);
    }
    *reinterpret_cast<uint2*>(q + (s >> 4) * 4096u + 256u * (lane >> 1) + 16u * (s & 15u) + 8u * (lane & 1u)) = make_uint2(lo, hi);
    int32_t sum = __dp4a((int)lo, 0x01010101, __dp4a((int)hi, 0x01010101, 0));
    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);      // lanes 4j .. 4j+3: sub-block j (32 values)
    if ((lane & 3u) == 0)
        *reinterpret_cast<int16_t*>(bs + (s >> 4) * 256u + 16u * (s & 15u) + 2u * (lane >> 2)) = (int16_t)sum;
    if (lane == 0) d[s] = db;
    const uint32_t u = fbits(db) & ~kSign;
    return u == 0u || u >= kSafeDx;
}

// The image of the one token x (RMS_NORM + MUL in front when a.rms), by the consumer warps.
// Returns (uniform over them) whether every nonzero scale is >= 2^-79.
template <int FMT, int NW>
__device__ __forceinline__ bool stage_x1(const MvArgs& a, uint8_t* q, float* d, uint8_t* bs, uint32_t* flags) {
    constexpr uint32_t kWarps = NW;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t nb = FMT == 0 ? a.K / 32u : a.K / 256u;
    const bool rms = a.rms != 0u, rms_w = a.rms_w != nullptr;
    const float sc = rms ? rms_scale_n<NW * 32u>(a) : 0.0f;
    bool ok = true;
    if (FMT == 0) {
        constexpr uint32_t B = 8;
        for (uint32_t i0 = warp; i0 < nb; i0 += B * kWarps) {
            float v[B], wv[B];
#pragma unroll
            for (uint32_t j = 0; j < B; ++j) {
                const uint32_t i = i0 + j * kWarps;
                v[j] = i < nb ? a.x[32u * i + lane] : 0.0f;
                wv[j] = (rms_w && i < nb) ? a.rms_w[32u * i + lane] : 0.0f;
            }
#pragma unroll
            for (uint32_t j = 0; j < B; ++j) {
                const uint32_t i = i0 + j * kWarps;
                if (i < nb) ok &= qact32_to_smem(rms ? rms_apply(v[j], wv[j], rms_w, sc) : v[j], i, lane, q, d);
            }
        }
    } else {
        // a warp's superblocks B at a time: every load of the batch is issued before the first
        // quantization, so long rows (several superblocks per warp) wait for one load latency
        constexpr uint32_t B = 3;
        for (uint32_t i0 = warp; i0 < nb; i0 += B * kWarps) {
            float v[B][8];
#pragma unroll
            for (uint32_t j = 0; j < B; ++j) {
                const uint32_t i = i0 + j * kWarps;
                if (i >= nb) break;
                const float* src = a.x + 256u * i + 8u * lane;
                if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
                    const float4 f0 = reinterpret_cast<const float4*>(src)[0], f1 = reinterpret_cast<const float4*>(src)[1];
                    v[j][0] = f0.x; v[j][1] = f0.y; v[j][2] = f0.z; v[j][3] = f0.w;
                    v[j][4] = f1.x; v[j][5] = f1.y; v[j][6] = f1.z; v[j][7] = f1.w;
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[j][e] = src[e];
                }
            }
#pragma unroll
            for (uint32_t j = 0; j < B; ++j) {
                const uint32_t i = i0 + j * kWarps;
                if (i >= nb) break;
                if (rms) {
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        v[j][e] = rms_apply(v[j][e], rms_w ? a.rms_w[256u * i + 8u * lane + e] : 0.0f, rms_w, sc);
                }
                ok &= qact256_img(v[j], i, lane, q, d, bs);
            }
        }
    }
    const uint32_t bad = __any_sync(0xFFFFFFFFu, !ok);
    if (lane == 0) flags[warp] = bad;
    asm volatile("bar.sync 1, %0;" ::"n"(NW * 32) : "memory");
    uint32_t any = 0;
#pragma unroll
    for (uint32_t w = 0; w < kWarps; w += 4) {
        const uint4 f = *reinterpret_cast<const uint4*>(flags + w);
        any |= f.x | f.y | f.z | f.w;
    }
    return any == 0u;
}

// Registers of a lane's activation for a one-unit row (Q4_K: superblock k, 16 chunks + its 8
// sub-block sums + scale; Q8_0: block 16 t + k of tiles t < 4, 2 chunks + scale each).
template <int FMT>
struct XReg;
template <>
struct XReg<1> {
    uint4 x[16];
    uint4 B;
    float dx;
};
template <>
struct XReg<0> {
    uint4 x[8];
    float dx[4];
};

// One unit (tiles t0 .. t0 + tpu - 1) of the lane's row: rq / rm address the row's tile 0 in shared
// memory (tile t at rq + t * qt, rm + t * mt).
template <int FMT, bool XR, bool FULL, bool SAFE>
__device__ __forceinline__ void unit_math(const Geo& G, const uint8_t* rq, const uint8_t* rm, uint32_t t0, uint32_t k,
                                          const uint8_t* q, const float* d, const uint8_t* bs, const XReg<FMT>& xr, float& p,
                                          int32_t* isum_row) {
    if constexpr (FMT == 1) {
        const uint32_t sb = 16u * t0 + k;
        if (!FULL && sb >= G.nb) return;
        const uint32_t rest = G.nb - 16u * t0, cs = (FULL || rest >= 16u) ? 256u : 16u * rest;
        const uint8_t* sq = rq + (size_t)t0 * 2048u + 16u * k;
        uint4 w[8];
#pragma unroll
        for (uint32_t j = 0; j < 8; ++j) w[j] = lds<uint4>(sq + j * cs);
        const uint4 m = lds<uint4>(rm + (size_t)t0 * 256u + 16u * k);
        const uint32_t sc_lo = m.y & 0x3F3F3F3Fu, mn_lo = m.z & 0x3F3F3F3Fu;
        const uint32_t sc_hi = (m.w & 0x0F0F0F0Fu) | ((m.y >> 2) & 0x30303030u);
        const uint32_t mn_hi = ((m.w >> 4) & 0x0F0F0F0Fu) | ((m.z >> 2) & 0x30303030u);
        const uint8_t* xq = q + (size_t)t0 * 4096u + 16u * k;
        int32_t S[8];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint4 a0 = w[2 * c], a1 = w[2 * c + 1];
            const uint4 l0 = make_uint4(a0.x & 0x0F0F0F0Fu, a0.y & 0x0F0F0F0Fu, a0.z & 0x0F0F0F0Fu, a0.w & 0x0F0F0F0Fu);
            const uint4 l1 = make_uint4(a1.x & 0x0F0F0F0Fu, a1.y & 0x0F0F0F0Fu, a1.z & 0x0F0F0F0Fu, a1.w & 0x0F0F0F0Fu);
            const uint4 h0 = make_uint4(a0.x & 0xF0F0F0F0u, a0.y & 0xF0F0F0F0u, a0.z & 0xF0F0F0F0u, a0.w & 0xF0F0F0F0u);
            const uint4 h1 = make_uint4(a1.x & 0xF0F0F0F0u, a1.y & 0xF0F0F0F0u, a1.z & 0xF0F0F0F0u, a1.w & 0xF0F0F0F0u);
            const uint4 x0 = XR ? xr.x[4 * c] : lds<uint4>(xq + 256u * (4 * c));
            const uint4 x1 = XR ? xr.x[4 * c + 1] : lds<uint4>(xq + 256u * (4 * c + 1));
            const uint4 x2 = XR ? xr.x[4 * c + 2] : lds<uint4>(xq + 256u * (4 * c + 2));
            const uint4 x3 = XR ? xr.x[4 * c + 3] : lds<uint4>(xq + 256u * (4 * c + 3));
            S[2 * c] = dot16s(l1, x1, dot16s(l0, x0, 0));
            S[2 * c + 1] = dot16us(h1, x3, dot16us(h0, x2, 0)) >> 4;
        }
        int32_t isum = 0;
#pragma unroll
        for (uint32_t j = 0; j < 4; ++j) isum += ubyte(sc_lo, j) * S[j] + ubyte(sc_hi, j) * S[4 + j];
        const uint4 B = XR ? xr.B : lds<uint4>(bs + (size_t)t0 * 256u + 16u * k);
        const int32_t msum = dp2a_hi(B.w, mn_hi, dp2a_lo(B.z, mn_hi, dp2a_hi(B.y, mn_lo, dp2a_lo(B.x, mn_lo, 0))));
        if (isum_row) {
            isum_row[2u * sb] = isum;
            isum_row[2u * sb + 1u] = msum;
        }
        const float Dx = XR ? xr.dx : d[sb];
        const float dw = h2f((uint16_t)(m.x & 0xFFFFu)), dmw = h2f((uint16_t)(m.x >> 16));
        const float t1v = mul_<SAFE>(mul_<SAFE>(dw, Dx), i2f(isum));
        const float t2v = mul_<SAFE>(mul_<SAFE>(dmw, Dx), i2f(msum));
        p = add_<SAFE>(p, sub_<SAFE>(t1v, t2v));
    } else {
#pragma unroll
        for (uint32_t ti = 0; ti < kTpuQ8; ++ti) {
            const uint32_t t = t0 + ti, b = 16u * t + k;
            if (!FULL && t >= G.tiles) break;
            if (FULL || b < G.nb) {
                const uint32_t rest = G.nb - 16u * t, cs = (FULL || rest >= 16u) ? 256u : 16u * rest;
                const uint8_t* sq = rq + (size_t)t * 512u + 16u * k;
                const uint4 w0 = lds<uint4>(sq), w1 = lds<uint4>(sq + cs);
                const float dw = h2f(lds<uint16_t>(rm + 2u * b));
                const uint8_t* xq = q + (size_t)t * 512u + 16u * k;
                const uint4 x0 = XR ? xr.x[2 * ti] : lds<uint4>(xq);
                const uint4 x1 = XR ? xr.x[2 * ti + 1] : lds<uint4>(xq + 256u);
                const int32_t isum = dot16s(w1, x1, dot16s(w0, x0, 0));
                if (isum_row) isum_row[b] = isum;
                const float Dx = XR ? xr.dx[ti] : d[b];
                p = add_<SAFE>(p, mul_<SAFE>(mul_<SAFE>(dw, Dx), i2f(isum)));
            }
        }
    }
}

// The consumer warps' walk over the chunks: every chunk in order (row group rg, k-chunk kc), the
// warp's pair of the row group (pair 16 rg + warp) over the chunk's units.
// EPI 0: y[row] = the MUL_MAT epilogue (addend / scale / softcap); EPI 1: also the isum hook,
// SWIGLU pairs and the fused all-gather (a separate instance keeps the common case's registers free).
template <int FMT, bool XR, bool FULL, bool SAFE, bool RING, int EPI, int NW>
__device__ __forceinline__ bool consume(const MvArgs& a, const Plan& P, uint8_t* slots, uint64_t* full, uint64_t* empty,
                                        uint32_t r_begin, uint32_t n, const uint8_t* q, const float* d, const uint8_t* bs,
                                        const XReg<FMT>& xr, float* team_rows) {
    constexpr uint32_t kWarps = NW;
    const Geo& G = P.g;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, k = lane & 15u, h = lane >> 4;
    const uint32_t isum_stride = FMT == 0 ? G.nb : 2u * G.nb;
    const uint32_t npairs = (n + 1u) / 2u, ngroups = (n + P.R - 1u) / P.R;
    float pacc = 0.0f;
    uint32_t c = 0, s = 0, ph = 0;              // chunk, its slot, the slot's phase parity
    uint32_t row0 = 0;                           // first row of the row group
    for (uint32_t rg = 0; rg < ngroups; ++rg, row0 += P.R) {
        // the row group's pairs go to warps (pair mod 16): this warp's pair, if any
        const uint32_t p0 = row0 >> 1;
        const uint32_t pr = p0 + ((warp + kWarps - (p0 % kWarps)) % kWarps);
        const uint32_t r = 2u * pr + h;          // the lane's row within the CTA
        const bool has = pr < min(npairs, p0 + (P.R >> 1)), rv = r < n;
        for (uint32_t kc = 0; kc < P.kchunks; ++kc, ++c) {
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(full + s, ph))) {     // a warp-uniform outcome
                if (lane == 0) atomicCAS(&g_mv_error, 0u, 3u);
                return false;
            }
            if (has) {
                const uint8_t* rq;
                const uint8_t* rm;
                if (RING) {     // the chunk holds tiles kc tt .. of rows row0 ..: tile t at (t - kc tt) qt
                    const uint8_t* sl = slots + (size_t)s * P.slot_bytes;
                    rq = sl + (size_t)(r - row0) * P.qstride - (size_t)kc * P.tt * G.qt;
                    rm = sl + (size_t)P.R * P.qstride + (size_t)(r - row0) * P.mstride - (size_t)kc * P.tt * G.mt;
                } else {
                    rq = slots + (size_t)r * G.qrow;
                    rm = slots + (size_t)P.rpc * G.qrow + (size_t)r * G.mrow;
                }
                int32_t* isum_row = (EPI == 1 && a.isum_out && rv) ? a.isum_out + (size_t)(r_begin + r) * isum_stride : nullptr;
                if (XR) {
                    unit_math<FMT, XR, FULL, SAFE>(G, rq, rm, 0u, k, q, d, bs, xr, pacc, isum_row);
                } else {
                    const uint32_t t_end = RING ? min(G.tiles, (kc + 1u) * P.tt) : G.tiles;
                    for (uint32_t t0 = RING ? kc * P.tt : 0u; t0 < t_end; t0 += G.tpu)
                        unit_math<FMT, XR, FULL, SAFE>(G, rq, rm, t0, k, q, d, bs, xr, pacc, isum_row);
                }
            }
            if (RING) {
                __syncwarp();
                if (lane == 0) mbar_arrive(empty + s);
                if (++s == P.ring) {
                    s = 0;
                    ph ^= 1u;
                }
            } else {
                ++s;
            }
        }
        if (has) {                               // the pair is complete: tree, epilogue, store
            float v = pacc;
            v = add_<SAFE>(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
            v = add_<SAFE>(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
            v = add_<SAFE>(v, __shfl_xor_sync(0xFFFFFFFFu, v, 4));
            v = add_<SAFE>(v, __shfl_xor_sync(0xFFFFFFFFu, v, 8));
            pacc = 0.0f;
            const uint32_t row = r_begin + r;
            if (EPI == 1 && a.swiglu_pairs) {        // gate (half 0) and up (half 1) rows
                const float up = __shfl_sync(0xFFFFFFFFu, v, 16);
                if (lane == 0 && rv) {
                    const float yv = canon(fmul(daz(silu_mv(canon(v))), daz(canon(up))));
                    if (a.team_world) team_rows[pr] = yv;
                    else a.y[row >> 1] = yv;
                }
            } else if (k == 0 && rv) {
                const float yv = mm_epilogue(v, a, 0u, row);
                if (EPI == 1 && a.team_world) team_rows[r] = yv;
                else a.y[row] = yv;
            }
        }
    }
    return true;
}

// The producer warp: the chunks' bulk copies (lane i copies row i of a ring chunk; resident chunks
// are two contiguous copies), refills of ring slots as the consumers release them, and at the end
// a bounded wait for every copy it issued.
template <bool RING>
__device__ __forceinline__ void produce(const MvArgs& a, const Plan& P, uint8_t* slots, uint64_t* full, uint64_t* empty,
                                        uint32_t r_begin, uint32_t n) {
    const Geo& G = P.g;
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t ngroups = (n + P.R - 1u) / P.R, nch = ngroups * P.kchunks;
    const uint8_t* meta = static_cast<const uint8_t*>(a.meta);
    uint32_t issued = 0;
    bool ok = true;
    for (uint32_t c = 0; c < nch; ++c) {
        const uint32_t rg = c / P.kchunks, kc = c - rg * P.kchunks;
        const uint32_t row0 = P.R * rg, rows = min(P.R, n - row0);
        uint32_t s = c;
        if (RING) {
            s = c % P.ring;
            if (c >= P.ring && !__all_sync(0xFFFFFFFFu, mbar_wait(empty + s, ((c / P.ring) - 1u) & 1u))) {
                if (lane == 0) atomicCAS(&g_mv_error, 0u, 3u);
                ok = false;
                break;
            }
            uint8_t* sl = slots + (size_t)s * P.slot_bytes;
            if (P.kchunks == 1u) {               // whole rows: one contiguous copy of quants, one of meta
                if (lane == 0) {
                    mbar_expect_tx(full + s, rows * (G.qrow + G.mrow));
                    bulk_g2s(sl, a.qs + (size_t)(r_begin + row0) * G.qrow, rows * G.qrow, full + s);
                    bulk_g2s(sl + (size_t)P.R * G.qrow, meta + (size_t)(r_begin + row0) * G.mrow, rows * G.mrow, full + s);
                }
                issued = c + 1u;
                continue;
            }
            const uint32_t t0 = kc * P.tt, t1 = min(G.tiles, t0 + P.tt);
            const uint32_t qb = min(16u * t1, G.nb) * G.bpb - 16u * t0 * G.bpb;
            const uint32_t mb = G.tpu == 1u ? (min(16u * t1, G.nb) - 16u * t0) * 16u
                                            : ((min(16u * t1, G.nb) - 16u * t0) * 2u + 15u) & ~15u;
            if (lane == 0) mbar_expect_tx(full + s, rows * (qb + mb));
            __syncwarp();
            if (lane < rows) {                   // one unit of each row: lane i copies row i
                const size_t grow = r_begin + row0 + lane;
                bulk_g2s(sl + (size_t)lane * P.qstride, a.qs + grow * G.qrow + (size_t)t0 * G.qt, qb, full + s);
                bulk_g2s(sl + (size_t)P.R * P.qstride + (size_t)lane * P.mstride, meta + grow * G.mrow + (size_t)t0 * G.mt, mb,
                         full + s);
            }
        } else if (lane == 0) {
            mbar_expect_tx(full + s, rows * (G.qrow + G.mrow));
            bulk_g2s(slots + (size_t)row0 * G.qrow, a.qs + (size_t)(r_begin + row0) * G.qrow, rows * G.qrow, full + s);
            bulk_g2s(slots + (size_t)P.rpc * G.qrow + (size_t)row0 * G.mrow, meta + (size_t)(r_begin + row0) * G.mrow,
                     rows * G.mrow, full + s);
        }
        issued = c + 1u;
    }
    // the CTA must not end while a copy is still writing its shared memory
    const uint32_t first = RING ? (issued > P.ring ? issued - P.ring : 0u) : 0u;
    for (uint32_t c = first; c < issued; ++c) {
        const uint32_t s = RING ? c % P.ring : c, ph = RING ? (c / P.ring) & 1u : 0u;
        if (!mbar_wait(full + s, ph)) {
            if (lane == 0) atomicCAS(&g_mv_error, 0u, 3u);
            break;
        }
    }
    (void)ok;
}

template <int FMT, bool XR, bool FULL, bool RING, int EPI, int NW>
__global__ void __launch_bounds__(Shape<NW>::kThreads, Shape<NW>::kMinBlocks) dec_kernel(MvArgs a, Plan P) {
    constexpr uint32_t kWarps = NW;
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u, k = lane & 15u;
    if (EPI == 0 && a.moe_pairs) {
        // MUL_MAT_ID: the expert ids come from the previous kernel, so every warp (the producer
        // included) waits for it before the expert's rows are known
        asm volatile("griddepcontrol.wait;" ::: "memory");
        const uint32_t p = blockIdx.y, t = p / a.n_used, j = p - t * a.n_used;
        const int32_t e = a.ids[(size_t)t * a.ids_stride + j];
        if (e < 0 || (uint32_t)e >= a.n_exp) {
            if (tid == 0) atomicCAS(&g_mv_error, 0u, 5u);     // an expert id outside the weight: not computed
            return;
        }
        a.qs += (size_t)e * a.n_rows * P.g.qrow;
        a.meta = static_cast<const uint8_t*>(a.meta) + (size_t)e * a.n_rows * P.g.mrow;
        a.x += (size_t)t * a.x_tok + (size_t)(j % a.x_slots) * a.x_slot;
        a.y += (size_t)t * a.y_tok + (size_t)j * a.y_slot;
    }
    const uint32_t r_begin = blockIdx.x * P.rpc;
    if (r_begin >= a.n_rows) return;
    const uint32_t n = min(a.n_rows - r_begin, P.rpc);
    uint8_t* slots = smem + P.slots_off;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + P.bars_off);
    uint64_t* empty = full + P.nbars;
    if (tid == 0) {
        for (uint32_t i = 0; i < P.nbars; ++i) {
            mbar_init(full + i, 1u);
            if (RING) mbar_init(empty + i, kWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    asm volatile("griddepcontrol.launch_dependents;");
    uint32_t* flags = reinterpret_cast<uint32_t*>(smem + P.flags_off);
    float* team_rows = reinterpret_cast<float*>(smem + P.team_off);
    if (warp == kWarps) {
        produce<RING>(a, P, slots, full, empty, r_begin, n);        // weights only: no wait for the previous kernel
    } else {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        // the team step, read only once the previous kernel (possibly a team launch that advances
        // it) has completed; the producer warp, which never waits, takes it from shared memory
        if (EPI == 1 && a.team_world && tid == 0) flags[NW] = *reinterpret_cast<volatile uint32_t*>(a.team_state);
        uint8_t* q = smem;
        float* d = reinterpret_cast<float*>(smem + P.qa_q);
        uint8_t* bs = smem + P.qa_q + P.qa_d;
        const bool safe = stage_x1<FMT, NW>(a, q, d, bs, flags);
        XReg<FMT> xr;
        if (XR) {
            if constexpr (FMT == 1) {
#pragma unroll
                for (int c = 0; c < 16; ++c) xr.x[c] = lds<uint4>(q + 16u * k + 256u * c);
                xr.B = lds<uint4>(bs + 16u * k);
                xr.dx = d[k];
            } else {
#pragma unroll
                for (uint32_t t = 0; t < kTpuQ8; ++t) {      // the image holds P.g.tiles tiles
                    if (t < P.g.tiles) {
                        xr.x[2 * t] = lds<uint4>(q + t * 512u + 16u * k);
                        xr.x[2 * t + 1] = lds<uint4>(q + t * 512u + 256u + 16u * k);
                        xr.dx[t] = d[16u * t + k];
                    }
                }
            }
        }
        if (safe) consume<FMT, XR, FULL, true, RING, EPI, NW>(a, P, slots, full, empty, r_begin, n, q, d, bs, xr, team_rows);
        else consume<FMT, XR, FULL, false, RING, EPI, NW>(a, P, slots, full, empty, r_begin, n, q, d, bs, xr, team_rows);
    }
    if (EPI == 1 && a.team_world)
        team_finish(a, 0u, flags + NW, team_rows, a.swiglu_pairs ? r_begin / 2u : r_begin,
                    a.swiglu_pairs ? (r_begin + n) / 2u : r_begin + n);
}

}  // namespace dec

// ---- host side ------------------------------------------------------------------------------------
size_t mv_smem_bytes(uint32_t fmt, uint32_t K, uint32_t T) { return make_plan(fmt, K).total(T); }

// One flag set per kernel instance and device (the template arguments make each instance's
// statics distinct).
template <int FMT, int MAXT>
static cudaError_t allow_smem() {
    static int done_dev[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && done_dev[dev] == dev + 1) return cudaSuccess;
    e = cudaFuncSetAttribute(matvec_kernel<FMT, MAXT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(200u * 1024u));
    if (e == cudaSuccess && dev < 64) done_dev[dev] = dev + 1;
    return e;
}

static int g_num_sms[64];

template <int FMT, int MAXT>
static cudaError_t launch_t(const MvArgs& a, cudaStream_t st) {
    const Plan P = make_plan(FMT, a.K);
    size_t smem = P.total(a.T);
    cudaError_t e = allow_smem<FMT, MAXT>();
    if (e != cudaSuccess) return e;
    int dev = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if (dev < 64 && g_num_sms[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        g_num_sms[dev] = n > 0 ? n : 148;
    }
    const uint32_t sms = dev < 64 ? (uint32_t)g_num_sms[dev] : 148u;
    // contiguous row ranges of even length, one CTA per SM
    uint32_t rpc = (a.n_rows + sms - 1u) / sms;
    rpc = (rpc + 1u) & ~1u;
    const uint32_t blocks = (a.n_rows + rpc - 1u) / rpc;
    if (a.team_world) smem += 4u * rpc;                       // the CTA's rows before they are sent
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, matvec_kernel<FMT, MAXT>, a, P, rpc);
}

template <int FMT>
static cudaError_t launch_fmt(const MvArgs& a, cudaStream_t st) {
    if (a.T <= 1) return launch_t<FMT, 1>(a, st);
    if (a.T <= 2) return launch_t<FMT, 2>(a, st);
    if (a.T <= 4) return launch_t<FMT, 4>(a, st);
    return launch_t<FMT, kMvMaxT>(a, st);
}

// ---- the one-token decode kernel: plan and launch ----
static int g_smem_optin[64];
static int g_smem_sm[64];

template <int FMT, bool XR, bool FULL, bool RING, int EPI, int NW>
static cudaError_t dec_launch(const MvArgs& a, const dec::Plan& P, uint32_t blocks, size_t smem, int dev, cudaStream_t st) {
    static int done_dev[64];
    if (dev < 64 && done_dev[dev] != dev + 1) {
        cudaError_t e = cudaFuncSetAttribute(dec::dec_kernel<FMT, XR, FULL, RING, EPI, NW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             g_smem_optin[dev]);
        if (e != cudaSuccess) return e;
        done_dev[dev] = dev + 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks, a.moe_pairs ? a.moe_pairs : 1u);
    cfg.blockDim = dim3(dec::Shape<NW>::kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, dec::dec_kernel<FMT, XR, FULL, RING, EPI, NW>, a, P);
}

template <int FMT, bool XR, bool FULL, int NW>
static cudaError_t dec_launch_ring(const MvArgs& a, const dec::Plan& P, uint32_t blocks, size_t smem, int dev, cudaStream_t st) {
    const bool general = a.isum_out || a.swiglu_pairs || a.team_world;
    if (P.ring) return general ? dec_launch<FMT, XR, FULL, true, 1, NW>(a, P, blocks, smem, dev, st)
                               : dec_launch<FMT, XR, FULL, true, 0, NW>(a, P, blocks, smem, dev, st);
    return general ? dec_launch<FMT, XR, FULL, false, 1, NW>(a, P, blocks, smem, dev, st)
                   : dec_launch<FMT, XR, FULL, false, 0, NW>(a, P, blocks, smem, dev, st);
}

// One token with QACT fused (a.x set): rows split evenly over the SMs in pairs; the CTA's rows all
// resident in shared memory when they fit its budget, else chunks of whole rows (or of one unit of
// 2 NW rows, for rows too long for three chunks) through a ring.
template <int NW>
static cudaError_t launch_dec_nw(uint32_t fmt, const MvArgs& a, int dev, uint32_t sms, cudaStream_t st) {
    using S = dec::Shape<NW>;
    const dec::Geo G(fmt, a.K);
    dec::Plan P{};
    P.g = G;
    P.rpc = (a.n_rows + sms - 1u) / sms;
    P.rpc = (P.rpc + 1u) & ~1u;
    const uint32_t blocks = (a.n_rows + P.rpc - 1u) / P.rpc;
    P.qa_q = G.tiles * (fmt == 0 ? 512u : 4096u);
    P.qa_d = (uint32_t)a16((size_t)G.nb * 4u);
    const uint32_t qa_bs = fmt == 0 ? 0u : G.tiles * 256u;
    P.flags_off = (uint32_t)a16((size_t)P.qa_q + P.qa_d + qa_bs);
    P.team_off = P.flags_off + 4u * NW + 16u;           // NW warp flags, then the team step
    const uint32_t team_bytes = a.team_world ? 4u * P.rpc : 0u;
    P.slots_off = (P.team_off + team_bytes + 127u) & ~127u;
    // the CTA's budget: the opt-in maximum, or half an SM's shared memory for two CTAs per SM
    const size_t budget = S::kMinBlocks == 1 ? (size_t)g_smem_optin[dev] : (size_t)g_smem_sm[dev] / 2u - 1024u - 256u;
    const size_t row_bytes = (size_t)G.qrow + G.mrow;
    const size_t resident = (size_t)P.rpc * row_bytes;
    const uint32_t ngroups = (P.rpc + S::kRowGroup - 1u) / S::kRowGroup;
    if (P.slots_off + 256u > budget) return cudaErrorInvalidValue;
    size_t slots_end;
    if (P.slots_off + resident + 16u * ngroups <= budget) {
        P.ring = 0;                              // the CTA's rows all resident
        P.R = S::kRowGroup;
        P.tt = G.tiles;
        P.kchunks = 1;
        P.qstride = G.qrow;
        P.mstride = G.mrow;
        P.nbars = ngroups;
        slots_end = P.slots_off + resident;
    } else {
        const size_t room = budget - P.slots_off - 256u;
        // whole-row chunks (contiguous copies) if three of at least two rows fit, else one unit of
        // 2 NW rows per chunk (a copy per row)
        uint32_t R = (uint32_t)std::min<size_t>(S::kRowGroup, room / (3u * row_bytes)) & ~1u;
        if (R >= 2u) {
            P.R = R;
            P.tt = G.tiles;
            P.kchunks = 1;
            P.qstride = G.qrow;
            P.mstride = G.mrow;
        } else {
            P.R = S::kRowGroup;
            P.tt = std::min(G.tpu, G.tiles);
            P.kchunks = (G.tiles + P.tt - 1u) / P.tt;
            P.qstride = P.tt * G.qt;
            P.mstride = P.tt * G.mt;
        }
        P.slot_bytes = P.R * (P.qstride + P.mstride);
        if (2u * (size_t)P.slot_bytes > room) return cudaErrorInvalidValue;
        P.ring = (uint32_t)std::min<size_t>(8u, room / P.slot_bytes);
        P.nbars = P.ring;
        slots_end = P.slots_off + (size_t)P.ring * P.slot_bytes;
    }
    P.bars_off = (uint32_t)((slots_end + 15u) & ~(size_t)15u);
    const size_t smem = P.bars_off + 16u * (size_t)P.nbars;
    // every unit of every row complete (no partial tile, no missing tile of a unit)
    const bool full = (G.nb % (16u * G.tpu)) == 0;
    const bool xr = fmt == 0 ? G.tiles <= dec::kTpuQ8 : G.tiles == 1;
    if constexpr (NW == 16) {       // x in registers needs the register budget of 17 warps
        if (fmt == 0 && xr) return full ? dec_launch_ring<0, true, true, NW>(a, P, blocks, smem, dev, st) : dec_launch_ring<0, true, false, NW>(a, P, blocks, smem, dev, st);
        if (fmt == 1 && xr) return full ? dec_launch_ring<1, true, true, NW>(a, P, blocks, smem, dev, st) : dec_launch_ring<1, true, false, NW>(a, P, blocks, smem, dev, st);
    }
    if (fmt == 0) return full ? dec_launch_ring<0, false, true, NW>(a, P, blocks, smem, dev, st) : dec_launch_ring<0, false, false, NW>(a, P, blocks, smem, dev, st);
    return full ? dec_launch_ring<1, false, true, NW>(a, P, blocks, smem, dev, st) : dec_launch_ring<1, false, false, NW>(a, P, blocks, smem, dev, st);
}

static cudaError_t launch_dec(uint32_t fmt, const MvArgs& a, cudaStream_t st) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 64) return cudaErrorInvalidDevice;
    if (g_num_sms[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        g_num_sms[dev] = n > 0 ? n : 148;
    }
    if (g_smem_optin[dev] == 0) {
        int n = 0, m = 0;
        e = cudaDeviceGetAttribute(&n, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&m, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
        if (e != cudaSuccess) return e;
        g_smem_sm[dev] = m;
        g_smem_optin[dev] = n - 1024;          // room for the kernel's static shared memory
    }
    // rows whose activation slice fits a lane's registers (one Q4_K tile, up to four Q8_0 tiles) run
    // 16 consumer warps with x in registers; longer rows read x from shared memory, and then 24
    // warps (fewer registers each) keep more row pairs in flight
    const dec::Geo G(fmt, a.K);
    const bool xr = fmt == 0 ? G.tiles <= dec::kTpuQ8 : G.tiles == 1;
    if (!xr) return launch_dec_nw<24>(fmt, a, dev, (uint32_t)g_num_sms[dev], st);
    return launch_dec_nw<16>(fmt, a, dev, (uint32_t)g_num_sms[dev], st);
}

// TSRC_MV_LEGACY=1 runs one-token MUL_MATs through the multi-token kernel (same bits; for comparison)
static bool dec_enabled() {
    static const bool on = std::getenv("TSRC_MV_LEGACY") == nullptr;
    return on;
}

cudaError_t launch_matvec(uint32_t fmt, const MvArgs& a, cudaStream_t st) {
    if (a.n_rows == 0 || a.T == 0) return cudaSuccess;
    if (a.T == 1 && a.x && dec_enabled()) return launch_dec(fmt, a, st);
    return fmt == 0 ? launch_fmt<0>(a, st) : launch_fmt<1>(a, st);
}

cudaError_t matvec_error(uint32_t* code, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(code, g_mv_error, sizeof(uint32_t));
    if (e == cudaSuccess && clear && *code) {
        const uint32_t zero = 0;
        e = cudaMemcpyToSymbol(g_mv_error, &zero, sizeof(uint32_t));
    }
    return e;
}

}  // namespace tsrc
