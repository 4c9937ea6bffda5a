// tsrc_matvec.cu -- decode (small-T) Q8_0 / Q4_K MUL_MAT on sm_100a.
//
// Numerics: the reference's MVM row rule bit for bit (jwkim04/tesseract-npu
// sw/sim/tsr_ref.c:533-635): per block i an exact int32 sum, the term
// t_i = (d_w (*) Dx_i) (*) f32(isum_i) [Q4_K: minus (dmin (*) Dx_i) (*) f32(msum_i)], term i
// added in order into partial p[i mod 16] (from +0), then the fixed tree ((p0+p1)+(p2+p3))+...,
// then the MVM epilogue (addend / scale / softcap, tsr_sim.c:1648-1670).
//
// Structure (an HBM stream; tsrc_layout.cuh has the tiled weight layout):
//   - each CTA owns a contiguous range of rows, cut into stages of 16 rows x a tile range;
//   - a producer warp moves stages into a shared-memory ring with bulk asynchronous copies
//     (cp.async.bulk, completion counted on an mbarrier; no multicast), starting at kernel entry,
//     before the activation is even available, so the first stages of every CTA are in flight
//     while the activation is quantized;
//   - 8 consumer warps: warp w takes rows 2w, 2w+1 of a stage; lane L serves row L/16 and block
//     16 t + (L % 16) of tile t, so it owns its block's whole integer sum (no cross-lane sums) and
//     accumulates exactly partial p[L % 16] of its row, tile by tile (the reference's order); the
//     16-partial tree is four xor-shuffle levels inside each half-warp;
//   - the quantized activation sits in shared memory in the same chunk-major tiles, so the 16
//     lanes of a half-warp read 256 contiguous bytes (conflict-free) at immediate offsets; for one
//     token the CTA quantizes x itself (QACT fused), otherwise it copies a QA image;
//   - fast path: if every nonzero activation scale Dx is >= 2^-79, every term and partial is 0 or
//     a multiple of 2^-126 of magnitude >= 2^-126 (|d_w| >= 2^-24 for a nonzero fp16), so no
//     result can be subnormal and the flush tests are skipped (a CTA-uniform choice; the values
//     are the same either way);
//   - every mbarrier wait is bounded; a wait that runs out records an error code (read by
//     tsrc_sync) and the CTA drains its copies in flight and returns.
#include <type_traits>

#include "tsrc_internal.h"
#include "tsrc_layout.cuh"
#include "tsrc_numerics.cuh"

namespace tsrc {

constexpr uint32_t kCWarps = 8;                     // consumer warps
constexpr uint32_t kThreads = (kCWarps + 1) * 32;   // + one producer warp
constexpr uint32_t kStageRows = 2 * kCWarps;        // 16
constexpr uint32_t kSafeDx = 0x18000000u;           // 2^-79
constexpr uint32_t kMaxStages = 4;
constexpr uint32_t kSpinLimit = 1u << 21;           // mbarrier polls (each suspends <= ~0.5 us)
constexpr uint32_t kErrConsumerWait = 1u, kErrProducerWait = 2u, kErrDrain = 3u;

__device__ unsigned int g_mv_error;                 // first error code of any launch (0 = none)

// ---- mbarrier and bulk-copy helpers -----------------------------------------------------------
__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity), "r"(500u)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, uint32_t code) {
    for (uint32_t i = 0; i < kSpinLimit; ++i)
        if (mbar_try_wait(b, parity)) return true;
    atomicCAS(&g_mv_error, 0u, code);
    return false;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(su32(dst)),
                 "l"(src), "r"(bytes), "r"(su32(bar))
                 : "memory");
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
    uint32_t stage_q, stage_m;         // bytes of a stage's quant / meta regions
    uint32_t pitch_q, pitch_m;         // per stage row
    uint32_t stages;                   // ring depth
    uint32_t qa_q, qa_d, qa_bs;        // per-token bytes of the activation image
    uint32_t whole;                    // 1: a stage holds whole rows (one contiguous copy)
    uint32_t tps;                      // tiles per stage
    __host__ __device__ size_t qa_bytes(uint32_t T) const { return (size_t)T * (qa_q + qa_d + qa_bs); }
    __host__ __device__ size_t ring_bytes() const { return (size_t)stages * (stage_q + stage_m); }
    __host__ __device__ size_t total(uint32_t T) const { return ring_bytes() + a16(qa_bytes(T)) + 2u * kMaxStages * 8u + 16u; }
};

__host__ __device__ inline Plan make_plan(uint32_t fmt, uint32_t K, uint32_t T, size_t budget) {
    const Layout L{fmt, K};
    Plan p{};
    p.tps = fmt == 0 ? 4u : 1u;
    p.whole = L.tiles() <= p.tps ? 1u : 0u;
    p.pitch_q = p.whole ? (uint32_t)L.qs_row_bytes() : p.tps * 16u * L.block_qs_bytes();
    p.pitch_m = p.whole ? (uint32_t)L.meta_row_bytes() : (uint32_t)a16((size_t)p.tps * 16u * L.meta_entry_bytes());
    p.stage_q = kStageRows * p.pitch_q;
    p.stage_m = kStageRows * p.pitch_m;
    p.qa_q = L.tiles() * (fmt == 0 ? 512u : 4096u);
    p.qa_d = (uint32_t)a16((size_t)L.blocks() * 4u);
    p.qa_bs = fmt == 0 ? 0u : L.tiles() * 256u;
    p.stages = kMaxStages;
    while (p.stages > 2 && p.total(T) > budget) --p.stages;
    return p;
}

// QACT A32 of block b (tsr_ref.c:472-487), one warp.
__device__ __forceinline__ void qact32_to_smem(const float* __restrict__ x, uint32_t b, uint32_t lane, uint8_t* q, float* d) {
    const float v = x[32u * b + lane];
    const uint32_t amax = __reduce_max_sync(0xFFFFFFFFu, amax_key(v));
    const float db = fdiv(ffrom(amax), 127.0f);
    const float id = (fbits(db) & ~kSign) ? frecip(db) : 0.0f;
    q[(b >> 4) * 512u + 256u * (lane >> 4) + 16u * (b & 15u) + (lane & 15u)] = (uint8_t)round_sat8(fmul(daz(v), id), false);
    if (lane == 0) d[b] = h2f(f2h(db));
}

// QACT A256 of superblock s (tsr_ref.c:488-518), one warp; lane l holds values 8 l .. 8 l + 7.
__device__ __forceinline__ void qact256_to_smem(const float* __restrict__ x, uint32_t s, uint32_t lane, uint8_t* q, float* d,
                                                uint8_t* bs) {
    const float* src = x + 256u * s + 8u * lane;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = src[i];
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
        for (int i = 0; i < 8; ++i) qv[i] = round_sat8(fmul(iscale, daz(v[i])), true);
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
}

// Fills the activation image (consumer threads only). Returns (uniform over the consumers)
// whether every nonzero scale is >= 2^-79.
template <int FMT>
__device__ __forceinline__ bool stage_qa(const MvArgs& a, const Qa& s, const Layout& L, uint32_t* flag) {
    const uint32_t K = a.K, T = a.T, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const uint32_t nb = L.blocks();
    if (tid == 0) *flag = 1u;
    if (a.x) {
        for (uint32_t i = warp; i < T * nb; i += kCWarps) {
            const uint32_t t = i / nb, b = i - t * nb;
            const float* xt = a.x + (size_t)t * a.x_stride;
            if (FMT == 0)
                qact32_to_smem(xt, b, lane, s.q + (size_t)t * s.q_tok, reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(s.d) + (size_t)t * s.d_tok));
            else
                qact256_to_smem(xt, b, lane, s.q + (size_t)t * s.q_tok,
                                reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(s.d) + (size_t)t * s.d_tok), s.bs + (size_t)t * s.bs_tok);
        }
    } else {
        for (uint32_t i = tid; i < T * (K / 16u); i += kCWarps * 32u) {    // 16-byte chunks of q
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
            reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(s.d) + (size_t)t * s.d_tok)[b] = a.dx[i];
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
    consumer_sync();
    bool ok = true;
    for (uint32_t i = tid; i < T * nb; i += kCWarps * 32u) {
        const uint32_t t = i / nb, b = i - t * nb;
        const uint32_t u = fbits(reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(s.d) + (size_t)t * s.d_tok)[b]) & ~kSign;
        ok = ok && (u == 0u || u >= kSafeDx);
    }
    if (!ok) atomicAnd(flag, 0u);
    consumer_sync();
    return *flag != 0u;
}

// ---- per-lane work on one stage -----------------------------------------------------------------
// Q8_0: tiles [t0, t1) of the stage; row_q / row_m: this lane's row in the stage buffers.
template <bool SAFE, int MAXT>
__device__ __forceinline__ void q8_stage(const uint8_t* row_q, const uint8_t* row_m, const Qa& s, const Layout& L, uint32_t T,
                                         uint32_t t0, uint32_t t1, bool whole, uint32_t k, float (&p)[MAXT], int32_t* isum_out) {
    const uint32_t nb = L.blocks();
    for (uint32_t t = t0; t < t1; ++t) {
        const uint32_t b = 16u * t + k;
        if (b >= nb) break;
        const uint32_t tl = whole ? t : t - t0;              // tile index inside the stage row
        const uint32_t nv = L.tile_blocks(t);
        const uint8_t* wq = row_q + (size_t)tl * 512u + 16u * k;
        const uint4 w0 = lds<uint4>(wq), w1 = lds<uint4>(wq + 16u * nv);
        const float dw = h2f(lds<uint16_t>(row_m + 2u * (16u * tl + k)));
#pragma unroll
        for (int tok = 0; tok < MAXT; ++tok) {
            if (tok < (int)T) {
                const uint8_t* xq = s.q + (size_t)tok * s.q_tok + (size_t)t * 512u + 16u * k;
                const int32_t isum = dot16s(w1, lds<uint4>(xq + 256u), dot16s(w0, lds<uint4>(xq), 0));
                if (isum_out && tok == 0) isum_out[b] = isum;
                const float Dx = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(s.d) + (size_t)tok * s.d_tok)[b];
                p[tok] = add_<SAFE>(p[tok], mul_<SAFE>(mul_<SAFE>(dw, Dx), i2f(isum)));
            }
        }
    }
}

// Q4_K: tile t of the stage (one per stage unless whole rows, then all tiles t0 .. t1).
template <bool SAFE, int MAXT>
__device__ __forceinline__ void q4_stage(const uint8_t* row_q, const uint8_t* row_m, const Qa& s, const Layout& L, uint32_t T,
                                         uint32_t t0, uint32_t t1, bool whole, uint32_t k, float (&p)[MAXT], int32_t* isum_out) {
    const uint32_t nsb = L.blocks();
    for (uint32_t t = t0; t < t1; ++t) {
        const uint32_t sb = 16u * t + k;
        if (sb >= nsb) break;
        const uint32_t tl = whole ? t : t - t0;
        const uint32_t cs = 16u * L.tile_blocks(t);          // chunk stride in this tile
        const uint8_t* wq = row_q + (size_t)tl * 2048u + 16u * k;
        uint4 w[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) w[j] = lds<uint4>(wq + (size_t)j * cs);
        const uint4 m = lds<uint4>(row_m + 16u * (16u * tl + k));
        const uint32_t sc_lo = m.y & 0x3F3F3F3Fu, mn_lo = m.z & 0x3F3F3F3Fu;
        const uint32_t sc_hi = (m.w & 0x0F0F0F0Fu) | ((m.y >> 2) & 0x30303030u);
        const uint32_t mn_hi = ((m.w >> 4) & 0x0F0F0F0Fu) | ((m.z >> 2) & 0x30303030u);
        const float dw = h2f((uint16_t)(m.x & 0xFFFFu)), dmw = h2f((uint16_t)(m.x >> 16));
#pragma unroll
        for (int tok = 0; tok < MAXT; ++tok) {
            if (tok < (int)T) {
                const uint8_t* xq = s.q + (size_t)tok * s.q_tok + (size_t)t * 4096u + 16u * k;
                int32_t S[8];
#pragma unroll
                for (int c = 0; c < 4; ++c) {      // qs bytes 32c .. 32c+31 = chunks 2c, 2c+1
                    const uint4 a0 = w[2 * c], a1 = w[2 * c + 1];
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
}

// ---- the kernel ---------------------------------------------------------------------------------
template <int FMT, int MAXT>
__global__ void __launch_bounds__(kThreads, 2) matvec_kernel(MvArgs a, Plan P, uint32_t rows_per_cta) {
    extern __shared__ __align__(128) uint8_t smem[];
    const Layout L{(uint32_t)FMT, a.K};
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const uint32_t r_begin = blockIdx.x * rows_per_cta;
    const uint32_t r_end = min(a.n_rows, r_begin + rows_per_cta);
    if (r_begin >= r_end) return;
    const uint32_t tiles = L.tiles();
    const uint32_t n_ranges = P.whole ? 1u : (tiles + P.tps - 1u) / P.tps;
    const uint32_t n_groups = (r_end - r_begin + kStageRows - 1u) / kStageRows;
    const uint32_t n_stages = n_groups * n_ranges;
    const uint32_t NS = P.stages;

    uint8_t* ring = smem;
    Qa qa;
    qa.q = smem + P.ring_bytes();
    qa.q_tok = P.qa_q;
    qa.d = reinterpret_cast<float*>(qa.q + (size_t)a.T * P.qa_q);
    qa.d_tok = P.qa_d;
    qa.bs = reinterpret_cast<uint8_t*>(qa.d) + (size_t)a.T * P.qa_d;
    qa.bs_tok = P.qa_bs;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + P.ring_bytes() + a16(P.qa_bytes(a.T)));
    uint64_t* empty = full + kMaxStages;
    uint32_t* flag = reinterpret_cast<uint32_t*>(empty + kMaxStages);

    if (tid == 0) {
        for (uint32_t s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1u);
            mbar_init(&empty[s], kCWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == kCWarps) {
        // ===== producer: stages of 16 rows x a tile range into the ring (weights only) =====
        uint32_t issued = 0;
        bool ok = true;
        for (uint32_t i = 0; i < n_stages && ok; ++i) {
            const uint32_t s = i % NS;
            if (i >= NS) ok = mbar_wait(&empty[s], ((i / NS) - 1u) & 1u, kErrProducerWait);
            ok = __all_sync(0xFFFFFFFFu, ok);
            if (!ok) break;
            const uint32_t g = i / n_ranges, rng = i - g * n_ranges;
            const uint32_t ra = r_begin + g * kStageRows, nr = min(kStageRows, r_end - ra);
            uint8_t* sq = ring + (size_t)s * (P.stage_q + P.stage_m);
            uint8_t* sm = sq + P.stage_q;
            uint32_t qb, mb, bytes;
            size_t qoff, moff;
            if (P.whole) {
                qb = nr * (uint32_t)L.qs_row_bytes();
                mb = nr * (uint32_t)L.meta_row_bytes();
                bytes = qb + mb;
                qoff = (size_t)ra * L.qs_row_bytes();
                moff = (size_t)ra * L.meta_row_bytes();
            } else {
                const uint32_t t0 = rng * P.tps, t1 = min(tiles, t0 + P.tps);
                const uint32_t b0 = 16u * t0, b1 = min(L.blocks(), 16u * t1);
                qb = (b1 - b0) * L.block_qs_bytes();
                mb = (uint32_t)a16((size_t)(b1 - b0) * L.meta_entry_bytes());
                bytes = nr * (qb + mb);
                qoff = (size_t)t0 * 16u * L.block_qs_bytes();
                moff = (size_t)b0 * L.meta_entry_bytes();
            }
            if (lane == 0) mbar_expect_tx(&full[s], bytes);
            __syncwarp();
            if (P.whole) {
                if (lane == 0) bulk_g2s(sq, a.qs + qoff, qb, &full[s]);
                if (lane == 1) bulk_g2s(sm, static_cast<const uint8_t*>(a.meta) + moff, mb, &full[s]);
            } else {
                if (lane < nr)
                    bulk_g2s(sq + (size_t)lane * P.pitch_q, a.qs + (size_t)(ra + lane) * L.qs_row_bytes() + qoff, qb, &full[s]);
                if (lane >= 16u && lane - 16u < nr)
                    bulk_g2s(sm + (size_t)(lane - 16u) * P.pitch_m,
                             static_cast<const uint8_t*>(a.meta) + (size_t)(ra + lane - 16u) * L.meta_row_bytes() + moff, mb, &full[s]);
            }
            issued = i + 1;
        }
        // drain: no copy of this CTA may still be in flight when it exits
        if (lane == 0) {
            const uint32_t first = issued > NS ? issued - NS : 0u;
            for (uint32_t i = first; i < issued; ++i)
                if (!mbar_wait(&full[i % NS], (i / NS) & 1u, kErrDrain)) break;
        }
        return;
    }

    // ===== consumers =====
    asm volatile("griddepcontrol.wait;" ::: "memory");   // the activation is ready
    const bool safe = stage_qa<FMT>(a, qa, L, flag);
    const uint32_t k = lane & 15u, half = lane >> 4;
    const uint32_t row_local = 2u * warp + half;
    float p[MAXT];
#pragma unroll
    for (int t = 0; t < MAXT; ++t) p[t] = 0.0f;
    for (uint32_t i = 0; i < n_stages; ++i) {
        const uint32_t s = i % NS;
        if (!__all_sync(0xFFFFFFFFu, mbar_wait(&full[s], (i / NS) & 1u, kErrConsumerWait))) break;
        const uint32_t g = i / n_ranges, rng = i - g * n_ranges;
        const uint32_t row = r_begin + g * kStageRows + row_local;
        const bool rv = row < r_end;
        const uint32_t t0 = P.whole ? 0u : rng * P.tps, t1 = P.whole ? tiles : min(tiles, t0 + P.tps);
        const uint8_t* sq = ring + (size_t)s * (P.stage_q + P.stage_m);
        const uint8_t* row_q = sq + (size_t)row_local * P.pitch_q;
        const uint8_t* row_m = sq + P.stage_q + (size_t)row_local * P.pitch_m;
        int32_t* isum_out = (a.isum_out && rv) ? a.isum_out + (size_t)row * L.blocks() * (FMT == 0 ? 1u : 2u) : nullptr;
        if (rv) {
            if constexpr (FMT == 0) {
                if (safe) q8_stage<true, MAXT>(row_q, row_m, qa, L, a.T, t0, t1, P.whole, k, p, isum_out);
                else q8_stage<false, MAXT>(row_q, row_m, qa, L, a.T, t0, t1, P.whole, k, p, isum_out);
            } else {
                if (safe) q4_stage<true, MAXT>(row_q, row_m, qa, L, a.T, t0, t1, P.whole, k, p, isum_out);
                else q4_stage<false, MAXT>(row_q, row_m, qa, L, a.T, t0, t1, P.whole, k, p, isum_out);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (rng == n_ranges - 1u) {            // the row pair is complete: tree, epilogue, store
#pragma unroll
            for (int t = 0; t < MAXT; ++t) {
                if (t < (int)a.T) {
                    const float v = tree16_lanes(p[t]);
                    if (k == 0 && rv) a.y[(size_t)t * a.y_stride + row] = mm_epilogue(v, a, (uint32_t)t, row);
                }
                p[t] = 0.0f;
            }
        }
    }
}

// ---- host side ------------------------------------------------------------------------------------
constexpr size_t kSmemPerCta = 113u * 1024u;      // two CTAs per SM (228 KB per SM)

size_t mv_smem_bytes(uint32_t fmt, uint32_t K, uint32_t T) { return make_plan(fmt, K, T, kSmemPerCta).total(T); }

template <typename F>
static cudaError_t allow_smem(F* kernel) {
    static int done_dev[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && done_dev[dev] == dev + 1) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(200u * 1024u));
    if (e == cudaSuccess && dev < 64) done_dev[dev] = dev + 1;
    return e;
}

static int g_num_sms[64];

template <int FMT, int MAXT>
static cudaError_t launch_t(const MvArgs& a, cudaStream_t st) {
    const Plan P = make_plan(FMT, a.K, a.T, kSmemPerCta);
    const size_t smem = P.total(a.T);
    cudaError_t e = allow_smem(matvec_kernel<FMT, MAXT>);
    if (e != cudaSuccess) return e;
    int dev = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if (dev < 64 && g_num_sms[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        g_num_sms[dev] = n > 0 ? n : 148;
    }
    const uint32_t sms = dev < 64 ? (uint32_t)g_num_sms[dev] : 148u;
    // contiguous row ranges of even length, two CTAs per SM
    uint32_t rpc = (a.n_rows + 2u * sms - 1u) / (2u * sms);
    rpc = (rpc + 1u) & ~1u;
    const uint32_t blocks = (a.n_rows + rpc - 1u) / rpc;
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

cudaError_t launch_matvec(uint32_t fmt, const MvArgs& a, cudaStream_t st) {
    if (a.n_rows == 0 || a.T == 0) return cudaSuccess;
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
