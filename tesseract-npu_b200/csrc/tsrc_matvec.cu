// tsrc_matvec.cu -- decode (small-T) Q8_0 / Q4_K MUL_MAT on sm_100a.
//
// Numerics: the reference's MVM row rule bit for bit (jwkim04/tesseract-npu
// sw/sim/tsr_ref.c:533-635): per block i an exact int32 sum, the term
// t_i = (d_w (*) Dx_i) (*) f32(isum_i) [Q4_K: minus (dmin (*) Dx_i) (*) f32(msum_i)], term i
// added in order into partial p[i mod 16] (from +0), then the fixed tree ((p0+p1)+(p2+p3))+...,
// then the MVM epilogue (addend / scale / softcap, tsr_sim.c:1648-1670).
//
// Mapping (an HBM stream; see tsrc_layout.cuh for the tiled weight layout):
//   - a warp owns a pair of rows; lane L serves row L/16 and block 16 t + (L % 16) of tile t, so
//     it accumulates exactly partial p[L % 16] of its row, tile by tile (the reference's order),
//     and owns its block's whole integer sum (no cross-lane reduction); the 16-partial tree is
//     four xor-shuffle levels inside each half-warp;
//   - persistent warps walk their row pairs tile group by tile group, with the next group's
//     128-bit non-allocating weight loads issued before the current group is computed;
//   - the quantized activation lives in shared memory, XOR-swizzled so that the 16 lanes reading
//     the same chunk of 16 different blocks hit distinct banks; for one token the CTA quantizes x
//     itself (QACT fused: no scratch buffer, no second launch), otherwise it stages a QA image;
//   - fast path: if every nonzero activation scale Dx of the call is >= 2^-79, every term and
//     partial is 0 or a multiple of 2^-126 of magnitude >= 2^-126 (|d_w| >= 2^-24 for a nonzero
//     fp16), so no result can be subnormal and the flush tests are skipped (CTA-uniform choice;
//     the exact same values either way).
#include <type_traits>

#include "tsrc_internal.h"
#include "tsrc_layout.cuh"
#include "tsrc_numerics.cuh"

namespace tsrc {

constexpr int kWarps = 8;                  // warps per CTA
constexpr int kThreads = kWarps * 32;
constexpr uint32_t kSafeDx = 0x18000000u;  // 2^-79

__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ int32_t dot16s(const uint4 w, const uint4 x, int32_t acc) {
    acc = __dp4a((int)w.x, (int)x.x, acc);
    acc = __dp4a((int)w.y, (int)x.y, acc);
    acc = __dp4a((int)w.z, (int)x.z, acc);
    acc = __dp4a((int)w.w, (int)x.w, acc);
    return acc;
}
// unsigned bytes of w (nibbles in place) times signed bytes of x
__device__ __forceinline__ int32_t dp4a_us(uint32_t a, uint32_t b, int32_t c) {
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

// f32 rules with the flush test only when the CTA is not on the fast path.
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

// ---- shared-memory QA image (per token): swizzled quants, scales, Q4_K sub-block sums --------
// Q8_0: byte e of block b at 32 b + 16 ((e >> 4) ^ ((b >> 2) & 1)) + (e & 15)
// Q4_K: byte e of superblock s at 256 s + 16 ((e >> 4) ^ (s & 7)) + (e & 15)
//       sub-block sum j of s at 32 s + 16 ((j >> 2) ^ ((s >> 2) & 1)) + 4 (j & 3)
__device__ __forceinline__ uint32_t swz_q8(uint32_t b, uint32_t c16) { return 32u * b + 16u * (c16 ^ ((b >> 2) & 1u)); }
__device__ __forceinline__ uint32_t swz_q4(uint32_t s, uint32_t c16) { return 256u * s + 16u * (c16 ^ (s & 7u)); }
__device__ __forceinline__ uint32_t swz_bs(uint32_t s, uint32_t h) { return 32u * s + 16u * (h ^ ((s >> 2) & 1u)); }

struct QaSmem {
    uint8_t* q;       // [T][K] swizzled
    float* d;         // [T][nb]
    int32_t* bsub;    // [T][nsb * 8] swizzled (Q4_K)
};

__host__ __device__ constexpr size_t a16(size_t n) { return (n + 15u) & ~(size_t)15u; }

size_t mv_smem_bytes(uint32_t fmt, uint32_t K, uint32_t T) {
    const uint32_t nb = fmt == 0 ? K / 32u : K / 256u;
    size_t s = a16((size_t)T * K) + a16((size_t)T * nb * 4u);
    if (fmt == 1) s += (size_t)T * nb * 32u;
    return s;
}

__device__ __forceinline__ QaSmem carve(uint8_t* smem, uint32_t fmt, uint32_t K, uint32_t T) {
    const uint32_t nb = fmt == 0 ? K / 32u : K / 256u;
    QaSmem s;
    s.q = smem;
    s.d = reinterpret_cast<float*>(smem + a16((size_t)T * K));
    s.bsub = reinterpret_cast<int32_t*>(smem + a16((size_t)T * K) + a16((size_t)T * nb * 4u));
    return s;
}

// QACT A32 of block b (tsr_ref.c:472-487), one warp, into the shared image of one token.
__device__ __forceinline__ void qact32_to_smem(const float* __restrict__ x, uint32_t b, uint32_t lane, uint8_t* q, float* d) {
    const float v = x[32u * b + lane];
    const uint32_t amax = __reduce_max_sync(0xFFFFFFFFu, amax_key(v));
    const float db = fdiv(ffrom(amax), 127.0f);
    const float id = (fbits(db) & ~kSign) ? frecip(db) : 0.0f;
    q[swz_q8(b, lane >> 4) + (lane & 15u)] = (uint8_t)round_sat8(fmul(daz(v), id), false);
    if (lane == 0) d[b] = h2f(f2h(db));
}

// QACT A256 of superblock s (tsr_ref.c:488-518), one warp, into the shared image of one token.
__device__ __forceinline__ void qact256_to_smem(const float* __restrict__ x, uint32_t s, uint32_t lane, uint8_t* q, float* d,
                                                int32_t* bsub) {
    const float* src = x + 256u * s + 8u * lane;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = src[i];
    uint32_t best = 0, best_i = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t kk = amax_key(v[i]);
        if (kk > best) { best = kk; best_i = (uint32_t)i; }
    }
    const uint32_t amax = __reduce_max_sync(0xFFFFFFFFu, best);
    const uint32_t owner = __reduce_min_sync(0xFFFFFFFFu, (best == amax && amax != 0u) ? lane : 32u);
    float mine = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) mine = ((uint32_t)i == best_i) ? v[i] : mine;
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
    *reinterpret_cast<uint2*>(q + swz_q4(s, lane >> 1) + 8u * (lane & 1u)) = make_uint2(lo, hi);
    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
    sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);     // lanes 4j..4j+3: sub-block j (32 values)
    if ((lane & 3u) == 0) {
        const uint32_t j = lane >> 2;
        bsub[(swz_bs(s, j >> 2) >> 2) + (j & 3u)] = sum;
    }
    if (lane == 0) d[s] = db;
}

// Fills the shared QA image of the call: QACT of the f32 tokens, or a copy of a QA image.
// Returns (CTA-uniform) whether every nonzero scale is >= 2^-79 (the fast path).
__device__ __forceinline__ bool stage_qa(const MvArgs& a, const QaSmem& s, uint32_t fmt) {
    const uint32_t K = a.K, T = a.T, warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t nb = fmt == 0 ? K / 32u : K / 256u;
    if (a.x) {
        for (uint32_t i = warp; i < T * nb; i += kWarps) {
            const uint32_t t = i / nb, b = i - t * nb;
            const float* xt = a.x + (size_t)t * a.x_stride;
            if (fmt == 0)
                qact32_to_smem(xt, b, lane, s.q + (size_t)t * K, s.d + (size_t)t * nb);
            else
                qact256_to_smem(xt, b, lane, s.q + (size_t)t * K, s.d + (size_t)t * nb, s.bsub + (size_t)t * nb * 8u);
        }
    } else {
        for (uint32_t i = threadIdx.x; i < T * K / 16u; i += kThreads) {    // 16-byte chunks
            const uint32_t t = i / (K / 16u), c = i - t * (K / 16u);
            const uint4 v = reinterpret_cast<const uint4*>(a.qx + (size_t)t * K)[c];
            const uint32_t off = fmt == 0 ? swz_q8(c >> 1, c & 1u) : swz_q4(c >> 4, c & 15u);
            *reinterpret_cast<uint4*>(s.q + (size_t)t * K + off) = v;
        }
        for (uint32_t i = threadIdx.x; i < T * nb; i += kThreads) s.d[i] = a.dx[i];
        if (fmt == 1) {
            for (uint32_t i = threadIdx.x; i < T * nb * 8u; i += kThreads) {
                const uint32_t t = i / (nb * 8u), r = i - t * nb * 8u, sb = r >> 3, j = r & 7u;
                const int32_t v = (int32_t)a.bsx[(size_t)t * (K / 16u) + 16u * sb + 2u * j] +
                                  (int32_t)a.bsx[(size_t)t * (K / 16u) + 16u * sb + 2u * j + 1u];
                s.bsub[(size_t)t * nb * 8u + (swz_bs(sb, j >> 2) >> 2) + (j & 3u)] = v;
            }
        }
    }
    __syncthreads();
    bool ok = true;
    for (uint32_t i = threadIdx.x; i < T * nb; i += kThreads) {
        const uint32_t u = fbits(s.d[i]) & ~kSign;
        ok = ok && (u == 0u || u >= kSafeDx);
    }
    return __syncthreads_and(ok) != 0;
}

// ---------------------------------------------------------------------------------------------
// Q8_0. A unit is a group of up to 4 tiles of one row pair; per lane: 2 x 128-bit quant loads
// and one fp16 scale per tile.
// ---------------------------------------------------------------------------------------------
constexpr uint32_t kQ8Tiles = 4;

struct Q8Unit {
    uint4 w[kQ8Tiles][2];
    uint32_t d[kQ8Tiles];     // fp16 scale in the low half
};

__device__ __forceinline__ void q8_load(const MvArgs& a, const Layout& L, uint32_t row, bool rv, uint32_t t0, uint32_t k,
                                        Q8Unit& u) {
    const uint32_t nb = L.blocks();
#pragma unroll
    for (uint32_t i = 0; i < kQ8Tiles; ++i) {
        const uint32_t b = 16u * (t0 + i) + k;
        if (rv && b < nb) {
            u.w[i][0] = ld_stream(a.qs + L.qs_off(row, b, 0));
            u.w[i][1] = ld_stream(a.qs + L.qs_off(row, b, 1));
            u.d[i] = __ldg(reinterpret_cast<const uint16_t*>(static_cast<const uint8_t*>(a.meta) + L.meta_off(row, b)));
        }
    }
}

template <bool SAFE, int MAXT>
__device__ __forceinline__ void q8_compute(const Q8Unit& u, const QaSmem& s, const Layout& L, uint32_t T, bool rv, uint32_t t0,
                                           uint32_t k, float (&p)[MAXT], int32_t* isum_out) {
    const uint32_t nb = L.blocks(), K = L.K;
#pragma unroll
    for (uint32_t i = 0; i < kQ8Tiles; ++i) {
        const uint32_t b = 16u * (t0 + i) + k;
        if (!rv || b >= nb) continue;
        const float dw = h2f((uint16_t)u.d[i]);
#pragma unroll
        for (int t = 0; t < MAXT; ++t) {
            if (t < (int)T) {
                const uint8_t* xq = s.q + (size_t)t * K;
                const uint4 x0 = *reinterpret_cast<const uint4*>(xq + swz_q8(b, 0));
                const uint4 x1 = *reinterpret_cast<const uint4*>(xq + swz_q8(b, 1));
                const int32_t isum = dot16s(u.w[i][1], x1, dot16s(u.w[i][0], x0, 0));
                if (isum_out && t == 0) isum_out[b] = isum;
                p[t] = add_<SAFE>(p[t], mul_<SAFE>(mul_<SAFE>(dw, s.d[(size_t)t * nb + b]), i2f(isum)));
            }
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Q4_K. A unit is one tile of one row pair; per lane: 8 x 128-bit quant loads (its superblock)
// and its 16-byte meta entry.
// ---------------------------------------------------------------------------------------------
struct Q4Unit {
    uint4 w[8];
    uint4 m;
};

__device__ __forceinline__ void q4_load(const MvArgs& a, const Layout& L, uint32_t row, bool rv, uint32_t t0, uint32_t k,
                                        Q4Unit& u) {
    const uint32_t sb = 16u * t0 + k;
    if (rv && sb < L.blocks()) {
#pragma unroll
        for (uint32_t j = 0; j < 8; ++j) u.w[j] = ld_stream(a.qs + L.qs_off(row, sb, j));
        u.m = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.meta) + L.meta_off(row, sb)));
    }
}

__device__ __forceinline__ int32_t byte_of(uint32_t w, int i) { return (int32_t)((w >> (8 * i)) & 0xFFu); }

template <bool SAFE, int MAXT>
__device__ __forceinline__ void q4_compute(const Q4Unit& u, const QaSmem& s, const Layout& L, uint32_t T, bool rv, uint32_t t0,
                                           uint32_t k, float (&p)[MAXT], int32_t* isum_out) {
    const uint32_t nsb = L.blocks(), K = L.K;
    const uint32_t sb = 16u * t0 + k;
    if (!rv || sb >= nsb) return;
    // 6-bit scales and mins of the 8 sub-blocks (ggml get_scale_min_k4), packed 4 per word
    const uint32_t sc_lo = u.m.y & 0x3F3F3F3Fu, mn_lo = u.m.z & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (u.m.w & 0x0F0F0F0Fu) | ((u.m.y >> 2) & 0x30303030u);
    const uint32_t mn_hi = ((u.m.w >> 4) & 0x0F0F0F0Fu) | ((u.m.z >> 2) & 0x30303030u);
    const float dw = h2f((uint16_t)(u.m.x & 0xFFFFu)), dmw = h2f((uint16_t)(u.m.x >> 16));
#pragma unroll
    for (int t = 0; t < MAXT; ++t) {
        if (t < (int)T) {
            const uint8_t* xq = s.q + (size_t)t * K;
            int32_t S[8];
#pragma unroll
            for (int c = 0; c < 4; ++c) {           // qs bytes 32c .. 32c+31: chunks 2c, 2c+1
                const uint4 w0 = u.w[2 * c], w1 = u.w[2 * c + 1];
                const uint4 xl0 = *reinterpret_cast<const uint4*>(xq + swz_q4(sb, 4u * c + 0u));
                const uint4 xl1 = *reinterpret_cast<const uint4*>(xq + swz_q4(sb, 4u * c + 1u));
                const uint4 xh0 = *reinterpret_cast<const uint4*>(xq + swz_q4(sb, 4u * c + 2u));
                const uint4 xh1 = *reinterpret_cast<const uint4*>(xq + swz_q4(sb, 4u * c + 3u));
                const uint4 l0 = make_uint4(w0.x & 0x0F0F0F0Fu, w0.y & 0x0F0F0F0Fu, w0.z & 0x0F0F0F0Fu, w0.w & 0x0F0F0F0Fu);
                const uint4 l1 = make_uint4(w1.x & 0x0F0F0F0Fu, w1.y & 0x0F0F0F0Fu, w1.z & 0x0F0F0F0Fu, w1.w & 0x0F0F0F0Fu);
                const uint4 h0 = make_uint4(w0.x & 0xF0F0F0F0u, w0.y & 0xF0F0F0F0u, w0.z & 0xF0F0F0F0u, w0.w & 0xF0F0F0F0u);
                const uint4 h1 = make_uint4(w1.x & 0xF0F0F0F0u, w1.y & 0xF0F0F0F0u, w1.z & 0xF0F0F0F0u, w1.w & 0xF0F0F0F0u);
                S[2 * c] = dot16s(l1, xl1, dot16s(l0, xl0, 0));
                S[2 * c + 1] = dot16us(h1, xh1, dot16us(h0, xh0, 0)) >> 4;   // high nibbles carry 16x
            }
            const int32_t* bt = s.bsub + (size_t)t * nsb * 8u;
            const int4 b0 = *reinterpret_cast<const int4*>(bt + (swz_bs(sb, 0) >> 2));
            const int4 b1 = *reinterpret_cast<const int4*>(bt + (swz_bs(sb, 1) >> 2));
            int32_t isum = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) isum += byte_of(sc_lo, j) * S[j] + byte_of(sc_hi, j) * S[4 + j];
            const int32_t msum = byte_of(mn_lo, 0) * b0.x + byte_of(mn_lo, 1) * b0.y + byte_of(mn_lo, 2) * b0.z +
                                 byte_of(mn_lo, 3) * b0.w + byte_of(mn_hi, 0) * b1.x + byte_of(mn_hi, 1) * b1.y +
                                 byte_of(mn_hi, 2) * b1.z + byte_of(mn_hi, 3) * b1.w;
            if (isum_out && t == 0) {
                isum_out[2u * sb] = isum;
                isum_out[2u * sb + 1u] = msum;
            }
            const float Dx = s.d[(size_t)t * nsb + sb];
            const float t1 = mul_<SAFE>(mul_<SAFE>(dw, Dx), i2f(isum));
            const float t2 = mul_<SAFE>(mul_<SAFE>(dmw, Dx), i2f(msum));
            p[t] = add_<SAFE>(p[t], sub_<SAFE>(t1, t2));
        }
    }
}

// ---------------------------------------------------------------------------------------------
// The kernel: FMT 0 = Q8_0, 1 = Q4_K.
// ---------------------------------------------------------------------------------------------
template <int FMT, int MAXT>
__global__ void __launch_bounds__(kThreads, 2) matvec_kernel(MvArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    const Layout L{(uint32_t)FMT, a.K};
    const uint32_t lane = threadIdx.x & 31u, k = lane & 15u, half = lane >> 4;
    const uint32_t gwarp = blockIdx.x * kWarps + (threadIdx.x >> 5);
    const uint32_t n_warps = gridDim.x * kWarps;
    const uint32_t n_pairs = (a.n_rows + 1u) / 2u;
    const uint32_t tiles = L.tiles();
    constexpr uint32_t TPU = FMT == 0 ? kQ8Tiles : 1u;          // tiles per unit
    const uint32_t units = (tiles + TPU - 1u) / TPU;
    using Unit = typename std::conditional<FMT == 0, Q8Unit, Q4Unit>::type;

    // prefetch the first unit (weights only: nothing an earlier kernel writes is read here)
    uint32_t pair = gwarp, ui = 0;
    Unit cur;
    {
        const uint32_t row = 2u * pair + half;
        const bool rv = pair < n_pairs && row < a.n_rows;
        if constexpr (FMT == 0) q8_load(a, L, row, rv, 0, k, cur); else q4_load(a, L, row, rv, 0, k, cur);
    }
    // the activation is read only after the previous kernel on the stream has completed
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const QaSmem s = carve(smem, FMT, a.K, a.T);
    const bool safe = stage_qa(a, s, FMT);
    if (gwarp >= n_pairs) return;

    float p[MAXT];
#pragma unroll
    for (int t = 0; t < MAXT; ++t) p[t] = 0.0f;
    while (pair < n_pairs) {
        const uint32_t row = 2u * pair + half;
        const bool rv = row < a.n_rows;
        // the next unit: the next tile group of this pair, else the first of the next pair
        uint32_t npair = pair, nui = ui + 1u;
        if (nui == units) { npair = pair + n_warps; nui = 0; }
        Unit nxt;
        {
            const uint32_t nrow = 2u * npair + half;
            const bool nrv = npair < n_pairs && nrow < a.n_rows;
            if constexpr (FMT == 0) q8_load(a, L, nrow, nrv, nui * TPU, k, nxt); else q4_load(a, L, nrow, nrv, nui * TPU, k, nxt);
        }
        int32_t* isum_out = nullptr;
        if (a.isum_out && rv) isum_out = a.isum_out + (size_t)row * L.blocks() * (FMT == 0 ? 1u : 2u);
        if constexpr (FMT == 0) {
            if (safe) q8_compute<true, MAXT>(cur, s, L, a.T, rv, ui * TPU, k, p, isum_out);
            else q8_compute<false, MAXT>(cur, s, L, a.T, rv, ui * TPU, k, p, isum_out);
        } else {
            if (safe) q4_compute<true, MAXT>(cur, s, L, a.T, rv, ui * TPU, k, p, isum_out);
            else q4_compute<false, MAXT>(cur, s, L, a.T, rv, ui * TPU, k, p, isum_out);
        }
        if (nui == 0) {            // the pair is complete: tree, epilogue, store
#pragma unroll
            for (int t = 0; t < MAXT; ++t) {
                if (t < (int)a.T) {
                    const float v = tree16_lanes(p[t]);
                    if (k == 0 && rv) a.y[(size_t)t * a.y_stride + row] = mm_epilogue(v, a, (uint32_t)t, row);
                }
                p[t] = 0.0f;
            }
        }
        pair = npair;
        ui = nui;
        cur = nxt;
    }
}

// The dynamic shared-memory limit is raised once per kernel and device (before any stream
// capture can be active: the first call of a shape is an ordinary launch).
template <typename F>
static cudaError_t allow_smem(F* kernel, size_t smem) {
    static int done_dev[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (smem <= 48u * 1024u || (dev < 64 && done_dev[dev] == dev + 1)) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e == cudaSuccess && dev < 64) done_dev[dev] = dev + 1;
    return e;
}

static int g_num_sms[64];

template <int FMT, int MAXT>
static cudaError_t launch_t(const MvArgs& a, cudaStream_t st) {
    const size_t smem = mv_smem_bytes(FMT, a.K, a.T);
    cudaError_t e = allow_smem(matvec_kernel<FMT, MAXT>, smem);
    if (e != cudaSuccess) return e;
    int dev = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if (dev < 64 && g_num_sms[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        g_num_sms[dev] = n > 0 ? n : 148;
    }
    const uint32_t sms = dev < 64 ? (uint32_t)g_num_sms[dev] : 148u;
    // persistent grid: at most 2 CTAs per SM; every warp gets ceil(pairs / warps) pairs
    const uint32_t n_pairs = (a.n_rows + 1u) / 2u;
    const uint32_t wmax = 2u * sms * kWarps;
    const uint32_t rounds = (n_pairs + wmax - 1u) / wmax;
    const uint32_t warps = (n_pairs + rounds - 1u) / rounds;
    const uint32_t blocks = (warps + kWarps - 1u) / kWarps;
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
    return cudaLaunchKernelEx(&cfg, matvec_kernel<FMT, MAXT>, a);
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

}  // namespace tsrc
