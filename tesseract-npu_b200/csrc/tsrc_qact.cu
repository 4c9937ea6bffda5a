// tsrc_qact.cu -- QACT on sm_100a: f32 activations -> q8 blocks, bit for bit the reference's
// tsr_qact (jwkim04/tesseract-npu sw/sim/tsr_ref.c:456-518).
//
//   A32  (Q8_0 weights): per 32 values amax = max |DAZ(x)| over non-NaN x, d = amax (/) 127,
//        id = d ? 1 (/) d : 0, q = round-half-away(x (*) id) saturated, D = f32(fp16(d)).
//   A256 (Q4_K weights): per 256 values max = the signed DAZ(x) of the first largest |x|,
//        iscale = -127 (/) max, q = round-half-even(iscale (*) x) saturated, d = 1 (/) iscale,
//        bs = int16 sums of 16 q; an all-zero block gives d = 0, q = 0, bs = 0. Optionally also the
//        sums of the eight 32-value sub-blocks p_j = bs_2j + bs_2j+1 (|p_j| <= 4064) as two int8
//        digits each, p_j = 64 hi_j + lo_j with lo_j = p_j & 63, hi_j = p_j >> 6 (in [-64, 63]), as
//        16 bytes per block {lo_0 .. lo_7, hi_0 .. hi_7}: the tensor-core operand of the Q4_K min sums.
// One warp per block; the reductions are exact (integer max on |x| bits, first index on ties).
#include "tsrc_internal.h"
#include "tsrc_numerics.cuh"

namespace tsrc {

__global__ void __launch_bounds__(256) qact_a32_kernel(const float* __restrict__ x, uint32_t K, uint32_t T,
                                                       uint32_t x_stride, int8_t* __restrict__ q,
                                                       float* __restrict__ d) {
    // let the dependent matvec launch now; it reads this kernel's output only after completion
    asm volatile("griddepcontrol.launch_dependents;");
    const uint32_t nb = K >> 5;
    const uint32_t gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint32_t lane = threadIdx.x & 31u;
    if (gw >= T * nb) return;
    const uint32_t t = gw / nb, b = gw - t * nb;
    const float v = x[(size_t)t * x_stride + 32u * b + lane];
    const uint32_t amax = __reduce_max_sync(0xFFFFFFFFu, amax_key(v));
    const float db = fdiv(ffrom(amax), 127.0f);
    const float id = (fbits(db) & ~kSign) ? frecip(db) : 0.0f;
    q[(size_t)t * K + 32u * b + lane] = (int8_t)round_away_sat8(fmul(daz(v), id));
    if (lane == 0) d[(size_t)t * nb + b] = h2f(f2h(db));
}

__global__ void __launch_bounds__(256) qact_a256_kernel(const float* __restrict__ x, uint32_t K, uint32_t T,
                                                        uint32_t x_stride, int8_t* __restrict__ q,
                                                        float* __restrict__ d, int16_t* __restrict__ bs,
                                                        int8_t* __restrict__ bsd) {
    asm volatile("griddepcontrol.launch_dependents;");
    const uint32_t nb = K >> 8;
    const uint32_t gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint32_t lane = threadIdx.x & 31u;
    if (gw >= T * nb) return;
    const uint32_t t = gw / nb, b = gw - t * nb;
    // lane holds values [8 lane, 8 lane + 8) of the block, in order
    const float4* src = reinterpret_cast<const float4*>(x + (size_t)t * x_stride + 256u * b + 8u * lane);
    const bool vec = ((reinterpret_cast<uintptr_t>(src) & 15u) == 0);
    float v[8];
    if (vec) {
        const float4 a0 = src[0], a1 = src[1];
        v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w; v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
    } else {
        const float* s = x + (size_t)t * x_stride + 256u * b + 8u * lane;
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = s[i];
    }
    uint32_t best = 0, best_i = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint32_t k = amax_key(v[i]);
        if (k > best) { best = k; best_i = (uint32_t)i; }
    }
    const uint32_t amax = __reduce_max_sync(0xFFFFFFFFu, best);
    // first occurrence of the largest |x|: the lowest lane holding it, its first index
    const uint32_t cand = (best == amax && amax != 0u) ? lane : 32u;
    const uint32_t owner = __reduce_min_sync(0xFFFFFFFFu, cand);
    const float mine = daz(v[best_i]);
    const float mx = __shfl_sync(0xFFFFFFFFu, mine, owner & 31u);
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
    int32_t s = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        lo |= ((uint32_t)qv[i] & 0xFFu) << (8 * i);
        hi |= ((uint32_t)qv[i + 4] & 0xFFu) << (8 * i);
        s += qv[i] + qv[i + 4];
    }
    *reinterpret_cast<uint2*>(q + (size_t)t * K + 256u * b + 8u * lane) = make_uint2(lo, hi);
    s += __shfl_xor_sync(0xFFFFFFFFu, s, 1);
    if ((lane & 1u) == 0) bs[(size_t)t * (K >> 4) + 16u * b + (lane >> 1)] = (int16_t)s;
    if (bsd) {
        const int32_t p = s + __shfl_xor_sync(0xFFFFFFFFu, s, 2);  // sub-block lane / 4: lanes 4 j .. 4 j + 3
        if ((lane & 3u) == 0) {
            int8_t* o = bsd + ((size_t)t * nb + b) * 16u;
            o[lane >> 2] = (int8_t)(p & 63);
            o[8u + (lane >> 2)] = (int8_t)(p >> 6);
        }
    }
    if (lane == 0) d[(size_t)t * nb + b] = db;
}

cudaError_t launch_qact(uint32_t kind, const float* x, uint32_t K, uint32_t T, uint32_t x_stride, int8_t* q, float* d,
                        int16_t* bs, cudaStream_t st, int8_t* bsd) {
    const uint32_t bsz = kind == 0 ? 32u : 256u;
    const uint64_t warps = (uint64_t)T * (K / bsz);
    const uint32_t blocks = (uint32_t)((warps + 7u) / 8u);
    if (blocks == 0) return cudaSuccess;
    if (kind == 0)
        qact_a32_kernel<<<blocks, 256, 0, st>>>(x, K, T, x_stride, q, d);
    else
        qact_a256_kernel<<<blocks, 256, 0, st>>>(x, K, T, x_stride, q, d, bs, bsd);
    return cudaGetLastError();
}

}  // namespace tsrc
