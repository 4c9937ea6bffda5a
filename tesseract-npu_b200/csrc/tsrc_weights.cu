// tsrc_weights.cu -- weight layout on the device and seeded synthetic weights.
//
// Layout: ggml rows (Q8_0: K/32 blocks {fp16 d, int8 qs[32]} = 34 B; Q4_K: K/256 superblocks
// {fp16 d, dmin, u8 scales[12], u8 qs[128]} = 144 B) <-> the tiled split layout of
// tsrc_layout.cuh; tsrc_weight_download (get_tensor) inverts the upload exactly.
//
// Synthetic weights: value (row n, column k) is a normal N(0, sigma^2) draw from Philox4x32-10
// (Salmon, Moraes, Dror, Shaw, SC'11) keyed by the seed, counter (n, k / 4), followed by the
// Box-Muller transform; blocks are then quantized on the device: Q8_0 with the A32 rule
// (ggml quantize_row_q8_0_ref), Q4_K with the sub-block min/scale encoder of the reference's
// test models (sw/ggml-tesseract/tests/gen_tiny_models.py:91-130). A row's values do not depend
// on the shard it is generated in.
#include "tsrc_internal.h"
#include "tsrc_layout.cuh"
#include "tsrc_numerics.cuh"

namespace tsrc {

// ---- layout ----------------------------------------------------------------------------------
// One thread per block (Q8_0) / superblock (Q4_K); b = block index within the row.
__global__ void repack_kernel(Layout L, const uint8_t* __restrict__ g, uint32_t n_rows, uint8_t* __restrict__ qs,
                              uint8_t* __restrict__ meta) {
    const uint32_t nb = L.blocks();
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)n_rows * nb) return;
    const uint32_t r = (uint32_t)(i / nb), b = (uint32_t)(i % nb);
    if (L.fmt == 0) {
        const uint8_t* src = g + i * 34u;
        *reinterpret_cast<uint16_t*>(meta + L.meta_off(r, b)) = (uint16_t)(src[0] | (src[1] << 8));
        for (uint32_t j = 0; j < 2; ++j) {
            uint32_t w[4];
            for (int e = 0; e < 4; ++e) {
                const uint8_t* p = src + 2 + 16 * j + 4 * e;
                w[e] = (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
            }
            *reinterpret_cast<uint4*>(qs + L.qs_off(r, b, j)) = make_uint4(w[0], w[1], w[2], w[3]);
        }
    } else {
        const uint4* src = reinterpret_cast<const uint4*>(g) + i * 9u;    // 144 B, 16-byte aligned
        *reinterpret_cast<uint4*>(meta + L.meta_off(r, b)) = src[0];
        for (uint32_t j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(qs + L.qs_off(r, b, j)) = src[1 + j];
    }
}

__global__ void unrepack_kernel(Layout L, const uint8_t* __restrict__ qs, const uint8_t* __restrict__ meta, uint32_t n_rows,
                                uint8_t* __restrict__ g) {
    const uint32_t nb = L.blocks();
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)n_rows * nb) return;
    const uint32_t r = (uint32_t)(i / nb), b = (uint32_t)(i % nb);
    if (L.fmt == 0) {
        uint8_t* dst = g + i * 34u;
        const uint16_t d = *reinterpret_cast<const uint16_t*>(meta + L.meta_off(r, b));
        dst[0] = (uint8_t)d;
        dst[1] = (uint8_t)(d >> 8);
        for (uint32_t j = 0; j < 2; ++j) {
            const uint8_t* c = qs + L.qs_off(r, b, j);
            for (int e = 0; e < 16; ++e) dst[2 + 16 * j + e] = c[e];
        }
    } else {
        uint4* dst = reinterpret_cast<uint4*>(g) + i * 9u;
        dst[0] = *reinterpret_cast<const uint4*>(meta + L.meta_off(r, b));
        for (uint32_t j = 0; j < 8; ++j) dst[1 + j] = *reinterpret_cast<const uint4*>(qs + L.qs_off(r, b, j));
    }
}

static inline uint32_t grid_for(uint64_t n, uint32_t bs) { return (uint32_t)((n + bs - 1u) / bs); }

cudaError_t launch_repack(uint32_t fmt, const uint8_t* ggml, uint32_t n_rows, uint32_t K, uint8_t* qs, uint8_t* meta,
                          cudaStream_t st) {
    const Layout L{fmt, K};
    const uint64_t n = (uint64_t)n_rows * L.blocks();
    if (n) repack_kernel<<<grid_for(n, 256), 256, 0, st>>>(L, ggml, n_rows, qs, meta);
    return cudaGetLastError();
}

cudaError_t launch_unrepack(uint32_t fmt, const uint8_t* qs, const uint8_t* meta, uint32_t n_rows, uint32_t K,
                            uint8_t* ggml, cudaStream_t st) {
    const Layout L{fmt, K};
    const uint64_t n = (uint64_t)n_rows * L.blocks();
    if (n) unrepack_kernel<<<grid_for(n, 256), 256, 0, st>>>(L, qs, meta, n_rows, ggml);
    return cudaGetLastError();
}

// ---- Philox4x32-10 + Box-Muller -------------------------------------------------------------
struct U4 {
    uint32_t x, y, z, w;
};

__device__ __forceinline__ U4 philox4x32_10(U4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
        const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
        c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c;
}

// Four N(0, 1) values for 4-value group q of row n.
__device__ __forceinline__ void normal4(uint64_t seed, uint32_t n, uint32_t q, float out[4]) {
    const U4 r = philox4x32_10(U4{q, n, 0x7473u, 0x72u}, (uint32_t)seed, (uint32_t)(seed >> 32));
    const float u0 = ((float)r.x + 1.0f) * 2.3283064e-10f, u1 = (float)r.y * 2.3283064e-10f;
    const float u2 = ((float)r.z + 1.0f) * 2.3283064e-10f, u3 = (float)r.w * 2.3283064e-10f;
    const float ra = sqrtf(-2.0f * logf(fminf(u0, 1.0f))), rb = sqrtf(-2.0f * logf(fminf(u2, 1.0f)));
    float s, c;
    sincospif(2.0f * u1, &s, &c);
    out[0] = ra * c;
    out[1] = ra * s;
    sincospif(2.0f * u3, &s, &c);
    out[2] = rb * c;
    out[3] = rb * s;
}

// One thread per Q8_0 block: A32 quantization of 32 normals (quantize_row_q8_0_ref).
__global__ void synth_q8_0_kernel(uint32_t K, uint32_t row0, uint32_t n_rows, uint64_t seed, float sigma,
                                  uint8_t* __restrict__ qs, uint8_t* __restrict__ meta) {
    const Layout L{0u, K};
    const uint32_t nb = K / 32u;
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)n_rows * nb) return;
    const uint32_t r = (uint32_t)(i / nb), b = (uint32_t)(i % nb);
    float v[32];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        float o[4];
        normal4(seed, row0 + r, b * 8u + (uint32_t)j, o);
#pragma unroll
        for (int e = 0; e < 4; ++e) v[4 * j + e] = o[e] * sigma;
    }
    uint32_t amax = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) amax = max(amax, amax_key(v[j]));
    const float db = fdiv(ffrom(amax), 127.0f);
    const float id = (fbits(db) & ~kSign) ? frecip(db) : 0.0f;
    uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 32; ++j) w[j >> 2] |= ((uint32_t)round_sat8(fmul(daz(v[j]), id), false) & 0xFFu) << (8 * (j & 3));
    *reinterpret_cast<uint4*>(qs + L.qs_off(r, b, 0)) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(qs + L.qs_off(r, b, 1)) = make_uint4(w[4], w[5], w[6], w[7]);
    *reinterpret_cast<uint16_t*>(meta + L.meta_off(r, b)) = f2h(db);
}

// One thread per Q4_K superblock (gen_tiny_models.py quantize_q4_k, in f32).
__global__ void synth_q4_K_kernel(uint32_t K, uint32_t row0, uint32_t n_rows, uint64_t seed, float sigma,
                                  uint8_t* __restrict__ qs, uint8_t* __restrict__ meta) {
    const Layout L{1u, K};
    const uint32_t nsb = K / 256u;
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)n_rows * nsb) return;
    const uint32_t r = (uint32_t)(i / nsb), s = (uint32_t)(i % nsb);
    float step[8], mins[8], smax = 0.0f, mmax = 0.0f;
    // pass 1: ranges of the 8 sub-blocks (values regenerated in pass 2: no 256-float array)
    for (int j = 0; j < 8; ++j) {
        float lo = 0.0f, hi = -3.0e38f;
        for (int q4 = 0; q4 < 8; ++q4) {
            float o[4];
            normal4(seed, row0 + r, s * 64u + (uint32_t)j * 8u + (uint32_t)q4, o);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float v = o[e] * sigma;
                lo = fminf(lo, v);
                hi = fmaxf(hi, v);
            }
        }
        step[j] = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
        mins[j] = -lo;
        smax = fmaxf(smax, step[j]);
        mmax = fmaxf(mmax, mins[j]);
    }
    const uint16_t hd = f2h(__fdiv_rn(smax, 63.0f)), hm = f2h(__fdiv_rn(mmax, 63.0f));
    const float dd = h2f(hd), dm = h2f(hm);
    uint32_t sc[8], mn[8];
    for (int j = 0; j < 8; ++j) {
        const float a = dd > 0.0f ? rintf(__fdiv_rn(step[j], dd)) : 0.0f;
        const float b = dm > 0.0f ? rintf(__fdiv_rn(mins[j], dm)) : 0.0f;
        sc[j] = (uint32_t)fminf(fmaxf(a, 0.0f), 63.0f);
        mn[j] = (uint32_t)fminf(fmaxf(b, 0.0f), 63.0f);
    }
    uint8_t m[16];
    m[0] = (uint8_t)hd; m[1] = (uint8_t)(hd >> 8); m[2] = (uint8_t)hm; m[3] = (uint8_t)(hm >> 8);
    for (int j = 0; j < 4; ++j) {
        m[4 + j] = (uint8_t)((sc[j] & 63u) | ((sc[j + 4] >> 4) << 6));
        m[8 + j] = (uint8_t)((mn[j] & 63u) | ((mn[j + 4] >> 4) << 6));
        m[12 + j] = (uint8_t)((sc[j + 4] & 15u) | ((mn[j + 4] & 15u) << 4));
    }
    uint8_t* mo = meta + L.meta_off(r, s);
    for (int j = 0; j < 16; ++j) mo[j] = m[j];
    uint8_t qo[128];
    for (int c = 0; c < 4; ++c) {               // bytes 32c .. 32c+31: sub-block 2c low, 2c+1 high
        const float s0 = __fmul_rn(dd, (float)sc[2 * c]), o0 = __fmul_rn(dm, (float)mn[2 * c]);
        const float s1 = __fmul_rn(dd, (float)sc[2 * c + 1]), o1 = __fmul_rn(dm, (float)mn[2 * c + 1]);
        for (int q4 = 0; q4 < 8; ++q4) {
            float lo4[4], hi4[4];
            normal4(seed, row0 + r, s * 64u + (uint32_t)(2 * c) * 8u + (uint32_t)q4, lo4);
            normal4(seed, row0 + r, s * 64u + (uint32_t)(2 * c + 1) * 8u + (uint32_t)q4, hi4);
            for (int e = 0; e < 4; ++e) {
                const float a = s0 > 0.0f ? rintf(__fdiv_rn(__fadd_rn(lo4[e] * sigma, o0), s0)) : 0.0f;
                const float b = s1 > 0.0f ? rintf(__fdiv_rn(__fadd_rn(hi4[e] * sigma, o1), s1)) : 0.0f;
                const uint32_t ql = (uint32_t)fminf(fmaxf(a, 0.0f), 15.0f), qh = (uint32_t)fminf(fmaxf(b, 0.0f), 15.0f);
                qo[32 * c + 4 * q4 + e] = (uint8_t)(ql | (qh << 4));
            }
        }
    }
    for (uint32_t j = 0; j < 8; ++j)
        for (int e = 0; e < 16; ++e) qs[L.qs_off(r, s, j) + e] = qo[16 * j + e];
}

cudaError_t launch_synth(uint32_t fmt, uint32_t K, uint32_t row0, uint32_t n_rows, uint64_t seed, float sigma,
                         uint8_t* qs, uint8_t* meta, cudaStream_t st) {
    if (fmt == 0) {
        const uint64_t n = (uint64_t)n_rows * (K / 32u);
        if (n) synth_q8_0_kernel<<<grid_for(n, 128), 128, 0, st>>>(K, row0, n_rows, seed, sigma, qs, meta);
    } else {
        const uint64_t n = (uint64_t)n_rows * (K / 256u);
        if (n) synth_q4_K_kernel<<<grid_for(n, 128), 128, 0, st>>>(K, row0, n_rows, seed, sigma, qs, meta);
    }
    return cudaGetLastError();
}

}  // namespace tsrc
