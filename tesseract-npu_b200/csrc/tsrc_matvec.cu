// tsrc_matvec.cu -- decode (small-T) Q8_0 / Q4_K matrix-vector products on sm_100a.
//
// Numerics are the reference's MVM row rule bit for bit (jwkim04/tesseract-npu
// sw/sim/tsr_ref.c:533-635): per block i an exact int32 sum, the term
// t_i = (d_w (*) Dx_i) (*) f32(isum_i) [Q4_K: minus (dmin (*) Dx) (*) f32(msum)], term i added
// in order into partial p[i mod 16] (from +0), then the fixed tree ((p0+p1)+(p2+p3))+... .
//
// Mapping (HBM-bound stream):
//   - one warp owns two weight rows; a "wave" is 16 consecutive blocks (Q8_0) / superblocks
//     (Q4_K) of both rows, loaded with coalesced 128-bit non-allocating loads before any math;
//   - the int8 dot products use dp4a (Q4_K nibbles unpacked in registers); exact partial sums
//     are combined with shuffles (integer sums: any order);
//   - the f32 part of the wave runs once per term: lane L takes row L/16, term L%16, so lane
//     L holds partial p[L%16] of its row across waves (term w0+k -> p[k]), the reference order;
//   - the tree is 4 xor-shuffle levels inside each 16-lane half (fadd is commutative).
// The quantized activations (QA of the T tokens) are staged in shared memory per CTA.
#include "tsrc_internal.h"
#include "tsrc_numerics.cuh"

namespace tsrc {

constexpr int kWarps = 8;                  // warps per CTA
__host__ __device__ constexpr size_t align16(size_t n) { return (n + 15u) & ~(size_t)15u; }
constexpr int kRowsPerWarp = 2;

__device__ __forceinline__ uint4 ld_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ int32_t dot16(const uint4 w, const uint4 x, int32_t acc) {
    acc = __dp4a((int)w.x, (int)x.x, acc);
    acc = __dp4a((int)w.y, (int)x.y, acc);
    acc = __dp4a((int)w.z, (int)x.z, acc);
    acc = __dp4a((int)w.w, (int)x.w, acc);
    return acc;
}

// Fixed 16-partial tree inside each 16-lane half of the warp (lanes k hold p[k]).
__device__ __forceinline__ float tree16_lanes(float v) {
    v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 1));
    v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 2));
    v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 4));
    v = fadd(v, __shfl_xor_sync(0xFFFFFFFFu, v, 8));
    return v;
}

// The MVM epilogues (tsr_sim.c:1648-1670; the ADD fusion of ggml-tesseract.cpp:2897-2914).
__device__ __forceinline__ float mm_epilogue(float v, const MvArgs& a, uint32_t t, uint32_t n) {
    if (a.flags & kMmAdd) v = fadd(daz(a.add[(size_t)t * a.add_stride + n]), v);
    if (a.flags & kMmSoftcap)
        v = fmul(tanh_vu(fmul(v, a.s0), g_expk_t64, g_expk_lk), a.s1);
    else if (a.flags & kMmScale)
        v = fmul(v, a.s1);
    return canon(v);
}

// ---------------------------------------------------------------------------------------------
// Q8_0: qs [n_rows][K] int8, d [n_rows][K/32] fp16. Wave = 16 blocks = 512 B per row; lane l of
// the wave reads bytes [16 l, 16 l + 16) = half (l & 1) of block l/2.
// ---------------------------------------------------------------------------------------------
template <int MAXT>
__global__ void __launch_bounds__(kWarps * 32, 2) mv_q8_0_kernel(MvArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    const uint32_t K = a.K, nb = K >> 5, T = a.T;
    int8_t* sq = reinterpret_cast<int8_t*>(smem);                 // [T][K]
    float* sd = reinterpret_cast<float*>(smem + (size_t)T * K);    // [T][nb]
    for (uint32_t i = threadIdx.x; i < T * K / 16u; i += blockDim.x)
        reinterpret_cast<uint4*>(sq)[i] = reinterpret_cast<const uint4*>(a.qx)[i];
    for (uint32_t i = threadIdx.x; i < T * nb; i += blockDim.x) sd[i] = a.dx[i];
    __syncthreads();

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t rowA = (blockIdx.x * kWarps + warp) * kRowsPerWarp;
    if (rowA >= a.n_rows) return;
    const bool hasB = rowA + 1u < a.n_rows;
    const uint32_t rowB = hasB ? rowA + 1u : rowA;
    const uint8_t* qA = a.qs + (size_t)rowA * K;
    const uint8_t* qB = a.qs + (size_t)rowB * K;
    const uint16_t* dW = reinterpret_cast<const uint16_t*>(a.meta);
    const uint32_t myrow = lane < 16u ? rowA : rowB;
    const uint32_t k = lane & 15u;

    float p[MAXT];
#pragma unroll
    for (int t = 0; t < MAXT; ++t) p[t] = 0.0f;

    for (uint32_t w0 = 0; w0 < nb; w0 += 16u) {
        const bool ldv = w0 + (lane >> 1) < nb;
        const uint4 z = make_uint4(0, 0, 0, 0);
        const uint4 wa = ldv ? ld_stream(qA + (size_t)w0 * 32u + 16u * lane) : z;
        const uint4 wb = ldv ? ld_stream(qB + (size_t)w0 * 32u + 16u * lane) : z;
        const uint32_t eb = w0 + k;
        const bool ev = eb < nb;
        const float dwf = ev ? h2f(__ldg(dW + (size_t)myrow * nb + eb)) : 0.0f;
#pragma unroll
        for (int t = 0; t < MAXT; ++t) {
            if (t < (int)T) {
                const uint4 xv = ldv ? *reinterpret_cast<const uint4*>(sq + (size_t)t * K + (size_t)w0 * 32u + 16u * lane) : z;
                int32_t sa = dot16(wa, xv, 0), sb = dot16(wb, xv, 0);
                sa += __shfl_xor_sync(0xFFFFFFFFu, sa, 1);
                sb += __shfl_xor_sync(0xFFFFFFFFu, sb, 1);
                const int32_t va = __shfl_sync(0xFFFFFFFFu, sa, 2u * k);
                const int32_t vb = __shfl_sync(0xFFFFFFFFu, sb, 2u * k);
                const int32_t isum = lane < 16u ? va : vb;
                if (ev) {
                    p[t] = fadd(p[t], fmul(fmul(dwf, sd[(size_t)t * nb + eb]), i2f(isum)));
                    if (a.isum_out && t == 0 && (lane < 16u || hasB))
                        a.isum_out[(size_t)myrow * nb + eb] = isum;
                }
            }
        }
    }
#pragma unroll
    for (int t = 0; t < MAXT; ++t) {
        if (t < (int)T) {
            const float v = tree16_lanes(p[t]);
            if (k == 0 && (lane == 0 || hasB)) a.y[(size_t)t * a.y_stride + myrow] = mm_epilogue(v, a, t, myrow);
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Q4_K: qs [n_rows][K/2] (the ggml qs bytes of each superblock, 128 B), meta [n_rows][K/256] x 16
// B ({d, dmin, scales[12]}). Wave = 16 superblocks in 4 steps of 4; in a step lane l reads 16 B
// at 16 (l & 7) of superblock 4 step + l/8: low nibbles = sub-block 2g values 16h .. 16h+15, high
// nibbles = sub-block 2g+1 values 16h .. 16h+15 (g = (l & 7)/2, h = l & 1).
// ---------------------------------------------------------------------------------------------
template <int MAXT>
__global__ void __launch_bounds__(kWarps * 32, 2) mv_q4_K_kernel(MvArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    const uint32_t K = a.K, nsb = K >> 8, T = a.T;
    // regions, each 16-byte aligned: q [T][K] | d [T][nsb] | sub-block sums [T][K/32] | exchange
    int8_t* sq = reinterpret_cast<int8_t*>(smem);
    float* sd = reinterpret_cast<float*>(smem + (size_t)T * K);
    int32_t* sbs = reinterpret_cast<int32_t*>(smem + (size_t)T * K + align16((size_t)T * nsb * 4u));
    uint4* xch = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(sbs) + (size_t)T * (K >> 5) * 4u);
    for (uint32_t i = threadIdx.x; i < T * K / 16u; i += blockDim.x)
        reinterpret_cast<uint4*>(sq)[i] = reinterpret_cast<const uint4*>(a.qx)[i];
    for (uint32_t i = threadIdx.x; i < T * nsb; i += blockDim.x) sd[i] = a.dx[i];
    for (uint32_t i = threadIdx.x; i < T * (K >> 5); i += blockDim.x)
        sbs[i] = (int32_t)a.bsx[2u * i] + (int32_t)a.bsx[2u * i + 1u];
    __syncthreads();

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t rowA = (blockIdx.x * kWarps + warp) * kRowsPerWarp;
    if (rowA >= a.n_rows) return;
    const bool hasB = rowA + 1u < a.n_rows;
    const uint32_t rowB = hasB ? rowA + 1u : rowA;
    const uint8_t* qA = a.qs + (size_t)rowA * (K >> 1);
    const uint8_t* qB = a.qs + (size_t)rowB * (K >> 1);
    const uint4* mA = reinterpret_cast<const uint4*>(a.meta) + (size_t)rowA * nsb;
    const uint4* mB = reinterpret_cast<const uint4*>(a.meta) + (size_t)rowB * nsb;
    const uint32_t grp = lane >> 3, sub = lane & 7u, g = sub >> 1, h = sub & 1u;
    const uint32_t myrow = lane < 16u ? rowA : rowB;
    const uint32_t k = lane & 15u;
    uint4* wx = xch + warp * 32u;

    float p[MAXT];
#pragma unroll
    for (int t = 0; t < MAXT; ++t) p[t] = 0.0f;

    for (uint32_t w0 = 0; w0 < nsb; w0 += 16u) {
        uint4 wq[2][4], wm[2][4];
        const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int it = 0; it < 4; ++it) {
            const uint32_t sb = w0 + 4u * it + grp;
            const bool v = sb < nsb;
            wq[0][it] = v ? ld_stream(qA + (size_t)sb * 128u + 16u * sub) : z;
            wq[1][it] = v ? ld_stream(qB + (size_t)sb * 128u + 16u * sub) : z;
            wm[0][it] = v ? __ldg(mA + sb) : z;
            wm[1][it] = v ? __ldg(mB + sb) : z;
        }
#pragma unroll
        for (int t = 0; t < MAXT; ++t) {
            if (t < (int)T) {
                const int8_t* xt = sq + (size_t)t * K;
                const int32_t* bt = sbs + (size_t)t * (K >> 5);
#pragma unroll
                for (int r = 0; r < 2; ++r) {
#pragma unroll
                    for (int it = 0; it < 4; ++it) {
                        const uint32_t sb = w0 + 4u * it + grp;
                        int32_t isum = 0, msum = 0;
                        if (sb < nsb) {
                            const int8_t* xs = xt + (size_t)sb * 256u + 64u * g + 16u * h;
                            const uint4 xlo = *reinterpret_cast<const uint4*>(xs);
                            const uint4 xhi = *reinterpret_cast<const uint4*>(xs + 32);
                            const uint4 w = wq[r][it];
                            const uint4 wl = make_uint4(w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, w.z & 0x0F0F0F0Fu,
                                                        w.w & 0x0F0F0F0Fu);
                            const uint4 wh = make_uint4((w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu,
                                                        (w.z >> 4) & 0x0F0F0F0Fu, (w.w >> 4) & 0x0F0F0F0Fu);
                            const int32_t slo = dot16(wl, xlo, 0), shi = dot16(wh, xhi, 0);
                            // 6-bit scales / mins of sub-blocks 2g, 2g+1 (ggml get_scale_min_k4)
                            const uint4 m = wm[r][it];
                            const uint32_t scw = g < 2u ? (m.y & 0x3F3F3F3Fu)
                                                        : ((m.w & 0x0F0F0F0Fu) | ((m.y >> 2) & 0x30303030u));
                            const uint32_t mnw = g < 2u ? (m.z & 0x3F3F3F3Fu)
                                                        : (((m.w >> 4) & 0x0F0F0F0Fu) | ((m.z >> 2) & 0x30303030u));
                            const uint32_t sh = (g & 1u) * 16u;
                            const int32_t sc0 = (int32_t)((scw >> sh) & 0xFFu), sc1 = (int32_t)((scw >> (sh + 8u)) & 0xFFu);
                            isum = sc0 * slo + sc1 * shi;
                            if (h == 0u) {
                                const int32_t m0 = (int32_t)((mnw >> sh) & 0xFFu), m1 = (int32_t)((mnw >> (sh + 8u)) & 0xFFu);
                                msum = m0 * bt[sb * 8u + 2u * g] + m1 * bt[sb * 8u + 2u * g + 1u];
                            }
                        }
                        isum += __shfl_xor_sync(0xFFFFFFFFu, isum, 1);
                        msum += __shfl_xor_sync(0xFFFFFFFFu, msum, 1);
                        isum += __shfl_xor_sync(0xFFFFFFFFu, isum, 2);
                        msum += __shfl_xor_sync(0xFFFFFFFFu, msum, 2);
                        isum += __shfl_xor_sync(0xFFFFFFFFu, isum, 4);
                        msum += __shfl_xor_sync(0xFFFFFFFFu, msum, 4);
                        if (sub == 0u) wx[r * 16 + 4 * it + grp] = make_uint4((uint32_t)isum, (uint32_t)msum, wm[r][it].x, 0u);
                    }
                }
                __syncwarp();
                const uint32_t sb = w0 + k;
                if (sb < nsb) {
                    const uint4 e = wx[lane];
                    const float Dx = sd[(size_t)t * nsb + sb];
                    const float t1 = fmul(fmul(h2f((uint16_t)(e.z & 0xFFFFu)), Dx), i2f((int32_t)e.x));
                    const float t2 = fmul(fmul(h2f((uint16_t)(e.z >> 16)), Dx), i2f((int32_t)e.y));
                    p[t] = fadd(p[t], fsub(t1, t2));
                    if (a.isum_out && t == 0 && (lane < 16u || hasB)) {
                        a.isum_out[((size_t)myrow * nsb + sb) * 2u] = (int32_t)e.x;
                        a.isum_out[((size_t)myrow * nsb + sb) * 2u + 1u] = (int32_t)e.y;
                    }
                }
                __syncwarp();
            }
        }
    }
#pragma unroll
    for (int t = 0; t < MAXT; ++t) {
        if (t < (int)T) {
            const float v = tree16_lanes(p[t]);
            if (k == 0 && (lane == 0 || hasB)) a.y[(size_t)t * a.y_stride + myrow] = mm_epilogue(v, a, t, myrow);
        }
    }
}

size_t mv_smem_bytes(uint32_t fmt, uint32_t K, uint32_t T) {
    if (fmt == 0) return (size_t)T * K + (size_t)T * (K / 32u) * 4u;
    return (size_t)T * K + align16((size_t)T * (K / 256u) * 4u) + (size_t)T * (K / 32u) * 4u + (size_t)kWarps * 32u * 16u;
}

// The dynamic shared-memory limit is raised once per kernel and device (before any stream
// capture can be active: the first call of a shape is an ordinary launch).
template <typename F>
static cudaError_t allow_smem(F* kernel, size_t smem) {
    static int done_dev[64];            // 1 + device index when set (zero-initialised)
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (smem <= 48u * 1024u || (dev < 64 && done_dev[dev] == dev + 1)) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e == cudaSuccess && dev < 64) done_dev[dev] = dev + 1;
    return e;
}

template <int MAXT>
static cudaError_t launch_mv_t(uint32_t fmt, const MvArgs& a, cudaStream_t st) {
    const uint32_t rows_per_cta = kWarps * kRowsPerWarp;
    const uint32_t blocks = (a.n_rows + rows_per_cta - 1u) / rows_per_cta;
    const size_t smem = mv_smem_bytes(fmt, a.K, a.T);
    cudaError_t e;
    if (fmt == 0) {
        if ((e = allow_smem(mv_q8_0_kernel<MAXT>, smem)) != cudaSuccess) return e;
        mv_q8_0_kernel<MAXT><<<blocks, kWarps * 32, smem, st>>>(a);
    } else {
        if ((e = allow_smem(mv_q4_K_kernel<MAXT>, smem)) != cudaSuccess) return e;
        mv_q4_K_kernel<MAXT><<<blocks, kWarps * 32, smem, st>>>(a);
    }
    return cudaGetLastError();
}

cudaError_t launch_matvec(uint32_t fmt, const MvArgs& a, cudaStream_t st) {
    if (a.n_rows == 0 || a.T == 0) return cudaSuccess;
    if (a.T <= 1) return launch_mv_t<1>(fmt, a, st);
    if (a.T <= 2) return launch_mv_t<2>(fmt, a, st);
    if (a.T <= 4) return launch_mv_t<4>(fmt, a, st);
    return launch_mv_t<kMvMaxT>(fmt, a, st);
}

}  // namespace tsrc
