// tsrc_mm_tc.cu -- prefill (many-token) Q8_0 / Q4_K MUL_MAT on the tcgen05 int8 tensor cores.
//
// Numerics: the reference's MVM row rule bit for bit (jwkim04/tesseract-npu sw/sim/tsr_ref.c:
// 533-635): for each token and row, block i contributes t_i = (d_w (*) Dx_i) (*) f32(isum_i) to
// partial p[i mod 16] (in order of i, from +0), then the fixed 16-partial tree. The exact int32
// block sums isum_i come from one tcgen05.mma (kind::i8, K = 32: one block) per block, written to
// a fresh TMEM tile (no accumulation across blocks: each block has its own scales). The f32 part
// runs in registers: blocks are visited partial by partial (i = j, j + 16, j + 32, ... for j = 0..15),
// so a thread needs one running partial per output plus a four-deep stack that folds the partials
// into the tree as they complete (((p0 + p1) + (p2 + p3)) + ...). Every factor is a multiple of
// 2^-24 (fp16 weight scales, the A32 activation scale stored as fp16, integer sums), so every
// product and sum is a multiple of 2^-48 and never subnormal: the flush tests are not needed.
//
// Work split: a CTA computes 128 rows x NT tokens; TMEM holds two 128 x NT int32 tiles (block s
// and block s + 1 alternate); warp w reads TMEM lanes 32 (w mod 4) .. + 31 (its rows) and columns
// 16 (w / 4) .. + 15 (its tokens). Operands go through a ring of kStages shared-memory stages,
// copied with cp.async into the canonical K-major, no-swizzle layout of the UMMA descriptors (8-row
// x 16-byte core matrices; the two 16-byte halves of a block 128 bytes apart, 8-row groups 256 bytes
// apart). One thread issues each MMA and commits it to an mbarrier; every wait on an mbarrier is
// bounded (error code 3 in the matvec error flag, reported by tsrc_sync).
#include "tsrc_internal.h"
#include "tsrc_layout.cuh"
#include "tsrc_numerics.cuh"

namespace tsrc {

namespace {

__device__ unsigned int g_tc_error;                // first error code of any launch (3: an MMA wait ran out)

constexpr uint32_t kStages = 6;                    // operand ring (blocks in flight: kStages - 2)
constexpr uint32_t kTileM = 128;
constexpr uint32_t kSpin = 1u << 22;               // mbarrier polls (~30 ns apart) before giving up

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// UMMA shared-memory descriptor: K-major, no swizzle; LBO = 128 B (K halves), SBO = 256 B (8-row groups)
__device__ __forceinline__ uint64_t umma_desc(const void* p) {
    const uint64_t a = (smem_u32(p) >> 4) & 0x3FFFu;
    return a | (uint64_t(128u >> 4) << 16) | (uint64_t(256u >> 4) << 32) | (uint64_t(1) << 46);
}

// instruction descriptor: s32 accumulator, signed int8 A and B, both K-major, M = 128, N = NT
template <uint32_t NT>
__device__ __forceinline__ uint32_t umma_idesc() {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((NT >> 3) << 17) | ((kTileM >> 4) << 24);
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t it = 0; it < kSpin; ++it) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
        __nanosleep(20);
    }
    return false;
}

// block of sequence position s in partial-major order (j = 0..15, then i = j, j + 16, ...)
struct Seq {
    uint32_t nb, q, rem;      // q = nb / 16, rem = nb % 16
    __device__ __forceinline__ uint32_t block(uint32_t s, uint32_t* j, bool* last) const {
        uint32_t jj, ii, cnt;
        if (s < rem * (q + 1u)) {
            jj = s / (q + 1u);
            ii = s - jj * (q + 1u);
            cnt = q + 1u;
        } else {
            const uint32_t s2 = s - rem * (q + 1u);
            jj = rem + s2 / q;
            ii = s2 - (jj - rem) * q;
            cnt = q;
        }
        *j = jj;
        *last = ii + 1u == cnt;
        return jj + 16u * ii;
    }
};

// folds partial j (value v) into the 16-partial tree kept as a four-level stack; after partial 15
// the tree's value is in L0
__device__ __forceinline__ void tree_push(float& L0, float& L1, float& L2, float& L3, uint32_t j, float v) {
    if ((j & 1u) == 0) { L0 = v; return; }
    v = fadd(L0, v);
    if ((j & 2u) == 0) { L1 = v; return; }
    v = fadd(L1, v);
    if ((j & 4u) == 0) { L2 = v; return; }
    v = fadd(L2, v);
    if ((j & 8u) == 0) { L3 = v; return; }
    L0 = fadd(L3, v);
}

template <uint32_t NT>
__global__ void __launch_bounds__(128 * (NT / 16), 1) mm_q8_tc_kernel(MvArgs a) {
    constexpr uint32_t WARPS = 4 * (NT / 16), THREADS = 32 * WARPS;
    constexpr uint32_t A_BYTES = kTileM * 32u, B_BYTES = NT * 32u;
    constexpr uint32_t TCOLS = 2 * NT <= 32 ? 32 : (2 * NT <= 64 ? 64 : 128);   // two tiles, a power of two
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* As = smem;                                               // [kStages][A_BYTES]
    uint8_t* Bs = As + kStages * A_BYTES;                             // [kStages][B_BYTES]
    float* DX = reinterpret_cast<float*>(Bs + kStages * B_BYTES);     // [kStages][NT]
    uint64_t* bars = reinterpret_cast<uint64_t*>(DX + kStages * NT);  // [2]
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const uint32_t row0 = blockIdx.x * kTileM, tok0 = blockIdx.y * NT;
    const uint32_t K = a.K, nb = K / 32u;
    const Layout L{0u, K};
    const Seq seq{nb, nb / 16u, nb % 16u};

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)), "r"(TCOLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[0])));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[1])));
        asm volatile("fence.mbarrier_init.release.cluster;");
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");     // the QA image comes from the previous kernel
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tslot;

    // stage fill: block of sequence position s into ring slot s % kStages (one commit group per thread)
    auto fill = [&](uint32_t s) {
        if (s < nb) {
            uint32_t j;
            bool last;
            const uint32_t b = seq.block(s, &j, &last), st = s % kStages;
            uint8_t* A = As + st * A_BYTES;
            uint8_t* B = Bs + st * B_BYTES;
            for (uint32_t c = tid; c < 2u * kTileM + 2u * NT; c += THREADS) {
                if (c < 2u * kTileM) {
                    const uint32_t r = c >> 1, h = c & 1u, row = row0 + r;
                    if (row < a.n_rows) cp_async16(A + (r >> 3) * 256u + h * 128u + (r & 7u) * 16u, a.qs + L.qs_off(row, b, h));
                } else {
                    const uint32_t i = c - 2u * kTileM, t = i >> 1, h = i & 1u, tok = tok0 + t;
                    if (tok < a.T) cp_async16(B + (t >> 3) * 256u + h * 128u + (t & 7u) * 16u, a.qx + (size_t)tok * K + 32u * b + 16u * h);
                }
            }
            for (uint32_t t = tid; t < NT; t += THREADS) DX[st * NT + t] = tok0 + t < a.T ? a.dx[(size_t)(tok0 + t) * nb + b] : 0.0f;
        }
        cp_async_commit();
    };

    // this thread's outputs: row, tokens 16 cq .. 16 cq + 15
    const uint32_t rq = warp & 3u, cq = warp >> 2;
    const uint32_t row = row0 + 32u * rq + lane;
    const uint8_t* meta = static_cast<const uint8_t*>(a.meta);
    float acc[16], L0[16], L1[16], L2[16], L3[16];
#pragma unroll
    for (uint32_t i = 0; i < 16; ++i) acc[i] = L0[i] = L1[i] = L2[i] = L3[i] = 0.0f;

    for (uint32_t s = 0; s + 2u < kStages; ++s) fill(s);
    uint32_t phase[2] = {0u, 0u};
    uint32_t jcur = 0;
    uint16_t dw_next = 0;
    {
        uint32_t j0;
        bool l0;
        const uint32_t b0 = seq.block(0, &j0, &l0);
        if (row < a.n_rows && nb) dw_next = *reinterpret_cast<const uint16_t*>(meta + L.meta_off(row, b0));
    }
    bool failed = false;
    for (uint32_t s = 0; s <= nb; ++s) {
        if (s < nb) {
            cp_async_wait<kStages - 3>();
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        asm volatile("tcgen05.fence::before_thread_sync;");
        __syncthreads();
        asm volatile("tcgen05.fence::after_thread_sync;");
        fill(s + kStages - 2u);                                  // slot of block s - 2: its MMA and reads are done
        if (s < nb && tid == 0) {
            const uint32_t st = s % kStages;
            const uint64_t da = umma_desc(As + st * A_BYTES), db = umma_desc(Bs + st * B_BYTES);
            const uint32_t d = tmem + (s & 1u) * NT;
            asm volatile(
                "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
                ::"r"(d), "l"(da), "l"(db), "r"(umma_idesc<NT>()), "r"(0u));
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         ::"r"(smem_u32(&bars[s & 1u])) : "memory");
        }
        if (s >= 1u) {
            const uint32_t sp = s - 1u, buf = sp & 1u;
            if (!mbar_wait(smem_u32(&bars[buf]), phase[buf])) failed = true;
            phase[buf] ^= 1u;
            asm volatile("tcgen05.fence::after_thread_sync;");
            uint32_t v[16];
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                  "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                : "r"(tmem + ((32u * rq) << 16) + buf * NT + 16u * cq));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            uint32_t j;
            bool last;
            seq.block(sp, &j, &last);
            const float dw = h2f(dw_next);
            if (sp + 1u < nb) {                                    // the next block's weight scale
                uint32_t jn;
                bool ln;
                const uint32_t bn = seq.block(sp + 1u, &jn, &ln);
                if (row < a.n_rows) dw_next = *reinterpret_cast<const uint16_t*>(meta + L.meta_off(row, bn));
            }
            const float* dxs = DX + (sp % kStages) * NT + 16u * cq;
#pragma unroll
            for (uint32_t i = 0; i < 16; ++i)
                acc[i] = fadd(acc[i], fmul(fmul(dw, dxs[i]), i2f((int32_t)v[i])));
            if (last) {                                            // partial j is complete
#pragma unroll
                for (uint32_t i = 0; i < 16; ++i) {
                    tree_push(L0[i], L1[i], L2[i], L3[i], j, acc[i]);
                    acc[i] = 0.0f;
                }
                jcur = j + 1u;
            }
        }
    }
    // partials nb .. 15 (fewer than 16 blocks) are +0
    for (uint32_t j = jcur; j < 16u; ++j) {
#pragma unroll
        for (uint32_t i = 0; i < 16; ++i) tree_push(L0[i], L1[i], L2[i], L3[i], j, 0.0f);
    }
    if (failed && lane == 0) atomicCAS(&g_tc_error, 0u, 3u);
    if (row < a.n_rows) {
#pragma unroll
        for (uint32_t i = 0; i < 16; ++i) {
            const uint32_t tok = tok0 + 16u * cq + i;
            if (tok < a.T) {
                float v = L0[i];
                if (a.flags & kMmAdd) v = fadd(daz(a.add[(size_t)tok * a.add_stride + row]), v);
                if (a.flags & kMmSoftcap) v = fmul(tanh_vu(fmul(v, a.s0), g_expk_t64, g_expk_lk), a.s1);
                else if (a.flags & kMmScale) v = fmul(v, a.s1);
                a.y[(size_t)tok * a.y_stride + row] = canon(v);
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS));
}

template <uint32_t NT>
size_t tc_smem() {
    return kStages * (kTileM * 32u + NT * 32u) + kStages * NT * 4u + 2u * 8u + 16u;
}

template <uint32_t NT>
cudaError_t launch_nt(const MvArgs& a, cudaStream_t st) {
    static int done_dev[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const size_t smem = tc_smem<NT>();
    if (dev < 64 && done_dev[dev] != dev + 1) {
        e = cudaFuncSetAttribute(mm_q8_tc_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        done_dev[dev] = dev + 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.n_rows + kTileM - 1u) / kTileM, (a.T + NT - 1u) / NT);
    cfg.blockDim = dim3(128u * (NT / 16u));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, mm_q8_tc_kernel<NT>, a);
}


// ---- Q4_K ---------------------------------------------------------------------------------------
// Per superblock (256 values) eight MMAs, one per 32-value sub-block j: A = the sub-block's nibbles
// expanded to int8 (0..15) in shared memory, B = the tokens' quantized activation of the same 32
// values; D = S_j[row][token] exactly. Then isum = sum_j sc_j S_j and msum = sum_j m_j (BS_2j +
// BS_2j+1) in int32 (exact, as tsr_ref.c:540-567), and the term d Dx isum - dmin Dx msum with the
// f32 rules (the A256 scale Dx is an arbitrary f32, so the flush tests stay).
template <uint32_t NT>
__global__ void __launch_bounds__(128 * (NT / 16), 1) mm_q4k_tc_kernel(MvArgs a) {
    constexpr uint32_t WARPS = 4 * (NT / 16), THREADS = 32 * WARPS;
    constexpr uint32_t RING = 4;
    constexpr uint32_t RAW = kTileM * 128u;            // the superblock's quants of 128 rows (16 KB)
    constexpr uint32_t ATILE = kTileM * 32u;           // one sub-block's expanded A tile
    constexpr uint32_t BTILE = NT * 32u;
    constexpr uint32_t TCOLS = 16 * NT <= 256 ? 256 : 512;   // two superblocks x 8 tiles
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* Raw = smem;                                                   // [RING][RAW]
    uint8_t* Ax = Raw + RING * RAW;                                        // [2][8][ATILE]
    uint8_t* Bs = Ax + 2u * 8u * ATILE;                                    // [RING][8][BTILE]
    float* DX = reinterpret_cast<float*>(Bs + RING * 8u * BTILE);          // [RING][NT]
    int32_t* BSS = reinterpret_cast<int32_t*>(DX + RING * NT);             // [RING][NT][8]
    uint64_t* bars = reinterpret_cast<uint64_t*>(BSS + RING * NT * 8u);    // [2]
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const uint32_t row0 = blockIdx.x * kTileM, tok0 = blockIdx.y * NT;
    const uint32_t K = a.K, nsb = K / 256u;
    const Layout L{1u, K};
    const Seq seq{nsb, nsb / 16u, nsb % 16u};

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)), "r"(TCOLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[0])));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[1])));
        asm volatile("fence.mbarrier_init.release.cluster;");
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tslot;

    auto fill = [&](uint32_t s) {
        if (s < nsb) {
            uint32_t j;
            bool last;
            const uint32_t sb = seq.block(s, &j, &last), st = s % RING;
            for (uint32_t c = tid; c < kTileM * 8u; c += THREADS) {          // 8 chunks of 16 B per row
                const uint32_t r = c >> 3, k = c & 7u, row = row0 + r;
                if (row < a.n_rows) cp_async16(Raw + st * RAW + r * 128u + k * 16u, a.qs + L.qs_off(row, sb, k));
            }
            for (uint32_t c = tid; c < 8u * NT * 2u; c += THREADS) {         // 8 sub-blocks x NT tokens x 2 halves
                const uint32_t jj = c / (2u * NT), rem = c - jj * 2u * NT, t = rem >> 1, h = rem & 1u, tok = tok0 + t;
                if (tok < a.T)
                    cp_async16(Bs + (st * 8u + jj) * BTILE + (t >> 3) * 256u + h * 128u + (t & 7u) * 16u,
                               a.qx + (size_t)tok * K + 256u * sb + 32u * jj + 16u * h);
            }
            for (uint32_t t = tid; t < NT; t += THREADS) {
                const uint32_t tok = tok0 + t;
                DX[st * NT + t] = tok < a.T ? a.dx[(size_t)tok * nsb + sb] : 0.0f;
#pragma unroll
                for (uint32_t jj = 0; jj < 8; ++jj) {
                    int32_t v = 0;
                    if (tok < a.T) {
                        const int16_t* b16 = a.bsx + (size_t)tok * (K / 16u) + 16u * sb + 2u * jj;
                        v = (int32_t)b16[0] + (int32_t)b16[1];
                    }
                    BSS[(st * NT + t) * 8u + jj] = v;
                }
            }
        }
        cp_async_commit();
    };
    // the raw quants of superblock s -> the eight expanded A tiles (low nibbles: sub-block 2c, high: 2c + 1)
    auto expand = [&](uint32_t s) {
        const uint32_t st = s % RING;
        uint8_t* A = Ax + (s & 1u) * 8u * ATILE;
        for (uint32_t c = tid; c < kTileM * 8u; c += THREADS) {
            const uint32_t r = c >> 3, k = c & 7u, cc = k >> 1, h = k & 1u;
            const uint4 w = *reinterpret_cast<const uint4*>(Raw + st * RAW + r * 128u + k * 16u);
            const uint4 lo = make_uint4(w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, w.z & 0x0F0F0F0Fu, w.w & 0x0F0F0F0Fu);
            const uint4 hi = make_uint4((w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu, (w.z >> 4) & 0x0F0F0F0Fu,
                                        (w.w >> 4) & 0x0F0F0F0Fu);
            const uint32_t off = (r >> 3) * 256u + h * 128u + (r & 7u) * 16u;
            *reinterpret_cast<uint4*>(A + (2u * cc) * ATILE + off) = lo;
            *reinterpret_cast<uint4*>(A + (2u * cc + 1u) * ATILE + off) = hi;
        }
    };

    const uint32_t rq = warp & 3u, cq = warp >> 2;
    const uint32_t row = row0 + 32u * rq + lane;
    const uint8_t* meta = static_cast<const uint8_t*>(a.meta);
    float acc[16], L0[16], L1[16], L2[16], L3[16];
#pragma unroll
    for (uint32_t i = 0; i < 16; ++i) acc[i] = L0[i] = L1[i] = L2[i] = L3[i] = 0.0f;

    for (uint32_t s = 0; s + 2u < RING; ++s) fill(s);
    uint32_t phase[2] = {0u, 0u};
    uint32_t jcur = 0;
    uint4 m_next = make_uint4(0, 0, 0, 0);
    if (nsb) {
        uint32_t j0;
        bool l0;
        const uint32_t sb0 = seq.block(0, &j0, &l0);
        if (row < a.n_rows) m_next = *reinterpret_cast<const uint4*>(meta + L.meta_off(row, sb0));
    }
    bool failed = false;
    for (uint32_t s = 0; s <= nsb; ++s) {
        if (s < nsb) {
            cp_async_wait<RING - 3>();
            __syncthreads();
            expand(s);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        asm volatile("tcgen05.fence::before_thread_sync;");
        __syncthreads();
        asm volatile("tcgen05.fence::after_thread_sync;");
        fill(s + RING - 2u);
        if (s < nsb && tid == 0) {
            const uint32_t st = s % RING;
#pragma unroll 1
            for (uint32_t jj = 0; jj < 8u; ++jj) {
                const uint64_t da = umma_desc(Ax + ((s & 1u) * 8u + jj) * ATILE);
                const uint64_t db = umma_desc(Bs + (st * 8u + jj) * BTILE);
                const uint32_t d = tmem + (s & 1u) * 8u * NT + jj * NT;
                asm volatile(
                    "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
                    ::"r"(d), "l"(da), "l"(db), "r"(umma_idesc<NT>()), "r"(0u));
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         ::"r"(smem_u32(&bars[s & 1u])) : "memory");
        }
        if (s >= 1u) {
            const uint32_t sp = s - 1u, buf = sp & 1u, st = sp % RING;
            if (!mbar_wait(smem_u32(&bars[buf]), phase[buf])) failed = true;
            phase[buf] ^= 1u;
            asm volatile("tcgen05.fence::after_thread_sync;");
            const uint4 m = m_next;
            if (sp + 1u < nsb) {
                uint32_t jn;
                bool ln;
                const uint32_t sbn = seq.block(sp + 1u, &jn, &ln);
                if (row < a.n_rows) m_next = *reinterpret_cast<const uint4*>(meta + L.meta_off(row, sbn));
            }
            const uint32_t sc_lo = m.y & 0x3F3F3F3Fu, mn_lo = m.z & 0x3F3F3F3Fu;
            const uint32_t sc_hi = (m.w & 0x0F0F0F0Fu) | ((m.y >> 2) & 0x30303030u);
            const uint32_t mn_hi = ((m.w >> 4) & 0x0F0F0F0Fu) | ((m.z >> 2) & 0x30303030u);
            int32_t isum[16];
#pragma unroll
            for (uint32_t i = 0; i < 16; ++i) isum[i] = 0;
#pragma unroll
            for (uint32_t jj = 0; jj < 8u; ++jj) {
                uint32_t v[16];
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                      "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                    : "r"(tmem + ((32u * rq) << 16) + buf * 8u * NT + jj * NT + 16u * cq));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                const int32_t sc = (int32_t)__byte_perm(jj < 4u ? sc_lo : sc_hi, 0u, 0x4440u | (jj & 3u));
#pragma unroll
                for (uint32_t i = 0; i < 16; ++i) isum[i] += sc * (int32_t)v[i];
            }
            uint32_t j;
            bool last;
            seq.block(sp, &j, &last);
            const float dw = h2f((uint16_t)(m.x & 0xFFFFu)), dmw = h2f((uint16_t)(m.x >> 16));
#pragma unroll
            for (uint32_t i = 0; i < 16; ++i) {
                const int32_t* bsv = BSS + (st * NT + 16u * cq + i) * 8u;
                int32_t msum = 0;
#pragma unroll
                for (uint32_t jj = 0; jj < 8u; ++jj)
                    msum += (int32_t)__byte_perm(jj < 4u ? mn_lo : mn_hi, 0u, 0x4440u | (jj & 3u)) * bsv[jj];
                const float Dx = DX[st * NT + 16u * cq + i];
                const float t1 = fmul(fmul(dw, Dx), i2f(isum[i]));
                const float t2 = fmul(fmul(dmw, Dx), i2f(msum));
                acc[i] = fadd(acc[i], fsub(t1, t2));
            }
            if (last) {
#pragma unroll
                for (uint32_t i = 0; i < 16; ++i) {
                    tree_push(L0[i], L1[i], L2[i], L3[i], j, acc[i]);
                    acc[i] = 0.0f;
                }
                jcur = j + 1u;
            }
        }
    }
    for (uint32_t j = jcur; j < 16u; ++j) {
#pragma unroll
        for (uint32_t i = 0; i < 16; ++i) tree_push(L0[i], L1[i], L2[i], L3[i], j, 0.0f);
    }
    if (failed && lane == 0) atomicCAS(&g_tc_error, 0u, 3u);
    if (row < a.n_rows) {
#pragma unroll
        for (uint32_t i = 0; i < 16; ++i) {
            const uint32_t tok = tok0 + 16u * cq + i;
            if (tok < a.T) {
                float v = L0[i];
                if (a.flags & kMmAdd) v = fadd(daz(a.add[(size_t)tok * a.add_stride + row]), v);
                if (a.flags & kMmSoftcap) v = fmul(tanh_vu(fmul(v, a.s0), g_expk_t64, g_expk_lk), a.s1);
                else if (a.flags & kMmScale) v = fmul(v, a.s1);
                a.y[(size_t)tok * a.y_stride + row] = canon(v);
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS));
}

template <uint32_t NT>
size_t q4k_smem() {
    return 4u * kTileM * 128u + 2u * 8u * kTileM * 32u + 4u * 8u * NT * 32u + 4u * NT * 4u + 4u * NT * 8u * 4u + 2u * 8u + 16u;
}

template <uint32_t NT>
cudaError_t launch_q4k_nt(const MvArgs& a, cudaStream_t st) {
    static int done_dev[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const size_t smem = q4k_smem<NT>();
    if (dev < 64 && done_dev[dev] != dev + 1) {
        e = cudaFuncSetAttribute(mm_q4k_tc_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        done_dev[dev] = dev + 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.n_rows + kTileM - 1u) / kTileM, (a.T + NT - 1u) / NT);
    cfg.blockDim = dim3(128u * (NT / 16u));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, mm_q4k_tc_kernel<NT>, a);
}

}  // namespace

cudaError_t tc_error(uint32_t* code, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(code, g_tc_error, sizeof(uint32_t));
    if (e == cudaSuccess && clear && *code) {
        const uint32_t zero = 0;
        e = cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(uint32_t));
    }
    return e;
}

// Q8_0 / Q4_K MUL_MAT of T tokens (their QA image in a.qx / a.dx / a.bsx) on the tensor cores.
cudaError_t launch_mm_tc(uint32_t fmt, const MvArgs& a, cudaStream_t st) {
    if (a.T == 0 || a.n_rows == 0 || fmt > 1u) return cudaErrorInvalidValue;
    if (fmt == 1u) return a.T <= 16 ? launch_q4k_nt<16>(a, st) : launch_q4k_nt<32>(a, st);
    if (a.T <= 16) return launch_nt<16>(a, st);
    if (a.T <= 32) return launch_nt<32>(a, st);
    if (a.T <= 48) return launch_nt<48>(a, st);
    return launch_nt<64>(a, st);
}

}  // namespace tsrc
