// tsrc_mm_tc.cu -- prefill (many-token) Q8_0 / Q4_K MUL_MAT on the tcgen05 int8 tensor cores.
//
// Numerics: the reference's MVM row rule bit for bit (jwkim04/tesseract-npu sw/sim/tsr_ref.c:
// 533-635): for each token and row, block i contributes t_i = (d_w (*) Dx_i) (*) f32(isum_i) to
// partial p[i mod 16] (in order of i, from +0), then the fixed 16-partial tree. The exact int32
// block sums come from tcgen05.mma (kind::i8): Q8_0 one K = 32 MMA per block into a fresh TMEM tile
// (each block has its own scales); Q4_K the superblock's scaled sums over K = 256 (its section below
// says how the 6-bit sub-block scales and mins reach the tensor cores exactly). The f32 part runs on
// the CUDA cores: blocks are visited partial by partial (i = j, j + 16, j + 32, ... for
// j = 0..15), so a thread keeps one running partial per output and folds the partials into the
// tree as they complete (((p0 + p1) + (p2 + p3)) + ...) through a four-level stack in TMEM.
// Q8_0: every factor is a multiple of 2^-24 (fp16 weight scales, the A32 activation scale stored as
// fp16, integer sums), so every product and sum is a multiple of 2^-48 and never subnormal: the
// flush tests are not needed.
//
// Work split: a CTA computes 128 rows x NT tokens with warp-specialised roles (a producer warp
// loading the operand tiles by TMA into rings of shared-memory stages in K-major, no-swizzle layouts
// of the UMMA descriptors -- 8-row x 16-byte core matrices, the strides between them set by each
// tensor map's box order --, one thread issuing the MMAs,
// epilogue warps reading TMEM lanes 32 (w mod 4) .. + 31 and token columns 16 (w / 4) .. + 15),
// handing work over through mbarriers. Every wait is bounded by the SM clock (~1 s); a wait that
// runs out sets a CTA-wide abort flag that ends every role's loop, and error code 3, reported by
// tsrc_sync.
#include <cuda.h>                                  // CUtensorMap (the encoder is reached through the runtime)

#include <algorithm>
#include <mutex>

#include "tsrc_internal.h"
#include "tsrc_layout.cuh"
#include "tsrc_numerics.cuh"

namespace tsrc {

namespace {

__device__ unsigned int g_tc_error;                // first error code of any launch (3: an MMA wait ran out)

constexpr uint32_t kTileM = 128;

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

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

// ---- pipeline primitives (warp-specialised kernels) --------------------------------------------
constexpr long long kWaitCycles = 1ll << 31;       // a wait gives up after ~1 s of SM clock

__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// arrive on b once every cp.async this thread has issued so far has landed (counted in the init count)
__device__ __forceinline__ void cp_async_arrive(uint64_t* b) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
// Bounded wait for the phase of the given parity. A CTA-wide abort flag ends every role's wait once
// one of them has given up (error code 3 in the tensor-core error flag).
__device__ __forceinline__ bool mbar_wait_ab(uint64_t* b, uint32_t parity, volatile uint32_t* abort_flag) {
    const uint32_t bar = smem_u32(b);
    long long t0 = 0;
    for (uint32_t it = 0;; ++it) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"     // the default suspend time
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
        // the abort flag and the clock every 64 polls: a poll is a shared-memory access, and warps
        // spinning here take issue slots and shared-memory bandwidth from the warps doing the work
        if ((it & 63u) != 0u) continue;
        if (*abort_flag) return false;
        if (it == 0) t0 = clock64();
        else if (clock64() - t0 > kWaitCycles) break;
    }
    *abort_flag = 1u;
    atomicCAS(&g_tc_error, 0u, 3u);
    return false;
}
__device__ __forceinline__ void mma_commit(uint64_t* b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void mma_i8(uint32_t d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
// waits for every tcgen05.ld of the thread: their registers are valid after it, not before
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// ---- TMA and TMEM helpers (both kernels) -------------------------------------------------------
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* m, int32_t c0, int32_t c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(m), "r"(c0), "r"(c1), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* m, int32_t c0, int32_t c1, int32_t c2, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(smem_u32(dst)), "l"(m), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* m, int32_t c0, int32_t c1, int32_t c2, int32_t c3,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
        ::"r"(smem_u32(dst)), "l"(m), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)) : "memory");
}
// Bounded wait that ignores the abort flag: the producer's last look at the loads it issued, so that
// no TMA write lands in this CTA's shared memory after it has exited
__device__ __forceinline__ void mbar_wait_drain(uint64_t* b, uint32_t parity) {
    const uint32_t bar = smem_u32(b);
    const long long t0 = clock64();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity), "r"(1000u)
            : "memory");
        if (ok || clock64() - t0 > kWaitCycles) return;
    }
}
// UMMA descriptor of a B image laid out by a b map (box {16, NT, 2, ...}): K-major, no swizzle,
// LBO = 16 NT (K halves), SBO = 128 (8-token groups)
template <uint32_t NT>
__device__ __forceinline__ uint64_t umma_desc_b(const void* p) {
    const uint64_t a = (smem_u32(p) >> 4) & 0x3FFFu;
    return a | (uint64_t((16u * NT) >> 4) << 16) | (uint64_t(128u >> 4) << 32) | (uint64_t(1) << 46);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
          "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])),
          "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
          "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
          "r"(__float_as_uint(v[15]))
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Folds partial j (16 values, one per token of the thread) into the 16-partial tree whose four stack
// levels live in TMEM columns s, s + CS, s + 2 CS, s + 3 CS of the thread's lane (the stacked, earlier
// partial is the left operand of each sum); after partial 15 the tree's value is level 0. FLUSH: the
// reference's flush test on every sum.
template <uint32_t CS, bool FLUSH>
__device__ __forceinline__ void tree_push_tmem(uint32_t s, uint32_t j, float (&v)[16]) {
#pragma unroll
    for (uint32_t lvl = 0; lvl < 4; ++lvl) {
        if (((j >> lvl) & 1u) == 0u) {
            tmem_st16(s + lvl * CS, v);
            tmem_wait_st();
            return;
        }
        uint32_t p[16];
        tmem_ld16(s + lvl * CS, p);
        tmem_wait_ld();
#pragma unroll
        for (uint32_t i = 0; i < 16; ++i)
            v[i] = FLUSH ? fadd(__uint_as_float(p[i]), v[i]) : __fadd_rn(__uint_as_float(p[i]), v[i]);
    }
    tmem_st16(s, v);
    tmem_wait_st();
}


// ---- Q8_0 ---------------------------------------------------------------------------------------
// Warp roles: E epilogue warps (warp w: TMEM lanes 32 (w mod 4) .., tokens 16 (w / 4) ..), one producer
// warp (lane 0 loads the weight and activation tiles of BPS consecutive blocks of the sequence by TMA
// into one of S ring stages; the lanes copy the blocks' activation and weight scales with cp.async and
// arrive when they have landed), one MMA warp (TMEM allocation; one thread issues the stage's MMAs into
// one of NB accumulator groups of BPS tiles). The partial trees' stacks live in TMEM after the
// accumulators. mbarriers: full[S] (producer -> MMA, epilogue), empty[S] (MMA commit + epilogue warps ->
// producer), tfull[NB] (MMA commit -> epilogue), tempty[NB] (epilogue warps -> MMA).
// Tensor maps (TMA, no swizzle, no multicast):
//  a:    the Q8_0 quants of the full 16-block tiles, dims {256 B of a chunk line, row, chunk, tile}
//        (strides {qrow, 256, 512}), box {16, 128, 2, 1}: block b of 128 rows lands as
//        smem[2048 chunk + 16 row + byte], the K-major UMMA layout with LBO = 2048, SBO = 128;
//  tail: the same for the last tile when it holds nv < 16 blocks (chunk stride 16 nv);
//  b:    the QA image, dims {16 B, token, 16-value half} (strides {K, 16}), box {16, NT, 2}: block b of
//        NT tokens lands as smem[16 NT half + 16 token + byte] (LBO = 16 NT, SBO = 128).
template <uint32_t NT>
struct Q8Cfg {
    static constexpr uint32_t E = 4u * (NT / 16u), P = 1u;
    static constexpr uint32_t WARPS = E + P + 1u;
    static constexpr uint32_t BPS = 4u;                  // blocks per stage: fewer barrier rounds per block
    static constexpr uint32_t S = 6u;
    static constexpr uint32_t NB = 1u;                   // with the stack: 128 / 256 / 512 TMEM columns
    static constexpr uint32_t A_BYTES = kTileM * 32u, B_BYTES = NT * 32u;
    static constexpr uint32_t B_OFF = BPS * A_BYTES;
    static constexpr uint32_t DX_OFF = B_OFF + BPS * B_BYTES, DW_OFF = DX_OFF + BPS * NT * 4u;
    static constexpr uint32_t STAGE = (DW_OFF + BPS * kTileM * 4u + 127u) & ~127u;
    static constexpr uint32_t CS = NT == 48u ? 64u : NT;   // TMEM columns per accumulator tile / stack level
    static constexpr uint32_t STK_COL = NB * BPS * CS, USED = STK_COL + 4u * CS;
    static constexpr uint32_t TCOLS = USED <= 128u ? 128u : USED <= 256u ? 256u : 512u;
    static constexpr size_t BAR_OFF = (size_t)S * STAGE;
    static constexpr size_t SMEM = BAR_OFF + (2u * S + 2u * NB) * 8u + 16u;
    static_assert(USED <= 512u, "TMEM columns");
    static_assert(SMEM <= 227u * 1024u, "shared memory");
    static_assert(NT <= 64u, "Dx copies: at most two per producer lane");
    static_assert(NT % 16u == 0u, "M = 128 MMAs take N in multiples of 16");
};

struct alignas(64) Q8Maps {
    CUtensorMap a, tail, b;
    uint32_t nfull;        // tiles of 16 blocks in a row; blocks from 16 nfull on are in the tail
};

// UMMA descriptor of an A tile laid out by the a map: K-major, no swizzle, LBO = 2048, SBO = 128
__device__ __forceinline__ uint64_t umma_desc_a8(const void* p) {
    const uint64_t a = (smem_u32(p) >> 4) & 0x3FFFu;
    return a | (uint64_t(2048u >> 4) << 16) | (uint64_t(128u >> 4) << 32) | (uint64_t(1) << 46);
}

template <uint32_t NT>
__global__ void __launch_bounds__(32 * Q8Cfg<NT>::WARPS, 1) mm_q8_tc_kernel(MvArgs a, const __grid_constant__ Q8Maps tm) {
    using C = Q8Cfg<NT>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
    uint64_t* empty = full + C::S;
    uint64_t* tfull = empty + C::S;
    uint64_t* tempty = tfull + C::NB;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(tempty + C::NB);
    volatile uint32_t* abort_flag = tslot + 1;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    // persistent CTAs: tile t = (row tile t mod rt, token tile t / rt) for t = blockIdx.x, + gridDim.x, ...
    const uint32_t rt = (a.n_rows + kTileM - 1u) / kTileM, n_tiles = rt * ((a.T + NT - 1u) / NT);
    const uint32_t K = a.K, nb = K / 32u, q = nb >> 4, rem = nb & 15u;
    const uint32_t nst = (nb + C::BPS - 1u) / C::BPS;      // stage uses per tile
    const Layout L{0u, K};

    if (warp == C::E + C::P) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)), "r"(C::TCOLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < C::S; ++i) {
            mbar_init(&full[i], 1u + 32u * C::P);                // the TMA issuer's expect_tx + every lane's scale copies
            mbar_init(&empty[i], 1u + C::E);
        }
        for (uint32_t i = 0; i < C::NB; ++i) {
            mbar_init(&tfull[i], 1u);
            mbar_init(&tempty[i], C::E);
        }
        *abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;");
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");     // the QA image comes from the previous kernel
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tslot;

    if (warp >= C::E && warp < C::E + C::P) {
        // ---- producer warp
        const uint32_t nfull = tm.nfull;
        uint32_t g = 0;                                          // stage uses issued, over all tiles
        bool quit = false;
        for (uint32_t tile = blockIdx.x; tile < n_tiles && !quit; tile += gridDim.x) {
            const uint32_t row0 = (tile % rt) * kTileM, tok0 = (tile / rt) * NT;
            const float* dxrow[2];
#pragma unroll
            for (uint32_t k = 0; k < 2u; ++k) dxrow[k] = a.dx + (size_t)min(tok0 + lane + 32u * k, a.T - 1u) * nb;
            const uint8_t* wrow[kTileM / 32u];
#pragma unroll
            for (uint32_t k = 0; k < kTileM / 32u; ++k)
                wrow[k] = static_cast<const uint8_t*>(a.meta) + (size_t)min(row0 + lane + 32u * k, a.n_rows - 1u) * L.meta_row_bytes();
            uint32_t j = 0, ii = 0, cnt = q + (rem > 0u ? 1u : 0u);
            for (uint32_t u = 0; u < nst; ++u, ++g) {
                const uint32_t st = g % C::S;
                if (g >= C::S && !mbar_wait_ab(&empty[st], ((g / C::S) - 1u) & 1u, abort_flag)) { quit = true; break; }
                uint8_t* sb = smem + (size_t)st * C::STAGE;
                const uint32_t nx = min(C::BPS, nb - u * C::BPS);    // blocks in this stage
                if (lane == 0) mbar_expect_tx(&full[st], nx * (C::A_BYTES + C::B_BYTES));
#pragma unroll
                for (uint32_t x = 0; x < C::BPS; ++x) {
                    if (x < nx) {
                        const uint32_t b = j + 16u * ii;
                        if (lane == 0) {
                            const bool in_full = (b >> 4) < nfull;
                            tma_load_4d(sb + x * C::A_BYTES, in_full ? &tm.a : &tm.tail, (int32_t)(16u * (b & 15u)), (int32_t)row0,
                                        0, in_full ? (int32_t)(b >> 4) : 0, &full[st]);
                            tma_load_3d(sb + C::B_OFF + x * C::B_BYTES, &tm.b, 0, (int32_t)tok0, (int32_t)(2u * b), &full[st]);
                        }
#pragma unroll
                        for (uint32_t k = 0; k < 2u; ++k)
                            if (lane + 32u * k < NT) cp_async4(sb + C::DX_OFF + x * NT * 4u + 4u * (lane + 32u * k), dxrow[k] + b);
#pragma unroll
                        for (uint32_t k = 0; k < kTileM / 32u; ++k)
                            cp_async4(sb + C::DW_OFF + x * kTileM * 4u + 4u * (lane + 32u * k), wrow[k] + 2u * (b & ~1u));
                        if (++ii == cnt) {
                            ++j;
                            ii = 0;
                            cnt = q + (j < rem ? 1u : 0u);
                        }
                    }
                }
                cp_async_arrive(&full[st]);                      // the stage is published when its copies land
            }
        }
        cp_async_wait<0>();
        if (lane == 0)      // the last loads into each stage have landed before the CTA may exit
            for (uint32_t v = g > C::S ? g - C::S : 0u; v < g; ++v) mbar_wait_drain(&full[v % C::S], (v / C::S) & 1u);
        __syncwarp();
    } else if (warp == C::E + C::P) {
        // ---- MMA issuer
        if (lane == 0) {
            uint32_t g = 0;
            bool quit = false;
            for (uint32_t tile = blockIdx.x; tile < n_tiles && !quit; tile += gridDim.x) {
                for (uint32_t u = 0; u < nst; ++u, ++g) {
                    const uint32_t st = g % C::S, buf = g % C::NB;
                    if (!mbar_wait_ab(&full[st], (g / C::S) & 1u, abort_flag)) { quit = true; break; }
                    if (g >= C::NB && !mbar_wait_ab(&tempty[buf], ((g / C::NB) - 1u) & 1u, abort_flag)) { quit = true; break; }
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    uint8_t* sb = smem + (size_t)st * C::STAGE;
#pragma unroll
                    for (uint32_t x = 0; x < C::BPS; ++x)
                        if (u * C::BPS + x < nb)
                            mma_i8(tmem + (buf * C::BPS + x) * C::CS, umma_desc_a8(sb + x * C::A_BYTES),
                                   umma_desc_b<NT>(sb + C::B_OFF + x * C::B_BYTES), umma_idesc<NT>(), 0u);
                    mma_commit(&tfull[buf]);
                    mma_commit(&empty[st]);
                }
            }
            if (g) {          // the last MMA (and with it every earlier one) has completed
                const uint32_t u = g - 1u;
                mbar_wait_ab(&tfull[u % C::NB], (u / C::NB) & 1u, abort_flag);
            }
        }
        __syncwarp();
    } else {
        // ---- epilogue: row = row0 + 32 rq + lane, tokens tok0 + 16 cq + i of each tile
        const uint32_t rq = warp & 3u, cq = warp >> 2;
        const uint32_t tl = tmem + ((32u * rq) << 16) + 16u * cq, ts = tl + C::STK_COL;
        uint32_t g = 0;
        bool aborted = false;
        for (uint32_t tile = blockIdx.x; tile < n_tiles && !aborted; tile += gridDim.x) {
            const uint32_t row = (tile % rt) * kTileM + 32u * rq + lane, tok0 = (tile / rt) * NT;
            float acc[16];
#pragma unroll
            for (uint32_t i = 0; i < 16; ++i) acc[i] = 0.0f;
            uint32_t j = 0, ii = 0, cnt = q + (rem > 0u ? 1u : 0u);
            for (uint32_t u = 0; u < nst; ++u, ++g) {
                const uint32_t st = g % C::S, buf = g % C::NB;
                if (!mbar_wait_ab(&tfull[buf], (g / C::NB) & 1u, abort_flag)) { aborted = true; break; }
                if (!mbar_wait_ab(&full[st], (g / C::S) & 1u, abort_flag)) { aborted = true; break; }
                asm volatile("tcgen05.fence::after_thread_sync;");
                const uint8_t* sb = smem + (size_t)st * C::STAGE;
                uint32_t v[C::BPS][16];
#pragma unroll
                for (uint32_t x = 0; x < C::BPS; ++x) tmem_ld16(tl + (buf * C::BPS + x) * C::CS, v[x]);
                tmem_wait_ld();
                asm volatile("tcgen05.fence::before_thread_sync;");
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[buf]);      // the accumulator group is free again
#pragma unroll
                for (uint32_t x = 0; x < C::BPS; ++x) {
                    if (u * C::BPS + x < nb) {
                        const float4* dx4 = reinterpret_cast<const float4*>(sb + C::DX_OFF + x * NT * 4u + 64u * cq);
                        const uint32_t dwp = reinterpret_cast<const uint32_t*>(sb + C::DW_OFF + x * kTileM * 4u)[32u * rq + lane];
                        const uint32_t b = j + 16u * ii;
                        const float dw = h2f((uint16_t)((b & 1u) ? (dwp >> 16) : (dwp & 0xFFFFu)));
#pragma unroll
                        for (uint32_t k = 0; k < 4; ++k) {
                            const float4 f = dx4[k];
                            const float d4[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
                            for (uint32_t e = 0; e < 4; ++e) {
                                const uint32_t i = 4u * k + e;
                                acc[i] = __fadd_rn(acc[i], __fmul_rn(__fmul_rn(dw, d4[e]), __int2float_rn((int32_t)v[x][i])));
                            }
                        }
                        if (++ii == cnt) {                       // partial j is complete
                            tree_push_tmem<C::CS, false>(ts, j, acc);
#pragma unroll
                            for (uint32_t i = 0; i < 16; ++i) acc[i] = 0.0f;
                            ++j;
                            ii = 0;
                            cnt = q + (j < rem ? 1u : 0u);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[st]);
            }
            if (aborted) break;
            for (; j < 16u; ++j) {                               // partials nb .. 15 (fewer than 16 blocks) are +0
                float z[16];
#pragma unroll
                for (uint32_t i = 0; i < 16; ++i) z[i] = 0.0f;
                tree_push_tmem<C::CS, false>(ts, j, z);
            }
            uint32_t out[16];
            tmem_ld16(ts, out);                                  // the tree's value: level 0
            tmem_wait_ld();
            if (row < a.n_rows) {
#pragma unroll
                for (uint32_t i = 0; i < 16; ++i) {
                    const uint32_t tok = tok0 + 16u * cq + i;
                    if (tok < a.T) {
                        float y = __uint_as_float(out[i]);
                        if (a.flags & kMmAdd) y = fadd(daz(a.add[(size_t)tok * a.add_stride + row]), y);
                        if (a.flags & kMmSoftcap) y = fmul(tanh_vu(fmul(y, a.s0), g_expk_t64, g_expk_lk), a.s1);
                        else if (a.flags & kMmScale) y = fmul(y, a.s1);
                        a.y[(size_t)tok * a.y_stride + row] = canon(y);
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == C::E + C::P) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TCOLS));
    }
}

// ---- Q4_K ---------------------------------------------------------------------------------------
// The reference's superblock term (tsr_ref.c:540-567): isum = sum_j sc_j S_j over the eight 32-value
// sub-blocks j (S_j = the int dot product of the nibbles and the activation), msum = sum_j m_j
// (BS_2j + BS_2j+1), both int32, then d Dx isum - dmin Dx msum with the f32 rules. All three integer
// sums come from the tensor cores, over the whole superblock (K = 256, eight K = 32 steps):
//  - with sc_j = 8 sh_j + sl_j (sh_j, sl_j in 0..7) the expanders write two int8 A images, sh_j q and
//    sl_j q (each at most 7 x 15 = 105, so one 32-bit multiply scales four packed nibbles without
//    carries between them); their chains give H = sum_j sh_j S_j and L = sum_j sl_j S_j, and
//    isum = 8 H + L is the same integer (|isum| < 2^31);
//  - msum = sum_j m_j p_j with the sub-block sums p_j = BS_2j + BS_2j+1 of the activation: QACT writes
//    p_j as two int8 digits, p_j = 64 hi_j + lo_j, 16 bytes per token and superblock; two K = 32 MMAs
//    with A rows {m_0 .. m_7, 0 ...} and {0 x 8, m_0 .. m_7, 0 ...} against the digit rows give
//    Dlo = sum_j m_j lo_j and Dhi = sum_j m_j hi_j, and msum = Dlo + 64 Dhi.
// So an output costs four TMEM values per superblock and a few f32 operations. The A256 scale Dx is
// an arbitrary f32: when every Dx of the CTA's tokens is 0 or at least 2^-79 in magnitude, every
// product and sum is a multiple of 2^-126 and the flush tests are skipped (SAFE); otherwise they run.
//
// Warp roles: E epilogue warps (32 rows x 16 tokens each), one producer warp (lane 0 loads the raw
// quants, the B tiles with the digit rows, and the 16-byte row metadata by TMA through the tensor maps
// below, whose box order lets the expanders read without bank conflicts; the lanes copy Dx with
// cp.async) into three rings: the raw quants (S entries, free once expanded), the B tiles (SB entries,
// free once the MMA has read them) and Dx and the metadata (SE entries, free once the expanders and the
// epilogue have used them), so that no copy waits for a later role than the one that reads it), X
// expander warps (one row per thread; a
// superblock in two halves of 128 values, each into one of NA slots holding the H and L images of
// four K steps; slot 0 also holds the two mins rows), one MMA warp. TMEM: one accumulator set (H, L,
// Dlo, Dhi: NT columns each; the epilogue frees it as soon as it has read it, so the next
// superblock's MMAs overlap the f32 work) and the four levels of the partial trees' stacks (NT
// columns each). The second K halves of the mins rows and of the digit rows are zero, written once.
// mbarriers: full/empty[S], bfull/bempty[SB], efull/eempty[SE], afull/aempty[NA], tfull/tempty[NB].
constexpr uint32_t kSafeDxQ4 = 0x18000000u;            // 2^-79

template <uint32_t NT>
struct Q4Cfg {
    static constexpr uint32_t E = 4u * (NT / 16u), P = 1u, X = 4u;
    static constexpr uint32_t WARPS = E + P + X + 1u, MMA_WARP = E + P + X;
    static constexpr uint32_t S = 3u, SB = 4u, SE = 6u, NB = 1u, NA = 2u;
    static constexpr uint32_t RAW = kTileM * 128u, BT = NT * 32u, ATILE = kTileM * 32u;
    // ring entries start on 128-byte boundaries (TMA destinations); META first, then Dx
    static constexpr uint32_t META_OFF = 0u, DX_OFF = kTileM * 16u, EPI = DX_OFF + ((NT * 4u + 127u) & ~127u);
    static constexpr uint32_t BENT = 9u * BT;            // B ring entry: eight sub-block tiles, the digit rows
    static constexpr size_t B_OFF = (size_t)S * RAW, E_OFF = B_OFF + (size_t)SB * BENT;
    static constexpr size_t AX_OFF = E_OFF + (size_t)SE * EPI, ASLOT = 10u * ATILE;   // H 0..3, L 0..3, mins lo, hi
    static constexpr size_t BAR_OFF = AX_OFF + NA * ASLOT;
    static constexpr size_t SMEM = BAR_OFF + (2u * S + 2u * SB + 2u * SE + 2u * NA + 2u * NB) * 8u + 16u;
    static constexpr uint32_t ACC_COLS = 4u * NT, STK_COL = NB * ACC_COLS, USED = STK_COL + 4u * NT;
    static constexpr uint32_t TCOLS = USED <= 128u ? 128u : USED <= 256u ? 256u : 512u;
    static_assert(USED <= 512u, "TMEM columns");
    static_assert(SMEM <= 227u * 1024u, "shared memory");
    static_assert(NT % 32u == 0u || NT < 32u, "Dx copies by the producer warp's lanes");
    static_assert(NA == 2u, "half 0 of every superblock (and the mins rows) in slot 0");
};

// Tensor maps of one launch (TMA, no swizzle, no multicast):
//  raw:  the Q4_K quants of the full 16-superblock tiles, dims {256 B of a chunk line, row, chunk, tile}
//        (strides {qrow, 256, 2048}), box {16, 128, 8, 1}: superblock b of 128 rows lands as
//        smem[2048 chunk + 16 row + byte], so the expanders' reads of one chunk of consecutive rows are
//        consecutive 16-byte words;
//  tail: the same for the last tile when it holds nv < 16 superblocks (chunk stride 16 nv);
//  b:    the QA image, dims {16 B, token, half, 32-value group} (strides {K, 16, 32}), box {16, NT, 2, 8}:
//        a superblock's B tiles land as smem[32 NT group + 16 NT half + 16 token + byte], the K-major
//        no-swizzle UMMA layout with LBO = 16 NT (K halves) and SBO = 128 (8-token groups);
//  meta: the 16-byte metadata, dims {16 nsb, row}, box {16, 128};
//  dig:  QACT's pair-sum digits, dims {16 nsb, token}, box {16, NT}: the first K half of the digit rows.
struct alignas(64) Q4Maps {
    CUtensorMap raw, tail, b, meta, dig;
    uint32_t nfull;        // tiles of 16 superblocks in a row; superblocks from 16 nfull on are in the tail
};

template <uint32_t NT, bool SAFE>
__device__ __forceinline__ void q4k_epilogue(const MvArgs& a, uint8_t* smem, uint64_t* efull, uint64_t* eempty,
                                             uint64_t* tfull, uint64_t* tempty, volatile uint32_t* abort_flag, uint32_t tmem,
                                             uint32_t warp, uint32_t lane) {
    using C = Q4Cfg<NT>;
    const uint32_t nsb = a.K / 256u, q = nsb >> 4, rem = nsb & 15u;
    const uint32_t rq = warp & 3u, cq = warp >> 2;
    const uint32_t row = blockIdx.x * kTileM + 32u * rq + lane, tok0 = blockIdx.y * NT;
    const uint32_t tl = tmem + ((32u * rq) << 16) + 16u * cq, ts = tl + C::STK_COL;
    float acc[16];
#pragma unroll
    for (uint32_t i = 0; i < 16; ++i) acc[i] = 0.0f;
    uint32_t j = 0, ii = 0, cnt = q + (rem > 0u ? 1u : 0u);
    bool aborted = false;
    for (uint32_t u = 0; u < nsb; ++u) {
        const uint32_t se = u % C::SE, buf = u % C::NB;
        if (!mbar_wait_ab(&tfull[buf], (u / C::NB) & 1u, abort_flag)) { aborted = true; break; }
        if (!mbar_wait_ab(&efull[se], (u / C::SE) & 1u, abort_flag)) { aborted = true; break; }
        asm volatile("tcgen05.fence::after_thread_sync;");
        uint32_t h[16], l[16];
        tmem_ld16(tl + buf * C::ACC_COLS, h);
        tmem_ld16(tl + buf * C::ACC_COLS + NT, l);
        const uint8_t* sb = smem + C::E_OFF + (size_t)se * C::EPI;
        const uint32_t mx = reinterpret_cast<const uint4*>(sb + C::META_OFF)[32u * rq + lane].x;
        const float dw = h2f((uint16_t)(mx & 0xFFFFu)), dmw = h2f((uint16_t)(mx >> 16));
        tmem_wait_ld();
#pragma unroll
        for (uint32_t i = 0; i < 16; ++i) h[i] = 8u * h[i] + l[i];            // isum = 8 H + L
        uint32_t g[16];
        tmem_ld16(tl + buf * C::ACC_COLS + 2u * NT, l);                     // Dlo
        tmem_ld16(tl + buf * C::ACC_COLS + 3u * NT, g);                     // Dhi
        tmem_wait_ld();
#pragma unroll
        for (uint32_t i = 0; i < 16; ++i) l[i] += 64u * g[i];              // msum = Dlo + 64 Dhi
        asm volatile("tcgen05.fence::before_thread_sync;");
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[buf]);
        const float4* dx4 = reinterpret_cast<const float4*>(sb + C::DX_OFF + 64u * cq);
#pragma unroll
        for (uint32_t k = 0; k < 4; ++k) {
            const float4 f = dx4[k];
            const float d4[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
            for (uint32_t e = 0; e < 4; ++e) {
                const uint32_t i = 4u * k + e;
                const int32_t isum = (int32_t)h[i], msum = (int32_t)l[i];
                const float Dx = d4[e];
                if (SAFE) {
                    const float t1 = __fmul_rn(__fmul_rn(dw, Dx), __int2float_rn(isum));
                    const float t2 = __fmul_rn(__fmul_rn(dmw, Dx), __int2float_rn(msum));
                    acc[i] = __fadd_rn(acc[i], __fsub_rn(t1, t2));
                } else {
                    const float t1 = fmul(fmul(dw, Dx), i2f(isum));
                    const float t2 = fmul(fmul(dmw, Dx), i2f(msum));
                    acc[i] = fadd(acc[i], fsub(t1, t2));
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&eempty[se]);
        if (++ii == cnt) {                                       // partial j is complete
            tree_push_tmem<NT, !SAFE>(ts, j, acc);
#pragma unroll
            for (uint32_t i = 0; i < 16; ++i) acc[i] = 0.0f;
            ++j;
            ii = 0;
            cnt = q + (j < rem ? 1u : 0u);
        }
    }
    if (aborted) return;
    for (; j < 16u; ++j) {                                       // partials nsb .. 15 are +0
        float z[16];
#pragma unroll
        for (uint32_t i = 0; i < 16; ++i) z[i] = 0.0f;
        tree_push_tmem<NT, !SAFE>(ts, j, z);
    }
    uint32_t out[16];
    tmem_ld16(ts, out);                                          // the tree's value: level 0
    tmem_wait_ld();
    if (row < a.n_rows) {
#pragma unroll
        for (uint32_t i = 0; i < 16; ++i) {
            const uint32_t tok = tok0 + 16u * cq + i;
            if (tok < a.T) {
                float y = __uint_as_float(out[i]);
                if (a.flags & kMmAdd) y = fadd(daz(a.add[(size_t)tok * a.add_stride + row]), y);
                if (a.flags & kMmSoftcap) y = fmul(tanh_vu(fmul(y, a.s0), g_expk_t64, g_expk_lk), a.s1);
                else if (a.flags & kMmScale) y = fmul(y, a.s1);
                a.y[(size_t)tok * a.y_stride + row] = canon(y);
            }
        }
    }
}

template <uint32_t NT>
__global__ void __launch_bounds__(32 * Q4Cfg<NT>::WARPS, 1) mm_q4k_tc_kernel(MvArgs a, const __grid_constant__ Q4Maps tm) {
    using C = Q4Cfg<NT>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
    uint64_t* empty = full + C::S;
    uint64_t* bfull = empty + C::S;
    uint64_t* bempty = bfull + C::SB;
    uint64_t* efull = bempty + C::SB;
    uint64_t* eempty = efull + C::SE;
    uint64_t* afull = eempty + C::SE;
    uint64_t* aempty = afull + C::NA;
    uint64_t* tfull = aempty + C::NA;
    uint64_t* tempty = tfull + C::NB;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(tempty + C::NB);
    volatile uint32_t* abort_flag = tslot + 1;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t row0 = blockIdx.x * kTileM, tok0 = blockIdx.y * NT;
    const uint32_t K = a.K, nsb = K / 256u, q = nsb >> 4, rem = nsb & 15u;
    const Layout L{1u, K};

    if (warp == C::MMA_WARP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)), "r"(C::TCOLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < C::S; ++i) {
            mbar_init(&full[i], 1u);                             // the TMA issuer's arrive.expect_tx
            mbar_init(&empty[i], C::X);
        }
        for (uint32_t i = 0; i < C::SB; ++i) {
            mbar_init(&bfull[i], 1u);
            mbar_init(&bempty[i], 1u);
        }
        for (uint32_t i = 0; i < C::SE; ++i) {
            mbar_init(&efull[i], 1u + 32u);                      // expect_tx (META) + every lane's Dx cp.async
            mbar_init(&eempty[i], C::E + C::X);
        }
        for (uint32_t i = 0; i < C::NA; ++i) {
            mbar_init(&afull[i], C::X);
            mbar_init(&aempty[i], 1u);
        }
        for (uint32_t i = 0; i < C::NB; ++i) {
            mbar_init(&tfull[i], 1u);
            mbar_init(&tempty[i], C::E);
        }
        *abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;");
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");     // the QA image comes from the previous kernels
    // SAFE: every activation scale of this CTA's tokens is 0 or at least 2^-79 in magnitude
    bool ok = true;
    for (uint32_t i = threadIdx.x; i < NT * nsb; i += 32u * C::WARPS) {
        const uint32_t t = i / nsb, tok = tok0 + t;
        if (tok < a.T) {
            const uint32_t u = __float_as_uint(a.dx[(size_t)tok * nsb + (i - t * nsb)]) & 0x7FFFFFFFu;
            ok = ok && (u == 0u || u >= kSafeDxQ4);
        }
    }
    // the zero second K halves of the digit rows (one per B ring entry) and of the mins rows (slot 0)
    for (uint32_t i = threadIdx.x; i < C::SB * NT + 2u * kTileM; i += 32u * C::WARPS) {
        uint8_t* z = i < C::SB * NT ? smem + C::B_OFF + (size_t)(i / NT) * C::BENT + 8u * C::BT + 16u * NT + 16u * (i % NT)
                                    : smem + C::AX_OFF + (8u + (i - C::SB * NT) / kTileM) * C::ATILE + 128u +
                                          ((i - C::SB * NT) % kTileM >> 3) * 256u + ((i - C::SB * NT) % 8u) * 16u;
        *reinterpret_cast<uint4*>(z) = make_uint4(0u, 0u, 0u, 0u);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;");
    const bool safe = __syncthreads_and(ok) != 0;
    asm volatile("tcgen05.fence::after_thread_sync;");
    const uint32_t tmem = *tslot;

    if (warp >= C::E && warp < C::E + C::P) {
        // ---- producer warp: lane 0 issues the TMA loads (META, raw quants, B tiles); the lanes copy Dx
        const uint32_t nfull = tm.nfull;
        uint32_t ne = 0, nr = 0, nb = 0;                         // loads issued into each ring
        for (uint32_t u = 0; u < nsb; ++u) {
            const uint32_t st = u % C::S, sbi = u % C::SB, se = u % C::SE;
            uint32_t jb;
            bool lb;
            const uint32_t sbk = Seq{nsb, q, rem}.block(u, &jb, &lb);
            if (u >= C::SE && !mbar_wait_ab(&eempty[se], ((u / C::SE) - 1u) & 1u, abort_flag)) break;
            uint8_t* eb = smem + C::E_OFF + (size_t)se * C::EPI;
            if (lane == 0) {
                mbar_expect_tx(&efull[se], kTileM * 16u);
                tma_load_2d(eb + C::META_OFF, &tm.meta, (int32_t)(16u * sbk), (int32_t)row0, &efull[se]);
            }
            ++ne;
#pragma unroll
            for (uint32_t t = lane; t < NT; t += 32u)
                cp_async4(eb + C::DX_OFF + 4u * t, a.dx + (size_t)min(tok0 + t, a.T - 1u) * nsb + sbk);
            cp_async_arrive(&efull[se]);                         // each entry is published when its copies land
            if (u >= C::S && !mbar_wait_ab(&empty[st], ((u / C::S) - 1u) & 1u, abort_flag)) break;
            if (lane == 0) {
                mbar_expect_tx(&full[st], C::RAW);
                const bool in_full = (sbk >> 4) < nfull;
                tma_load_4d(smem + (size_t)st * C::RAW, in_full ? &tm.raw : &tm.tail, (int32_t)(16u * (sbk & 15u)),
                            (int32_t)row0, 0, in_full ? (int32_t)(sbk >> 4) : 0, &full[st]);
            }
            ++nr;
            if (u >= C::SB && !mbar_wait_ab(&bempty[sbi], ((u / C::SB) - 1u) & 1u, abort_flag)) break;
            if (lane == 0) {
                uint8_t* bb = smem + C::B_OFF + (size_t)sbi * C::BENT;
                mbar_expect_tx(&bfull[sbi], 8u * C::BT + 16u * NT);
                tma_load_4d(bb, &tm.b, 0, (int32_t)tok0, 0, (int32_t)(8u * sbk), &bfull[sbi]);
                tma_load_2d(bb + 8u * C::BT, &tm.dig, (int32_t)(16u * sbk), (int32_t)tok0, &bfull[sbi]);
            }
            ++nb;
        }
        cp_async_wait<0>();
        if (lane == 0) {
            // the last load into each ring entry has landed before the CTA may exit (on every path: a
            // consumer has waited for it already unless a wait gave up)
            for (uint32_t v = ne > C::SE ? ne - C::SE : 0u; v < ne; ++v) mbar_wait_drain(&efull[v % C::SE], (v / C::SE) & 1u);
            for (uint32_t v = nr > C::S ? nr - C::S : 0u; v < nr; ++v) mbar_wait_drain(&full[v % C::S], (v / C::S) & 1u);
            for (uint32_t v = nb > C::SB ? nb - C::SB : 0u; v < nb; ++v) mbar_wait_drain(&bfull[v % C::SB], (v / C::SB) & 1u);
        }
        __syncwarp();
    } else if (warp >= C::E + C::P && warp < C::MMA_WARP) {
        // ---- expanders: thread r owns row r of the tile
        const uint32_t r = (warp - C::E - C::P) * 32u + lane;
        const uint32_t off = (r >> 3) * 256u + (r & 7u) * 16u;
        for (uint32_t u = 0; u < nsb; ++u) {
            const uint32_t st = u % C::S, se = u % C::SE;
            if (!mbar_wait_ab(&efull[se], (u / C::SE) & 1u, abort_flag)) break;
            const uint4 m = reinterpret_cast<const uint4*>(smem + C::E_OFF + (size_t)se * C::EPI + C::META_OFF)[r];
            __syncwarp();
            if (lane == 0) mbar_arrive(&eempty[se]);
            // the eight 6-bit scales (sub-blocks 0..3 in sc_lo, 4..7 in sc_hi, a byte each), split 8 sh + sl
            const uint32_t sc_lo = m.y & 0x3F3F3F3Fu, sc_hi = (m.w & 0x0F0F0F0Fu) | ((m.y >> 2) & 0x30303030u);
            const uint32_t shw[2] = {(sc_lo >> 3) & 0x07070707u, (sc_hi >> 3) & 0x07070707u};
            const uint32_t slw[2] = {sc_lo & 0x07070707u, sc_hi & 0x07070707u};
            const uint32_t mn_lo = m.z & 0x3F3F3F3Fu, mn_hi = ((m.w >> 4) & 0x0F0F0F0Fu) | ((m.z >> 2) & 0x30303030u);
            if (!mbar_wait_ab(&full[st], (u / C::S) & 1u, abort_flag)) break;
            const uint8_t* raw = smem + (size_t)st * C::RAW + r * 16u;         // chunk k at + 2048 k
            bool quit = false;
#pragma unroll
            for (uint32_t hf = 0; hf < 2u; ++hf) {               // values 128 hf .. 128 hf + 127: sub-blocks 4 hf .. 4 hf + 3
                const uint32_t hc = 2u * u + hf, slot = hc % C::NA;
                if (hc >= C::NA && !mbar_wait_ab(&aempty[slot], ((hc / C::NA) - 1u) & 1u, abort_flag)) { quit = true; break; }
                uint8_t* ax = smem + C::AX_OFF + slot * C::ASLOT + off;
#pragma unroll
                for (uint32_t kq = 0; kq < 4u; ++kq) {           // chunk k: low nibbles -> sub-block 2 (k / 2), high -> +1
                    const uint32_t k = 4u * hf + kq, c = k >> 1, h = k & 1u;
                    const uint4 w = *reinterpret_cast<const uint4*>(raw + k * 2048u);
                    const uint4 lo = make_uint4(w.x & 0x0F0F0F0Fu, w.y & 0x0F0F0F0Fu, w.z & 0x0F0F0F0Fu, w.w & 0x0F0F0F0Fu);
                    const uint4 hi = make_uint4((w.x >> 4) & 0x0F0F0F0Fu, (w.y >> 4) & 0x0F0F0F0Fu, (w.z >> 4) & 0x0F0F0F0Fu,
                                                (w.w >> 4) & 0x0F0F0F0Fu);
                    const uint32_t sa = 2u * c, sbb = 2u * c + 1u;   // sub-blocks of the low and high nibbles
                    const uint32_t ha = (shw[sa >> 2] >> (8u * (sa & 3u))) & 0xFFu, la = (slw[sa >> 2] >> (8u * (sa & 3u))) & 0xFFu;
                    const uint32_t hb = (shw[sbb >> 2] >> (8u * (sbb & 3u))) & 0xFFu, lb = (slw[sbb >> 2] >> (8u * (sbb & 3u))) & 0xFFu;
                    const uint32_t ka = sa - 4u * hf, kb = sbb - 4u * hf;   // K steps within the half
                    *reinterpret_cast<uint4*>(ax + ka * C::ATILE + h * 128u) = make_uint4(lo.x * ha, lo.y * ha, lo.z * ha, lo.w * ha);
                    *reinterpret_cast<uint4*>(ax + (4u + ka) * C::ATILE + h * 128u) = make_uint4(lo.x * la, lo.y * la, lo.z * la, lo.w * la);
                    *reinterpret_cast<uint4*>(ax + kb * C::ATILE + h * 128u) = make_uint4(hi.x * hb, hi.y * hb, hi.z * hb, hi.w * hb);
                    *reinterpret_cast<uint4*>(ax + (4u + kb) * C::ATILE + h * 128u) = make_uint4(hi.x * lb, hi.y * lb, hi.z * lb, hi.w * lb);
                }
                if (hf == 0u) {                                  // the mins rows: {m_0 .. m_7, 0 x 8}, {0 x 8, m_0 .. m_7}
                    *reinterpret_cast<uint4*>(ax + 8u * C::ATILE) = make_uint4(mn_lo, mn_hi, 0u, 0u);
                    *reinterpret_cast<uint4*>(ax + 9u * C::ATILE) = make_uint4(0u, 0u, mn_lo, mn_hi);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&afull[slot]);
            }
            if (quit) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }
    } else if (warp == C::MMA_WARP) {
        if (lane == 0) {
            uint32_t issued = 0;
            bool quit = false;
            for (uint32_t u = 0; u < nsb && !quit; ++u) {
                const uint32_t sbi = u % C::SB, buf = u % C::NB;
                if (!mbar_wait_ab(&bfull[sbi], (u / C::SB) & 1u, abort_flag)) break;
                if (u >= C::NB && !mbar_wait_ab(&tempty[buf], ((u / C::NB) - 1u) & 1u, abort_flag)) break;
                uint8_t* bb = smem + C::B_OFF + (size_t)sbi * C::BENT;
                const uint32_t dh = tmem + buf * C::ACC_COLS, dl = dh + NT, dlo = dh + 2u * NT, dhi = dh + 3u * NT;
#pragma unroll
                for (uint32_t hf = 0; hf < 2u; ++hf) {
                    const uint32_t hc = 2u * u + hf, slot = hc % C::NA;
                    if (!mbar_wait_ab(&afull[slot], (hc / C::NA) & 1u, abort_flag)) { quit = true; break; }
                    asm volatile("tcgen05.fence::after_thread_sync;");
                    uint8_t* ax = smem + C::AX_OFF + slot * C::ASLOT;
#pragma unroll
                    for (uint32_t ks = 0; ks < 4u; ++ks) {
                        const uint32_t acc = (hf | ks) != 0u ? 1u : 0u;
                        const uint64_t db = umma_desc_b<NT>(bb + (4u * hf + ks) * C::BT);
                        mma_i8(dh, umma_desc(ax + ks * C::ATILE), db, umma_idesc<NT>(), acc);
                        mma_i8(dl, umma_desc(ax + (4u + ks) * C::ATILE), db, umma_idesc<NT>(), acc);
                    }
                    if (hf == 0u) {                                  // the min sums' digit MMAs
                        const uint64_t dd = umma_desc_b<NT>(bb + 8u * C::BT);
                        mma_i8(dlo, umma_desc(ax + 8u * C::ATILE), dd, umma_idesc<NT>(), 0u);
                        mma_i8(dhi, umma_desc(ax + 9u * C::ATILE), dd, umma_idesc<NT>(), 0u);
                    }
                    mma_commit(&aempty[slot]);
                }
                if (quit) break;
                mma_commit(&tfull[buf]);
                mma_commit(&bempty[sbi]);
                ++issued;
            }
            if (issued) {
                const uint32_t u = issued - 1u;
                mbar_wait_ab(&tfull[u % C::NB], (u / C::NB) & 1u, abort_flag);
            }
        }
        __syncwarp();
    } else if (safe) {
        q4k_epilogue<NT, true>(a, smem, efull, eempty, tfull, tempty, abort_flag, tmem, warp, lane);
    } else {
        q4k_epilogue<NT, false>(a, smem, efull, eempty, tfull, tempty, abort_flag, tmem, warp, lane);
    }
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == C::MMA_WARP) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TCOLS));
    }
}


// cuTensorMapEncodeTiled, from the driver through the runtime (no link against libcuda)
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                   const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// a rank-R uint8 tiled map, no swizzle; dims / strides in bytes (strides of dims 1 .. R-1)
template <int R>
bool encode_u8(CUtensorMap* m, const void* base, const cuuint64_t (&dims)[R], const cuuint64_t (&strides)[R - 1],
               const cuuint32_t (&box)[R]) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return false;
    cuuint32_t es[R];
    for (int i = 0; i < R; ++i) es[i] = 1;
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, (cuuint32_t)R, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <uint32_t NT>
bool make_q4_maps(const MvArgs& a, Q4Maps* tm) {
    const Layout L{1u, a.K};
    const uint32_t nsb = a.K / 256u, nfull = nsb / 16u, nv = nsb % 16u;
    const cuuint64_t qrow = L.qs_row_bytes(), rows = a.n_rows;
    *tm = Q4Maps{};
    tm->nfull = nfull;
    if (nfull && !encode_u8<4>(&tm->raw, a.qs, {256, rows, 8, nfull}, {qrow, 256, 2048}, {16, kTileM, 8, 1})) return false;
    if (nv && !encode_u8<4>(&tm->tail, a.qs + (size_t)nfull * 2048u, {16ull * nv, rows, 8, 1}, {qrow, 16ull * nv, 128ull * nv},
                            {16, kTileM, 8, 1}))
        return false;
    if (!encode_u8<4>(&tm->b, a.qx, {16, a.T, 2, a.K / 32u}, {a.K, 16, 32}, {16, NT, 2, 8})) return false;
    if (!encode_u8<2>(&tm->dig, a.bsd, {16ull * nsb, a.T}, {16ull * nsb}, {16, NT})) return false;
    return encode_u8<2>(&tm->meta, a.meta, {16ull * nsb, rows}, {L.meta_row_bytes()}, {16, kTileM});
}

template <uint32_t NT>
cudaError_t launch_q4k_nt(const MvArgs& a, cudaStream_t st) {
    using C = Q4Cfg<NT>;
    static int done_dev[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && done_dev[dev] != dev + 1) {
        e = cudaFuncSetAttribute(mm_q4k_tc_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
        if (e != cudaSuccess) return e;
        done_dev[dev] = dev + 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.n_rows + kTileM - 1u) / kTileM, (a.T + NT - 1u) / NT);
    cfg.blockDim = dim3(32u * C::WARPS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    Q4Maps tm;
    if (!make_q4_maps<NT>(a, &tm)) return cudaErrorInvalidValue;
    return cudaLaunchKernelEx(&cfg, mm_q4k_tc_kernel<NT>, a, tm);
}

template <uint32_t NT>
bool make_q8_maps(const MvArgs& a, Q8Maps* tm) {
    const Layout L{0u, a.K};
    const uint32_t nb = a.K / 32u, nfull = nb / 16u, nv = nb % 16u;
    const cuuint64_t qrow = L.qs_row_bytes(), rows = a.n_rows;
    *tm = Q8Maps{};
    tm->nfull = nfull;
    if (nfull && !encode_u8<4>(&tm->a, a.qs, {256, rows, 2, nfull}, {qrow, 256, 512}, {16, kTileM, 2, 1})) return false;
    if (nv && !encode_u8<4>(&tm->tail, a.qs + (size_t)nfull * 512u, {16ull * nv, rows, 2, 1}, {qrow, 16ull * nv, 32ull * nv},
                            {16, kTileM, 2, 1}))
        return false;
    return encode_u8<3>(&tm->b, a.qx, {16, a.T, a.K / 16u}, {a.K, 16}, {16, NT, 2});
}

template <uint32_t NT>
cudaError_t launch_nt(const MvArgs& a, cudaStream_t st) {
    using C = Q8Cfg<NT>;
    static int done_dev[64];
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && done_dev[dev] != dev + 1) {
        e = cudaFuncSetAttribute(mm_q8_tc_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
        if (e != cudaSuccess) return e;
        done_dev[dev] = dev + 1;
    }
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    const uint64_t tiles = (uint64_t)((a.n_rows + kTileM - 1u) / kTileM) * ((a.T + NT - 1u) / NT);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((uint32_t)std::min<uint64_t>(tiles, (uint64_t)std::max(sms, 1)), 1);   // persistent CTAs
    cfg.blockDim = dim3(32u * C::WARPS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    Q8Maps tm;
    if (!make_q8_maps<NT>(a, &tm)) return cudaErrorInvalidValue;
    return cudaLaunchKernelEx(&cfg, mm_q8_tc_kernel<NT>, a, tm);
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
    if (fmt == 1u) return a.T <= 16 ? launch_q4k_nt<16>(a, st) : a.T <= 32 ? launch_q4k_nt<32>(a, st) : launch_q4k_nt<64>(a, st);
    if (a.T <= 16) return launch_nt<16>(a, st);
    if (a.T <= 32) return launch_nt<32>(a, st);
    // 64-, 48- or 32-token tiles: the width with the least (tiles per persistent CTA) x (tokens per tile
    // + 16, the per-block work that does not grow with the width: the weight tile, the MMA issue),
    // ties to the wider, so that neither a grid just past a whole number of SMs (config 4 FFN: 304
    // tiles of 64 on 148 SMs) nor a narrow matrix (896 rows: 56 tiles of 64) leaves SMs idle
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint64_t rt = (a.n_rows + kTileM - 1u) / kTileM, sm = sms > 0 ? (uint64_t)sms : 148u;
    auto cost = [&](uint64_t nt) { return (rt * ((a.T + nt - 1u) / nt) + sm - 1u) / sm * (nt + 16u); };
    const uint64_t c64 = cost(64), c48 = cost(48), c32 = cost(32);
    if (c32 < c48 && c32 < c64) return launch_nt<32>(a, st);
    return c48 < c64 ? launch_nt<48>(a, st) : launch_nt<64>(a, st);
}

}  // namespace tsrc
