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

// ---- pipeline primitives (warp-specialised kernels) --------------------------------------------
constexpr long long kWaitCycles = 1ll << 31;       // a wait gives up after ~1 s of SM clock

__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
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
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity), "r"(1000u)
            : "memory");
        if (ok) return true;
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
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]),
          "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Folds partial j (16 values, one per token of the thread) into the 16-partial tree whose four
// stack levels live in TMEM columns lv, lv + NT, lv + 2 NT, lv + 3 NT (the thread's lane); after
// partial 15 the tree's value is level 0. FLUSH: the reference's flush test on every sum.
template <bool FLUSH, uint32_t NT>
__device__ __forceinline__ void tree_push_tmem(uint32_t lv, uint32_t j, float (&v)[16]) {
    uint32_t w[16];
#pragma unroll
    for (uint32_t lvl = 0; lvl < 4; ++lvl) {
        if (((j >> lvl) & 1u) == 0u) {
            tmem_st16(lv + lvl * NT, v);
            return;
        }
        tmem_ld16(lv + lvl * NT, w);
#pragma unroll
        for (uint32_t i = 0; i < 16; ++i) v[i] = FLUSH ? fadd(__uint_as_float(w[i]), v[i]) : __fadd_rn(__uint_as_float(w[i]), v[i]);
    }
    tmem_st16(lv, v);
}

// exact int32 -> f32 for |v| < 2^22 (block sums of Q8_0: |v| <= 32 * 128 * 128 = 2^19)
__device__ __forceinline__ float small_i2f(int32_t v) {
    return __fsub_rn(__int_as_float(v + 0x4B400000), 12582912.0f);
}

// ---- Q8_0 ---------------------------------------------------------------------------------------
// Warp roles: E epilogue warps (warp w: TMEM lanes 32 (w mod 4) .., tokens 16 (w / 4) ..), P producer
// warps (cp.async of the block's A / B operand tiles, activation scales and weight scales into a
// ring of S stages; a stage is published when the producer's copies of it have landed), one MMA
// warp (TMEM allocation; one thread issues each block's MMA into one of NB accumulator tiles).
// mbarriers: full[S] (producers -> MMA, epilogue), empty[S] (MMA commit + epilogue warps ->
// producers), tfull[NB] (MMA commit -> epilogue), tempty[NB] (epilogue warps -> MMA).
template <uint32_t NT>
struct Q8Cfg {
    static constexpr uint32_t E = 4u * (NT / 16u);
    static constexpr uint32_t P = 2u;
    static constexpr uint32_t WARPS = E + P + 1u;
    static constexpr uint32_t S = 16u;
    static constexpr uint32_t LAG = 8u;                // producer: stages in flight before publishing
    static constexpr uint32_t NB = 4u;
    static constexpr uint32_t A_BYTES = kTileM * 32u, B_BYTES = NT * 32u;
    static constexpr uint32_t DX_OFF = A_BYTES + B_BYTES, DW_OFF = DX_OFF + NT * 4u;
    static constexpr uint32_t STAGE = DW_OFF + kTileM * 4u;
    static constexpr uint32_t TCOLS = 8u * NT;         // NB accumulator tiles + 4 tree levels
    static constexpr size_t BAR_OFF = (size_t)S * STAGE;
    static constexpr size_t NEED = BAR_OFF + (2u * S + 2u * NB) * 8u + 16u;
    // 512 TMEM columns: one CTA per SM (more shared memory than half the SM's)
    static constexpr size_t SMEM = (TCOLS == 512u && NEED < 120u * 1024u) ? 120u * 1024u : NEED;
};

template <uint32_t NT>
__global__ void __launch_bounds__(32 * Q8Cfg<NT>::WARPS, 1) mm_q8_tc_kernel(MvArgs a) {
    using C = Q8Cfg<NT>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
    uint64_t* empty = full + C::S;
    uint64_t* tfull = empty + C::S;
    uint64_t* tempty = tfull + C::NB;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(tempty + C::NB);
    volatile uint32_t* abort_flag = tslot + 1;

    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t row0 = blockIdx.x * kTileM, tok0 = blockIdx.y * NT;
    const uint32_t K = a.K, nb = K / 32u, q = nb >> 4, rem = nb & 15u;
    const Layout L{0u, K};

    if (warp == C::E + C::P) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)), "r"(C::TCOLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < C::S; ++i) {
            mbar_init(&full[i], C::P);
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
    bool aborted = false;

    if (warp >= C::E && warp < C::E + C::P) {
        // ---- producers: lane pl copies A chunks of rows (pl / 2) + 32 P k, half pl & 1, ...
        constexpr uint32_t LN = 32u * C::P, AR = 256u / LN, BR = (2u * NT + LN - 1u) / LN, WR = kTileM / LN;
        const uint32_t pl = (warp - C::E) * 32u + lane, h = pl & 1u;
        const uint8_t* arow[AR];
        uint32_t adst[AR];
#pragma unroll
        for (uint32_t k = 0; k < AR; ++k) {
            const uint32_t r = (pl >> 1) + (LN / 2u) * k;
            arow[k] = a.qs + (size_t)min(row0 + r, a.n_rows - 1u) * L.qs_row_bytes();
            adst[k] = (r >> 3) * 256u + h * 128u + (r & 7u) * 16u;
        }
        const int8_t* brow[BR];
        uint32_t bdst[BR];
#pragma unroll
        for (uint32_t k = 0; k < BR; ++k) {
            const uint32_t t = (pl >> 1) + (LN / 2u) * k;
            brow[k] = a.qx + (size_t)min(tok0 + t, a.T - 1u) * K + 16u * h;
            bdst[k] = t < NT ? C::A_BYTES + (t >> 3) * 256u + h * 128u + (t & 7u) * 16u : 0xFFFFFFFFu;
        }
        const float* dxrow = a.dx + (size_t)min(tok0 + (pl < NT ? pl : 0u), a.T - 1u) * nb;
        const uint8_t* wrow[WR];
#pragma unroll
        for (uint32_t k = 0; k < WR; ++k)
            wrow[k] = static_cast<const uint8_t*>(a.meta) + (size_t)min(row0 + pl + LN * k, a.n_rows - 1u) * L.meta_row_bytes();
        uint32_t j = 0, ii = 0, cnt = q + (rem > 0u ? 1u : 0u), issued = 0;
        for (uint32_t s = 0; s < nb; ++s) {
            const uint32_t st = s % C::S;
            if (s >= C::S && !mbar_wait_ab(&empty[st], ((s / C::S) - 1u) & 1u, abort_flag)) { aborted = true; break; }
            const uint32_t b = j + 16u * ii;
            uint8_t* sb = smem + (size_t)st * C::STAGE;
            const size_t aoff = L.qs_off(0u, b, h);
#pragma unroll
            for (uint32_t k = 0; k < AR; ++k) cp_async16(sb + adst[k], arow[k] + aoff);
#pragma unroll
            for (uint32_t k = 0; k < BR; ++k)
                if (bdst[k] != 0xFFFFFFFFu) cp_async16(sb + bdst[k], brow[k] + 32u * b);
            if (pl < NT) cp_async4(sb + C::DX_OFF + 4u * pl, dxrow + b);
#pragma unroll
            for (uint32_t k = 0; k < WR; ++k) cp_async4(sb + C::DW_OFF + 4u * (pl + LN * k), wrow[k] + 2u * (b & ~1u));
            cp_async_commit();
            ++issued;
            if (s >= C::LAG) {
                cp_async_wait<C::LAG>();
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[(s - C::LAG) % C::S]);
            }
            if (++ii == cnt) {
                ++j;
                ii = 0;
                cnt = q + (j < rem ? 1u : 0u);
            }
        }
        cp_async_wait<0>();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0)
            for (uint32_t s = issued > C::LAG ? issued - C::LAG : 0u; s < issued; ++s) mbar_arrive(&full[s % C::S]);
    } else if (warp == C::E + C::P) {
        // ---- MMA issuer
        if (lane == 0) {
            uint32_t issued = 0;
            for (uint32_t s = 0; s < nb; ++s) {
                const uint32_t st = s % C::S, buf = s % C::NB;
                if (!mbar_wait_ab(&full[st], (s / C::S) & 1u, abort_flag)) break;
                if (s >= C::NB && !mbar_wait_ab(&tempty[buf], ((s / C::NB) - 1u) & 1u, abort_flag)) break;
                asm volatile("tcgen05.fence::after_thread_sync;");
                uint8_t* sb = smem + (size_t)st * C::STAGE;
                mma_i8(tmem + buf * NT, umma_desc(sb), umma_desc(sb + C::A_BYTES), umma_idesc<NT>(), 0u);
                mma_commit(&tfull[buf]);
                mma_commit(&empty[st]);
                ++issued;
            }
            if (issued) {     // the last MMA (and with it every earlier one) has completed
                const uint32_t s = issued - 1u;
                mbar_wait_ab(&tfull[s % C::NB], (s / C::NB) & 1u, abort_flag);
            }
        }
        __syncwarp();
    } else {
        // ---- epilogue: row = row0 + 32 rq + lane, tokens tok0 + 16 cq + i
        const uint32_t rq = warp & 3u, cq = warp >> 2;
        const uint32_t row = row0 + 32u * rq + lane;
        const uint32_t tl = tmem + ((32u * rq) << 16);
        const uint32_t lv = tl + C::NB * NT + 16u * cq;
        float acc[16];
#pragma unroll
        for (uint32_t i = 0; i < 16; ++i) acc[i] = 0.0f;
        uint32_t j = 0, ii = 0, cnt = q + (rem > 0u ? 1u : 0u);
        for (uint32_t s = 0; s < nb; ++s) {
            const uint32_t st = s % C::S, buf = s % C::NB;
            if (!mbar_wait_ab(&tfull[buf], (s / C::NB) & 1u, abort_flag)) { aborted = true; break; }
            asm volatile("tcgen05.fence::after_thread_sync;");
            uint32_t v[16];
            tmem_ld16(tl + buf * NT + 16u * cq, v);
            asm volatile("tcgen05.fence::before_thread_sync;");
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[buf]);
            if (!mbar_wait_ab(&full[st], (s / C::S) & 1u, abort_flag)) { aborted = true; break; }
            const uint8_t* sb = smem + (size_t)st * C::STAGE;
            const float4* dx4 = reinterpret_cast<const float4*>(sb + C::DX_OFF + 64u * cq);
            const float4 x0 = dx4[0], x1 = dx4[1], x2 = dx4[2], x3 = dx4[3];
            const uint32_t dwp = reinterpret_cast<const uint32_t*>(sb + C::DW_OFF)[32u * rq + lane];
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
            const uint32_t b = j + 16u * ii;
            const float dw = h2f((uint16_t)((b & 1u) ? (dwp >> 16) : (dwp & 0xFFFFu)));
            const float dx[16] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w, x2.x, x2.y, x2.z, x2.w, x3.x, x3.y, x3.z, x3.w};
#pragma unroll
            for (uint32_t i = 0; i < 16; ++i)
                acc[i] = __fadd_rn(acc[i], __fmul_rn(__fmul_rn(dw, dx[i]), small_i2f((int32_t)v[i])));
            if (++ii == cnt) {                                   // partial j is complete
                tree_push_tmem<false, NT>(lv, j, acc);
#pragma unroll
                for (uint32_t i = 0; i < 16; ++i) acc[i] = 0.0f;
                ++j;
                ii = 0;
                cnt = q + (j < rem ? 1u : 0u);
            }
        }
        if (!aborted) {
            for (; j < 16u; ++j) {                               // partials nb .. 15 (fewer than 16 blocks) are +0
                float z[16];
#pragma unroll
                for (uint32_t i = 0; i < 16; ++i) z[i] = 0.0f;
                tree_push_tmem<false, NT>(lv, j, z);
            }
            uint32_t r[16];
            tmem_ld16(lv, r);
            if (row < a.n_rows) {
#pragma unroll
                for (uint32_t i = 0; i < 16; ++i) {
                    const uint32_t tok = tok0 + 16u * cq + i;
                    if (tok < a.T) {
                        float y = __uint_as_float(r[i]);
                        if (a.flags & kMmAdd) y = fadd(daz(a.add[(size_t)tok * a.add_stride + row]), y);
                        if (a.flags & kMmSoftcap) y = fmul(tanh_vu(fmul(y, a.s0), g_expk_t64, g_expk_lk), a.s1);
                        else if (a.flags & kMmScale) y = fmul(y, a.s1);
                        a.y[(size_t)tok * a.y_stride + row] = canon(y);
                    }
                }
            }
        }
    }
    (void)aborted;
    asm volatile("tcgen05.fence::before_thread_sync;");
    __syncthreads();
    if (warp == C::E + C::P) {
        asm volatile("tcgen05.fence::after_thread_sync;");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TCOLS));
    }
}

template <uint32_t NT>
cudaError_t launch_nt(const MvArgs& a, cudaStream_t st) {
    using C = Q8Cfg<NT>;
    static int done_dev[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && done_dev[dev] != dev + 1) {
        e = cudaFuncSetAttribute(mm_q8_tc_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
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
    return launch_nt<64>(a, st);
}

}  // namespace tsrc
