// tsrc_fa.cu -- flash attention over a q8_0 KV cache on sm_100a, bit-exact with the reference's
// composite FA (jwkim04/tesseract-npu sw/sim/tsr_ref_at.c:774-860, design doc AT §6.6).
//
// The reference runs, per query tile and per chunk of cell groups (the chunk planner, rules 1-8 of
// sw/sim/include/tsr_fa_plan.h; host side in tsrc_fa_plan.cu): ATTQK (scores, row max MAXOUT
// floored at -2^100), ASMAX (EXP of the scaled difference), ATTPV + LSUM per channel (the groups
// u = c mod C of the chunk) as block-floating-point sums per 64-cell segment, then AMERGE (channel
// tree CTREE, online merge with the running max) and finally ANORM. Every f32 operation follows
// the reference's rules (tsrc_numerics.cuh); every sum that the reference makes exact is an
// integer sum here too, so the result does not depend on how the work is spread over threads.
//
// Work split (one launch of fa_chunk_kernel, then one of fa_merge_kernel; both are programmatic
// dependent launches: each starts its prologue while the kernel before it finishes):
//   - a thread-block cluster per (work item = query tile x chunk, KV head g), one CTA per channel
//     (cluster rank = channel); the CTA prefetches its groups' K and V bytes into L2 on entry,
//     before it waits for the kernel it depends on;
//   - a CTA computes the scores of its channel's cells for RB rows (query heads of g x tokens of
//     the tile) at a time, the cluster exchanges the per-channel row maxima through distributed
//     shared memory (the chunk max is a max over all channels), then the CTA applies EXP and runs
//     the channel's segments, one warp per (segment, 64-value slice), folding the segment
//     results in order, and writes its channel result and row sums to global scratch;
//   - fa_merge_kernel<C> reduces the C channel results of every chunk (CTREE), merges the
//     chunks of a tile in execution order (AMERGE) and normalises (ANORM), one thread per output
//     value, over the whole GPU.
#include <cooperative_groups.h>

#include "tsrc_internal.h"
#include "tsrc_numerics.cuh"

namespace cg = cooperative_groups;

namespace tsrc {

namespace {

// Warps of a chunk CTA: 16 for few large items (decode: the latency of one item matters), 4 or 2
// for many small ones (a prompt's query tiles: four or eight CTAs per SM hide each other's latency).
constexpr uint32_t kFaWarpsLarge = 16, kFaWarpsSmall = 4, kFaWarpsTiny = 2;
constexpr uint32_t kNegInf = 0xFF800000u;
constexpr uint32_t kMFloor = 0xF1800000u;      // -2^100: MAXOUT's floor (sw/sim/include/tsr_tables.h:89)
constexpr uint32_t kLFloor = 0x00800000u;      // 2^-126: ANORM's floor of the row sum (tsr_tables.h:90)
constexpr uint32_t kFlCausal = 1u, kFlSlide = 2u;
constexpr uint32_t kWdStride = 80u;             // bytes per row of a W-digit table (64 cells + pad: no bank conflicts)

// MAXT (VU §6.8; tsr_ref_at.c:318-325): NaN -> canonical NaN, else the larger value, -0 < +0.
__device__ __forceinline__ float maxt(float a, float b) {
    const uint32_t ua = fbits(daz(a)), ub = fbits(daz(b));
    if ((ua & ~kSign) > kExp || (ub & ~kSign) > kExp) return ffrom(kCanonNaN);
    const uint32_t ka = (ua & kSign) ? ~ua : (ua | kSign);
    const uint32_t kb = (ub & kSign) ? ~ub : (ub | kSign);
    return ffrom(ka >= kb ? ua : ub);
}

// Block floating point (tsr_ref_at.c:380-430): RNE_int(w * 2^(23 - es)) of a finite w whose
// exponent is <= es (zero for a zero w), and RNE to 24 bits of A * 2^k with underflow to a signed
// zero below 2^-126 and overflow to infinity.
//
// bf_int: w is zero or normal (flushed), so w * 2^(23 - es) is w with 23 - es added to its exponent
// field; when the new field is <= 125 the value is below 1/2 and rounds to 0, otherwise it is a
// normal float below 2^24 and the hardware conversion rounds it to the nearest integer, ties to even.
__device__ __forceinline__ int32_t bf_int(float w, int32_t es) {
    const uint32_t u = fbits(w);
    const int32_t ew = (int32_t)((u >> 23) & 0xFFu);
    if (ew == 0 || ew + 23 - es <= 125) return 0;
    return __float2int_rn(ffrom(u + ((uint32_t)(23 - es) << 23)));
}

// bf_f: A * 2^k is exact in double (|A| < 2^53 here), and one conversion rounds it to 24 bits. When
// k < -60 the value is first scaled by 2^64 so that the rounded value stays a normal float and the
// comparison with 2^-126 (2^-62 scaled) sees it; A = 0 gives +0.
__device__ __forceinline__ double pow2d(int32_t j) { return __longlong_as_double((long long)(j + 1023) << 52); }
__device__ __forceinline__ float bf_f(int64_t A, int32_t k) {
    const bool small = k < -60;
    float f = __double2float_rn(__dmul_rn(__ll2double_rn(A), pow2d(small ? k + 64 : k)));
    if (small) f = fabsf(f) < 0x1p-62f ? ffrom(fbits(f) & kSign) : __fmul_rn(f, 0x1p-64f);
    return f;
}

// The four balanced base-256 digits of |W| <= 2^24 (W = d0 + 2^8 d1 + 2^16 d2 + 2^24 d3, d0..d2 in
// [-128, 127]) as the bytes of one word: adding 128 to digits 0-2 makes them the unsigned bytes of
// W + 0x808080, and flipping their top bits gives the signed digits back.
__device__ __forceinline__ uint32_t digits4(int32_t W) { return ((uint32_t)W + 0x00808080u) ^ 0x00808080u; }

__device__ __forceinline__ bool nonfinite(uint32_t u) { return (u & kExp) == kExp; }

// maxt over a warp (every lane gets the result)
// MAXT as an unsigned key: the largest key is the MAXT of the values (NaN above every number,
// -0 below +0), so a maximum over many values is one integer max (a warp reduction, an atomic).
__device__ __forceinline__ uint32_t maxt_key(float x) {
    const uint32_t u = fbits(daz(x));
    if ((u & ~kSign) > kExp) return 0xFFFFFFFFu;
    return (u & kSign) ? ~u : (u | kSign);
}
__device__ __forceinline__ float maxt_val(uint32_t k) {
    if (k == 0xFFFFFFFFu) return ffrom(kCanonNaN);
    return ffrom((k & kSign) ? (k & ~kSign) : ~k);
}

__device__ __forceinline__ int32_t dot32(const uint4 a0, const uint4 a1, const uint4 b0, const uint4 b1) {
    int32_t s = 0;
    s = __dp4a((int)a0.x, (int)b0.x, s);
    s = __dp4a((int)a0.y, (int)b0.y, s);
    s = __dp4a((int)a0.z, (int)b0.z, s);
    s = __dp4a((int)a0.w, (int)b0.w, s);
    s = __dp4a((int)a1.x, (int)b1.x, s);
    s = __dp4a((int)a1.y, (int)b1.y, s);
    s = __dp4a((int)a1.z, (int)b1.z, s);
    s = __dp4a((int)a1.w, (int)b1.w, s);
    return s;
}

// The fixed 16-partial tree (tsr_ref.c:592-606) of ND terms p[b] = fadd(+0, term_b), zeros after,
// for QK terms t_b = (dK dQ) f32(isum): dK and dQ are fp16 values, so dK dQ is exact and >= 2^-48
// when nonzero, every term and every sum of terms is 0 or a multiple of 2^-71 (never subnormal: no
// flush can trigger) and no partial is -0 after its first addition (+0 + -0 = +0). The tree thus
// reduces to the pairwise sums of the live partials, with the flush tests left out.
template <int ND>
__device__ __forceinline__ float tree16_qk(const float (&t)[ND]) {
    float v[ND];
#pragma unroll
    for (int i = 0; i < ND; ++i) v[i] = __fadd_rn(t[i], 0.0f);
#pragma unroll
    for (int n = ND; n > 1; n /= 2)
#pragma unroll
        for (int k = 0; k < n / 2; ++k) v[k] = __fadd_rn(v[2 * k], v[2 * k + 1]);
    return v[0];
}

__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Shared-memory plan of fa_chunk_kernel (host and device agree).
struct FaSmem {
    uint32_t qx_off, dx_off, s_off, w_off, cv_off, vq_off, vs_off, misc_off, total;
};

__host__ __device__ inline uint32_t fa_a16(uint32_t n) { return (n + 15u) & ~15u; }
// values of a 64-cell segment whose V quants one warp stages: its 64-value slice (4 KB)
__host__ __device__ inline uint32_t fa_vp(uint32_t) { return 64u; }
// segments a round of the P.V phase runs at once: one warp per (segment, 64-value slice)
__host__ __device__ inline uint32_t fa_segs(uint32_t D, uint32_t W) { return W / (D / 64u); }
// rows of a W-digit table: RB rows x 4 digits (an 8-wide tensor-core tile wraps around a 4-row
// table; the extra output columns are not used)
__host__ __device__ inline uint32_t fa_wd_rows(uint32_t D) { return 4u * (512u / D); }

__host__ __device__ inline FaSmem fa_smem(uint32_t D, uint32_t ncell_max, uint32_t W) {
    const uint32_t RB = 512u / D, ND = D / 32u;
    FaSmem s{};
    uint32_t o = fa_a16(64u * 4u + 4u * 8u);                    // EXPK tables
    s.qx_off = o;
    o += fa_a16(RB * D);                                        // qx [RB][D]
    s.dx_off = o;
    o += fa_a16(RB * ND * 4u);                                  // dx [RB][ND]
    s.s_off = o;
    o += fa_a16(RB * ncell_max * 4u);                           // S [RB][ncell_max]
    s.w_off = o;
    o += fa_a16(W * 2u * fa_wd_rows(D) * kWdStride);            // W digits [warp][2][rows][kWdStride] (its slice)
    s.cv_off = o;
    o += fa_a16(fa_segs(D, W) * RB * D * 4u);                   // CV [segment of the round][RB][D]
    s.vq_off = o;
    o += fa_a16(W * 64u * fa_vp(D));                            // V quants of a segment [warp][4 groups][VP][16]
    s.vs_off = o;
    o += fa_a16(W * 64u * ND * 2u);                             // V scales of a segment [warp][64][ND]
    s.misc_off = o;
    // mx [2][RB] (max keys), mk [RB], ls [segments][RB], lacc [RB], es [warps][RB], fl [warps][RB]
    o += 4u * (2u * RB + RB + W * RB + RB + 2u * W * RB);
    s.total = fa_a16(o);
    return s;
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)), "l"(gmem_src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// The cluster barrier in two halves: arrive once this CTA is done reading its peers' shared
// memory, wait before it exits (a peer's shared memory must outlive every remote read of it).
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------------------------------
template <int D, uint32_t W>
__global__ void __launch_bounds__(W * 32u, W <= kFaWarpsTiny ? 8 : (W <= kFaWarpsSmall ? 4 : 1)) fa_chunk_kernel(FaLaunch a) {
    constexpr uint32_t kFaWarps = W, kFaThreads = W * 32u;
    constexpr uint32_t ND = D / 32, NSL = D / 64, RB = 512 / D;
    extern __shared__ __align__(16) uint8_t smem[];
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t C = a.C, cc = cluster.block_rank();
    const uint32_t ig = blockIdx.x / C, item = ig / a.n_head_kv, g = ig - item * a.n_head_kv;
    const FaItem it = a.n_items <= kFaInlineItems ? a.inl_items[item] : a.items[item];
    const uint32_t G = a.G, rows = it.Tq * G, rows_max = a.Tq0 * G;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;

    // the channel's groups: u = ufirst + C k, k < nu
    const uint32_t ufirst = it.u0 + (cc + C - it.u0 % C) % C;
    const uint32_t nu = ufirst < it.u0 + it.n ? (it.u0 + it.n - ufirst + C - 1u) / C : 0u;
    const uint32_t ncell = 16u * nu;
    const uint32_t ncell_max = 16u * ((it.n + C - 1u) / C);
    const FaSmem P = fa_smem(D, ncell_max, W);
    constexpr uint32_t VP = 64u;                               // fa_vp(D): a warp's 64-value slice
    constexpr uint32_t SEGS = kFaWarps / NSL;                  // fa_segs(D, W)
    static_assert(SEGS >= 1, "a round needs at least one segment");
    const uint32_t wseg = warp / NSL, wsl = warp - wseg * NSL; // the warp's segment of a round and slice
    constexpr uint32_t kWdRows = 4u * RB;                      // fa_wd_rows(D)
    constexpr uint32_t kNT = kWdRows < 8u ? 1u : kWdRows / 8u; // 8-wide tensor-core tiles of the W digits
    constexpr uint32_t kWdWarp = 2u * kWdRows * kWdStride;

    const size_t head_cells = (size_t)g * a.n_cells;
    // K and V of the channel's visible groups: HBM -> L2 now
    for (uint32_t i = tid; i < 4u * nu; i += kFaThreads) {
        const uint32_t k = i >> 2, which = i & 3u, u = ufirst + C * k;
        if (16u * u >= a.n_kv) continue;
        const size_t c0 = head_cells + 16u * u;
        if (which == 0) prefetch_l2(a.kq + c0 * D, 16u * D);
        else if (which == 1) prefetch_l2(a.vq + c0 * D, 16u * D);
        else if (which == 2) prefetch_l2(a.kd + c0 * ND, 32u * ND);
        else prefetch_l2(a.vd + c0 * ND, 32u * ND);
    }

    uint32_t* t64s = reinterpret_cast<uint32_t*>(smem);
    uint64_t* lks = reinterpret_cast<uint64_t*>(smem + 256);
    int8_t* qx = reinterpret_cast<int8_t*>(smem + P.qx_off);
    float* dx = reinterpret_cast<float*>(smem + P.dx_off);
    float* S = reinterpret_cast<float*>(smem + P.s_off);
    uint8_t* Wbase = smem + P.w_off;
    float* CV = reinterpret_cast<float*>(smem + P.cv_off);
    int8_t* vqs = reinterpret_cast<int8_t*>(smem + P.vq_off) + warp * 64u * VP;
    uint16_t* vss = reinterpret_cast<uint16_t*>(smem + P.vs_off) + warp * 64u * ND;
    uint32_t* mx = reinterpret_cast<uint32_t*>(smem + P.misc_off);   // [2][RB] the CTA's row max keys
    float* mk = reinterpret_cast<float*>(mx + 2u * RB);              // [RB]
    float* ls = mk + RB;                                             // [segments][RB]
    float* lacc = ls + kFaWarps * RB;                            // [RB]
    int32_t* esw = reinterpret_cast<int32_t*>(lacc + RB);        // [warps][RB]
    uint32_t* flw = reinterpret_cast<uint32_t*>(esw + kFaWarps * RB);
    if (tid < 64) t64s[tid] = g_expk_t64[tid];
    if (tid < 4) lks[tid] = g_expk_lk[tid];
    // the next kernel may start its own prologue; q, the KV cache and the mask copy are read only
    // after the kernel this one depends on has finished
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");

    const uint32_t nseg = (nu + 3u) / 4u;
    const float scale = a.scale;

    // cell of the channel's local index j (cells of group k are 16 k .. 16 k + 15)
    auto cell_of = [&](uint32_t j) { return 16u * (ufirst + C * (j >> 4)) + (j & 15u); };
    // this warp's copies of segment sg into shared memory: of each of its groups the quants of
    // values [ph VP, ph VP + VP) (16 cells each, value-major), and (with scales) the fp16 scales of
    // all its cells; one commit group
    auto stage_v = [&](uint32_t sg, uint32_t ph, bool scales) {
        const uint32_t ng = min(4u, nu - 4u * sg);
        for (uint32_t c = lane; c < ng * VP; c += 32u) {         // VP 16-byte chunks per group
            const uint32_t kk = c / VP, off = (c % VP) * 16u;
            const int8_t* src = a.vq + (head_cells + 16u * (ufirst + C * (4u * sg + kk))) * D + (size_t)ph * VP * 16u;
            cp_async16(vqs + kk * VP * 16u + off, src + off);
        }
        if (scales) {
            for (uint32_t c = lane; c < ng * 2u * ND; c += 32u) {    // a group's scales: 32 ND bytes
                const uint32_t kk = c / (2u * ND), off = (c % (2u * ND)) * 16u;
                const uint8_t* src = reinterpret_cast<const uint8_t*>(a.vd + (head_cells + 16u * (ufirst + C * (4u * sg + kk))) * ND);
                cp_async16(reinterpret_cast<uint8_t*>(vss) + kk * 32u * ND + off, src + off);
            }
        }
        cp_async_commit();
    };

    float* ok_ch = a.ok + (((size_t)item * a.n_head_kv + g) * C + cc) * rows_max * D;
    float* lk_ch = a.lk + (((size_t)item * a.n_head_kv + g) * C + cc) * rows_max;
    bool arrived = false;
    uint32_t pass = 0;
    constexpr uint32_t kFloorKey = ~kMFloor;                    // maxt_key(-2^100)
    for (uint32_t r0 = 0; r0 < rows; r0 += RB, ++pass) {
        const uint32_t nr = min(RB, rows - r0);
        // this pass's max slot (the slots alternate between passes: a peer reads a slot between the
        // barrier of its pass and the next pass's barrier, which this CTA has passed by now)
        uint32_t* slot = mx + (pass & 1u) * RB;
        if (tid < RB) slot[tid] = kFloorKey;
        // ---- QACT A32 of the pass's query rows (tsr_ref.c:472-487): one warp per 32-block ----
        constexpr uint32_t kQB = (RB * ND + kFaWarps - 1u) / kFaWarps;     // blocks per warp
        float qv[kQB];
#pragma unroll
        for (uint32_t i = 0; i < kQB; ++i) {
            const uint32_t bi = warp + i * kFaWarps;
            const uint32_t r = bi / ND, b = bi - r * ND, ri = r0 + r;
            const uint32_t t = ri / G, h = g * G + (ri - t * G);
            qv[i] = bi < nr * ND ? a.q[((size_t)(it.q0 + t) * a.n_head + h) * D + 32u * b + lane] : 0.0f;
        }
#pragma unroll
        for (uint32_t i = 0; i < kQB; ++i) {
            const uint32_t bi = warp + i * kFaWarps;
            if (bi >= nr * ND) break;
            const uint32_t r = bi / ND, b = bi - r * ND;
            const float v = qv[i];
            const uint32_t amax = __reduce_max_sync(0xFFFFFFFFu, amax_key(v));
            const float db = fdiv(ffrom(amax), 127.0f);
            const float id = (fbits(db) & ~kSign) ? frecip(db) : 0.0f;
            qx[r * D + 32u * b + lane] = (int8_t)round_away_sat8(fmul(daz(v), id));
            if (lane == 0) dx[r * ND + b] = h2f(f2h(db));
        }
        __syncthreads();

        // ---- ATTQK (+ AMASK for GENERAL chunks) and the CTA's row maxima ----
        uint32_t rkey[RB];
#pragma unroll
        for (uint32_t r = 0; r < RB; ++r) rkey[r] = kFloorKey;
        // D <= 128: a cell's K bytes stay in registers across the rows, and the thread's next cell is
        // loaded while this one is computed; larger D reads them per row (L1 hits after the first row)
        constexpr uint32_t KW = D <= 128 ? 2 * ND : 1, KD = D <= 128 ? ND : 1;
        uint4 kwn[KW];
        uint16_t kdn[KD];
        auto load_k = [&](uint32_t j) {
            if constexpr (D <= 128) {
                const uint32_t cell = cell_of(j);
                if (cell < a.n_kv) {
                    const uint4* kr = reinterpret_cast<const uint4*>(a.kq + (head_cells + cell) * D);
                    const uint16_t* kdr = a.kd + (head_cells + cell) * ND;
#pragma unroll
                    for (uint32_t i = 0; i < KW; ++i) kwn[i] = kr[i];
#pragma unroll
                    for (uint32_t i = 0; i < KD; ++i) kdn[i] = kdr[i];
                }
            }
        };
        if (tid < ncell) load_k(tid);
        for (uint32_t j = tid; j < ncell; j += kFaThreads) {
            const uint32_t cell = cell_of(j);
            const int64_t jr = (int64_t)cell - 16 * (int64_t)it.u0;         // cell within the chunk
            const int8_t* kr = a.kq + (head_cells + cell) * D;
            const uint16_t* kdr = a.kd + (head_cells + cell) * ND;
            const bool live = cell < a.n_kv;
            uint4 kw[KW];
            uint16_t kd[KD];
#pragma unroll
            for (uint32_t i = 0; i < KW; ++i) kw[i] = kwn[i];
#pragma unroll
            for (uint32_t i = 0; i < KD; ++i) kd[i] = kdn[i];
            if (j + kFaThreads < ncell) load_k(j + kFaThreads);
#pragma unroll
            for (uint32_t r = 0; r < RB; ++r) {
                if (r >= nr) break;
                const uint32_t ri = r0 + r, t = ri / G;
                const int64_t dq = (int64_t)it.Tq - 1 - t;
                float s = ffrom(kNegInf);
                bool vis = true;
                if (!it.general) {
                    const int64_t lo = max((int64_t)0, (int64_t)it.c_lo - ((it.flags & kFlSlide) ? dq : 0));
                    const int64_t hi = (int64_t)it.c_hi - ((it.flags & kFlCausal) ? dq : 0);
                    vis = jr >= lo && jr < hi;
                }
                if (vis && live) {
                    float terms[ND];
#pragma unroll
                    for (uint32_t b = 0; b < ND; ++b) {
                        uint4 w0, w1;
                        uint16_t dk;
                        if constexpr (D <= 128) {
                            w0 = kw[2 * b];
                            w1 = kw[2 * b + 1];
                            dk = kd[b];
                        } else {
                            w0 = reinterpret_cast<const uint4*>(kr)[2 * b];
                            w1 = reinterpret_cast<const uint4*>(kr)[2 * b + 1];
                            dk = kdr[b];
                        }
                        const uint4* xq = reinterpret_cast<const uint4*>(qx + r * D + 32u * b);
                        const int32_t isum = dot32(w0, w1, xq[0], xq[1]);
                        terms[b] = __fmul_rn(__fmul_rn(h2f(dk), dx[r * ND + b]), i2f(isum));
                    }
                    s = tree16_qk<ND>(terms);
                }
                if (it.general) {
                    const float m = cell < a.n_kv ? a.maskf[(size_t)(it.q0 + t) * a.maskf_stride + cell] : ffrom(kNegInf);
                    s = fbits(m) == kNegInf ? ffrom(kNegInf) : fadd(s, m);
                }
                S[r * ncell_max + j] = s;
                rkey[r] = max(rkey[r], maxt_key(s));
            }
        }
        // round 0's V slices, in flight during the maximum and EXP (issued after ATTQK, whose K
        // loads they would otherwise compete with); one round holds every segment: staged once
        if (wseg < nseg && (pass == 0 || nseg > SEGS)) stage_v(wseg, wsl, true);
        // the CTA's row maxima: a warp reduction and a shared-memory atomic per row
#pragma unroll
        for (uint32_t r = 0; r < RB; ++r) {
            const uint32_t k = __reduce_max_sync(0xFFFFFFFFu, rkey[r]);
            if (lane == 0 && r < nr) atomicMax(slot + r, k);
        }
        // ---- the chunk maximum: MAXOUT over every channel of the chunk ----
        // (the cluster barrier also orders every thread's atomics of this CTA before the reads)
        cluster_arrive();
        cluster_wait();
        if (tid < RB) {
            uint32_t mv[16];                 // every channel's max in flight at once
#pragma unroll
            for (uint32_t c = 0; c < 16; ++c) mv[c] = c < C ? *cluster.map_shared_rank(slot + tid, c) : kFloorKey;
            uint32_t km = kFloorKey;
#pragma unroll
            for (uint32_t c = 0; c < 16; ++c) km = max(km, mv[c]);
            const float m = maxt_val(km);
            mk[tid] = m;
            if (cc == 0 && tid < nr) a.mk[((size_t)item * a.n_head_kv + g) * rows_max + r0 + tid] = m;
        }
        if (r0 + RB >= rows) {               // the last pass: no more remote reads
            cluster_arrive();
            arrived = true;
        }
        __syncthreads();
        // ---- ASMAX: p = EXP(fmul(fsub(s, m), scale)) ----
#pragma unroll 4
        for (uint32_t i = tid; i < nr * ncell; i += kFaThreads) {
            const uint32_t r = i / ncell, j = i - r * ncell;
            float* sp = &S[r * ncell_max + j];
            *sp = expk(fmul(fsub(*sp, mk[r]), scale), 0u, t64s, lks);
        }
        if (tid < RB) lacc[tid] = 0.0f;
        __syncthreads();

        // ---- ATTPV + LSUM, results folded in segment order ----
        // A round holds up to SEGS segments; warp (wseg, wsl) stages the V quants of slice wsl of
        // the round's segment wseg (and the segment's scales). Then every warp takes work units
        // of the round in turn: first (segment, slice, row) -- the W digits of the row and, for
        // slice 0, its LSUM -- then (segment, slice, 16-value tile) -- the tensor-core products
        // of the tile for every row.
        constexpr uint32_t kPer = RB * D / kFaThreads;        // (row, value) pairs folded per thread
        constexpr uint32_t kMt = VP / 16u;                    // 16-value tiles of a slice
        float oacc[kPer];
#pragma unroll
        for (uint32_t i = 0; i < kPer; ++i) oacc[i] = 0.0f;
        for (uint32_t sg0 = 0; sg0 < nseg; sg0 += SEGS) {
            const uint32_t nsr = min(SEGS, nseg - sg0);        // segments of this round
            if (sg0 > 0 && wseg < nsr) stage_v(sg0 + wseg, wsl, true);
            cp_async_wait_all();
            __syncthreads();
            // W digits (+ LSUM) of unit (segment s, slice sl, row r)
#pragma unroll 1
            for (uint32_t u = warp; u < nsr * NSL * nr; u += kFaWarps) {
                const uint32_t r = u % nr, ss = u / nr, sl = ss % NSL, s = ss / NSL, sg = sg0 + s;
                const uint32_t owner = s * NSL + sl;           // the warp that staged (s, sl)
                const uint16_t* vsso = reinterpret_cast<const uint16_t*>(smem + P.vs_off) + owner * 64u * ND;
                uint8_t* Wd = Wbase + owner * kWdWarp;
                const uint32_t ng = min(4u, nu - 4u * sg), nc = 16u * ng;
                {
                    // w = p (*) dV of the lane's two cells and the slice's two blocks
                    float w[2][2];
                    int32_t le = -1000;
                    bool bad0 = false, bad1 = false, any = false;
#pragma unroll
                    for (uint32_t h = 0; h < 2; ++h) {
                        const uint32_t i = lane + 32u * h;
                        const float p = i < nc ? S[r * ncell_max + 64u * sg + i] : 0.0f;
                        const bool pz = (fbits(p) & kExp) == 0;
                        const uint32_t pr = i < nc ? *reinterpret_cast<const uint32_t*>(vsso + i * ND + 2u * sl) : 0u;
#pragma unroll
                        for (uint32_t e = 0; e < 2; ++e) {
                            const float wv = pz ? 0.0f : fmul(p, h2f((uint16_t)(e ? pr >> 16 : pr & 0xFFFFu)));
                            w[h][e] = wv;
                            const uint32_t uu = fbits(wv);
                            if (nonfinite(uu)) {
                                if (e == 0) bad0 = true;
                                else bad1 = true;
                            } else if (uu & ~kSign) {
                                le = max(le, (int32_t)((uu >> 23) & 0xFFu) - 127);
                                any = true;
                            }
                        }
                    }
                    const int32_t es = (int32_t)__reduce_max_sync(0xFFFFFFFFu, (uint32_t)(le + 1000)) - 1000;
                    const uint32_t fl3 = __reduce_or_sync(0xFFFFFFFFu, (bad0 ? 1u : 0u) | (bad1 ? 2u : 0u) | (any ? 4u : 0u));
                    bad0 = (fl3 & 1u) != 0;
                    bad1 = (fl3 & 2u) != 0;
                    any = (fl3 & 4u) != 0;
                    // W = RNE_int(w 2^(23 - es)) (|W| <= 2^24) as four balanced base-256 digits,
                    // the B operand of the int8 tensor-core products: table (owner, e), row r*4 + digit
#pragma unroll
                    for (uint32_t h = 0; h < 2; ++h)
#pragma unroll
                        for (uint32_t e = 0; e < 2; ++e) {
                            const int32_t Wv = (any && !(e ? bad1 : bad0)) ? bf_int(w[h][e], es) : 0;
                            const uint32_t dg = digits4(Wv);
                            uint8_t* col = Wd + (e * kWdRows + r * 4u) * kWdStride + lane + 32u * h;
                            col[0] = (uint8_t)dg;
                            col[kWdStride] = (uint8_t)(dg >> 8);
                            col[2u * kWdStride] = (uint8_t)(dg >> 16);
                            col[3u * kWdStride] = (uint8_t)(dg >> 24);
                        }
                    if (lane == 0) {
                        esw[owner * RB + r] = es;
                        flw[owner * RB + r] = (bad0 ? 1u : 0u) | (bad1 ? 2u : 0u) | (any ? 4u : 0u);
                    }
                }
                // LSUM of the segment (tsr_ref_at.c:520-553), with slice 0's unit
                if (sl == 0) {
                    int32_t le = -1000;
                    bool bad = false, any = false;
                    float pv[2];
#pragma unroll
                    for (uint32_t h = 0; h < 2; ++h) {
                        const uint32_t i = lane + 32u * h;
                        pv[h] = i < nc ? daz(S[r * ncell_max + 64u * sg + i]) : 0.0f;
                        const uint32_t uu = fbits(pv[h]);
                        if (nonfinite(uu)) bad = true;
                        else if (uu & ~kSign) {
                            le = max(le, (int32_t)((uu >> 23) & 0xFFu) - 127);
                            any = true;
                        }
                    }
                    const int32_t ep = (int32_t)__reduce_max_sync(0xFFFFFFFFu, (uint32_t)(le + 1000)) - 1000;
                    const uint32_t fl2 = __reduce_or_sync(0xFFFFFFFFu, (bad ? 1u : 0u) | (any ? 2u : 0u));
                    bad = (fl2 & 1u) != 0;
                    any = (fl2 & 2u) != 0;
                    int32_t part = 0;
                    if (!bad && any) part = bf_int(pv[0], ep) + bf_int(pv[1], ep);
                    const int32_t sum = __reduce_add_sync(0xFFFFFFFFu, part);
                    if (lane == 0) ls[s * RB + r] = bad ? ffrom(kCanonNaN) : !any ? 0.0f : bf_f((int64_t)sum, ep - 23);
                }
            }
            __syncthreads();
            // exact sums A[r][v] = sum_cells W * qV on the int8 tensor cores (m16n8k32): A operand
            // = V^T (16 values x 32 cells, from the value-major groups), B operand = the W digits
            // (32 cells x 8 = 2 rows x 4 digits); digit sums are exact in int32 (|.| <= 2^20)
            const uint32_t gid = lane >> 2, tig = lane & 3u;
#pragma unroll 1
            for (uint32_t u = warp; u < nsr * NSL * kMt; u += kFaWarps) {
                const uint32_t mt = u % kMt, ss = u / kMt, sl = ss % NSL, s = ss / NSL, sg = sg0 + s;
                const uint32_t owner = s * NSL + sl;
                const int8_t* vqo = reinterpret_cast<const int8_t*>(smem + P.vq_off) + owner * 64u * VP;
                const uint8_t* Wd = Wbase + owner * kWdWarp;
                const uint32_t ng = min(4u, nu - 4u * sg), nks = (ng + 1u) / 2u;
                float* cvw = CV + s * RB * D;
                const uint32_t v0 = sl * VP + 16u * mt, e = (16u * mt) / 32u;
                const uint8_t* Wt_se = Wd + e * kWdRows * kWdStride;
                int32_t acc[kNT][4];
#pragma unroll
                for (uint32_t nt = 0; nt < kNT; ++nt)
#pragma unroll
                    for (uint32_t j = 0; j < 4; ++j) acc[nt][j] = 0;
                for (uint32_t ks = 0; ks < nks; ++ks) {
                    const uint8_t* va = reinterpret_cast<const uint8_t*>(vqo) + ((2u * ks) * VP + 16u * mt + gid) * 16u + tig * 4u;
                    const uint32_t a0 = *reinterpret_cast<const uint32_t*>(va);
                    const uint32_t a1 = *reinterpret_cast<const uint32_t*>(va + 8u * 16u);
                    const uint32_t a2 = *reinterpret_cast<const uint32_t*>(va + VP * 16u);
                    const uint32_t a3 = *reinterpret_cast<const uint32_t*>(va + VP * 16u + 8u * 16u);
#pragma unroll
                    for (uint32_t nt = 0; nt < kNT; ++nt) {
                        const uint8_t* wb = Wt_se + ((nt * 8u + gid) % kWdRows) * kWdStride + 32u * ks + tig * 4u;
                        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(wb);
                        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(wb + 16u);
                        asm volatile(
                            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                            "{%0,%1,%2,%3};"
                            : "+r"(acc[nt][0]), "+r"(acc[nt][1]), "+r"(acc[nt][2]), "+r"(acc[nt][3])
                            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
                    }
                }
                // digits 0,1 sit in even lanes (tig even), 2,3 in the odd neighbour: even lanes
                // finish value gid, odd lanes value gid + 8
                const bool odd = (tig & 1u) != 0;
#pragma unroll
                for (uint32_t nt = 0; nt < kNT; ++nt) {
                    const int32_t s0 = odd ? acc[nt][0] : acc[nt][2], s1 = odd ? acc[nt][1] : acc[nt][3];
                    const int32_t o0 = __shfl_xor_sync(0xFFFFFFFFu, s0, 1), o1 = __shfl_xor_sync(0xFFFFFFFFu, s1, 1);
                    int64_t Av;
                    if (!odd) Av = (int64_t)acc[nt][0] + ((int64_t)acc[nt][1] << 8) + ((int64_t)o0 << 16) + ((int64_t)o1 << 24);
                    else Av = (int64_t)o0 + ((int64_t)o1 << 8) + ((int64_t)acc[nt][2] << 16) + ((int64_t)acc[nt][3] << 24);
                    const uint32_t r = nt * 2u + (tig >> 1), v = v0 + gid + (odd ? 8u : 0u);
                    if (r < nr) {
                        const int32_t es = esw[owner * RB + r];
                        const uint32_t fl = flw[owner * RB + r];
                        const bool bad = (fl >> e) & 1u, any = (fl & 4u) != 0;
                        cvw[r * D + v] = bad ? ffrom(kCanonNaN) : !any ? 0.0f : bf_f(Av, es - 23);
                    }
                }
            }
            __syncthreads();
            // fold this round's segments in order: o = fadd(o, cv), l = fadd(l, v)
            const uint32_t nw = min(SEGS, nseg - sg0);
#pragma unroll
            for (uint32_t i = 0; i < kPer; ++i) {
                const uint32_t pidx = tid + i * kFaThreads, r = pidx / D;
                if (r < nr)
                    for (uint32_t w = 0; w < nw; ++w) oacc[i] = fadd(oacc[i], CV[w * RB * D + pidx]);
            }
            if (tid < nr) {
                float l = lacc[tid];
                for (uint32_t w = 0; w < nw; ++w) l = fadd(l, ls[w * RB + tid]);
                lacc[tid] = l;
            }
            __syncthreads();
        }
        // ---- the channel's result and row sums of the pass's rows ----
#pragma unroll
        for (uint32_t i = 0; i < kPer; ++i) {
            const uint32_t pidx = tid + i * kFaThreads;
            if (pidx < nr * D) ok_ch[(size_t)r0 * D + pidx] = oacc[i];
        }
        if (tid < nr) lk_ch[r0 + tid] = lacc[tid];
    }
    if (!arrived) cluster_arrive();
    cluster_wait();
}

// CTREE (tsr_ref_at.c:588-598) of N values: pairwise by levels, an unpaired last element passes
// through.
template <uint32_t N>
__device__ __forceinline__ float ctree(float (&v)[N]) {
    uint32_t n = N;
#pragma unroll
    for (uint32_t lvl = 0; lvl < 5; ++lvl) {
        if (n <= 1u) break;
#pragma unroll
        for (uint32_t k = 0; k < (N + 1u) / 2u; ++k) {
            if (2u * k + 1u < n) v[k] = fadd(v[2u * k], v[2u * k + 1u]);
            else if (2u * k + 1u == n) v[k] = v[2u * k];
        }
        n = (n + 1u) / 2u;
    }
    return v[0];
}

// CTREE of the C channel results of each chunk, AMERGE over the chunks of each tile in execution
// order, then ANORM (tsr_ref_at.c:588-641). One thread per output value; the values of two chunks
// are loaded before they are folded.
template <uint32_t C>
__global__ void __launch_bounds__(256) fa_merge_kernel(FaLaunch a) {
    asm volatile("griddepcontrol.launch_dependents;");
    const uint32_t G = a.G, D = a.D, rows_max = a.Tq0 * G;
    const size_t per_tile = (size_t)a.n_head_kv * rows_max * D;
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (size_t)a.n_tiles * per_tile) return;
    const uint32_t tile = (uint32_t)(idx / per_tile);
    size_t rem = idx - (size_t)tile * per_tile;
    const uint32_t g = (uint32_t)(rem / ((size_t)rows_max * D));
    rem -= (size_t)g * rows_max * D;
    const uint32_t ri = (uint32_t)(rem / D), v = (uint32_t)(rem - (size_t)ri * D);
    const bool inl = a.n_items <= kFaInlineItems;
    const uint32_t i0 = inl ? a.inl_tiles[tile] : a.tile_items[tile], i1 = inl ? a.inl_tiles[tile + 1] : a.tile_items[tile + 1];
    const FaItem first = inl ? a.inl_items[i0] : a.items[i0];
    if (ri >= first.Tq * G) return;
    const float scale = a.scale;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    float O = 0.0f, lrun = 0.0f, mrun = 0.0f;
    constexpr uint32_t kB = 2;
    for (uint32_t k0 = i0; k0 < i1; k0 += kB) {
        float ok[kB][C], lk[kB][C], mkk[kB];
#pragma unroll
        for (uint32_t j = 0; j < kB; ++j) {
            if (k0 + j < i1) {
                const size_t hb = (size_t)(k0 + j) * a.n_head_kv + g;
#pragma unroll
                for (uint32_t c = 0; c < C; ++c) {
                    ok[j][c] = a.ok[((hb * C + c) * rows_max + ri) * D + v];
                    lk[j][c] = a.lk[(hb * C + c) * rows_max + ri];
                }
                mkk[j] = a.mk[hb * rows_max + ri];
            }
        }
#pragma unroll
        for (uint32_t j = 0; j < kB; ++j) {
            if (k0 + j >= i1) break;
            const float oj = ctree<C>(ok[j]), lj = ctree<C>(lk[j]);
            if (k0 + j == i0) {
                O = oj;
                lrun = lj;
                mrun = mkk[j];
            } else {
                const float mn = maxt(mrun, mkk[j]);
                const float ea = expk(fmul(fsub(mrun, mn), scale), 0u, g_expk_t64, g_expk_lk);
                const float eb = expk(fmul(fsub(mkk[j], mn), scale), 0u, g_expk_t64, g_expk_lk);
                lrun = fadd(fmul(lrun, ea), fmul(lj, eb));
                mrun = mn;
                O = fadd(fmul(O, ea), fmul(oj, eb));
            }
        }
    }
    const float rinv = frecip(maxt(lrun, ffrom(kLFloor)));
    const uint32_t t = ri / G, h = g * G + (ri - t * G);
    a.out[((size_t)(first.q0 + t) * a.n_head + h) * D + v] = canon(fmul(O, rinv));
}

using MergeFn = void (*)(FaLaunch);
constexpr MergeFn kMerge[16] = {fa_merge_kernel<1>,  fa_merge_kernel<2>,  fa_merge_kernel<3>,  fa_merge_kernel<4>,
                                fa_merge_kernel<5>,  fa_merge_kernel<6>,  fa_merge_kernel<7>,  fa_merge_kernel<8>,
                                fa_merge_kernel<9>,  fa_merge_kernel<10>, fa_merge_kernel<11>, fa_merge_kernel<12>,
                                fa_merge_kernel<13>, fa_merge_kernel<14>, fa_merge_kernel<15>, fa_merge_kernel<16>};

// f32 mask copy of the GENERAL path (tsr_ref_at.c:694-715): fdiv(f32(mask), scale), -inf kept.
__global__ void fa_maskf_kernel(const uint16_t* m16, uint32_t stride, uint32_t T, uint32_t n_kv, float scale, float* out) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)T * n_kv) return;
    const uint32_t t = (uint32_t)(i / n_kv), j = (uint32_t)(i - (size_t)t * n_kv);
    const uint16_t h = m16[(size_t)t * stride + j];
    out[(size_t)t * n_kv + j] = h == 0xFC00u ? ffrom(kNegInf) : fdiv(h2f(h), scale);
}

// The kernel's attributes, set once per device: the largest shared-memory plan any call can need
// and non-portable cluster sizes (C up to 16).
template <int D, uint32_t W>
cudaError_t fa_attributes() {
    static int done_dev[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 64 && done_dev[dev] == dev + 1) return cudaSuccess;
    e = cudaFuncSetAttribute(fa_chunk_kernel<D, W>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(227u * 1024u));
    if (e == cudaSuccess) e = cudaFuncSetAttribute(fa_chunk_kernel<D, W>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e == cudaSuccess && dev < 64) done_dev[dev] = dev + 1;
    return e;
}

template <int D, uint32_t W>
cudaError_t launch_chunks_w(const FaLaunch& a, uint32_t ncell_max, cudaStream_t st) {
    const FaSmem P = fa_smem(D, ncell_max, W);
    cudaError_t e = fa_attributes<D, W>();
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_items * a.n_head_kv * a.C);
    cfg.blockDim = dim3(W * 32u);
    cfg.dynamicSmemBytes = P.total;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a.C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (a.C > 8) {        // a non-portable cluster size: make sure one cluster can be resident
        int n = 0;
        e = cudaOccupancyMaxActiveClusters(&n, (const void*)fa_chunk_kernel<D, W>, &cfg);
        if (e != cudaSuccess) return e;
        if (n == 0) return cudaErrorInvalidConfiguration;
    }
    return cudaLaunchKernelEx(&cfg, fa_chunk_kernel<D, W>, a);
}

// 2-warp CTAs (head sizes up to 128) when the call has enough of them to fill every SM eight times
// over, 4-warp CTAs at four times (a prompt), else 16-warp CTAs (decode)
template <int D>
cudaError_t launch_chunks(const FaLaunch& a, uint32_t ncell_max, cudaStream_t st) {
    if constexpr (D <= 256) {
        int dev = 0, sms = 148;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const uint64_t ctas = (uint64_t)a.n_items * a.n_head_kv * a.C;
        if constexpr (D <= 128)
            if (ctas >= 8u * (uint64_t)sms) return launch_chunks_w<D, kFaWarpsTiny>(a, ncell_max, st);
        if (ctas >= 4u * (uint64_t)sms) return launch_chunks_w<D, kFaWarpsSmall>(a, ncell_max, st);
    }
    return launch_chunks_w<D, kFaWarpsLarge>(a, ncell_max, st);
}

}  // namespace

size_t fa_smem_bytes(uint32_t D, uint32_t n_max_groups, uint32_t C) {
    return fa_smem(D, 16u * ((n_max_groups + C - 1u) / C), kFaWarpsLarge).total;
}

cudaError_t launch_fa_maskf(const uint16_t* m16, uint32_t stride, uint32_t T, uint32_t n_kv, float scale, float* out,
                            cudaStream_t st) {
    const size_t n = (size_t)T * n_kv;
    if (n == 0) return cudaSuccess;
    fa_maskf_kernel<<<(unsigned)((n + 255u) / 256u), 256, 0, st>>>(m16, stride, T, n_kv, scale, out);
    return cudaGetLastError();
}

const void* fa_merge_fn(uint32_t C) { return C >= 1u && C <= 16u ? reinterpret_cast<const void*>(kMerge[C - 1u]) : nullptr; }

const void* fa_chunk_fn(uint32_t D, uint32_t warps) {
    const bool small = warps == kFaWarpsSmall, tiny = warps == kFaWarpsTiny;
    switch (D) {
        case 64: return tiny ? reinterpret_cast<const void*>(fa_chunk_kernel<64, kFaWarpsTiny>)
                      : small ? reinterpret_cast<const void*>(fa_chunk_kernel<64, kFaWarpsSmall>)
                              : reinterpret_cast<const void*>(fa_chunk_kernel<64, kFaWarpsLarge>);
        case 128: return tiny ? reinterpret_cast<const void*>(fa_chunk_kernel<128, kFaWarpsTiny>)
                       : small ? reinterpret_cast<const void*>(fa_chunk_kernel<128, kFaWarpsSmall>)
                               : reinterpret_cast<const void*>(fa_chunk_kernel<128, kFaWarpsLarge>);
        case 256: return tiny ? nullptr
                       : small ? reinterpret_cast<const void*>(fa_chunk_kernel<256, kFaWarpsSmall>)
                               : reinterpret_cast<const void*>(fa_chunk_kernel<256, kFaWarpsLarge>);
        case 512: return (small || tiny) ? nullptr : reinterpret_cast<const void*>(fa_chunk_kernel<512, kFaWarpsLarge>);
        default: return nullptr;
    }
}

cudaError_t launch_fa(const FaLaunch& a, uint32_t n_max_groups, cudaStream_t st) {
    const uint32_t ncell_max = 16u * ((n_max_groups + a.C - 1u) / a.C);
    cudaError_t e;
    switch (a.D) {
        case 64: e = launch_chunks<64>(a, ncell_max, st); break;
        case 128: e = launch_chunks<128>(a, ncell_max, st); break;
        case 256: e = launch_chunks<256>(a, ncell_max, st); break;
        case 512: e = launch_chunks<512>(a, ncell_max, st); break;
        default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    if (a.C < 1u || a.C > 16u) return cudaErrorInvalidValue;
    const size_t n = (size_t)a.n_tiles * a.n_head_kv * a.Tq0 * a.G * a.D;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((n + 255u) / 256u));
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kMerge[a.C - 1u], a);
}

}  // namespace tsrc
