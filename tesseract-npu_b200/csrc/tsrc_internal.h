// tsrc_internal.h -- declarations shared by the library's translation units (not part of the ABI).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

struct tsrc_ctx;
struct tsrc_kv;
struct tsrc_fa_cfg;

namespace tsrc {

constexpr uint32_t kMmAdd = 0x1u;
constexpr uint32_t kMmScale = 0x2u;
constexpr uint32_t kMmSoftcap = 0x4u;
constexpr uint32_t kMvMaxT = 8;            // tokens per matvec launch (larger T is tiled)

// Arguments of one matvec launch over a weight shard (device pointers).
struct MvArgs {
    const uint8_t* qs;        // weight quants: Q8_0 [n_rows][K]; Q4_K [n_rows][K/2]
    const void* meta;         // Q8_0: fp16 d [n_rows][K/32]; Q4_K: 16 B {d, dmin, scales} [n_rows][K/256]
    uint32_t n_rows, K;
    const float* x;           // f32 tokens (x[t * x_stride + k]): the kernel runs QACT itself; or NULL:
    uint32_t x_stride;
    const int8_t* qx;         // QA of T tokens: q [T][K]
    const float* dx;          //                 d [T][K/bs]
    const int16_t* bsx;       //                 bs [T][K/16] (Q4_K)
    const int8_t* bsd;        //                 Q4_K on the tensor cores: pair-sum digits [T][K/256][16]
    uint32_t T;
    float* y;                 // y [t * y_stride + n]
    uint32_t y_stride;
    const float* add;         // addend [t * add_stride + n] (kMmAdd)
    uint32_t add_stride;
    uint32_t flags;
    float s0, s1;
    int32_t* isum_out;        // optional: the kernel's exact block sums of token 0
    // RMS_NORM (+ MUL) of the token fused in front of QACT (T = 1; rms = 0: off): the activation is
    // y_j = canon(FM(fmul(daz(x_j), scale), w_j)) with the RMS_NORM kind's scale (tsrc_vu.cu)
    const float* rms_w;       // the norm weight, or NULL (no MUL)
    float rms_eps, rms_inv_n;
    uint32_t rms;
    // SWIGLU of row pairs as the epilogue (T = 1; 0: off): rows 2j, 2j + 1 are gate_j, up_j and
    // y[j] = canon(FM(SILU(gate_j), up_j)), the SWIGLU kind's value (tsrc_vu.cu); y has n_rows / 2
    uint32_t swiglu_pairs;
    // fused all-gather over a team of GPUs (one token; team_world = 0: off). Row n of the shard
    // is stored into every rank's staging buffer at team_row0 + n (half (step & 1) of [2][team_n])
    // as one 64-bit word {value bits, step + 1}; every CTA then copies its share of the full
    // vector into y once each word of the share carries this step's tag.
    unsigned long long* const* team_y;  // device array [world]: each rank's staging [2][team_n] tagged words
    uint32_t* team_state;     // this rank: [0] steps done, [1] CTAs finished in this launch
    uint32_t team_world, team_rank, team_row0, team_n;
    uint32_t team_half;       // words per staging half (the team's capacity; calls of any N alternate halves)
    // MUL_MAT_ID (one token per slot; moe_pairs = 0: off): grid row p = (t, j) of moe_pairs = T n_used
    // runs expert e = ids[t ids_stride + j] -- rows [e n_rows, (e + 1) n_rows) of the stacked weight --
    // on x + t x_tok + (j mod x_slots) x_slot, into y + t y_tok + j y_slot
    const int32_t* ids;
    uint32_t moe_pairs, n_used, n_exp, ids_stride, x_slots, x_slot, x_tok, y_slot, y_tok;
};

cudaError_t launch_qact(uint32_t kind, const float* x, uint32_t K, uint32_t T, uint32_t x_stride, int8_t* q, float* d,
                        int16_t* bs, cudaStream_t st, int8_t* bsd = nullptr);
cudaError_t launch_matvec(uint32_t fmt, const MvArgs& a, cudaStream_t st);
// All-gather of a plain vector over a team (the tagged-word exchange of the fused MUL_MAT, without
// the MUL_MAT): src [n_local] of this rank lands at dst[offset .. offset + n_local) on every rank.
struct TeamGather {
    unsigned long long* const* team_y;
    uint32_t* team_state;
    uint32_t world, rank, half;
    const float* src;
    uint32_t n_local, offset, n;
    float* dst;
    uint32_t T, src_stride, dst_stride;   // T token rows: src [T][src_stride], dst [T][dst_stride]; T n <= half
};
cudaError_t launch_team_gather(const TeamGather& g, cudaStream_t st);
}  // namespace tsrc
struct tsrc_team;
struct tsrc_weight;
namespace tsrc {
// tsrc_team.cu: the model runner's tensor-parallel steps (see there)
int team_info(const tsrc_team* t, uint32_t* rank, uint32_t* world, uint32_t* n_max);
int team_mul_mat(tsrc_ctx* ctx, tsrc_team* t, const tsrc_weight* w, const float* x, float* y, const float* add,
                 const float* rms_w, float eps, float inv_n, bool rms, void* stream);
// RMS_NORM in front and SWIGLU of row pairs behind, the pairs' outputs gathered over the team at
// [out0, out0 + n_rows / 2) of y (out_n values)
int team_mul_mat_swiglu(tsrc_ctx* ctx, tsrc_team* t, const tsrc_weight* w, const float* x, float* y, uint32_t out0,
                        uint32_t out_n, const float* rms_w, float eps, float inv_n, void* stream);
// tsrc_api.cu: one-token MUL_MAT with RMS_NORM in front and SWIGLU of row pairs behind
int mul_mat_rms_swiglu(tsrc_ctx* ctx, const tsrc_weight* w, const float* x, const float* norm_w, float eps, float inv_n,
                       float* y, void* stream);
// a copy of w with its two halves of rows interleaved (row j of the first half -> 2j, of the
// second -> 2j + 1); w is freed
int weight_interleave_halves(tsrc_ctx* ctx, tsrc_weight* w, tsrc_weight** out);
int weight_rows(const tsrc_weight* w, uint32_t* N, uint32_t* row0, uint32_t* n_rows);
int team_gather(tsrc_team* t, const float* src, uint32_t n_local, uint32_t offset, float* dst, uint32_t n, void* stream);
// T token rows of such vectors (row strides in floats), several rows per team step
int team_gather_rows(tsrc_team* t, const float* src, uint32_t src_stride, uint32_t n_local, uint32_t offset, float* dst,
                     uint32_t dst_stride, uint32_t n, uint32_t T, void* stream);
// tsrc_api.cu: a weight whose rows are row ranges [r0[i], r0[i] + n[i]) of one synthetic N-row
// matrix, stacked in that order (the rows equal those of tsrc_weight_synth's full matrix)
int weight_synth_ranges(tsrc_ctx* ctx, uint32_t fmt, uint32_t N, uint32_t K, const uint32_t* r0, const uint32_t* n,
                        uint32_t count, uint64_t seed, float sigma, tsrc_weight** out);
// Many-token MUL_MAT on the tcgen05 tensor cores (Q8_0; the QA image in qx / dx, any T).
cudaError_t launch_mm_tc(uint32_t fmt, const MvArgs& a, cudaStream_t st);

// tsrc_vu.cu: RMS_NORM, ROPE, VOP, GET_ROWS
cudaError_t launch_rms_norm(const float* x, uint32_t xs, float* y, uint32_t ys, const float* w, uint32_t n, uint32_t rows,
                            float eps, float inv_n, cudaStream_t st);
cudaError_t launch_rope(const float* x, uint32_t xs, float* y, uint32_t ys, const int32_t* pos, uint32_t T, uint32_t n_heads,
                        uint32_t hd, uint32_t nd, uint32_t neox, float ts, float m, cudaStream_t st);
// ROPE from per-position tables [n_pos][n_dims / 2] of c_i and s_i (filled by launch_rope_table)
cudaError_t launch_rope_table(uint32_t n_pos, uint32_t nd, float ts, float m, float* cs_tab, float* sn_tab, cudaStream_t st);
cudaError_t launch_rope_apply(const float* x, uint32_t xs, float* y, uint32_t ys, const int32_t* pos, uint32_t T,
                              uint32_t n_heads, uint32_t hd, uint32_t nd, uint32_t neox, const float* cs_tab,
                              const float* sn_tab, cudaStream_t st);
cudaError_t launch_vop(uint32_t func, const float* a, uint32_t as, const float* b, uint32_t bs, float* y, uint32_t ys,
                       uint32_t n, uint32_t rows, cudaStream_t st);
cudaError_t launch_get_rows(uint32_t fmt, const uint8_t* qs, const void* meta, uint32_t n_rows, uint32_t K, const int32_t* ids,
                            uint32_t T, float* y, uint32_t ys, cudaStream_t st);
cudaError_t vu_error(uint32_t* code, bool clear);

// records msg as the C ABI's last error and returns code (tsrc_api.cu)
int api_fail(int code, const char* msg);
cudaError_t tc_error(uint32_t* code, bool clear);
size_t mv_smem_bytes(uint32_t fmt, uint32_t K, uint32_t T);
// The first error code any matvec launch recorded on the current device (0 = none).
cudaError_t matvec_error(uint32_t* code, bool clear);

// Weight layout (tsrc_weights.cu): ggml rows <-> this library's split layout.
cudaError_t launch_repack(uint32_t fmt, const uint8_t* ggml, uint32_t n_rows, uint32_t K, uint8_t* qs, uint8_t* meta,
                          cudaStream_t st);
cudaError_t launch_unrepack(uint32_t fmt, const uint8_t* qs, const uint8_t* meta, uint32_t n_rows, uint32_t K,
                            uint8_t* ggml, cudaStream_t st);
cudaError_t launch_synth(uint32_t fmt, uint32_t K, uint32_t row0, uint32_t n_rows, uint64_t seed, float sigma,
                         uint8_t* qs, uint8_t* meta, cudaStream_t st);

// ---- flash attention (tsrc_fa.cu, tsrc_fa_plan.cu, tsrc_kv.cu) ----------------------------------
// One work item: a query tile [q0, q0 + Tq) and one chunk of its plan (groups [u0, u0 + n) of 16
// cells; c_lo / c_hi the ATTQK bounds relative to cell 16 u0; flags causal 1 / slide 2; general:
// the chunk runs ATTQK without bounds and then adds the f32 mask copy).
struct FaItem {
    uint32_t q0, Tq, u0, n, c_lo, c_hi, flags, general;
};

constexpr uint32_t kFaInlineItems = 32;   // plans up to this size travel in the kernel parameters

struct FaLaunch {
    const float* q;             // [T][n_head][D] f32
    uint32_t T, n_head, n_head_kv, D, G, C, n_kv, n_cells;
    const int8_t* kq;           // K quants [n_head_kv][n_cells][D]
    const uint16_t* kd;         // K scales (fp16) [n_head_kv][n_cells][D/32]
    const int8_t* vq;           // V quants [n_head_kv][n_cells / 16][D][16] (value-major per group)
    const uint16_t* vd;         // V scales, as K
    const float* maskf;         // f32 mask copy [T][maskf_stride] (GENERAL chunks only)
    uint32_t maskf_stride;
    float scale;
    const FaItem* items;        // work items, tile by tile, chunks in execution order
    uint32_t n_items;
    const uint32_t* tile_items; // [n_tiles + 1]: items of tile i are [tile_items[i], tile_items[i + 1])
    uint32_t n_tiles, Tq0;
    float* ok;                  // channel results  [n_items][n_head_kv][C][Tq0 G][D]
    float* lk;                  // channel row sums [n_items][n_head_kv][C][Tq0 G]
    float* mk;                  // chunk maxima     [n_items][n_head_kv][Tq0 G]
    float* out;                 // [T][n_head][D] f32
    // small plans: the items and tile offsets themselves (no host -> device copy, so a call can be
    // captured in a CUDA graph); used when n_items <= kFaInlineItems
    FaItem inl_items[kFaInlineItems];
    uint32_t inl_tiles[kFaInlineItems + 1];
};

cudaError_t launch_fa(const FaLaunch& a, uint32_t n_max_groups, cudaStream_t st);
// the kernels launch_fa runs (to find their nodes in a captured CUDA graph)
// the chunk kernel of head size D with CTAs of `warps` warps (16; 4 or 2 for calls with many items)
const void* fa_chunk_fn(uint32_t D, uint32_t warps);
const void* fa_merge_fn(uint32_t C);
// tsrc_flash_attn up to the kernel launches (tsrc_api.cu)
int fa_setup(::tsrc_ctx* ctx, const ::tsrc_kv* kv, const float* q, uint32_t T, uint32_t n_head, uint32_t n_kv,
             const uint16_t* mask, uint32_t mask_stride, float scale, uint32_t new_lo, uint32_t new_hi,
             const ::tsrc_fa_cfg* cfg, float* out, cudaStream_t st, FaLaunch* la, uint32_t* n_max_groups);
size_t fa_smem_bytes(uint32_t D, uint32_t n_max_groups, uint32_t C);
cudaError_t launch_fa_maskf(const uint16_t* m16, uint32_t stride, uint32_t T, uint32_t n_kv, float scale, float* out,
                            cudaStream_t st);

// The host-side plan of one FA call (the reference's pass rule, mask summary and chunk planner).
struct FaPlanIn {
    uint32_t C, t_max, pcap, k_max;
    uint32_t T, D, n_head, n_head_kv, n_kv;
    uint32_t plan_n_head_kv;    // KV heads of the whole model (E of the plan and the shape checks)
    const uint16_t* mask;       // host f16 mask [T][mask_stride], or NULL (every cell < n_kv visible)
    size_t mask_stride;
    uint32_t new_lo, new_hi;    // cells written by this launch: their chunks run last
};
struct FaPlanOut {
    uint32_t Tq0, G, n_tiles, n_max_groups;
    bool general;               // some chunk runs the GENERAL path (needs the f32 mask copy)
};
// 0, or a TSRC_E_* code with a message in *why.
int fa_plan(const FaPlanIn& in, FaPlanOut* out, FaItem** items, uint32_t* n_items, uint32_t** tile_items, const char** why);
void fa_plan_free(FaItem* items, uint32_t* tile_items);

#ifdef __CUDACC__
// Byte offset of (cell, value k of head g) in a KV quant plane of n_cells cells per head (head-major;
// K cell-major [head][cell][D]; vt: the V plane's value-major 16-cell groups [head][group][D][16]).
__device__ __forceinline__ size_t kv_qoff(bool vt, uint32_t g, uint32_t n_cells, uint32_t D, size_t cell, uint32_t k) {
    const size_t hc = (size_t)g * n_cells + cell;
    return vt ? (hc - (cell & 15u)) * D + (size_t)k * 16u + (cell & 15u) : hc * D + k;
}
#endif

// ROPE of the q and k heads of T fused q | k | v rows (in place, from the per-position tables),
// then KVST of each token's k and v rows into a layer's K and V planes: one launch for what the
// decoder layer's ROPE, ROPE and two SET_ROWS nodes do (tsrc_vu.cu). err: the KVST error flag.
struct RopeKvst {
    float* qkv;
    uint32_t stride;            // floats per token row
    const int32_t* pos;         // [T]
    uint32_t n_rot_heads, hd, nd, neox;   // q heads + k heads are rotated
    const float *cs_tab, *sn_tab;
    uint32_t k_off, v_off;      // the k and v rows inside a token row
    const int64_t* cells;       // [T] or NULL: cell0 + t
    uint32_t cell0, n_head_kv, n_cells;   // n_cells: the planes' cells per head (padded to 16)
    int8_t *kq, *vq;
    uint16_t *kd, *vd;
    unsigned int* err;
};
cudaError_t launch_rope_kvst(const RopeKvst& a, uint32_t T, cudaStream_t st);
// fills n_head_kv, n_cells and the plane pointers of `a` from a cache (tsrc_api.cu); cells of the cache
int kv_fill_planes(const ::tsrc_kv* kv, RopeKvst* a);
uint32_t kv_cells(const ::tsrc_kv* kv);
cudaError_t kv_error_flag(unsigned int** err);

// KV cache planes (tsrc_kv.cu): KVST of f32 rows (QACT A32), and ggml q8_0 rows <-> planes.
// vt: the V plane (value-major inside each 16-cell group); K is cell-major.
cudaError_t launch_kv_store(const float* rows, uint32_t n, uint32_t row_stride, const int64_t* cells, uint32_t cell0,
                            uint32_t n_head_kv, uint32_t D, uint32_t n_cells, bool vt, int8_t* q, uint16_t* d, cudaStream_t st);
cudaError_t launch_kv_from_ggml(const uint8_t* ggml, uint32_t n, uint32_t cell0, uint32_t n_head_kv, uint32_t D,
                                uint32_t n_cells, bool vt, int8_t* q, uint16_t* d, cudaStream_t st);
cudaError_t launch_kv_to_ggml(const int8_t* q, const uint16_t* d, uint32_t n, uint32_t cell0, uint32_t n_head_kv, uint32_t D,
                              uint32_t n_cells, bool vt, uint8_t* ggml, cudaStream_t st);
// The first error a KVST launch recorded on the current device (0 = none, 1 = a cell index
// outside the cache).
cudaError_t kv_error(uint32_t* code, bool clear);

}  // namespace tsrc
