// tsro.h — CPU restatement of the Tesseract hot-path numerics (TEST INFRASTRUCTURE ONLY).
//
// This library is the parity oracle of the B200 build. Only the tests, the smoke check and the
// CPU-baseline leg of the bench load it; the product (the CUDA C-ABI library) never links or calls
// it, and there is no CPU fallback built on it.
//
// It restates, in plain C11 built with -ffp-contract=off -fno-fast-math, the reference's bit-exact
// definitions (jwkim04/tesseract-npu, sw/sim):
//   - the f32 rules of sw/sim/include/tsr_ref.h:47-70 (DAZ inputs, RNE, flush of subnormal
//     results after gradual rounding, canonical NaN 0x7FC00000),
//   - QACT A32 / A256 of sw/sim/tsr_ref.c:456-518,
//   - the Q8_0 / Q4_K block terms and the 16-partial row dot of sw/sim/tsr_ref.c:526-635,
//   - EXPK / TANH of sw/sim/tsr_ref_math.c:78-161 and :206-229,
//   - flash attention over a q8_0 KV cache, sw/sim/tsr_ref_at.c (tsro_fa.c).
// Data is passed in plain arrays in the layouts the GPU path uses (ggml blocks for weights and KV
// rows; QA split into q[K] int8, d[K/bs] f32 and, for A256, bs[K/16] int16), not in the FPGA's
// repacked beats: the numerics do not depend on that layout.
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TSRO_FMT_Q8_0 0u
#define TSRO_FMT_Q4_K 1u
#define TSRO_QA_A32   0u
#define TSRO_QA_A256  1u

// ---- f32 rules (tsr_ref.c:54-104) -----------------------------------------------------------
float    tsro_fadd(float a, float b);
float    tsro_fsub(float a, float b);
float    tsro_fmul(float a, float b);
float    tsro_fdiv(float a, float b);
float    tsro_frecip(float a);
float    tsro_i32_to_f32(int32_t v);
float    tsro_fp16_to_f32(uint16_t h);
uint16_t tsro_f32_to_fp16(float f);
float    tsro_tree16(const float p[16]);

// ---- VU math (tsr_ref_math.c) ---------------------------------------------------------------
float    tsro_expk(float v, unsigned kappa);   // kappa: 0 P1 (+1), 1 N1 (-1), 2 N2 (-2), 3 NG (-C2G)
float    tsro_exp(float x);
float    tsro_tanh(float x);

// ---- decoder-layer vector kinds (tsro_vu.c; tsr_ref_vu.c, tsr_ref_math.c, tsr_ref.c) ------------
float    tsro_fsqrt(float a);
// RMS_NORM + MUL on rows x n (contiguous rows): RED.SUMSQ post RMS then FM(FM(x, s), w) (w may be NULL)
void     tsro_rms_norm(const float * x, float * y, const float * w, uint32_t n, uint32_t rows, float eps, float inv_n);
void     tsro_sincos(float t, float * s, float * c);
// ROPE recurrence form; mode 0 NORM, 1 NEOX; x, y: [T][n_heads][hd] (y may be x)
void     tsro_rope(const float * x, float * y, const int32_t * pos, uint32_t T, uint32_t n_heads, uint32_t hd, uint32_t nd,
                   uint32_t mode, float ts, float m);
// VOP: func 0 ADD, 2 MUL, 6 SILU (b unused), 7 SWIGLU
void     tsro_vop(uint32_t func, const float * a, const float * b, float * y, size_t n);
// one ggml row (K/32 block_q8_0 or K/256 block_q4_K) -> K f32 values
void     tsro_dequant_row(uint32_t fmt, const uint8_t * row, uint32_t K, float * y);

// ---- QACT (tsr_ref.c:456-518) ----------------------------------------------------------------
// A32: q[K], d[K/32] (d = f32(fp16(amax/127))). A256: q[K], d[K/256], bs[K/16].
void     tsro_qact_a32(const float * x, uint32_t K, int8_t * q, float * d);
void     tsro_qact_a256(const float * x, uint32_t K, int8_t * q, float * d, int16_t * bs);

// ---- Row dot products (tsr_ref.c:526-635) -----------------------------------------------------
// row: K/32 ggml block_q8_0 (34 B) or K/256 block_q4_K (144 B). isum (may be NULL) receives the
// exact int32 block sums: Q8_0 one per block; Q4_K two per superblock {sum sc_j*S_j, sum m_j*BS}.
float    tsro_dot_q8_0(const uint8_t * row, uint32_t K, const int8_t * q, const float * d, int32_t * isum);
float    tsro_dot_q4_K(const uint8_t * row, uint32_t K, const int8_t * q, const float * d, const int16_t * bs,
                       int32_t * isum);

// ---- MUL_MAT kind composite (sw/ctrl/ref/mulmat_ref.hpp:8-13, tsr_sim.c:1639-1670) ------------
// y[t][n] = epilogue(dot(W row n, QACT(x_t))). flags: TSRO_MM_ADD -> fadd(add[t*add_stride + n], dot)
// (add_stride 0 repeats row 0); TSRO_MM_SCALE -> fmul(v, s1); TSRO_MM_SOFTCAP -> fmul(tanh(fmul(v, s0)), s1).
// w: N rows of ggml blocks, row-major. Rows are split over `threads` host threads (results are
// identical for any thread count). Returns 0, or -1 for bad arguments.
#define TSRO_MM_ADD     0x1u
#define TSRO_MM_SCALE   0x2u
#define TSRO_MM_SOFTCAP 0x4u
int      tsro_matvec(uint32_t fmt, const uint8_t * w, uint32_t N, uint32_t K, const float * x, uint32_t T,
                     const float * add, uint32_t add_stride, uint32_t flags, float s0, float s1, float * y,
                     int threads);

// ---- Flash attention over a q8_0 KV cache (tsr_ref_at.c, tsro_fa.c) ---------------------------
// The composite of tsr_ref_at.c:774-860 (AT §6.6) with the chunk planner of tsr_fa_plan.h, on a
// ggml-layout cache: K and V are [kv_size][E/32] block_q8_0 (E = n_head_kv * D); cell j of the
// op's view is row j. q: [T][n_head][D] f32; out: the same. mask: F16 [T][mask_stride] or NULL
// (then every row sees cells [0, n_kv)). C / t_max / pcap: the device parameters the chunk plan
// depends on (the U200 image: 4, 4 (T_MAX of the FA kind), 9344). Returns 0 or a TSRO_FA_E_* code.
#define TSRO_FA_OK      0
#define TSRO_FA_E_SHAPE 1
#define TSRO_FA_E_MASK  2
#define TSRO_FA_E_NOMEM 3
#define TSRO_FA_E_MSUM  4
typedef struct tsro_fa_params {
    uint32_t C, t_max, pcap;
    uint32_t T, D, n_head, n_head_kv, n_kv;
    float    scale;
    uint32_t new_lo, new_hi;   // cells written in this launch (their chunks run last); lo == hi: none
} tsro_fa_params;
int      tsro_fa(const tsro_fa_params * p, const float * q, const uint8_t * k_rows, const uint8_t * v_rows,
                 const uint16_t * mask, size_t mask_stride, float * out);
// The exact int32 QK block sums of ATTQK (AT §6.2): isum[h][j][b] = sum_i qK[j][h/G*D + 32b + i] *
// qQ[h*D + 32b + i] for token 0 (decode), heads h < n_head, cells j < n_kv, blocks b < D/32.
void     tsro_fa_qk_isums(const tsro_fa_params * p, const float * q, const uint8_t * k_rows, int32_t * isum);

// ---- Synthetic data (seeded, independent of the GPU) ------------------------------------------
// ggml Q4_K blocks of one f32 row (K % 256 == 0) with the sub-block min/scale encoder of
// the reference's test models (sw/ggml-tesseract/tests/gen_tiny_models.py:91-130).
void     tsro_quantize_q4_K(const float * x, uint32_t K, uint8_t * blocks);
// ggml Q8_0 blocks of one f32 row (K % 32 == 0): {fp16(d), q} from QACT A32 (the identity
// tsr_ref.h:122-127 states with quantize_row_q8_0_ref).
void     tsro_quantize_q8_0(const float * x, uint32_t K, uint8_t * blocks);

#ifdef __cplusplus
}
#endif
