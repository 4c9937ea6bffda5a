// tsrc.h -- C ABI of the B200 (sm_100a) hot path of the Tesseract stack: Q8_0 / Q4_K matrix-vector
// products (MUL_MAT) and flash attention over a q8_0 KV cache (FLASH_ATTN_EXT, SET_ROWS).
//
// This is the seam a ggml backend adapter (the rewrite of jwkim04/tesseract-npu
// sw/ggml-tesseract/ggml-tesseract.cpp) calls in place of the reference's op-list lowering,
// transport and firmware: the adapter keeps the ggml backend interface llama.cpp reaches through
// -ngl (registration, buffer types, supports_op, graph_compute) and calls these functions from
// set_tensor / graph_compute. Plain C types only: pointers, sizes and an opaque CUDA stream
// (cudaStream_t passed as void *; NULL = the legacy default stream).
//
// Numerics: every result is the reference's bit for bit (the spec's f32 rules: DAZ inputs, RNE,
// flush of subnormal results, canonical NaN 0x7FC00000; QACT A32 / A256; the 16-partial row dot of
// sw/sim/tsr_ref.c:592-635), for any input bytes.
//
// Errors: every function returns TSRC_OK (0) or a negative TSRC_E_* code and then sets a message
// that tsrc_last_error() returns (per thread). Nothing aborts and no C++ exception crosses the ABI.
// Kernels are queued on the given stream; functions that take host buffers synchronise as noted.
// Threading: a context may be used from one thread at a time (the reference serialises every call
// with one device mutex, ggml-tesseract.cpp:3932).
#pragma once

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define TSRC_API __attribute__((visibility("default")))
#else
#define TSRC_API
#endif

#define TSRC_OK             0
#define TSRC_E_ARG         (-1)   // a NULL handle / pointer, or a value out of range
#define TSRC_E_SHAPE       (-2)   // a shape the path does not support (the supports_op refusals)
#define TSRC_E_CUDA        (-3)   // a CUDA runtime error (message carries cudaGetErrorString)
#define TSRC_E_NOMEM       (-4)   // device or host allocation failed
#define TSRC_E_NODEV       (-5)   // no usable sm_100 device
#define TSRC_E_DEVICE      (-6)   // a kernel reported an error (a bounded wait ran out)

#define TSRC_FMT_Q8_0  0u         // ggml block_q8_0: {fp16 d; int8 qs[32]}, 34 B per 32 weights
#define TSRC_FMT_Q4_K  1u         // ggml block_q4_K: {fp16 d, dmin; u8 scales[12]; u8 qs[128]}, 144 B per 256

#define TSRC_QA_A32    0u         // QACT kind of Q8_0 (block 32, round half away, d = fp16(amax/127))
#define TSRC_QA_A256   1u         // QACT kind of Q4_K (block 256, round half even, int16 sums of 16)

// tsrc_mul_mat flags (the MVM epilogues, sw/sim/tsr_sim.c:1648-1670; MUL_MAT + ADD fusion,
// ggml-tesseract.cpp:2897-2914)
#define TSRC_MM_ADD     0x1u      // y = fadd(add[t * add_stride + n], dot)
#define TSRC_MM_SCALE   0x2u      // y = fmul(dot, s1)
#define TSRC_MM_SOFTCAP 0x4u      // y = fmul(tanh(fmul(dot, s0)), s1)

typedef struct tsrc_ctx tsrc_ctx;
typedef struct tsrc_weight tsrc_weight;
typedef struct tsrc_team tsrc_team;

// Last error message of the calling thread ("" if none). Replaces the reference's GGML_ABORT text
// (ggml-tesseract.cpp:2260-2271) as a returned status.
TSRC_API const char * tsrc_last_error(void);

// Library version string ("tsrc <major>.<minor> sm_100a").
TSRC_API const char * tsrc_version(void);

// Opens CUDA device `device` (must be sm_100). Replaces tsr_dev_open_locked (ggml-tesseract.cpp:463)
// and the backend init (tsr_dev_init_backend, :4079).
TSRC_API int tsrc_open(int device, tsrc_ctx ** out);
// Releases the context and every weight still attached to it (tsr_backend_free, :3799).
TSRC_API int tsrc_close(tsrc_ctx * ctx);
// Waits for the work queued on `stream` (NULL: the whole device) and reports a kernel-side error
// (TSRC_E_DEVICE: a bounded wait inside a kernel ran out; the flag is cleared). The reference's
// transport had launch timeouts for the same purpose (sw/transport/tsr_kdev.cpp:1452-1531).
TSRC_API int tsrc_sync(tsrc_ctx * ctx, void * stream);

// ---- weights (the WEIGHTS buffer's set_tensor / get_tensor, ggml-tesseract.cpp:1905, :1947) -----

// Uploads rows [row0, row0 + n_rows) of an N x K ggml weight (rows packed: K/32*34 or K/256*144
// bytes each, host memory at ggml_rows, which holds exactly those rows) and repacks them on the
// device into this library's layout. row0 / n_rows give a row shard for tensor parallelism (the
// reference's symmetric row split, sw/sim/tsr_ref.c:335-357); pass 0 / N for the whole tensor.
// Synchronous. Replaces tsr_store_weight_rows / tsr_repack_row (ggml-tesseract.cpp:852,
// sw/sim/tsr_ref.c:296-314).
TSRC_API int tsrc_weight_upload(tsrc_ctx * ctx, uint32_t fmt, const void * ggml_rows, uint32_t N, uint32_t K,
                       uint32_t row0, uint32_t n_rows, tsrc_weight ** out);
// The same from ggml rows already in device memory (e.g. a staging buffer); runs on `stream` and
// returns when the weight is in place.
TSRC_API int tsrc_weight_upload_device(tsrc_ctx * ctx, uint32_t fmt, const void * ggml_rows_dev, uint32_t N, uint32_t K,
                              uint32_t row0, uint32_t n_rows, void * stream, tsrc_weight ** out);
// Seeded synthetic weight generated on the device (counter-based Philox4x32-10 normal values of
// standard deviation sigma, quantized to fmt on the device); rows [row0, row0+n_rows) of an N x K
// tensor, identical to the same rows of an unsharded generation. For benches and tests. Runs on
// `stream` and returns when the weight is in place.
TSRC_API int tsrc_weight_synth(tsrc_ctx * ctx, uint32_t fmt, uint32_t N, uint32_t K, uint32_t row0, uint32_t n_rows,
                      uint64_t seed, float sigma, void * stream, tsrc_weight ** out);
// ggml tensor types at load time (tsr_dev_fmt_for_type / tsr_type_loadable / tsr_row_to_dev_blocks,
// sw/ggml-tesseract/tsr-weights.h:14-30). ggml_type is ggml.h's enum value. Q8_0 (8) and Q4_K (12)
// load as shipped; F32 (0), F16 (1), BF16 (30), Q4_0 (2), Q4_1 (3), Q5_0 (6), Q5_1 (7), Q5_K (13)
// and Q6_K (14) are converted to Q8_0 on the host: ggml's to_float of the type, then
// quantize_row_q8_0_ref. Other types are refused with TSRC_E_SHAPE.
// Block geometry of a type and the device format it loads as (TSRC_FMT_*).
TSRC_API int tsrc_ggml_type_info(uint32_t ggml_type, uint32_t * block_elems, uint32_t * block_bytes, uint32_t * dev_fmt);
// Host-only: n_rows rows of K values of ggml_type (ggml layout, packed) -> rows of the device format's
// ggml blocks at dst (K / 32 * 34 bytes a row for Q8_0, K / 256 * 144 for Q4_K; native types are
// copied). Large tensors are converted on several host threads.
TSRC_API int tsrc_ggml_rows_to_dev(uint32_t ggml_type, const void * src, uint32_t n_rows, uint32_t K, void * dst);
// tsrc_weight_upload for rows of any loadable ggml type (converted on the host first when the type is
// not native). Synchronous.
TSRC_API int tsrc_weight_upload_ggml(tsrc_ctx * ctx, uint32_t ggml_type, const void * ggml_rows, uint32_t N, uint32_t K,
                                     uint32_t row0, uint32_t n_rows, tsrc_weight ** out);
// Reads the shard back as ggml rows (n_rows rows) into host memory (get_tensor; the inverse repack,
// tsr_unrepack_row, sw/sim/tsr_ref.c:316-333). Synchronous.
TSRC_API int tsrc_weight_download(const tsrc_weight * w, void * ggml_rows);
// fmt, N, K, row0, n_rows and the device bytes the shard occupies (any pointer may be NULL).
TSRC_API int tsrc_weight_info(const tsrc_weight * w, uint32_t * fmt, uint32_t * N, uint32_t * K, uint32_t * row0,
                     uint32_t * n_rows, uint64_t * device_bytes);
TSRC_API int tsrc_weight_free(tsrc_weight * w);

// ---- MUL_MAT (tsr_lower_mul_mat, ggml-tesseract.cpp:2790-2928; kind_mulmat, sw/ctrl/kernels/k_mulmat.cpp) ----

// For t < T: y[t * y_stride + n] = epilogue(dot(W row n, QACT(x[t * x_stride .. + K]))) for the
// shard's rows n < n_rows (y row t holds the shard's outputs only). Strides are in floats (0 =
// dense: K for x, n_rows for y, n_rows for add, or 0 = row 0 for every token when add_stride is
// 0). x, y, add are device pointers; y must not overlap x or add. s0 / s1: TSRC_MM_SOFTCAP /
// TSRC_MM_SCALE factors. ADD cannot be combined with SCALE or SOFTCAP (the reference refuses it,
// tsr_sim.c chk_mvm). Queued on `stream`; no host synchronisation.
TSRC_API int tsrc_mul_mat(tsrc_ctx * ctx, const tsrc_weight * w, const float * x, uint32_t T, uint32_t x_stride, float * y,
                 uint32_t y_stride, const float * add, uint32_t add_stride, uint32_t flags, float s0, float s1,
                 void * stream);

// The MVM tile op alone (ex_mvm, sw/sim/tsr_sim.c:1623-1671): tsrc_mul_mat on activations already
// quantized by tsrc_qact (q [T][K], d [T][K/bs], bs [T][K/16] for Q4_K, dense), same epilogues
// and strides. T <= 8 per call. Device pointers, queued on `stream`.
TSRC_API int tsrc_mvm(tsrc_ctx * ctx, const tsrc_weight * w, const int8_t * q, const float * d, const int16_t * bs,
                      uint32_t T, float * y, uint32_t y_stride, const float * add, uint32_t add_stride, uint32_t flags,
                      float s0, float s1, void * stream);

// tsrc_mul_mat for callers that cannot allocate device memory (no counterpart in the reference,
// whose device memory is planned by the backend). Same arguments, results and errors as
// tsrc_mul_mat, but the quantized activations live in a fixed 1 MiB array compiled into this
// library (present on every device that loads it until the process exits) instead of a scratch
// buffer the context allocates: the call itself allocates nothing. The image of one token of K
// values takes about 1.2 K bytes, so K up to 65536 works for any T (tokens are processed at most
// 8 at a time); a larger image is refused with TSRC_E_SHAPE. The first call on a device looks up
// the array's device address (cudaGetSymbolAddress): make it before any stream capture. All calls
// share the array: calls that may run at the same time on one device (other streams, other
// contexts) race and must be serialised by the caller; calls queued on one stream are ordered.
// Device memory and copies for hosts that do not link the CUDA runtime themselves (the C++ runtime
// front end, include/tsrc_rt.hpp): a buffer on the context's device; an asynchronous copy between host
// and device memory on `stream` (to_device 1: host -> device, 0: device -> host; tsrc_sync waits).
TSRC_API int tsrc_dev_alloc(tsrc_ctx * ctx, size_t bytes, void ** out);
TSRC_API int tsrc_dev_free(tsrc_ctx * ctx, void * p);
TSRC_API int tsrc_copy(tsrc_ctx * ctx, void * dst, const void * src, size_t bytes, uint32_t to_device, void * stream);

// MUL_MAT_ID (ggml's expert-routed product, the reference's MUL_MAT_ID kind: tsr_lower_mul_mat_id_node,
// sw/ggml-tesseract/ggml-tesseract.cpp:3317-3350): w holds n_exp experts of N / n_exp rows each, stacked
// (upload ggml's 3D expert tensor [n_exp][N/n_exp][K] as N rows). For token t < T and slot j < n_used,
// with e = ids[t * ids_stride + j] (device int32, written by the router before the call):
//   y[t * y_tok_stride + j * y_slot_stride + n] = MUL_MAT of expert e's row n with
//   x[t * x_tok_stride + (j mod x_slots) * x_slot_stride ..]   (x_slots 1: one activation row per token
//   shared by its slots, or n_used: one per slot)
// -- each (t, j) exactly as a one-token tsrc_mul_mat of that expert (same bits). Strides in floats / ints,
// 0 = dense. An id outside [0, n_exp) leaves its outputs unwritten; tsrc_sync then returns TSRC_E_ARG.
// At most 65535 (token, slot) pairs per call. Queued on `stream`.
TSRC_API int tsrc_mul_mat_id(tsrc_ctx * ctx, const tsrc_weight * w, uint32_t n_exp, const float * x, uint32_t x_slots,
                             uint32_t x_slot_stride, uint32_t x_tok_stride, const int32_t * ids, uint32_t ids_stride,
                             uint32_t n_used, uint32_t T, float * y, uint32_t y_slot_stride, uint32_t y_tok_stride, void * stream);
TSRC_API int tsrc_mul_mat_noalloc(tsrc_ctx * ctx, const tsrc_weight * w, const float * x, uint32_t T, uint32_t x_stride,
                                  float * y, uint32_t y_stride, const float * add, uint32_t add_stride, uint32_t flags,
                                  float s0, float s1, void * stream);

// Why a MUL_MAT of this weight shape could not run here (NULL if it can): the B200 counterpart of
// the MUL_MAT branch of supports_op (ggml-tesseract.cpp:4199-4299).
TSRC_API const char * tsrc_mul_mat_unsupported(uint32_t fmt, uint64_t N, uint64_t K, uint64_t T);

// ---- test hooks (the reference exposes the same through get_proc_address, ggml-tesseract.cpp:4409-4431) ----

// QACT alone (tsr_qact, sw/sim/tsr_ref.c:456-518): T vectors of K floats (x_stride floats apart, 0
// = K) -> q [T][K] int8, d [T][K/bs] f32, bs [T][K/16] int16 (A256 only; NULL for A32). Device
// pointers, queued on `stream`.
TSRC_API int tsrc_qact(tsrc_ctx * ctx, uint32_t kind, const float * x, uint32_t K, uint32_t T, uint32_t x_stride,
              int8_t * q, float * d, int16_t * bs, void * stream);
// MUL_MAT of one token (x: K device floats -> y: n_rows floats) that also writes the kernel's own
// exact int32 block sums: Q8_0 isum[n][K/32]; Q4_K isum[n][K/256][2] = {sum sc_j*S_j,
// sum m_j*(BS_2j + BS_2j+1)} (the integer parts of sw/sim/tsr_ref.c:533-567), so that a test can
// check them bit for bit. Device pointers, queued on `stream`.
TSRC_API int tsrc_mul_mat_isums(tsrc_ctx * ctx, const tsrc_weight * w, const float * x, float * y, int32_t * isum,
                       void * stream);
// Connects a team with other teams of the same process and GPU (members[r] = rank r's team, this
// one included) instead of IPC handles: for tests of the team's exchange on one GPU (only
// one rank's launches may run there: ranks wait for each other, and two of them on one GPU are
// not guaranteed to run at the same time).
TSRC_API int tsrc_team_connect_local(tsrc_team * team, const tsrc_team * const * members);

// ---- tensor parallelism: MUL_MAT with the all-gather fused in (no counterpart in the reference,
// whose channels live on one card) ------------------------------------------------------------------
// A team is one rank's side of a group of `world` GPUs of one box (one process per GPU). Each rank
// creates its buffer (writing a TSRC_TEAM_HANDLE_BYTES CUDA IPC handle), the ranks exchange the
// handles (e.g. an all-gather over torch.distributed), and each rank connects with all of them
// (world x TSRC_TEAM_HANDLE_BYTES bytes in rank order).
#define TSRC_TEAM_HANDLE_BYTES 64
TSRC_API int tsrc_team_create(tsrc_ctx * ctx, uint32_t rank, uint32_t world, uint32_t n_max, void * handle_out,
                              tsrc_team ** out);
TSRC_API int tsrc_team_connect(tsrc_team * team, const void * handles);
TSRC_API int tsrc_team_free(tsrc_team * team);
// MUL_MAT of one token over this rank's row shard of an N-row weight (N <= n_max) whose rows go
// to every rank: y (device, N floats) receives the whole vector on every rank, bit for bit the
// single-GPU result. The shard's rows are stored into every rank's buffer by the matvec kernel
// itself (P2P stores over NVLink, each value with its step's tag in one 64-bit word); every CTA
// copies its share of the vector out once the share's words carry the step's tag (a bounded wait:
// a rank that does not take part makes tsrc_sync return TSRC_E_DEVICE). Every rank must make the same sequence of calls; queued on `stream`, no host sync. (The
// reference's row split: sw/sim/tsr_ref.c:335-357; its host then had all rows in one memory.)
TSRC_API int tsrc_mul_mat_allgather(tsrc_ctx * ctx, tsrc_team * team, const tsrc_weight * w, const float * x, float * y,
                                    void * stream);

// ---- q8_0 KV cache (one layer) -------------------------------------------------------------------
// A cache holds n_cells cells of E = n_head_kv * head_dim values for K and for V, each value stored
// as ggml's q8_0 holds it ({fp16 d; int8 qs[32]} per 32 values); the device layout is the
// library's own. Replaces the reference's KV plane buffer (ggml-tesseract tsr-kvbuf, plane layout
// sw/sim/tsr_ref_at.c:91-212) behind the ggml KV tensors.
typedef struct tsrc_kv tsrc_kv;

#define TSRC_KV_K 0u
#define TSRC_KV_V 1u

// Allocates a zeroed cache (head_dim 64, 128, 256 or 512; E / 64 <= 511).
TSRC_API int tsrc_kv_create(tsrc_ctx * ctx, uint32_t n_head_kv, uint32_t head_dim, uint32_t n_cells, tsrc_kv ** out);
// Synchronises the device, then frees the cache.
TSRC_API int tsrc_kv_free(tsrc_kv * kv);
// SET_ROWS into a q8_0 cache / the KVST op (sw/sim/tsr_ref_at.c:244-264): n f32 rows of E values
// (device memory, row_stride floats apart, 0 = E) quantized with QACT A32 and stored at cells
// cells[i] (device int64, ggml's row-index tensor) or, with cells = NULL, at cell0 + i. Queued on
// `stream`. A device-side cell index outside the cache is not stored and makes the next tsrc_sync
// return TSRC_E_ARG.
TSRC_API int tsrc_kv_set_rows(tsrc_ctx * ctx, tsrc_kv * kv, uint32_t which, const float * rows, uint32_t n,
                              uint32_t row_stride, const int64_t * cells, uint32_t cell0, void * stream);
// The ggml q8_0 image of cells [cell0, cell0 + n): host rows of E/32 blocks of 34 bytes (the
// backend's set_tensor / get_tensor of a KV tensor, ggml-tesseract.cpp:1905-1947). Synchronous.
TSRC_API int tsrc_kv_set_bytes(tsrc_kv * kv, uint32_t which, const void * ggml_rows, uint32_t cell0, uint32_t n);
TSRC_API int tsrc_kv_get_bytes(const tsrc_kv * kv, uint32_t which, void * ggml_rows, uint32_t cell0, uint32_t n);

// ---- flash attention over the cache (FLASH_ATTN_EXT) ---------------------------------------------
// The attention configuration the reference's output depends on (tsr_att_cfg, sw/sim/include/
// tsr_ref_at.h:262-267): channels C (1..16), T_MAX (1..8), PCAP, K_MAX (0 = not checked). NULL
// selects the release image's {4, 4, 9344, 32768, 0}. plan_n_head_kv: the model's KV heads when
// the cache holds only a shard of them (tensor parallelism by KV heads): the chunk plan and the
// shape checks depend on E = n_head_kv * head_dim of the whole model, so every shard plans as the
// single device does and the shards' outputs are the single-device output bit for bit; 0 = the
// cache's own n_head_kv.
typedef struct tsrc_fa_cfg {
    uint32_t C, t_max, pcap, k_max;
    uint32_t plan_n_head_kv;
} tsrc_fa_cfg;

// out[t][h][:] = softmax(scale * q[t][h] . K[:, h / G]^T + mask[t]) V[:, h / G] over cells [0, n_kv),
// computed as the reference's composite FA (tsr_ref_fa, sw/sim/tsr_ref_at.c:774-860) bit for bit:
// QACT A32 of q, chunks of 16-cell groups from the chunk planner, exact block sums, EXPK, block
// floating point P.V, the channel tree and the online merge. q and out: device f32 [T][n_head]
// [head_dim]. mask: HOST f16 [T][mask_stride] (0 / -0 visible, -inf hidden, other values added
// after division by scale -- the GENERAL path), as the backend sees it in set_tensor; NULL makes
// cells [0, n_kv) visible to every token. Cells [new_lo, new_hi) were written by this step: chunks
// holding them run last (lo == hi: none). Queued on `stream` (the plan and, for a GENERAL mask,
// the mask are copied to the device first). Replaces tsr_lower_fa (sw/ggml-tesseract/
// tsr-build.cpp:673-773) and the FLASH_ATTN kind (sw/ctrl/kernels/k_fattn.cpp).
TSRC_API int tsrc_flash_attn(tsrc_ctx * ctx, const tsrc_kv * kv, const float * q, uint32_t T, uint32_t n_head,
                             uint32_t n_kv, const uint16_t * mask, uint32_t mask_stride, float scale,
                             uint32_t new_lo, uint32_t new_hi, const tsrc_fa_cfg * cfg, float * out, void * stream);

// ---- the decoder layer's vector kinds (VU ops of the reference's kinds) ----------------------------
// Every f32 result follows the reference's vector-unit rules (DAZ inputs, RNE, FTZ results,
// canonical NaN; sw/sim/include/tsr_ref_vu.h). Operands are device f32 rows of n values at the
// given strides (in floats; 0 = n); y may be x (in place). Queued on `stream`.

// RMS_NORM + MUL (the RMS_NORM kind, sw/ctrl/ref/rmsnorm_ref.hpp:44; op list kind 0x14):
// y[r][j] = FM(FM(x[r][j], s_r), w[j]) with s_r = RC(SQ(FA(FM(tree128(sum sq), inv_n), eps))),
// the 128-partial pairwise tree of RED.SUMSQ (tsr_ref_vu.c:171-263). w = NULL: no weight MUL.
// inv_n is 1/n as the backend computes it (tsr-build.cpp:405).
TSRC_API int tsrc_rms_norm(tsrc_ctx * ctx, const float * x, uint32_t x_stride, float * y, uint32_t y_stride,
                           const float * w, uint32_t n, uint32_t rows, float eps, float inv_n, void * stream);
// RMS_NORM + MUL of one token followed by its MUL_MAT, in one launch: y = MUL_MAT(W, RMS_NORM(x) * w)
// with the values of tsrc_rms_norm (n = K) then tsrc_mul_mat (T = 1), bit for bit. No single
// counterpart in the reference, whose graph runs the RMS_NORM kind and then the MUL_MAT kind
// (ggml-tesseract tsr-build.cpp:405, ggml-tesseract.cpp:2790-2928); the normalised row never
// goes through device memory. add / flags / s0 / s1 as tsrc_mul_mat; device pointers, on `stream`.
TSRC_API int tsrc_mul_mat_rms(tsrc_ctx * ctx, const tsrc_weight * wt, const float * x, const float * norm_w, float eps,
                              float inv_n, float * y, const float * add, uint32_t flags, float s0, float s1, void * stream);

#define TSRC_ROPE_NORM 0u          // adjacent pairs (2i, 2i + 1)  (TSR_ROPE_MODE_NORM)
#define TSRC_ROPE_NEOX 1u          // half-split pairs (i, i + n_dims / 2)
// ROPE (the ROPE kind, sw/ctrl/ref/rope_ref.hpp:29; tsr_ref_rope, tsr_ref_vu.c:308-376), recurrence
// form: T tokens of n_heads heads of head_dim values; token t at position pos[t] (device int32);
// theta_0 = f32(pos), theta_(i+1) = FM(theta_i, ts) with ts = powf(freq_base, -2 / n_dims) as the
// backend computes it (tsr-build.cpp:547); c_i = FM(attn_factor, COS), s_i = FM(attn_factor, SIN).
TSRC_API int tsrc_rope(tsrc_ctx * ctx, const float * x, uint32_t x_stride, float * y, uint32_t y_stride,
                       const int32_t * pos, uint32_t T, uint32_t n_heads, uint32_t head_dim, uint32_t n_dims,
                       uint32_t mode, float ts, float attn_factor, void * stream);

#define TSRC_VOP_ADD    0u         // FA(a, b)          (TSR_VOP_FUNC_ADD)
#define TSRC_VOP_MUL    2u         // FM(a, b)
#define TSRC_VOP_SILU   6u         // FM(a, SIG(a)), SIG(a) = RC(FA(1, EXPK(a, -1)))
#define TSRC_VOP_SWIGLU 7u         // FM(SILU(a), b)    (ggml's swiglu: silu(gate) * up)
// Elementwise VOP over rows x n (tsr_ref_vop, tsr_ref_vu.c:104-160); b is not read by SILU.
TSRC_API int tsrc_vop(tsrc_ctx * ctx, uint32_t func, const float * a, uint32_t a_stride, const float * b,
                      uint32_t b_stride, float * y, uint32_t y_stride, uint32_t n, uint32_t rows, void * stream);

// GET_ROWS of a quantized weight (the token embedding; DQROW, tsr_dequant_row, sw/sim/tsr_ref.c:
// 369-401): y[t][:] = the f32 values of row ids[t] (device int32; rows of the weight's shard).
// An id outside the shard is not written and makes the next tsrc_sync return TSRC_E_ARG.
TSRC_API int tsrc_get_rows(tsrc_ctx * ctx, const tsrc_weight * w, const int32_t * ids, uint32_t T, float * y,
                           uint32_t y_stride, void * stream);

// ---- an end-to-end decoder model through the kinds above (llama.cpp's llama / qwen2 graphs) --------
// A random-init model of the given shape, every matrix quantized to fmt, run layer by layer through
// GET_ROWS, RMS_NORM + MUL, MUL_MAT (+ bias), ROPE, SET_ROWS into a per-layer q8_0 KV cache,
// FLASH_ATTN_EXT, MUL_MAT + residual, SWIGLU, MUL_MAT + residual, the output norm and head. It is
// the device-side counterpart of llama.cpp with -ngl all on the reference backend (the model's
// graph_compute of every node, ggml-tesseract.cpp:3929-3966), for the decode tokens/s measurement.
typedef struct tsrc_model tsrc_model;
typedef struct tsrc_model_cfg {
    uint32_t n_layer, n_embd, n_ff, n_head, n_head_kv, head_dim, n_vocab;
    uint32_t fmt;            // TSRC_FMT_Q8_0 or TSRC_FMT_Q4_K for every matrix (K multiples of 256 for Q4_K)
    uint32_t rope_mode;      // TSRC_ROPE_NORM (llama) or TSRC_ROPE_NEOX (qwen2); n_dims = head_dim
    float rope_base;         // freq_base; ts = powf(freq_base, -2 / head_dim) on the host
    float rms_eps;
    uint32_t qkv_bias;       // f32 biases on q, k, v (qwen2)
    uint32_t tied_head;      // the head is the token embedding (qwen2.5-0.5B)
    uint32_t n_ctx;          // KV cells per layer
    tsrc_fa_cfg fa;          // C = 0: the release image's {4, 4, 9344, 32768, 0}
} tsrc_model_cfg;
#define TSRC_MODEL_GLOBAL 0xFFFFFFFFu   // tsrc_model_weight layer: which 0 = token embedding, 1 = head

// Weights from tsrc_weight_synth(seed * 1000 + 1 / + 2 for the embedding / head; seed * 1000 +
// 16 (l + 1) + i for layer l's i = 0 [q | k | v] rows, 1 o, 2 [gate | up] rows, 3 down; sigma 0.02);
// f32 vectors from tsrc_model_f32_value.
TSRC_API int tsrc_model_create(tsrc_ctx * ctx, const tsrc_model_cfg * cfg, uint64_t seed, tsrc_model ** out);
// The same model split over a connected team (no counterpart in the reference, whose channels live
// on one card): this rank holds the q heads and KV heads [rank, rank + 1) x (heads / world) (n_head_kv
// must split evenly) with their q / k / v rows and cache, and the symmetric row shards (R = ceil(N /
// world), sw/sim/tsr_ref.c:335-357) of o, gate / up (of n_ff), down and the head; every exchange is
// the team's tagged-word gather (the attention output and the SWIGLU row, then o, down and the head
// fused with their gathers). tsrc_model_decode runs one token; tsrc_model_forward any T (a prompt:
// tensor-core MUL_MATs of the rank's rows, then gathers of T rows, as many rows per team step as
// n_max holds): logits (all n_vocab) on every rank equal the single-GPU model's. The team's n_max
// must hold max(n_vocab, n_ff, n_head * head_dim, n_embd); a multiple of it speeds prompts up.
TSRC_API int tsrc_model_create_tp(tsrc_ctx * ctx, const tsrc_model_cfg * cfg, uint64_t seed, tsrc_team * team,
                                  tsrc_model ** out);
TSRC_API int tsrc_model_free(tsrc_model * m);
// Layer `layer`'s q8_0 KV cache (owned by the model; a tensor-parallel rank's holds its KV heads),
// e.g. to load cells written elsewhere with tsrc_kv_set_rows / tsrc_kv_set_bytes.
TSRC_API int tsrc_model_kv(const tsrc_model * m, uint32_t layer, tsrc_kv ** out);
// Runs tokens ids[0..T) (device int32) at positions pos0 .. pos0 + T - 1: their K / V rows are stored
// at cells pos0 .. and attention is causal over cells [0, pos0 + t]. logits (device f32 [n_vocab])
// receives the head output of the last token. Queued on `stream`.
TSRC_API int tsrc_model_forward(tsrc_model * m, const int32_t * ids, uint32_t T, uint32_t pos0, float * logits,
                                void * stream);
// One decode token (T = 1) through a CUDA graph of the whole step: the first call (and any call
// whose ids / logits pointers, stream or FA plan shape differ from the captured ones) captures the
// step; later calls rewrite the position and the FA plans in the instantiated graph and launch it,
// so a token costs one graph launch on the host. Same results as tsrc_model_forward(m, ids, 1, ...).
TSRC_API int tsrc_model_decode(tsrc_model * m, const int32_t * ids, uint32_t pos0, float * logits, void * stream);
// The model's weight handles (owned by the model): layer < n_layer, which 0 = the q, k, v rows
// stacked (n_head + 2 n_head_kv heads), 1 = o, 2 = the gate and up rows interleaved (row 2j gate_j,
// 2j + 1 up_j; 2 n_ff rows: the MUL_MAT applies SWIGLU to the pairs as its epilogue), 3 = down;
// or TSRC_MODEL_GLOBAL.
TSRC_API int tsrc_model_weight(const tsrc_model * m, uint32_t layer, uint32_t which, tsrc_weight ** out);
// Replaces a weight of a single-device model with rows of a loadable ggml type (host memory; the
// load of a GGUF model's tensors, llama.cpp's set_tensor of each weight). layer / which as
// tsrc_model_weight; N x K must be the weight's shape. which 0 takes the q, k, v rows stacked (q rows,
// then k, then v); which 2 the gate rows then the up rows (the model interleaves them); the head
// (TSRC_MODEL_GLOBAL, 1) exists only without a tied head. The next decode token captures a new graph.
TSRC_API int tsrc_model_set_weight(tsrc_model * m, uint32_t layer, uint32_t which, uint32_t ggml_type, const void * rows,
                                   uint32_t N, uint32_t K);
// Replaces an f32 vector of a single-device model (host memory, n values): which 0 attn_norm, 1
// ffn_norm (n_embd), 2 the q | k | v bias (n_head + 2 n_head_kv heads; models with qkv_bias), 5 the
// output norm (layer = n_layer), as tsrc_model_f32_value numbers them.
TSRC_API int tsrc_model_set_f32(tsrc_model * m, uint32_t layer, uint32_t which, const float * values, uint32_t n);
// The host-computed ROPE theta scale and attention scale the model passes to the kinds.
TSRC_API int tsrc_model_params(const tsrc_model * m, float * ts, float * kq_scale);
// f32 vector element i of the model: which 0 attn_norm, 1 ffn_norm, 2 the q | k | v bias (layer l),
// 5 output norm (layer = n_layer): splitmix64 of (seed, layer, which, i) -> 1 + 0.25 u for the
// norms, 0.1 u for the biases, u uniform in [-1, 1) on 24 bits.
TSRC_API float tsrc_model_f32_value(uint64_t seed, uint32_t layer, uint32_t which, uint32_t i);

#ifdef __cplusplus
}
#endif
