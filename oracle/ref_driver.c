// ref_driver.c — batch drivers over the REFERENCE's own C library (TEST INFRASTRUCTURE ONLY).
//
// Compiled together with the reference's sw/sim/tsr_ref.c, tsr_ref_at.c and tsr_ref_math.c (where
// they lie, see Makefile `ref`) into oracle/_ref/libtsr_refdrv.so. It only sequences calls to the
// reference's public functions (tsr_ref.h, tsr_ref_at.h, tsr_ref_math.h) so that tests can pin the
// restatement (libtsro.so) and the bench can time the reference's CPU path:
//   - QACT: tsr_qact into the reference's QA image, split into q / d / bs arrays;
//   - MUL_MAT: tsr_repack_row once, then tsr_qact + tsr_dot_row per row on `threads` host threads
//     (the composite of sw/ctrl/ref/mulmat_ref.hpp:8-13 with the MVM epilogues of tsr_sim.c:1648-1670);
//   - FA: ggml q8_0 rows packed into KV planes (tsr_kv_pack_row), the mask summary
//     (tsr_msum_build_f16, tsr_msum_mask_f32), then tsr_ref_fa.
#include "tsr_ref.h"
#include "tsr_ref_at.h"
#include "tsr_ref_math.h"

#include <pthread.h>
#include <stdlib.h>
#include <string.h>

void refdrv_expk_n(const float * v, size_t n, unsigned kappa, float * out) {
    for (size_t i = 0; i < n; ++i) out[i] = tsr_m_expk(v[i], kappa);
}
void refdrv_tanh_n(const float * v, size_t n, float * out) {
    for (size_t i = 0; i < n; ++i) out[i] = tsr_m_tanh(v[i]);
}
void refdrv_fp_n(int op, const float * a, const float * b, size_t n, float * out) {
    for (size_t i = 0; i < n; ++i) {
        switch (op) {
        case 0: out[i] = tsr_fadd(a[i], b[i]); break;
        case 1: out[i] = tsr_fsub(a[i], b[i]); break;
        case 2: out[i] = tsr_fmul(a[i], b[i]); break;
        case 3: out[i] = tsr_fdiv(a[i], b[i]); break;
        default: out[i] = tsr_frecip(a[i]); break;
        }
    }
}
void refdrv_f32_to_fp16_n(const float * a, size_t n, uint16_t * out) {
    for (size_t i = 0; i < n; ++i) out[i] = tsr_f32_to_fp16(a[i]);
}

// QACT of one token into arrays: q[K], d[K/bs], bs[K/16] (A256 only; may be NULL for A32).
void refdrv_qact(uint32_t kind, const float * x, uint32_t K, int8_t * q, float * d, int16_t * bs) {
    uint8_t * qa = (uint8_t *)aligned_alloc(64, (size_t)tsr_qa_lines(kind, K) * 64u);
    tsr_qact(kind, x, K, qa);
    memcpy(q, tsr_qa_qs(kind, K, qa), K);
    memcpy(d, tsr_qa_d(kind, K, qa), (size_t)(K / tsr_qa_block_size(kind)) * sizeof(float));
    if (kind == TSR_QA_A256 && bs) memcpy(bs, tsr_qa_bs(kind, K, qa), (size_t)(K / 16u) * sizeof(int16_t));
    free(qa);
}

size_t refdrv_row_bytes(uint32_t fmt, uint32_t K) { return (size_t)tsr_row_beats(fmt, K) * TSR_BEAT_BYTES; }

// ggml blocks of N rows -> the reference's device row images (tsr_repack_row), row-major.
void refdrv_repack(uint32_t fmt, const uint8_t * ggml, uint32_t N, uint32_t K, uint8_t * dst) {
    const size_t gb = (size_t)(K / tsr_fmt_block_size(fmt)) * tsr_fmt_ggml_block_bytes(fmt);
    const size_t rb = refdrv_row_bytes(fmt, K);
    for (uint32_t n = 0; n < N; ++n) tsr_repack_row(fmt, ggml + (size_t)n * gb, K, dst + (size_t)n * rb);
}

typedef struct mm_job {
    uint32_t fmt, N, K, T, flags, add_stride;
    const uint8_t * rows;
    const uint8_t * qa;
    size_t qa_bytes;
    const float * add;
    float s0, s1;
    float * y;
    uint32_t lo, hi;
} mm_job;

static void * mm_rows(void * arg) {
    const mm_job * j = (const mm_job *)arg;
    const size_t rb = refdrv_row_bytes(j->fmt, j->K);
    for (uint32_t n = j->lo; n < j->hi; ++n) {
        for (uint32_t t = 0; t < j->T; ++t) {
            float v = tsr_dot_row(j->fmt, j->rows + (size_t)n * rb, j->K, j->qa + (size_t)t * j->qa_bytes);
            if (j->flags & 1u) v = tsr_fadd(j->add[(size_t)t * j->add_stride + n], v);
            if (j->flags & 4u) v = tsr_fmul(tsr_m_tanh(tsr_fmul(v, j->s0)), j->s1);
            else if (j->flags & 2u) v = tsr_fmul(v, j->s1);
            j->y[(size_t)t * j->N + n] = v;
        }
    }
    return NULL;
}

// y[t][n] for repacked rows (refdrv_repack); flags 1 ADD, 2 SCALE, 4 SOFTCAP as tsro_matvec.
int refdrv_matvec_repacked(uint32_t fmt, const uint8_t * rows, uint32_t N, uint32_t K, const float * x, uint32_t T,
                           const float * add, uint32_t add_stride, uint32_t flags, float s0, float s1, float * y,
                           int threads) {
    const uint32_t kind = tsr_qa_kind_for_fmt(fmt);
    const size_t qab = (size_t)tsr_qa_lines(kind, K) * 64u;
    uint8_t * qa = (uint8_t *)aligned_alloc(64, qab * T);
    if (!qa) return -1;
    for (uint32_t t = 0; t < T; ++t) tsr_qact(kind, x + (size_t)t * K, K, qa + (size_t)t * qab);
    if (threads < 1) threads = 1;
    if ((uint32_t)threads > N) threads = (int)N;
    mm_job * jobs = (mm_job *)calloc((size_t)threads, sizeof(mm_job));
    pthread_t * th = (pthread_t *)calloc((size_t)threads, sizeof(pthread_t));
    const uint32_t per = (N + (uint32_t)threads - 1u) / (uint32_t)threads;
    for (int i = 0; i < threads; ++i) {
        mm_job j = { fmt, N, K, T, flags, add_stride, rows, qa, qab, add, s0, s1, y, 0, 0 };
        j.lo = (uint32_t)i * per < N ? (uint32_t)i * per : N;
        j.hi = j.lo + per < N ? j.lo + per : N;
        jobs[i] = j;
        if (i > 0) pthread_create(&th[i], NULL, mm_rows, &jobs[i]);
    }
    mm_rows(&jobs[0]);
    for (int i = 1; i < threads; ++i) pthread_join(th[i], NULL);
    free(jobs); free(th); free(qa);
    return 0;
}

// ---------------------------------------------------------------------------------------------
// Flash attention through tsr_ref_fa
// ---------------------------------------------------------------------------------------------
typedef struct refdrv_fa {
    tsr_att_cfg cfg;
    tsr_kv_geom geom;
    uint8_t * kpl[16];
    uint8_t * vpl[16];
    uint32_t * msum_words;
    tsr_msum msum;
    float * mask_f32;
    uint32_t T, D, G, n_kv, new_run[1][2], n_new;
    float scale;
} refdrv_fa;

void refdrv_fa_free(refdrv_fa * f) {
    if (!f) return;
    for (int c = 0; c < 16; ++c) { free(f->kpl[c]); free(f->vpl[c]); }
    free(f->msum_words);
    free(f->mask_f32);
    free(f);
}

// Planes from ggml q8_0 rows [kv_size][E/32 blocks]; mask F16 [T][mask_stride] or NULL (all of
// [0, n_kv) visible). new_lo < new_hi names the cells written in this launch.
refdrv_fa * refdrv_fa_prepare(uint32_t C, uint32_t t_max, uint32_t pcap, uint32_t T, uint32_t D, uint32_t n_head,
                              uint32_t n_head_kv, uint32_t n_kv, uint32_t kv_size, float scale,
                              const uint8_t * k_rows, const uint8_t * v_rows, const uint16_t * mask,
                              size_t mask_stride, uint32_t new_lo, uint32_t new_hi) {
    refdrv_fa * f = (refdrv_fa *)calloc(1, sizeof *f);
    if (!f) return NULL;
    f->cfg = (tsr_att_cfg){ C, t_max, pcap, 32768u };
    const uint32_t E = n_head_kv * D;
    if (kv_size < n_kv) kv_size = n_kv;
    f->geom = (tsr_kv_geom){ E, C, tsr_kv_lg_min(kv_size ? kv_size : 1u, C) };
    const size_t pb = (size_t)tsr_kv_plane_beats(&f->geom) * TSR_BEAT_BYTES;
    for (uint32_t c = 0; c < C; ++c) {
        f->kpl[c] = (uint8_t *)calloc(pb, 1);
        f->vpl[c] = (uint8_t *)calloc(pb, 1);
    }
    const size_t rb = (size_t)(E / 32u) * 34u;
    for (uint32_t j = 0; j < kv_size; ++j) {
        tsr_kv_pack_row(TSR_KV_K, &f->geom, f->kpl, j, (const tsr_block_q8_0 *)(k_rows + (size_t)j * rb));
        tsr_kv_pack_row(TSR_KV_V, &f->geom, f->vpl, j, (const tsr_block_q8_0 *)(v_rows + (size_t)j * rb));
    }
    uint16_t * zero = NULL;
    if (!mask) {
        zero = (uint16_t *)calloc((size_t)T * (n_kv ? n_kv : 1u), sizeof(uint16_t));
        mask = zero;
        mask_stride = n_kv;
    }
    f->msum_words = (uint32_t *)calloc(tsr_msum_words(T), sizeof(uint32_t));
    tsr_msum_build_f16(mask, mask_stride, n_kv, T, 1u, f->msum_words);
    tsr_msum_view(f->msum_words, tsr_msum_words(T), &f->msum);
    f->mask_f32 = (float *)calloc((size_t)T * 16u * ((n_kv + 15u) / 16u + 1u), sizeof(float));
    tsr_msum_mask_f32(mask, mask_stride, n_kv, T, scale, f->mask_f32);
    free(zero);
    f->T = T; f->D = D; f->G = n_head / n_head_kv; f->n_kv = n_kv; f->scale = scale;
    f->new_run[0][0] = new_lo; f->new_run[0][1] = new_hi;
    f->n_new = new_hi > new_lo ? 1u : 0u;
    return f;
}

int refdrv_fa_run(const refdrv_fa * f, const float * q, float * out) {
    const tsr_fa_args a = {
        f->T, f->D, f->G, f->scale, q, f->geom.E, f->geom.LG,
        (const uint8_t * const *)f->kpl, (const uint8_t * const *)f->vpl,
        &f->msum, f->mask_f32, f->n_new ? (const uint32_t (*)[2])f->new_run : NULL, f->n_new, out, NULL,
    };
    return tsr_ref_fa(&f->cfg, &a);
}
