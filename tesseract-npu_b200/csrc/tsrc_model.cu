// tsrc_model.cu -- a random-init decoder-only transformer (Llama / Qwen2 layer graph) run through the
// C ABI's kinds, for end-to-end prefill and decode: the graph llama.cpp builds for these
// architectures (llm_build_llama / llm_build_qwen2 of the pinned llama.cpp) with every node on the
// device: GET_ROWS, RMS_NORM + MUL, MUL_MAT (+ bias ADD), ROPE, SET_ROWS into the q8_0 KV cache,
// FLASH_ATTN_EXT, MUL_MAT + residual ADD, RMS_NORM + MUL, MUL_MAT gate / up, SWIGLU, MUL_MAT down +
// residual ADD; then the output RMS_NORM + MUL and the head MUL_MAT of the last token.
//
// Each residual ADD is the MUL_MAT's addend epilogue (fadd(x, dot): the same value as the ADD
// node); for one token each RMS_NORM + MUL runs inside the MUL_MAT that consumes it
// (tsrc_mul_mat_rms: the same values, one launch and no round trip of the normalised row). q, k and v are one MUL_MAT over the rows of the three matrices stacked (every output row is
// its own dot product, so the values are those of three MUL_MATs), and so are gate and up; ROPE of
// q and k is one launch over their heads, with c_i and s_i of every position precomputed once per
// model by the same device code (a table lookup instead of the per-token angle recurrence). Weights come from tsrc_weight_synth (seeded); the f32 vectors (norm weights, biases) from
// splitmix64 (tsrc_model_f32_value), so a checker can rebuild them.
#include <algorithm>
#include <cmath>
#include <initializer_list>
#include <cstdio>
#include <cstring>
#include <vector>

#include "tsrc_internal.h"
#include "../../include/tsrc.h"

struct tsrc_model {
    tsrc_ctx* ctx;
    tsrc_model_cfg c;
    float ts, kq_scale;
    tsrc_weight* tok_embd = nullptr;
    tsrc_weight* output = nullptr;                       // NULL with a tied head
    float* f32 = nullptr;                                // every f32 vector, one allocation
    float* out_norm = nullptr;
    struct Layer {
        tsrc_weight *wqkv, *wo, *wgu, *wd;               // [q | k | v] rows, o, [gate | up] rows, down
        float *attn_norm, *ffn_norm, *bqkv;
        tsrc_kv* kv;
    };
    std::vector<Layer> layers;
    int32_t* pos = nullptr;                              // 0 .. n_ctx - 1 (device)
    float* rope_tab = nullptr;                           // c_i then s_i of every position [2][n_ctx][head_dim / 2]
    float* buf = nullptr;                                // activations for t_alloc tokens
    uint32_t t_alloc = 0;
    float *x, *h, *qkv, *q, *att, *gu, *act;          // gu: (gate, up) pairs interleaved; act: their SWIGLU
    std::vector<uint16_t> mask;                          // host causal mask of a multi-token call
    // decode graph (tsrc_model_decode): one token's kernels captured once; per token the position
    // kernel's argument and the FA nodes' plans are rewritten in the instantiated graph
    int32_t* dstate = nullptr;                           // device: [0] position (int32), [2..3] cell (int64)
    cudaStream_t own = nullptr;                          // a blocking stream for callers on the legacy stream
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t gexec = nullptr;
    const int32_t* g_ids = nullptr;
    float* g_logits = nullptr;
    cudaStream_t g_stream = nullptr;
    cudaGraphNode_t pos_node = nullptr;
    cudaKernelNodeParams pos_params{};
    struct FaNode {
        cudaGraphNode_t node;
        cudaKernelNodeParams params;
        tsrc::FaLaunch arg;
    };
    std::vector<FaNode> fa_nodes;
    uint32_t g_n_items = 0, g_n_tiles = 0, g_Tq0 = 0, g_nmax = 0;
    const void* g_ok = nullptr;
    // tensor parallelism (tsrc_model_create_tp): this rank's heads and row ranges
    tsrc_team* team = nullptr;
    uint32_t rank = 0, world = 1;
    uint32_t hq_loc = 0, hkv_loc = 0, f0 = 0, f_n = 0;   // local q / kv heads; gate / up rows [f0, f0 + f_n)
    tsrc_weight* head_shard = nullptr;                   // rows of the head (the embedding when tied)
    float* tp_bias = nullptr;                            // [n_layer][local q | k | v] bias slices
    float* tp_act = nullptr;                             // the gathered SWIGLU row [F]
};

namespace {

uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}


// f32 vector kinds of the model (tsrc_model_f32_value)
constexpr uint32_t kVecAttnNorm = 0, kVecFfnNorm = 1, kVecBqkv = 2, kVecOutNorm = 5;

}  // namespace

// the decode graph's per-token state: the token's position and its KV cell
__global__ void model_state_kernel(int32_t* st, int32_t pos) {
    st[0] = pos;
    reinterpret_cast<int64_t*>(st)[1] = (int64_t)pos;
}

extern "C" {

float tsrc_model_f32_value(uint64_t seed, uint32_t layer, uint32_t which, uint32_t i) {
    const uint64_t z = splitmix64(seed ^ ((uint64_t)layer << 40) ^ ((uint64_t)which << 32) ^ i);
    const float u = (float)(z >> 40) * (1.0f / 16777216.0f) * 2.0f - 1.0f;   // [-1, 1), 24 random bits
    return (which == kVecAttnNorm || which == kVecFfnNorm || which == kVecOutNorm) ? 1.0f + 0.25f * u : 0.1f * u;
}

int tsrc_model_free(tsrc_model* m) {
    if (!m) return TSRC_OK;
    cudaDeviceSynchronize();
    for (auto& L : m->layers) {
        tsrc_weight* ws[] = {L.wqkv, L.wo, L.wgu, L.wd};
        for (tsrc_weight* w : ws)
            if (w) tsrc_weight_free(w);
        if (L.kv) tsrc_kv_free(L.kv);
    }
    if (m->tok_embd) tsrc_weight_free(m->tok_embd);
    if (m->output) tsrc_weight_free(m->output);
    if (m->head_shard) tsrc_weight_free(m->head_shard);
    cudaFree(m->tp_bias);
    cudaFree(m->tp_act);
    if (m->gexec) cudaGraphExecDestroy(m->gexec);
    if (m->graph) cudaGraphDestroy(m->graph);
    cudaFree(m->dstate);
    if (m->own) cudaStreamDestroy(m->own);
    cudaFree(m->f32);
    cudaFree(m->pos);
    cudaFree(m->rope_tab);
    cudaFree(m->buf);
    delete m;
    return TSRC_OK;
}

}  // extern "C"

static int model_create(tsrc_ctx* ctx, const tsrc_model_cfg* cfg, uint64_t seed, tsrc_team* team, tsrc_model** out) {
    if (!ctx || !cfg || !out) return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_create: NULL argument");
    *out = nullptr;
    const tsrc_model_cfg& c = *cfg;
    if (c.n_layer == 0 || c.n_embd == 0 || c.n_ff == 0 || c.n_head == 0 || c.n_head_kv == 0 || c.n_head % c.n_head_kv ||
        c.n_vocab == 0 || c.n_ctx == 0 || (c.fmt != TSRC_FMT_Q8_0 && c.fmt != TSRC_FMT_Q4_K) || c.rope_mode > TSRC_ROPE_NEOX)
        return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_create: a shape field is zero or out of range");
    uint32_t rank = 0, world = 1, n_max = 0;
    if (team) {
        int rc = tsrc::team_info(team, &rank, &world, &n_max);
        if (rc) return rc;
        if (c.n_head_kv % world) return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_create_tp: the KV heads do not split over the ranks");
        const uint32_t need = std::max(std::max(c.n_vocab, c.n_ff), std::max(c.n_head * c.head_dim, c.n_embd));
        if (n_max < need)
            return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_create_tp: the team's n_max is below max(n_vocab, n_ff, n_head * head_dim, n_embd)");
    }
    tsrc_model* m = new tsrc_model();
    m->ctx = ctx;
    m->c = c;
    m->team = team;
    m->rank = rank;
    m->world = world;
    m->ts = powf(c.rope_base, -2.0f / (float)c.head_dim);       // the backend's theta scale (host libm)
    m->kq_scale = 1.0f / sqrtf((float)c.head_dim);              // llama.cpp's kq_scale
    const uint32_t E = c.n_embd, D = c.head_dim, Hq = c.n_head * D, Hkv = c.n_head_kv * D, F = c.n_ff;
    const float sigma = 0.02f;
    int rc = TSRC_OK;
    auto synth = [&](uint32_t N, uint32_t K, uint64_t s, tsrc_weight** w) {
        if (rc == TSRC_OK) rc = tsrc_weight_synth(ctx, c.fmt, N, K, 0, N, s, sigma, nullptr, w);
    };
    // a rank's share of the rows (the symmetric split R = ceil(N / world), sw/sim/tsr_ref.c:335-357)
    auto shard = [&](uint32_t N, uint32_t* r0, uint32_t* n) {
        const uint32_t R = (N + world - 1u) / world;
        *r0 = std::min(N, rank * R);
        *n = std::min(N, *r0 + R) - *r0;
    };
    auto synth_shard = [&](uint32_t N, uint32_t K, uint64_t s, tsrc_weight** w) {
        uint32_t r0 = 0, n = 0;
        shard(N, &r0, &n);
        if (rc == TSRC_OK) rc = tsrc_weight_synth(ctx, c.fmt, N, K, r0, n, s, sigma, nullptr, w);
    };
    auto synth_ranges = [&](uint32_t N, uint32_t K, std::initializer_list<uint32_t> r0, std::initializer_list<uint32_t> n,
                            uint64_t s, tsrc_weight** w) {
        if (rc == TSRC_OK)
            rc = tsrc::weight_synth_ranges(ctx, c.fmt, N, K, r0.begin(), n.begin(), (uint32_t)r0.size(), s, sigma, w);
    };
    m->hq_loc = c.n_head / world;
    m->hkv_loc = c.n_head_kv / world;
    shard(F, &m->f0, &m->f_n);
    synth(c.n_vocab, E, seed * 1000u + 1u, &m->tok_embd);
    if (!c.tied_head && !team) synth(c.n_vocab, E, seed * 1000u + 2u, &m->output);
    if (team) synth_shard(c.n_vocab, E, seed * 1000u + (c.tied_head ? 1u : 2u), &m->head_shard);
    // f32 vectors: per layer attn_norm, ffn_norm (E) and the q | k | v bias (Hq + 2 Hkv); out_norm (E)
    const size_t per_layer = 2u * E + (c.qkv_bias ? (size_t)Hq + 2u * Hkv : 0u);
    const size_t n_f32 = per_layer * c.n_layer + E;
    std::vector<float> host(n_f32);
    m->layers.resize(c.n_layer);
    if (rc == TSRC_OK && cudaMalloc(&m->f32, n_f32 * sizeof(float)) != cudaSuccess) rc = TSRC_E_NOMEM;
    size_t o = 0;
    auto vec = [&](uint32_t layer, uint32_t which, uint32_t n) {
        float* p = m->f32 + o;
        for (uint32_t i = 0; i < n; ++i) host[o + i] = tsrc_model_f32_value(seed, layer, which, i);
        o += n;
        return p;
    };
    for (uint32_t l = 0; l < c.n_layer && rc == TSRC_OK; ++l) {
        tsrc_model::Layer& L = m->layers[l];
        std::memset(&L, 0, sizeof L);
        const uint64_t s = seed * 1000u + 16u * (l + 1u);
        if (team) {
            const uint32_t qn = m->hq_loc * D, kn = m->hkv_loc * D;
            synth_ranges(Hq + 2u * Hkv, E, {rank * qn, Hq + rank * kn, Hq + Hkv + rank * kn}, {qn, kn, kn}, s + 0, &L.wqkv);
            synth_shard(E, Hq, s + 1, &L.wo);
            synth_ranges(2u * F, E, {m->f0, F + m->f0}, {m->f_n, m->f_n}, s + 2, &L.wgu);
            synth_shard(E, F, s + 3, &L.wd);
        } else {
            synth(Hq + 2u * Hkv, E, s + 0, &L.wqkv);
            synth(E, Hq, s + 1, &L.wo);
            synth(2u * F, E, s + 2, &L.wgu);
            synth(E, F, s + 3, &L.wd);
        }
        // gate and up rows interleaved (gate_j, up_j adjacent): the MUL_MAT kernel's warp then holds
        // both values of a SWIGLU pair and applies it as its epilogue
        if (rc == TSRC_OK) rc = tsrc::weight_interleave_halves(ctx, L.wgu, &L.wgu);
        L.attn_norm = vec(l, kVecAttnNorm, E);
        L.ffn_norm = vec(l, kVecFfnNorm, E);
        if (c.qkv_bias) L.bqkv = vec(l, kVecBqkv, Hq + 2u * Hkv);
        if (rc == TSRC_OK) rc = tsrc_kv_create(ctx, c.n_head_kv / world, D, c.n_ctx, &L.kv);
    }
    m->out_norm = vec(c.n_layer, kVecOutNorm, E);
    if (rc == TSRC_OK && cudaMemcpy(m->f32, host.data(), n_f32 * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess)
        rc = TSRC_E_CUDA;
    if (team && rc == TSRC_OK) {
        // the rank's q | k | v bias slices, and its SWIGLU / gathered activation rows
        const uint32_t qn = m->hq_loc * D, kn = m->hkv_loc * D, qkv_loc = qn + 2u * kn;
        if (c.qkv_bias) {
            std::vector<float> hb((size_t)c.n_layer * qkv_loc);
            for (uint32_t l = 0; l < c.n_layer; ++l) {
                float* d = hb.data() + (size_t)l * qkv_loc;
                for (uint32_t i = 0; i < qn; ++i) d[i] = tsrc_model_f32_value(seed, l, kVecBqkv, rank * qn + i);
                for (uint32_t i = 0; i < kn; ++i) d[qn + i] = tsrc_model_f32_value(seed, l, kVecBqkv, Hq + rank * kn + i);
                for (uint32_t i = 0; i < kn; ++i) d[qn + kn + i] = tsrc_model_f32_value(seed, l, kVecBqkv, Hq + Hkv + rank * kn + i);
            }
            if (cudaMalloc(&m->tp_bias, hb.size() * sizeof(float)) != cudaSuccess ||
                cudaMemcpy(m->tp_bias, hb.data(), hb.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess)
                rc = TSRC_E_NOMEM;
        }
        if (rc == TSRC_OK && cudaMalloc(&m->tp_act, (size_t)F * sizeof(float)) != cudaSuccess) rc = TSRC_E_NOMEM;
    }
    std::vector<int32_t> pos(c.n_ctx);
    for (uint32_t i = 0; i < c.n_ctx; ++i) pos[i] = (int32_t)i;
    if (rc == TSRC_OK && (cudaMalloc(&m->pos, c.n_ctx * sizeof(int32_t)) != cudaSuccess ||
                          cudaMemcpy(m->pos, pos.data(), c.n_ctx * sizeof(int32_t), cudaMemcpyHostToDevice) != cudaSuccess))
        rc = TSRC_E_NOMEM;
    const size_t half = D / 2u;
    if (rc == TSRC_OK && cudaMalloc(&m->rope_tab, 2u * c.n_ctx * half * sizeof(float)) != cudaSuccess) rc = TSRC_E_NOMEM;
    if (rc == TSRC_OK &&
        (tsrc::launch_rope_table(c.n_ctx, D, m->ts, 1.0f, m->rope_tab, m->rope_tab + c.n_ctx * half, nullptr) != cudaSuccess ||
         cudaDeviceSynchronize() != cudaSuccess))
        rc = tsrc::api_fail(TSRC_E_CUDA, "tsrc_model_create: ROPE tables");
    if (rc != TSRC_OK) {
        tsrc_model_free(m);
        return rc;
    }
    *out = m;
    return TSRC_OK;
}

extern "C" {

int tsrc_model_create(tsrc_ctx* ctx, const tsrc_model_cfg* cfg, uint64_t seed, tsrc_model** out) {
    return model_create(ctx, cfg, seed, nullptr, out);
}

int tsrc_model_create_tp(tsrc_ctx* ctx, const tsrc_model_cfg* cfg, uint64_t seed, tsrc_team* team, tsrc_model** out) {
    if (!team) return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_create_tp: NULL team");
    return model_create(ctx, cfg, seed, team, out);
}

int tsrc_model_kv(const tsrc_model* m, uint32_t layer, tsrc_kv** out) {
    if (!m || !out || layer >= m->c.n_layer) return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_kv: no such layer");
    *out = m->layers[layer].kv;
    return TSRC_OK;
}

int tsrc_model_weight(const tsrc_model* m, uint32_t layer, uint32_t which, tsrc_weight** out) {
    if (!m || !out) return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_weight: NULL argument");
    *out = nullptr;
    if (layer == TSRC_MODEL_GLOBAL) {
        if (which == 0u) *out = m->tok_embd;
        else if (which == 1u) *out = m->c.tied_head ? m->tok_embd : m->output;
        return *out ? TSRC_OK : TSRC_E_ARG;
    }
    if (layer >= m->c.n_layer || which > 3u) return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_weight: no such weight");
    const tsrc_model::Layer& L = m->layers[layer];
    tsrc_weight* ws[] = {L.wqkv, L.wo, L.wgu, L.wd};
    *out = ws[which];
    return TSRC_OK;
}

int tsrc_model_params(const tsrc_model* m, float* ts, float* kq_scale) {
    if (!m) return TSRC_E_ARG;
    if (ts) *ts = m->ts;
    if (kq_scale) *kq_scale = m->kq_scale;
    return TSRC_OK;
}

}  // extern "C"

namespace {

int ensure_buffers(tsrc_model* m, uint32_t T) {
    const tsrc_model_cfg& c = m->c;
    const uint32_t E = c.n_embd, D = c.head_dim, Hq = c.n_head * D, Hkv = c.n_head_kv * D, F = c.n_ff;
    const uint32_t QKV = Hq + 2u * Hkv;
    if (T > m->t_alloc) {
        cudaDeviceSynchronize();
        cudaFree(m->buf);
        m->buf = nullptr;
        const size_t per = 2u * E + QKV + 2u * Hq + 3u * F;
        if (cudaMalloc(&m->buf, per * T * sizeof(float)) != cudaSuccess) {
            m->t_alloc = 0;
            return tsrc::api_fail(TSRC_E_NOMEM, "tsrc_model_forward: activation buffers");
        }
        m->t_alloc = T;
        float* p = m->buf;
        m->x = p; p += (size_t)E * T;
        m->h = p; p += (size_t)E * T;
        m->qkv = p; p += (size_t)QKV * T;
        m->q = p; p += (size_t)Hq * T;
        m->att = p; p += (size_t)Hq * T;
        m->gu = p; p += 2u * (size_t)F * T;
        m->act = p;
    }
    return TSRC_OK;
}

// The model's graph for T tokens at pos0. pos: device positions of the tokens; cells: device KV
// cells of the tokens (NULL: cells pos0 .. pos0 + T - 1).
int forward_body(tsrc_model* m, const int32_t* ids, uint32_t T, uint32_t pos0, float* logits, void* stream, const int32_t* pos,
                 const int64_t* cells) {
    const tsrc_model_cfg& c = m->c;
    tsrc_ctx* ctx = m->ctx;
    const uint32_t E = c.n_embd, D = c.head_dim, Hq = c.n_head * D, Hkv = c.n_head_kv * D, F = c.n_ff;
    const uint32_t QKV = Hq + 2u * Hkv;
    const uint32_t n_kv = pos0 + T;
    const uint16_t* mask = nullptr;
    if (T > 1) {                                          // causal: token t sees cells [0, pos0 + t]
        m->mask.assign((size_t)T * n_kv, 0xFC00u);
        for (uint32_t t = 0; t < T; ++t)
            std::fill(m->mask.begin() + (size_t)t * n_kv, m->mask.begin() + (size_t)t * n_kv + pos0 + t + 1u, (uint16_t)0u);
        mask = m->mask.data();
    }
    const float inv_n = 1.0f / (float)E;
    const size_t half = D / 2u;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    tsrc_fa_cfg fa = c.fa;
    if (fa.C == 0) fa = tsrc_fa_cfg{4u, 4u, 9344u, 32768u, 0u};
    int rc = tsrc_get_rows(ctx, m->tok_embd, ids, T, m->x, E, stream);
#define TSRC_M(call) \
    if (rc == TSRC_OK) rc = (call)
#define TSRC_MC(call, what) \
    if (rc == TSRC_OK && (call) != cudaSuccess) rc = tsrc::api_fail(TSRC_E_CUDA, what)
    if (m->team && T > 1) {
        // a prompt over the team: every rank holds all T rows of the residual stream x. Per layer:
        // RMS_NORM; q / k / v of this rank's heads (tensor-core MUL_MAT for T > 8) with its bias
        // slice; ROPE + KVST into its KV heads; FA of its q heads (planned with the model's E); then
        // the exchanges of T rows each: the attention output (gather), o rows + residual (gather
        // into x), gate / up pairs of its F slice and SWIGLU (gather), down rows + residual (gather
        // into x). The head runs on the last token as in decode. Every value is one GPU's result,
        // so the logits are the single GPU's.
        tsrc_team* tm = m->team;
        const uint32_t qn = m->hq_loc * D, kn = m->hkv_loc * D, qkv_loc = qn + 2u * kn;
        uint32_t on = 0, o0 = 0, dn = 0, d0 = 0, wN = 0;
        if (rc == TSRC_OK) rc = tsrc::weight_rows(m->layers[0].wo, &wN, &o0, &on);
        if (rc == TSRC_OK) rc = tsrc::weight_rows(m->layers[0].wd, &wN, &d0, &dn);
        fa.plan_n_head_kv = c.n_head_kv;
        for (uint32_t l = 0; l < c.n_layer; ++l) {
            const tsrc_model::Layer& L = m->layers[l];
            const float* bias = m->tp_bias ? m->tp_bias + (size_t)l * qkv_loc : nullptr;
            TSRC_M(tsrc_rms_norm(ctx, m->x, E, m->h, E, L.attn_norm, E, T, c.rms_eps, inv_n, stream));
            TSRC_M(tsrc_mul_mat(ctx, L.wqkv, m->h, T, E, m->qkv, qkv_loc, bias, 0, bias ? TSRC_MM_ADD : 0u, 1.0f, 1.0f, stream));
            tsrc::RopeKvst rk{};
            rk.qkv = m->qkv;
            rk.stride = qkv_loc;
            rk.pos = pos;
            rk.n_rot_heads = m->hq_loc + m->hkv_loc;
            rk.hd = D;
            rk.nd = D;
            rk.neox = c.rope_mode;
            rk.cs_tab = m->rope_tab;
            rk.sn_tab = m->rope_tab + (size_t)c.n_ctx * half;
            rk.k_off = qn;
            rk.v_off = qn + kn;
            rk.cells = cells;
            rk.cell0 = pos0;
            if (rc == TSRC_OK && !cells && (uint64_t)pos0 + T > tsrc::kv_cells(L.kv))
                rc = tsrc::api_fail(TSRC_E_ARG, "tsrc_model_forward: cells outside the cache");
            TSRC_M(tsrc::kv_fill_planes(L.kv, &rk));
            TSRC_MC(tsrc::launch_rope_kvst(rk, T, st), "tsrc_model_forward: ROPE + KVST launch");
            // FA takes q rows [T][heads][D] contiguous: the rank's q rows go to att first
            TSRC_MC(cudaMemcpy2DAsync(m->att, (size_t)qn * 4u, m->qkv, (size_t)qkv_loc * 4u, (size_t)qn * 4u, T,
                                      cudaMemcpyDeviceToDevice, st), "tsrc_model_forward: q copy");
            TSRC_M(tsrc_flash_attn(ctx, L.kv, m->att, T, m->hq_loc, n_kv, mask, n_kv, m->kq_scale, pos0, n_kv, &fa, m->q, stream));
            TSRC_M(tsrc::team_gather_rows(tm, m->q, qn, qn, m->rank * qn, m->att, Hq, Hq, T, stream));
            TSRC_M(tsrc_mul_mat(ctx, L.wo, m->att, T, Hq, m->h, on, m->x + o0, E, TSRC_MM_ADD, 1.0f, 1.0f, stream));
            TSRC_M(tsrc::team_gather_rows(tm, m->h, on, on, o0, m->x, E, E, T, stream));
            TSRC_M(tsrc_rms_norm(ctx, m->x, E, m->h, E, L.ffn_norm, E, T, c.rms_eps, inv_n, stream));
            TSRC_M(tsrc_mul_mat(ctx, L.wgu, m->h, T, E, m->gu, 2u * m->f_n, nullptr, 0, 0u, 1.0f, 1.0f, stream));
            TSRC_MC(tsrc::launch_vop(8u, m->gu, 2u * m->f_n, nullptr, 0u, m->act, m->f_n, m->f_n, T, st),
                    "tsrc_model_forward: SWIGLU launch");
            TSRC_M(tsrc::team_gather_rows(tm, m->act, m->f_n, m->f_n, m->f0, m->gu, F, F, T, stream));
            TSRC_M(tsrc_mul_mat(ctx, L.wd, m->gu, T, F, m->h, dn, m->x + d0, E, TSRC_MM_ADD, 1.0f, 1.0f, stream));
            TSRC_M(tsrc::team_gather_rows(tm, m->h, dn, dn, d0, m->x, E, E, T, stream));
        }
        const float* xl = m->x + (size_t)(T - 1u) * E;
        TSRC_M(tsrc::team_mul_mat(ctx, tm, m->head_shard, xl, logits, nullptr, m->out_norm, c.rms_eps, inv_n, true, stream));
        return rc;
    }
    if (m->team) {
        // one token over the team: q / k / v of this rank's heads, its KV heads' cache and FA, then
        // the exchanges: attention output (gather), o rows (+ residual, fused gather), gate / up row
        // pairs of this rank's F slice with SWIGLU as their epilogue (fused gather), down rows
        // (+ residual, fused gather), head rows (fused gather). Every row is one GPU's dot product:
        // the logits are the single GPU's.
        tsrc_team* tm = m->team;
        const uint32_t qn = m->hq_loc * D, kn = m->hkv_loc * D, qkv_loc = qn + 2u * kn;
        float* att_loc = m->q;
        float* act_all = m->tp_act;
        fa.plan_n_head_kv = c.n_head_kv;
        for (uint32_t l = 0; l < c.n_layer; ++l) {
            const tsrc_model::Layer& L = m->layers[l];
            const float* bias = m->tp_bias ? m->tp_bias + (size_t)l * qkv_loc : nullptr;
            TSRC_M(tsrc_mul_mat_rms(ctx, L.wqkv, m->x, L.attn_norm, c.rms_eps, inv_n, m->qkv, bias, bias ? TSRC_MM_ADD : 0u,
                                    1.0f, 1.0f, stream));
            tsrc::RopeKvst rk{};
            rk.qkv = m->qkv;
            rk.stride = qkv_loc;
            rk.pos = pos;
            rk.n_rot_heads = m->hq_loc + m->hkv_loc;
            rk.hd = D;
            rk.nd = D;
            rk.neox = c.rope_mode;
            rk.cs_tab = m->rope_tab;
            rk.sn_tab = m->rope_tab + (size_t)c.n_ctx * half;
            rk.k_off = qn;
            rk.v_off = qn + kn;
            rk.cells = cells;
            rk.cell0 = pos0;
            if (rc == TSRC_OK && !cells && (uint64_t)pos0 + 1u > tsrc::kv_cells(L.kv))
                rc = tsrc::api_fail(TSRC_E_ARG, "tsrc_model_forward: cells outside the cache");
            TSRC_M(tsrc::kv_fill_planes(L.kv, &rk));
            TSRC_MC(tsrc::launch_rope_kvst(rk, 1, st), "tsrc_model_forward: ROPE + KVST launch");
            TSRC_M(tsrc_flash_attn(ctx, L.kv, m->qkv, 1, m->hq_loc, n_kv, nullptr, n_kv, m->kq_scale, pos0, n_kv, &fa, att_loc,
                                   stream));
            TSRC_M(tsrc::team_gather(tm, att_loc, qn, m->rank * qn, m->att, Hq, stream));
            TSRC_M(tsrc::team_mul_mat(ctx, tm, L.wo, m->att, m->x, m->x, nullptr, 0.0f, 0.0f, false, stream));
            TSRC_M(tsrc::team_mul_mat_swiglu(ctx, tm, L.wgu, m->x, act_all, m->f0, F, L.ffn_norm, c.rms_eps, inv_n, stream));
            TSRC_M(tsrc::team_mul_mat(ctx, tm, L.wd, act_all, m->x, m->x, nullptr, 0.0f, 0.0f, false, stream));
        }
        TSRC_M(tsrc::team_mul_mat(ctx, tm, m->head_shard, m->x, logits, nullptr, m->out_norm, c.rms_eps, inv_n, true, stream));
        return rc;
    }
    for (uint32_t l = 0; l < c.n_layer; ++l) {
        const tsrc_model::Layer& L = m->layers[l];
        if (T == 1) {                                     // one token: RMS_NORM + MUL fused into the MUL_MAT
            TSRC_M(tsrc_mul_mat_rms(ctx, L.wqkv, m->x, L.attn_norm, c.rms_eps, inv_n, m->qkv, L.bqkv,
                                    L.bqkv ? TSRC_MM_ADD : 0u, 1.0f, 1.0f, stream));
        } else {
            TSRC_M(tsrc_rms_norm(ctx, m->x, E, m->h, E, L.attn_norm, E, T, c.rms_eps, inv_n, stream));
            TSRC_M(tsrc_mul_mat(ctx, L.wqkv, m->h, T, E, m->qkv, QKV, L.bqkv, 0, L.bqkv ? TSRC_MM_ADD : 0u, 1.0f, 1.0f, stream));
        }
        {   // ROPE of q and k, SET_ROWS of k and v into the layer's q8_0 cache: one launch
            tsrc::RopeKvst rk{};
            rk.qkv = m->qkv;
            rk.stride = QKV;
            rk.pos = pos;
            rk.n_rot_heads = c.n_head + c.n_head_kv;
            rk.hd = D;
            rk.nd = D;
            rk.neox = c.rope_mode;
            rk.cs_tab = m->rope_tab;
            rk.sn_tab = m->rope_tab + (size_t)c.n_ctx * half;
            rk.k_off = Hq;
            rk.v_off = Hq + Hkv;
            rk.cells = cells;
            rk.cell0 = pos0;
            if (rc == TSRC_OK && !cells && (uint64_t)pos0 + T > tsrc::kv_cells(L.kv))
                rc = tsrc::api_fail(TSRC_E_ARG, "tsrc_model_forward: cells outside the cache");
            TSRC_M(tsrc::kv_fill_planes(L.kv, &rk));
            TSRC_MC(tsrc::launch_rope_kvst(rk, T, st), "tsrc_model_forward: ROPE + KVST launch");
        }
        const float* q = m->qkv;
        if (T > 1) {                                      // FA takes q rows [T][n_head][D] contiguous
            TSRC_MC(cudaMemcpy2DAsync(m->q, (size_t)Hq * 4u, m->qkv, (size_t)QKV * 4u, (size_t)Hq * 4u, T, cudaMemcpyDeviceToDevice, st),
                    "tsrc_model_forward: q copy");
            q = m->q;
        }
        TSRC_M(tsrc_flash_attn(ctx, L.kv, q, T, c.n_head, n_kv, mask, n_kv, m->kq_scale, pos0, n_kv, &fa, m->att, stream));
        TSRC_M(tsrc_mul_mat(ctx, L.wo, m->att, T, Hq, m->x, E, m->x, E, TSRC_MM_ADD, 1.0f, 1.0f, stream));
        if (T == 1) {                                     // RMS_NORM, gate / up and SWIGLU: one launch
            TSRC_M(tsrc::mul_mat_rms_swiglu(ctx, L.wgu, m->x, L.ffn_norm, c.rms_eps, inv_n, m->act, stream));
        } else {
            TSRC_M(tsrc_rms_norm(ctx, m->x, E, m->h, E, L.ffn_norm, E, T, c.rms_eps, inv_n, stream));
            TSRC_M(tsrc_mul_mat(ctx, L.wgu, m->h, T, E, m->gu, 2u * F, nullptr, 0, 0u, 1.0f, 1.0f, stream));
            TSRC_MC(tsrc::launch_vop(8u, m->gu, 2u * F, nullptr, 0u, m->act, F, F, T, st), "tsrc_model_forward: SWIGLU launch");
        }
        TSRC_M(tsrc_mul_mat(ctx, L.wd, m->act, T, F, m->x, E, m->x, E, TSRC_MM_ADD, 1.0f, 1.0f, stream));
    }
    // the last token: output norm and head
    const float* xl = m->x + (size_t)(T - 1u) * E;
    TSRC_M(tsrc_mul_mat_rms(ctx, c.tied_head ? m->tok_embd : m->output, xl, m->out_norm, c.rms_eps, inv_n, logits, nullptr, 0u,
                            1.0f, 1.0f, stream));
#undef TSRC_MC
#undef TSRC_M
    return rc;
}

bool same_plan(const tsrc_model* m, const tsrc::FaLaunch& a, uint32_t nmax) {
    return a.n_items == m->g_n_items && a.n_tiles == m->g_n_tiles && a.Tq0 == m->g_Tq0 && nmax == m->g_nmax &&
           a.n_items <= tsrc::kFaInlineItems && (const void*)a.ok == m->g_ok;
}

void drop_graph(tsrc_model* m) {
    if (m->gexec) cudaGraphExecDestroy(m->gexec);
    if (m->graph) cudaGraphDestroy(m->graph);
    m->gexec = nullptr;
    m->graph = nullptr;
    m->fa_nodes.clear();
    m->pos_node = nullptr;
}

// captures one decode token at pos0 (the FA plans of that position) and instantiates it
int capture_decode(tsrc_model* m, const int32_t* ids, uint32_t pos0, float* logits, cudaStream_t st, const tsrc::FaLaunch& a0,
                   uint32_t nmax) {
    drop_graph(m);
    if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess)
        return tsrc::api_fail(TSRC_E_CUDA, "tsrc_model_decode: stream capture");
    model_state_kernel<<<1, 1, 0, st>>>(m->dstate, (int32_t)pos0);
    int rc = forward_body(m, ids, 1, pos0, logits, st, m->dstate, reinterpret_cast<const int64_t*>(m->dstate + 2));
    cudaGraph_t g = nullptr;
    const cudaError_t e = cudaStreamEndCapture(st, &g);
    if (rc != TSRC_OK || e != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        return rc != TSRC_OK ? rc : tsrc::api_fail(TSRC_E_CUDA, "tsrc_model_decode: capture failed");
    }
    m->graph = g;
    if (cudaGraphInstantiate(&m->gexec, g, 0) != cudaSuccess) {
        drop_graph(m);
        return tsrc::api_fail(TSRC_E_CUDA, "tsrc_model_decode: graph instantiation");
    }
    size_t n = 0;
    cudaGraphGetNodes(g, nullptr, &n);
    std::vector<cudaGraphNode_t> nodes(n);
    cudaGraphGetNodes(g, nodes.data(), &n);
    const void* fchunk = tsrc::fa_chunk_fn(m->c.head_dim, 16u);
    const void* fchunk_s = tsrc::fa_chunk_fn(m->c.head_dim, 4u);
    const void* fchunk_t = tsrc::fa_chunk_fn(m->c.head_dim, 2u);
    const void* fmerge = tsrc::fa_merge_fn(a0.C);
    const void* fstate = reinterpret_cast<const void*>(model_state_kernel);
    for (cudaGraphNode_t nd : nodes) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(nd, &t) != cudaSuccess || t != cudaGraphNodeTypeKernel) continue;
        cudaKernelNodeParams p{};
        if (cudaGraphKernelNodeGetParams(nd, &p) != cudaSuccess) continue;
        if (p.func == fchunk || (fchunk_s && p.func == fchunk_s) || (fchunk_t && p.func == fchunk_t) || p.func == fmerge) {
            tsrc_model::FaNode f;
            f.node = nd;
            f.params = p;
            f.arg = *static_cast<const tsrc::FaLaunch*>(p.kernelParams[0]);
            m->fa_nodes.push_back(f);
        } else if (p.func == fstate) {
            m->pos_node = nd;
            m->pos_params = p;
        }
    }
    if (!m->pos_node || m->fa_nodes.size() != 2u * m->c.n_layer) {
        drop_graph(m);
        return tsrc::api_fail(TSRC_E_CUDA, "tsrc_model_decode: the captured graph lacks the expected kernels");
    }
    m->g_ids = ids;
    m->g_logits = logits;
    m->g_stream = st;
    m->g_n_items = a0.n_items;
    m->g_n_tiles = a0.n_tiles;
    m->g_Tq0 = a0.Tq0;
    m->g_nmax = nmax;
    m->g_ok = a0.ok;
    return TSRC_OK;
}

}  // namespace

extern "C" {

int tsrc_model_forward(tsrc_model* m, const int32_t* ids, uint32_t T, uint32_t pos0, float* logits, void* stream) {
    if (!m || !ids || !logits || T == 0) return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_forward: NULL argument or T = 0");
    if ((uint64_t)pos0 + T > m->c.n_ctx) return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_forward: positions beyond n_ctx");
    int rc = ensure_buffers(m, T);
    if (rc) return rc;
    return forward_body(m, ids, T, pos0, logits, stream, m->pos + pos0, nullptr);
}

int tsrc_model_decode(tsrc_model* m, const int32_t* ids, uint32_t pos0, float* logits, void* stream) {
    if (!m || !ids || !logits) return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_decode: NULL argument");
    const tsrc_model_cfg& c = m->c;
    if ((uint64_t)pos0 + 1u > c.n_ctx) return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_decode: position beyond n_ctx");
    int rc = ensure_buffers(m, 1);
    if (rc) return rc;
    if (!m->dstate && cudaMalloc(&m->dstate, 16) != cudaSuccess) return tsrc::api_fail(TSRC_E_NOMEM, "tsrc_model_decode: state");
    // a graph cannot be captured on the legacy default stream: a NULL stream runs on the model's
    // own blocking stream, which that stream orders with
    if (!stream && !m->own && cudaStreamCreate(&m->own) != cudaSuccess)
        return tsrc::api_fail(TSRC_E_CUDA, "tsrc_model_decode: stream");
    const cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : m->own;
    // the plan of this position (the same for every layer: same shapes and n_kv)
    tsrc_fa_cfg fa = c.fa;
    if (fa.C == 0) fa = tsrc_fa_cfg{4u, 4u, 9344u, 32768u, 0u};
    tsrc::FaLaunch a0;
    uint32_t nmax = 0;
    if (m->team) fa.plan_n_head_kv = c.n_head_kv;         // shards plan as the single device does
    rc = tsrc::fa_setup(m->ctx, m->layers[0].kv, m->qkv, 1, m->team ? m->hq_loc : c.n_head, pos0 + 1u, nullptr, 0, m->kq_scale,
                        pos0, pos0 + 1u, &fa, m->team ? m->q : m->att, st, &a0, &nmax);
    if (rc) return rc;
    if (a0.n_items > tsrc::kFaInlineItems) return forward_body(m, ids, 1, pos0, logits, st, m->pos + pos0, nullptr);
    if (!m->gexec || ids != m->g_ids || logits != m->g_logits || st != m->g_stream || !same_plan(m, a0, nmax)) {
        rc = capture_decode(m, ids, pos0, logits, st, a0, nmax);
        if (rc) return rc;
    } else {
        int32_t p = (int32_t)pos0;
        void* pa[2] = {&m->dstate, &p};
        cudaKernelNodeParams pp = m->pos_params;
        pp.kernelParams = pa;
        if (cudaGraphExecKernelNodeSetParams(m->gexec, m->pos_node, &pp) != cudaSuccess)
            return tsrc::api_fail(TSRC_E_CUDA, "tsrc_model_decode: position update");
        for (auto& f : m->fa_nodes) {
            tsrc::FaLaunch a = f.arg;                    // this node's layer pointers, the new plan
            a.n_kv = a0.n_kv;
            a.n_items = a0.n_items;
            a.n_tiles = a0.n_tiles;
            a.Tq0 = a0.Tq0;
            std::memcpy(a.inl_items, a0.inl_items, sizeof a.inl_items);
            std::memcpy(a.inl_tiles, a0.inl_tiles, sizeof a.inl_tiles);
            void* ka[1] = {&a};
            cudaKernelNodeParams kp = f.params;
            kp.kernelParams = ka;
            if (cudaGraphExecKernelNodeSetParams(m->gexec, f.node, &kp) != cudaSuccess)
                return tsrc::api_fail(TSRC_E_CUDA, "tsrc_model_decode: FA plan update");
        }
    }
    if (cudaGraphLaunch(m->gexec, st) != cudaSuccess) return tsrc::api_fail(TSRC_E_CUDA, "tsrc_model_decode: graph launch");
    return TSRC_OK;
}

int tsrc_model_set_weight(tsrc_model* m, uint32_t layer, uint32_t which, uint32_t ggml_type, const void* rows, uint32_t N,
                          uint32_t K) {
    if (!m || !rows) return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_set_weight: NULL argument");
    if (m->team) return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_set_weight: single-device models only");
    const tsrc_model_cfg& c = m->c;
    const uint32_t E = c.n_embd, Hq = c.n_head * c.head_dim, Hkv = c.n_head_kv * c.head_dim, F = c.n_ff;
    tsrc_weight** slot = nullptr;
    uint32_t eN = 0, eK = 0;
    if (layer == TSRC_MODEL_GLOBAL) {
        if (which == 0u) {
            slot = &m->tok_embd;
        } else if (which == 1u && !c.tied_head) {
            slot = &m->output;
        } else {
            return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_set_weight: no such global weight (a tied head is the embedding)");
        }
        eN = c.n_vocab;
        eK = E;
    } else {
        if (layer >= c.n_layer || which > 3u) return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_set_weight: no such weight");
        tsrc_model::Layer& L = m->layers[layer];
        tsrc_weight** slots[] = {&L.wqkv, &L.wo, &L.wgu, &L.wd};
        const uint32_t ns[] = {Hq + 2u * Hkv, E, 2u * F, E}, ks[] = {E, Hq, E, F};
        slot = slots[which];
        eN = ns[which];
        eK = ks[which];
    }
    if (N != eN || K != eK) return tsrc::api_fail(TSRC_E_SHAPE, "tsrc_model_set_weight: the rows do not have the weight's shape");
    tsrc_weight* w = nullptr;
    int rc = tsrc_weight_upload_ggml(m->ctx, ggml_type, rows, N, K, 0, N, &w);
    if (rc) return rc;
    if (layer != TSRC_MODEL_GLOBAL && which == 2u) {      // gate rows then up rows -> interleaved pairs
        rc = tsrc::weight_interleave_halves(m->ctx, w, &w);
        if (rc) {
            tsrc_weight_free(w);
            return rc;
        }
    }
    drop_graph(m);                                       // the captured step holds the old weight
    tsrc_weight_free(*slot);
    *slot = w;
    return TSRC_OK;
}

int tsrc_model_set_f32(tsrc_model* m, uint32_t layer, uint32_t which, const float* values, uint32_t n) {
    if (!m || !values) return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_set_f32: NULL argument");
    if (m->team) return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_set_f32: single-device models only");
    const tsrc_model_cfg& c = m->c;
    const uint32_t E = c.n_embd, Hq = c.n_head * c.head_dim, Hkv = c.n_head_kv * c.head_dim;
    float* dst = nullptr;
    uint32_t en = 0;
    if (which == kVecOutNorm && layer == c.n_layer) {
        dst = m->out_norm;
        en = E;
    } else if (layer < c.n_layer && (which == kVecAttnNorm || which == kVecFfnNorm)) {
        dst = which == kVecAttnNorm ? m->layers[layer].attn_norm : m->layers[layer].ffn_norm;
        en = E;
    } else if (layer < c.n_layer && which == kVecBqkv && c.qkv_bias) {
        dst = m->layers[layer].bqkv;
        en = Hq + 2u * Hkv;
    } else {
        return tsrc::api_fail(TSRC_E_ARG, "tsrc_model_set_f32: no such vector");
    }
    if (n != en) return tsrc::api_fail(TSRC_E_SHAPE, "tsrc_model_set_f32: wrong length");
    if (cudaMemcpy(dst, values, (size_t)n * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess)
        return tsrc::api_fail(TSRC_E_CUDA, "tsrc_model_set_f32: copy");
    return TSRC_OK;
}

}  // extern "C"
