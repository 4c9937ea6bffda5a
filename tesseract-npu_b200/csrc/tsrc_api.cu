// tsrc_api.cu -- the C ABI (include/tsrc.h): argument checks, device memory, launches.
//
// Host side of the B200 path. It stands where the reference's ggml backend lowered a node into
// an op-list record and ran it through the transport and the firmware
// (jwkim04/tesseract-npu sw/ggml-tesseract/ggml-tesseract.cpp:2790-2928 for MUL_MAT); here a
// call is a queue of kernel launches on the caller's stream. Refusals mirror supports_op
// (:4199-4299) as TSRC_E_SHAPE with the reason in tsrc_last_error().
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <string>

#include "../../include/tsrc.h"
#include "tsrc_internal.h"
#include "tsrc_layout.cuh"

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

}  // namespace

namespace tsrc {
// the C ABI's error record, for the library's other translation units (the model runner)
int api_fail(int code, const char* msg) {
    g_err = msg;
    return code;
}
}  // namespace tsrc

namespace {

int cuda_fail(cudaError_t e, const char* what) {
    return fail(TSRC_E_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

#define TSRC_CUDA(call, what)                      \
    do {                                           \
        cudaError_t e_ = (call);                   \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

constexpr uint32_t kKMax = 65536;             // shared-memory bound of one token's QA image
constexpr size_t kSmemBudget = 200u * 1024u;  // dynamic shared memory one matvec CTA may use

uint32_t block_of(uint32_t fmt) { return fmt == TSRC_FMT_Q8_0 ? 32u : 256u; }
size_t ggml_row_bytes(uint32_t fmt, uint32_t K) {
    return fmt == TSRC_FMT_Q8_0 ? (size_t)(K / 32u) * 34u : (size_t)(K / 256u) * 144u;
}
size_t qs_row_bytes(uint32_t fmt, uint32_t K) { return tsrc::Layout{fmt, K}.qs_row_bytes(); }
size_t meta_row_bytes(uint32_t fmt, uint32_t K) { return tsrc::Layout{fmt, K}.meta_row_bytes(); }
size_t align256(size_t n) { return (n + 255u) & ~(size_t)255u; }

// The tensor-core prefill path is on unless TSRC_NO_TC is set (then many tokens run through the
// matvec kernel, eight per launch; both give the same bits).
bool tc_enabled() {
    static const bool on = std::getenv("TSRC_NO_TC") == nullptr;
    return on;
}

// s0 / s1 enter the f32 rules as inputs: DAZ them once on the host.
float daz_host(float v) {
    uint32_t u;
    std::memcpy(&u, &v, 4);
    if ((u & 0x7F800000u) == 0) u &= 0x80000000u;
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}

// Bytes of the QA image of T tokens (q | d | bs, each 256-byte aligned).
size_t qa_bytes(uint32_t fmt, uint32_t K, uint32_t T) {
    return align256((size_t)T * K) + align256((size_t)T * (K / block_of(fmt)) * 4u) + align256((size_t)T * (K / 16u) * 2u);
}

}  // namespace

struct tsrc_weight {
    tsrc_ctx* ctx;
    uint32_t fmt, N, K, row0, n_rows;
    uint8_t* qs;
    uint8_t* meta;
    size_t bytes;
};

struct tsrc_kv {
    tsrc_ctx* ctx;
    uint32_t n_head_kv, D, n_cells, n_alloc;   // n_alloc: n_cells rounded up to 16 (zero padding)
    int8_t* q[2];                               // [K, V] quants [n_head_kv][n_alloc][D]
    uint16_t* d[2];                             //        scales [n_head_kv][n_alloc][D/32]
    uint8_t* mem;
    size_t bytes;
};

struct tsrc_ctx {
    int device;
    cudaDeviceProp prop;
    uint8_t* scratch = nullptr;   // QA images of the tokens of one call
    size_t scratch_bytes = 0;
    uint8_t* fa_scratch = nullptr;   // FA work items, channel partials, mask copies of one call
    size_t fa_scratch_bytes = 0;
    std::set<tsrc_weight*> weights;
    std::set<tsrc_kv*> kvs;
};

namespace {

int use_device(const tsrc_ctx* ctx) {
    int cur = -1;
    TSRC_CUDA(cudaGetDevice(&cur), "cudaGetDevice");
    if (cur != ctx->device) TSRC_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    return TSRC_OK;
}

int ensure_scratch(tsrc_ctx* ctx, size_t bytes) {
    if (bytes <= ctx->scratch_bytes) return TSRC_OK;
    if (ctx->scratch) {
        // the previous buffer may still be read by queued kernels
        TSRC_CUDA(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
        cudaFree(ctx->scratch);
        ctx->scratch = nullptr;
        ctx->scratch_bytes = 0;
    }
    const size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    cudaError_t e = cudaMalloc(&ctx->scratch, want);
    if (e != cudaSuccess) return fail(TSRC_E_NOMEM, "cudaMalloc of %zu scratch bytes: %s", want, cudaGetErrorString(e));
    ctx->scratch_bytes = want;
    return TSRC_OK;
}

const char* shape_reason(uint32_t fmt, uint64_t N, uint64_t K, uint64_t T) {
    if (fmt != TSRC_FMT_Q8_0 && fmt != TSRC_FMT_Q4_K) return "MUL_MAT: the weight type has no device format (Q8_0 and Q4_K only)";
    if (K == 0 || K % block_of(fmt) != 0) return "MUL_MAT: K is not a positive multiple of the block size (32 Q8_0, 256 Q4_K)";
    if (K > kKMax) return "MUL_MAT: K exceeds 65536 (one token's quantized activation must fit shared memory)";
    if (N == 0 || N > 0xFFFFFFFFull) return "MUL_MAT: N is 0 or does not fit 32 bits";
    if (T > 0xFFFFFFFFull) return "MUL_MAT: too many tokens";
    return nullptr;
}

int new_weight(tsrc_ctx* ctx, uint32_t fmt, uint32_t N, uint32_t K, uint32_t row0, uint32_t n_rows, tsrc_weight** out) {
    if (!ctx || !out) return fail(TSRC_E_ARG, "NULL context or output handle");
    if (const char* why = shape_reason(fmt, N, K, 1)) return fail(TSRC_E_SHAPE, "%s", why);
    if (n_rows == 0 || (uint64_t)row0 + n_rows > N) return fail(TSRC_E_ARG, "row shard [%u, %u+%u) outside [0, %u)", row0, row0, n_rows, N);
    int rc = use_device(ctx);
    if (rc) return rc;
    const size_t qb = align256(qs_row_bytes(fmt, K) * n_rows), mb = align256(meta_row_bytes(fmt, K) * n_rows);
    uint8_t* mem = nullptr;
    cudaError_t e = cudaMalloc(&mem, qb + mb);
    if (e != cudaSuccess) return fail(TSRC_E_NOMEM, "cudaMalloc of %zu weight bytes: %s", qb + mb, cudaGetErrorString(e));
    e = cudaMemset(mem, 0, qb + mb);      // the padding of partial tiles
    if (e != cudaSuccess) {
        cudaFree(mem);
        return cuda_fail(e, "cudaMemset");
    }
    tsrc_weight* w = new tsrc_weight{ctx, fmt, N, K, row0, n_rows, mem, mem + qb, qb + mb};
    ctx->weights.insert(w);
    *out = w;
    return TSRC_OK;
}

void drop_weight(tsrc_weight* w) {
    if (!w) return;
    cudaFree(w->qs);
    w->ctx->weights.erase(w);
    delete w;
}

void drop_kv(tsrc_kv* kv) {
    if (!kv) return;
    cudaFree(kv->mem);
    kv->ctx->kvs.erase(kv);
    delete kv;
}

int ensure_fa_scratch(tsrc_ctx* ctx, size_t bytes) {
    if (bytes <= ctx->fa_scratch_bytes) return TSRC_OK;
    if (ctx->fa_scratch) {
        TSRC_CUDA(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
        cudaFree(ctx->fa_scratch);
        ctx->fa_scratch = nullptr;
        ctx->fa_scratch_bytes = 0;
    }
    const size_t want = std::max<size_t>(bytes, 4u << 20);
    cudaError_t e = cudaMalloc(&ctx->fa_scratch, want);
    if (e != cudaSuccess) return fail(TSRC_E_NOMEM, "cudaMalloc of %zu FA scratch bytes: %s", want, cudaGetErrorString(e));
    ctx->fa_scratch_bytes = want;
    return TSRC_OK;
}

bool kv_geometry_ok(uint32_t n_head_kv, uint32_t D) {
    return (D == 64 || D == 128 || D == 256 || D == 512) && n_head_kv >= 1 && n_head_kv * D / 64u <= 511u;
}

}  // namespace

namespace tsrc {

int set_error(int code, const char* msg) { return fail(code, "%s", msg); }

// Makes the context's device current (for translation units that do not see tsrc_ctx) and returns
// its ordinal in *dev.
int ctx_device(const tsrc_ctx* ctx, int* dev) {
    int rc = use_device(ctx);
    if (rc) return rc;
    *dev = ctx->device;
    return TSRC_OK;
}

int weight_synth_ranges(tsrc_ctx* ctx, uint32_t fmt, uint32_t N, uint32_t K, const uint32_t* r0, const uint32_t* n,
                        uint32_t count, uint64_t seed, float sigma, tsrc_weight** out) {
    uint32_t total = 0;
    for (uint32_t i = 0; i < count; ++i) {
        if ((uint64_t)r0[i] + n[i] > N) return fail(TSRC_E_ARG, "weight_synth_ranges: range outside [0, %u)", N);
        total += n[i];
    }
    tsrc_weight* w = nullptr;
    int rc = new_weight(ctx, fmt, total, K, 0, total, &w);
    if (rc) return rc;
    cudaError_t e = cudaSuccess;
    uint32_t at = 0;
    for (uint32_t i = 0; i < count && e == cudaSuccess; ++i) {
        e = launch_synth(fmt, K, r0[i], n[i], seed, sigma, w->qs + qs_row_bytes(fmt, K) * at, w->meta + meta_row_bytes(fmt, K) * at,
                         nullptr);
        at += n[i];
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        drop_weight(w);
        return cuda_fail(e, "synth launch");
    }
    *out = w;
    return TSRC_OK;
}

int weight_interleave_halves(tsrc_ctx* ctx, tsrc_weight* w, tsrc_weight** out) {
    if (w->n_rows & 1u) return fail(TSRC_E_ARG, "weight_interleave_halves: odd row count");
    tsrc_weight* o = nullptr;
    int rc = new_weight(ctx, w->fmt, w->N, w->K, w->row0, w->n_rows, &o);
    if (rc) return rc;
    const size_t qr = qs_row_bytes(w->fmt, w->K), mr = meta_row_bytes(w->fmt, w->K), h = w->n_rows / 2u;
    cudaError_t e = cudaMemcpy2D(o->qs, 2u * qr, w->qs, qr, qr, h, cudaMemcpyDeviceToDevice);
    if (e == cudaSuccess) e = cudaMemcpy2D(o->qs + qr, 2u * qr, w->qs + h * qr, qr, qr, h, cudaMemcpyDeviceToDevice);
    if (e == cudaSuccess) e = cudaMemcpy2D(o->meta, 2u * mr, w->meta, mr, mr, h, cudaMemcpyDeviceToDevice);
    if (e == cudaSuccess) e = cudaMemcpy2D(o->meta + mr, 2u * mr, w->meta + h * mr, mr, mr, h, cudaMemcpyDeviceToDevice);
    if (e != cudaSuccess) {
        drop_weight(o);
        return cuda_fail(e, "weight_interleave_halves");
    }
    drop_weight(w);
    *out = o;
    return TSRC_OK;
}

int weight_rows(const tsrc_weight* w, uint32_t* N, uint32_t* row0, uint32_t* n_rows) {
    *N = w->N;
    *row0 = w->row0;
    *n_rows = w->n_rows;
    return TSRC_OK;
}

// The argument checks of a MUL_MAT call (the same rules as tsrc_mul_mat) and the per-call launch
// fields; for entry points that run the kernels with their own activation scratch.
int mm_check(tsrc_ctx* ctx, const tsrc_weight* w, const float* x, uint32_t T, uint32_t* x_stride, float* y, uint32_t* y_stride,
             const float* add, uint32_t add_stride, uint32_t flags, float s0, float s1, MvArgs* base, uint32_t* fmt,
             const char* who) {
    if (!ctx || !w || !x || !y) return fail(TSRC_E_ARG, "%s: NULL argument", who);
    if (w->ctx != ctx) return fail(TSRC_E_ARG, "%s: the weight belongs to another context", who);
    if (T == 0) {                        // nothing to do, and no further checks (as tsrc_mul_mat)
        *fmt = w->fmt;
        return TSRC_OK;
    }
    if (flags & ~(TSRC_MM_ADD | TSRC_MM_SCALE | TSRC_MM_SOFTCAP)) return fail(TSRC_E_ARG, "%s: undefined flag bits 0x%x", who, flags);
    if ((flags & TSRC_MM_ADD) && (flags & (TSRC_MM_SCALE | TSRC_MM_SOFTCAP)))
        return fail(TSRC_E_ARG, "%s: an addend cannot be combined with SCALE or SOFTCAP", who);
    if ((flags & TSRC_MM_SCALE) && (flags & TSRC_MM_SOFTCAP)) return fail(TSRC_E_ARG, "%s: SCALE and SOFTCAP are exclusive", who);
    if ((flags & TSRC_MM_ADD) && !add) return fail(TSRC_E_ARG, "%s: TSRC_MM_ADD without an addend", who);
    if (*x_stride == 0) *x_stride = w->K;
    if (*y_stride == 0) *y_stride = w->n_rows;
    if (*x_stride < w->K || *y_stride < w->n_rows) return fail(TSRC_E_ARG, "%s: a stride is shorter than its row", who);
    if ((flags & TSRC_MM_ADD) && add_stride != 0 && add_stride < w->n_rows) return fail(TSRC_E_ARG, "%s: addend stride", who);
    int rc = use_device(ctx);
    if (rc) return rc;
    *fmt = w->fmt;
    MvArgs a{};
    a.qs = w->qs;
    a.meta = w->meta;
    a.n_rows = w->n_rows;
    a.K = w->K;
    a.y_stride = *y_stride;
    a.add_stride = add_stride;
    a.flags = flags;
    a.s0 = daz_host(s0);
    a.s1 = daz_host(s1);
    *base = a;
    return TSRC_OK;
}

int mul_mat_rms_swiglu(tsrc_ctx* ctx, const tsrc_weight* w, const float* x, const float* norm_w, float eps, float inv_n,
                       float* y, void* stream) {
    MvArgs a{};
    uint32_t fmt = 0, x_stride = 0, y_stride = 0;
    int rc = mm_check(ctx, w, x, 1, &x_stride, y, &y_stride, nullptr, 0, 0u, 1.0f, 1.0f, &a, &fmt, "mul_mat_rms_swiglu");
    if (rc != TSRC_OK) return rc;
    if (w->n_rows & 1u) return fail(TSRC_E_ARG, "mul_mat_rms_swiglu: odd row count");
    a.x = x;
    a.x_stride = x_stride;
    a.T = 1;
    a.y = y;
    a.rms = 1u;
    a.rms_w = norm_w;
    a.rms_eps = daz_host(eps);
    a.rms_inv_n = daz_host(inv_n);
    a.swiglu_pairs = 1u;
    cudaError_t e = launch_matvec(fmt, a, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? TSRC_OK : cuda_fail(e, "matvec launch");
}

}  // namespace tsrc

namespace tsrc {
// the planes of a cache for a fused ROPE + KVST launch (tsrc_model.cu)
int kv_fill_planes(const tsrc_kv* kv, RopeKvst* a) {
    if (!kv) return TSRC_E_ARG;
    a->n_head_kv = kv->n_head_kv;
    a->n_cells = kv->n_alloc;
    a->kq = kv->q[TSRC_KV_K];
    a->vq = kv->q[TSRC_KV_V];
    a->kd = kv->d[TSRC_KV_K];
    a->vd = kv->d[TSRC_KV_V];
    return kv_error_flag(&a->err) == cudaSuccess ? TSRC_OK : fail(TSRC_E_CUDA, "KVST error flag");
}
uint32_t kv_cells(const tsrc_kv* kv) { return kv->n_cells; }
}  // namespace tsrc

extern "C" {

const char* tsrc_last_error(void) { return g_err.c_str(); }

const char* tsrc_version(void) { return "tsrc 0.1 sm_100a"; }

int tsrc_open(int device, tsrc_ctx** out) {
    if (!out) return fail(TSRC_E_ARG, "tsrc_open: NULL output handle");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) return fail(TSRC_E_NODEV, "no CUDA device (%s)", cudaGetErrorString(e));
    if (device < 0 || device >= n) return fail(TSRC_E_NODEV, "device %d not in [0, %d)", device, n);
    tsrc_ctx* ctx = new tsrc_ctx();
    ctx->device = device;
    e = cudaGetDeviceProperties(&ctx->prop, device);
    if (e != cudaSuccess) {
        delete ctx;
        return cuda_fail(e, "cudaGetDeviceProperties");
    }
    if (ctx->prop.major != 10) {
        const int maj = ctx->prop.major, mnr = ctx->prop.minor;
        delete ctx;
        return fail(TSRC_E_NODEV, "device %d is sm_%d%d; this library is built for sm_100a only", device, maj, mnr);
    }
    e = cudaSetDevice(device);
    if (e != cudaSuccess) {
        delete ctx;
        return cuda_fail(e, "cudaSetDevice");
    }
    *out = ctx;
    return TSRC_OK;
}

int tsrc_close(tsrc_ctx* ctx) {
    if (!ctx) return fail(TSRC_E_ARG, "tsrc_close: NULL context");
    use_device(ctx);
    cudaDeviceSynchronize();
    while (!ctx->weights.empty()) drop_weight(*ctx->weights.begin());
    while (!ctx->kvs.empty()) drop_kv(*ctx->kvs.begin());
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->fa_scratch) cudaFree(ctx->fa_scratch);
    delete ctx;
    return TSRC_OK;
}

int tsrc_sync(tsrc_ctx* ctx, void* stream) {
    if (!ctx) return fail(TSRC_E_ARG, "tsrc_sync: NULL context");
    int rc = use_device(ctx);
    if (rc) return rc;
    cudaError_t e = stream ? cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) : cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "synchronize");
    uint32_t code = 0;
    e = tsrc::matvec_error(&code, true);
    if (e != cudaSuccess) return cuda_fail(e, "reading the kernel error flag");
    if (code == 5) return fail(TSRC_E_ARG, "tsrc_mul_mat_id: an expert id outside [0, n_exp) (those pairs were not computed)");
    if (code) return fail(TSRC_E_DEVICE, "a matvec kernel gave up a bounded wait (code %u%s)", code,
                          code == 2 ? ": a team peer did not signal its step"
                                    : code == 3 ? ": a weight copy into shared memory did not complete" : "");
    e = tsrc::tc_error(&code, true);
    if (e != cudaSuccess) return cuda_fail(e, "reading the tensor-core kernel error flag");
    if (code) return fail(TSRC_E_DEVICE, "a tensor-core MUL_MAT kernel gave up waiting for its MMA (code %u)", code);
    e = tsrc::kv_error(&code, true);
    if (e != cudaSuccess) return cuda_fail(e, "reading the KV error flag");
    if (code) return fail(TSRC_E_ARG, "tsrc_kv_set_rows: a cell index outside the cache (those rows were not stored)");
    e = tsrc::vu_error(&code, true);
    if (e != cudaSuccess) return cuda_fail(e, "reading the vector-kind error flag");
    if (code) return fail(TSRC_E_ARG, "tsrc_get_rows: a token id outside the weight (that row was not written)");
    return TSRC_OK;
}

// ---- vector kinds ---------------------------------------------------------------------------------
int tsrc_rms_norm(tsrc_ctx* ctx, const float* x, uint32_t x_stride, float* y, uint32_t y_stride, const float* w, uint32_t n,
                  uint32_t rows, float eps, float inv_n, void* stream) {
    if (!ctx || !x || !y) return fail(TSRC_E_ARG, "tsrc_rms_norm: NULL argument");
    if (n == 0 || rows == 0) return TSRC_OK;
    if (x_stride == 0) x_stride = n;
    if (y_stride == 0) y_stride = n;
    if (x_stride < n || y_stride < n) return fail(TSRC_E_ARG, "tsrc_rms_norm: stride below n");
    if (n > 51200u) return fail(TSRC_E_SHAPE, "tsrc_rms_norm: n %u above 51200 (one row in shared memory)", n);
    int rc = use_device(ctx);
    if (rc) return rc;
    cudaError_t e = tsrc::launch_rms_norm(x, x_stride, y, y_stride, w, n, rows, daz_host(eps), daz_host(inv_n),
                                          static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? TSRC_OK : cuda_fail(e, "rms_norm launch");
}

int tsrc_mul_mat_rms(tsrc_ctx* ctx, const tsrc_weight* w, const float* x, const float* norm_w, float eps, float inv_n, float* y,
                     const float* add, uint32_t flags, float s0, float s1, void* stream) {
    tsrc::MvArgs a{};
    uint32_t fmt = 0, x_stride = 0, y_stride = 0;
    int rc = tsrc::mm_check(ctx, w, x, 1, &x_stride, y, &y_stride, add, 0, flags, s0, s1, &a, &fmt, "tsrc_mul_mat_rms");
    if (rc != TSRC_OK) return rc;
    a.x = x;
    a.x_stride = x_stride;
    a.T = 1;
    a.y = y;
    a.add = (flags & TSRC_MM_ADD) ? add : nullptr;
    a.rms = 1u;
    a.rms_w = norm_w;
    a.rms_eps = daz_host(eps);
    a.rms_inv_n = daz_host(inv_n);
    cudaError_t e = tsrc::launch_matvec(fmt, a, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? TSRC_OK : cuda_fail(e, "matvec launch");
}

int tsrc_rope(tsrc_ctx* ctx, const float* x, uint32_t x_stride, float* y, uint32_t y_stride, const int32_t* pos, uint32_t T,
              uint32_t n_heads, uint32_t head_dim, uint32_t n_dims, uint32_t mode, float ts, float attn_factor, void* stream) {
    if (!ctx || !x || !y || !pos) return fail(TSRC_E_ARG, "tsrc_rope: NULL argument");
    if (mode > TSRC_ROPE_NEOX) return fail(TSRC_E_ARG, "tsrc_rope: undefined mode %u", mode);
    if (head_dim == 0 || (head_dim & 15u) || head_dim > 1024u) return fail(TSRC_E_ARG, "tsrc_rope: head_dim %u", head_dim);
    if (n_dims == 0 || n_dims > head_dim || n_dims % (mode == TSRC_ROPE_NEOX ? 32u : 16u))
        return fail(TSRC_E_ARG, "tsrc_rope: n_dims %u", n_dims);
    if (T == 0 || n_heads == 0) return TSRC_OK;
    const uint32_t row = n_heads * head_dim;
    if (x_stride == 0) x_stride = row;
    if (y_stride == 0) y_stride = row;
    if (x_stride < row || y_stride < row) return fail(TSRC_E_ARG, "tsrc_rope: stride below n_heads * head_dim");
    int rc = use_device(ctx);
    if (rc) return rc;
    cudaError_t e = tsrc::launch_rope(x, x_stride, y, y_stride, pos, T, n_heads, head_dim, n_dims, mode, daz_host(ts),
                                      daz_host(attn_factor), static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? TSRC_OK : cuda_fail(e, "rope launch");
}

int tsrc_vop(tsrc_ctx* ctx, uint32_t func, const float* a, uint32_t a_stride, const float* b, uint32_t b_stride, float* y,
             uint32_t y_stride, uint32_t n, uint32_t rows, void* stream) {
    if (!ctx || !a || !y) return fail(TSRC_E_ARG, "tsrc_vop: NULL argument");
    if (func != TSRC_VOP_ADD && func != TSRC_VOP_MUL && func != TSRC_VOP_SILU && func != TSRC_VOP_SWIGLU)
        return fail(TSRC_E_ARG, "tsrc_vop: function %u not supported", func);
    if (func != TSRC_VOP_SILU && !b) return fail(TSRC_E_ARG, "tsrc_vop: function %u reads b", func);
    if (n == 0 || rows == 0) return TSRC_OK;
    if (a_stride == 0) a_stride = n;
    if (b_stride == 0) b_stride = n;
    if (y_stride == 0) y_stride = n;
    if (a_stride < n || y_stride < n || (b && b_stride < n)) return fail(TSRC_E_ARG, "tsrc_vop: stride below n");
    int rc = use_device(ctx);
    if (rc) return rc;
    cudaError_t e = tsrc::launch_vop(func, a, a_stride, func == TSRC_VOP_SILU ? nullptr : b, b_stride, y, y_stride, n, rows,
                                     static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? TSRC_OK : cuda_fail(e, "vop launch");
}

int tsrc_get_rows(tsrc_ctx* ctx, const tsrc_weight* w, const int32_t* ids, uint32_t T, float* y, uint32_t y_stride, void* stream) {
    if (!ctx || !w || !ids || !y) return fail(TSRC_E_ARG, "tsrc_get_rows: NULL argument");
    if (w->ctx != ctx) return fail(TSRC_E_ARG, "tsrc_get_rows: the weight belongs to another context");
    if (T == 0) return TSRC_OK;
    if (y_stride == 0) y_stride = w->K;
    if (y_stride < w->K) return fail(TSRC_E_ARG, "tsrc_get_rows: stride below K");
    int rc = use_device(ctx);
    if (rc) return rc;
    cudaError_t e = tsrc::launch_get_rows(w->fmt, w->qs, w->meta, w->n_rows, w->K, ids, T, y, y_stride,
                                          static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? TSRC_OK : cuda_fail(e, "get_rows launch");
}

int tsrc_weight_upload_device(tsrc_ctx* ctx, uint32_t fmt, const void* ggml_rows_dev, uint32_t N, uint32_t K, uint32_t row0,
                              uint32_t n_rows, void* stream, tsrc_weight** out) {
    if (!ggml_rows_dev) return fail(TSRC_E_ARG, "tsrc_weight_upload_device: NULL rows");
    if (fmt == TSRC_FMT_Q4_K && (reinterpret_cast<uintptr_t>(ggml_rows_dev) & 15u))
        return fail(TSRC_E_ARG, "tsrc_weight_upload_device: Q4_K rows must be 16-byte aligned in device memory");
    tsrc_weight* w = nullptr;
    int rc = new_weight(ctx, fmt, N, K, row0, n_rows, &w);
    if (rc) return rc;
    cudaError_t e = tsrc::launch_repack(fmt, static_cast<const uint8_t*>(ggml_rows_dev), n_rows, K, w->qs, w->meta,
                                        static_cast<cudaStream_t>(stream));
    // the matvec streams weights before it waits on earlier kernels: the weight must be complete
    if (e == cudaSuccess) e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        drop_weight(w);
        return cuda_fail(e, "repack launch");
    }
    *out = w;
    return TSRC_OK;
}

int tsrc_weight_upload(tsrc_ctx* ctx, uint32_t fmt, const void* ggml_rows, uint32_t N, uint32_t K, uint32_t row0,
                       uint32_t n_rows, tsrc_weight** out) {
    if (!ctx || !ggml_rows || !out) return fail(TSRC_E_ARG, "tsrc_weight_upload: NULL argument");
    if (const char* why = shape_reason(fmt, N, K, 1)) return fail(TSRC_E_SHAPE, "%s", why);
    if (n_rows == 0 || (uint64_t)row0 + n_rows > N) return fail(TSRC_E_ARG, "row shard outside the tensor");
    int rc = use_device(ctx);
    if (rc) return rc;
    tsrc_weight* w = nullptr;
    rc = new_weight(ctx, fmt, N, K, row0, n_rows, &w);
    if (rc) return rc;
    // stage in pieces of at most 256 MiB of ggml rows
    const size_t rb = ggml_row_bytes(fmt, K);
    const uint32_t rows_per = (uint32_t)std::max<size_t>(1, (256u << 20) / rb);
    uint8_t* stage = nullptr;
    const size_t sb = (size_t)std::min<uint32_t>(rows_per, n_rows) * rb;
    cudaError_t e = cudaMalloc(&stage, sb);
    if (e != cudaSuccess) {
        drop_weight(w);
        return fail(TSRC_E_NOMEM, "cudaMalloc of %zu staging bytes: %s", sb, cudaGetErrorString(e));
    }
    for (uint32_t r = 0; r < n_rows && e == cudaSuccess; r += rows_per) {
        const uint32_t nr = std::min(rows_per, n_rows - r);
        e = cudaMemcpy(stage, static_cast<const uint8_t*>(ggml_rows) + (size_t)r * rb, (size_t)nr * rb, cudaMemcpyHostToDevice);
        if (e == cudaSuccess)
            e = tsrc::launch_repack(fmt, stage, nr, K, w->qs + qs_row_bytes(fmt, K) * r, w->meta + meta_row_bytes(fmt, K) * r, 0);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
    }
    cudaFree(stage);
    if (e != cudaSuccess) {
        drop_weight(w);
        return cuda_fail(e, "weight upload");
    }
    *out = w;
    return TSRC_OK;
}

int tsrc_weight_synth(tsrc_ctx* ctx, uint32_t fmt, uint32_t N, uint32_t K, uint32_t row0, uint32_t n_rows, uint64_t seed,
                      float sigma, void* stream, tsrc_weight** out) {
    tsrc_weight* w = nullptr;
    int rc = new_weight(ctx, fmt, N, K, row0, n_rows, &w);
    if (rc) return rc;
    cudaError_t e = tsrc::launch_synth(fmt, K, row0, n_rows, seed, sigma, w->qs, w->meta, static_cast<cudaStream_t>(stream));
    if (e == cudaSuccess) e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        drop_weight(w);
        return cuda_fail(e, "synth launch");
    }
    *out = w;
    return TSRC_OK;
}

int tsrc_weight_download(const tsrc_weight* w, void* ggml_rows) {
    if (!w || !ggml_rows) return fail(TSRC_E_ARG, "tsrc_weight_download: NULL argument");
    int rc = use_device(w->ctx);
    if (rc) return rc;
    const size_t bytes = ggml_row_bytes(w->fmt, w->K) * w->n_rows;
    uint8_t* stage = nullptr;
    cudaError_t e = cudaMalloc(&stage, bytes);
    if (e != cudaSuccess) return fail(TSRC_E_NOMEM, "cudaMalloc of %zu staging bytes", bytes);
    e = tsrc::launch_unrepack(w->fmt, w->qs, w->meta, w->n_rows, w->K, stage, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(ggml_rows, stage, bytes, cudaMemcpyDeviceToHost);
    cudaFree(stage);
    if (e != cudaSuccess) return cuda_fail(e, "weight download");
    return TSRC_OK;
}

int tsrc_weight_info(const tsrc_weight* w, uint32_t* fmt, uint32_t* N, uint32_t* K, uint32_t* row0, uint32_t* n_rows,
                     uint64_t* device_bytes) {
    if (!w) return fail(TSRC_E_ARG, "tsrc_weight_info: NULL weight");
    if (fmt) *fmt = w->fmt;
    if (N) *N = w->N;
    if (K) *K = w->K;
    if (row0) *row0 = w->row0;
    if (n_rows) *n_rows = w->n_rows;
    if (device_bytes) *device_bytes = w->bytes;
    return TSRC_OK;
}

int tsrc_weight_free(tsrc_weight* w) {
    if (!w) return fail(TSRC_E_ARG, "tsrc_weight_free: NULL weight");
    use_device(w->ctx);
    cudaDeviceSynchronize();
    drop_weight(w);
    return TSRC_OK;
}

const char* tsrc_mul_mat_unsupported(uint32_t fmt, uint64_t N, uint64_t K, uint64_t T) { return shape_reason(fmt, N, K, T); }

// MUL_MAT_ID (expert-routed MUL_MAT): one token per (token, slot) pair through the one-token
// kernel, the pair's expert chosen on the device from ids
static int mul_mat_id_impl(tsrc_ctx* ctx, const tsrc_weight* w, uint32_t n_exp, const float* x, uint32_t x_slots,
                           uint32_t x_slot_stride, uint32_t x_tok_stride, const int32_t* ids, uint32_t ids_stride, uint32_t n_used,
                           uint32_t T, float* y, uint32_t y_slot_stride, uint32_t y_tok_stride, void* stream) {
    if (!ctx || !w || !x || !ids || !y) return fail(TSRC_E_ARG, "tsrc_mul_mat_id: NULL argument");
    if (w->ctx != ctx) return fail(TSRC_E_ARG, "tsrc_mul_mat_id: the weight belongs to another context");
    if (T == 0) return TSRC_OK;
    if (n_exp == 0 || n_used == 0 || w->row0 != 0 || w->n_rows != w->N || w->N % n_exp)
        return fail(TSRC_E_ARG, "tsrc_mul_mat_id: the weight must be whole and hold n_exp experts of equal row counts");
    if (x_slots != 1u && x_slots != n_used) return fail(TSRC_E_ARG, "tsrc_mul_mat_id: x_slots must be 1 or n_used");
    if ((uint64_t)T * n_used > 65535u) return fail(TSRC_E_SHAPE, "tsrc_mul_mat_id: more than 65535 (token, slot) pairs");
    if (std::getenv("TSRC_MV_LEGACY")) return fail(TSRC_E_SHAPE, "tsrc_mul_mat_id: not available with TSRC_MV_LEGACY");
    const uint32_t K = w->K, fmt = w->fmt, Ne = w->N / n_exp;
    if (const char* why = tsrc_mul_mat_unsupported(fmt, Ne, K, 1))
        return fail(TSRC_E_SHAPE, "tsrc_mul_mat_id: %s", why);
    if (x_slot_stride == 0) x_slot_stride = K;
    if (x_tok_stride == 0) x_tok_stride = x_slots * x_slot_stride;
    if (ids_stride == 0) ids_stride = n_used;
    if (y_slot_stride == 0) y_slot_stride = Ne;
    if (y_tok_stride == 0) y_tok_stride = n_used * y_slot_stride;
    if ((x_slots > 1u && x_slot_stride < K) || (T > 1u && x_tok_stride < K) || ids_stride < n_used ||
        (n_used > 1u && y_slot_stride < Ne) || (T > 1u && y_tok_stride < Ne))
        return fail(TSRC_E_ARG, "tsrc_mul_mat_id: a stride is shorter than its row");
    int rc = use_device(ctx);
    if (rc) return rc;
    tsrc::MvArgs a{};
    a.qs = w->qs;
    a.meta = w->meta;
    a.n_rows = Ne;
    a.K = K;
    a.x = x;
    a.x_stride = K;
    a.T = 1;
    a.y = y;
    a.y_stride = Ne;
    a.ids = ids;
    a.moe_pairs = T * n_used;
    a.n_used = n_used;
    a.n_exp = n_exp;
    a.ids_stride = ids_stride;
    a.x_slots = x_slots;
    a.x_slot = x_slot_stride;
    a.x_tok = x_tok_stride;
    a.y_slot = y_slot_stride;
    a.y_tok = y_tok_stride;
    cudaError_t e = tsrc::launch_matvec(fmt, a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "MUL_MAT_ID launch");
    return TSRC_OK;
}

static int mul_mat_impl(tsrc_ctx* ctx, const tsrc_weight* w, const float* x, uint32_t T, uint32_t x_stride, float* y,
                        uint32_t y_stride, const float* add, uint32_t add_stride, uint32_t flags, float s0, float s1,
                        int32_t* isum_out, void* stream) {
    if (!ctx || !w || !x || !y) return fail(TSRC_E_ARG, "tsrc_mul_mat: NULL argument");
    if (w->ctx != ctx) return fail(TSRC_E_ARG, "tsrc_mul_mat: the weight belongs to another context");
    if (T == 0) return TSRC_OK;
    if (flags & ~(TSRC_MM_ADD | TSRC_MM_SCALE | TSRC_MM_SOFTCAP)) return fail(TSRC_E_ARG, "tsrc_mul_mat: undefined flag bits 0x%x", flags);
    if ((flags & TSRC_MM_ADD) && (flags & (TSRC_MM_SCALE | TSRC_MM_SOFTCAP)))
        return fail(TSRC_E_ARG, "tsrc_mul_mat: an addend cannot be combined with SCALE or SOFTCAP");
    if ((flags & TSRC_MM_SCALE) && (flags & TSRC_MM_SOFTCAP)) return fail(TSRC_E_ARG, "tsrc_mul_mat: SCALE and SOFTCAP are exclusive");
    if ((flags & TSRC_MM_ADD) && !add) return fail(TSRC_E_ARG, "tsrc_mul_mat: TSRC_MM_ADD without an addend");
    const uint32_t K = w->K, fmt = w->fmt;
    if (x_stride == 0) x_stride = K;
    if (y_stride == 0) y_stride = w->n_rows;
    if (x_stride < K || y_stride < w->n_rows) return fail(TSRC_E_ARG, "tsrc_mul_mat: a stride is shorter than its row");
    if ((flags & TSRC_MM_ADD) && add_stride != 0 && add_stride < w->n_rows) return fail(TSRC_E_ARG, "tsrc_mul_mat: addend stride");
    int rc = use_device(ctx);
    if (rc) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (T == 1) {
        // decode: the matvec kernel quantizes the token itself (one launch, no scratch)
        tsrc::MvArgs a{};
        a.qs = w->qs;
        a.meta = w->meta;
        a.n_rows = w->n_rows;
        a.K = K;
        a.x = x;
        a.x_stride = x_stride;
        a.T = 1;
        a.y = y;
        a.y_stride = y_stride;
        a.add = (flags & TSRC_MM_ADD) ? add : nullptr;
        a.add_stride = add_stride;
        a.flags = flags;
        a.s0 = daz_host(s0);
        a.s1 = daz_host(s1);
        a.isum_out = isum_out;
        cudaError_t e = tsrc::launch_matvec(fmt, a, st);
        if (e != cudaSuccess) return cuda_fail(e, "matvec launch");
        return TSRC_OK;
    }
    if (T > tsrc::kMvMaxT && !isum_out && tc_enabled()) {
        // prefill: QACT of every token, then one tensor-core MUL_MAT over all of them
        const bool q4 = fmt == TSRC_FMT_Q4_K;
        rc = ensure_scratch(ctx, qa_bytes(fmt, K, T) + (q4 ? align256((size_t)T * (K / 16u)) : 0u));
        if (rc) return rc;
        int8_t* q = reinterpret_cast<int8_t*>(ctx->scratch);
        float* d = reinterpret_cast<float*>(ctx->scratch + align256((size_t)T * K));
        int16_t* bs = reinterpret_cast<int16_t*>(ctx->scratch + align256((size_t)T * K) + align256((size_t)T * (K / block_of(fmt)) * 4u));
        int8_t* bsd = q4 ? reinterpret_cast<int8_t*>(ctx->scratch + qa_bytes(fmt, K, T)) : nullptr;
        cudaError_t e = tsrc::launch_qact(fmt == TSRC_FMT_Q8_0 ? 0u : 1u, x, K, T, x_stride, q, d, bs, st, bsd);
        if (e != cudaSuccess) return cuda_fail(e, "QACT launch");
        tsrc::MvArgs a{};
        a.qs = w->qs;
        a.meta = w->meta;
        a.n_rows = w->n_rows;
        a.K = K;
        a.qx = q;
        a.dx = d;
        a.bsx = bs;
        a.bsd = bsd;
        a.T = T;
        a.y = y;
        a.y_stride = y_stride;
        a.add = (flags & TSRC_MM_ADD) ? add : nullptr;
        a.add_stride = add_stride;
        a.flags = flags;
        a.s0 = daz_host(s0);
        a.s1 = daz_host(s1);
        e = tsrc::launch_mm_tc(fmt, a, st);
        if (e != cudaSuccess) return cuda_fail(e, "tensor-core MUL_MAT launch");
        return TSRC_OK;
    }
    // several tokens: one QACT launch per tile of tokens into the scratch image, then the matvec
    uint32_t tt = tsrc::kMvMaxT;
    while (tt > 1 && tsrc::mv_smem_bytes(fmt, K, tt) > kSmemBudget) --tt;
    tt = std::min(tt, T);
    rc = ensure_scratch(ctx, qa_bytes(fmt, K, tt));
    if (rc) return rc;
    int8_t* q = reinterpret_cast<int8_t*>(ctx->scratch);
    float* d = reinterpret_cast<float*>(ctx->scratch + align256((size_t)tt * K));
    int16_t* bs = reinterpret_cast<int16_t*>(ctx->scratch + align256((size_t)tt * K) + align256((size_t)tt * (K / block_of(fmt)) * 4u));
    for (uint32_t t0 = 0; t0 < T; t0 += tt) {
        const uint32_t n = std::min(tt, T - t0);
        cudaError_t e = tsrc::launch_qact(fmt == TSRC_FMT_Q8_0 ? 0u : 1u, x + (size_t)t0 * x_stride, K, n, x_stride, q, d, bs, st);
        if (e != cudaSuccess) return cuda_fail(e, "QACT launch");
        tsrc::MvArgs a{};
        a.qs = w->qs;
        a.meta = w->meta;
        a.n_rows = w->n_rows;
        a.K = K;
        a.qx = q;
        a.dx = d;
        a.bsx = bs;
        a.T = n;
        a.y = y + (size_t)t0 * y_stride;
        a.y_stride = y_stride;
        a.add = (flags & TSRC_MM_ADD) ? add + (size_t)t0 * add_stride : nullptr;
        a.add_stride = add_stride;
        a.flags = flags;
        a.s0 = daz_host(s0);
        a.s1 = daz_host(s1);
        a.isum_out = t0 == 0 ? isum_out : nullptr;
        e = tsrc::launch_matvec(fmt, a, st);
        if (e != cudaSuccess) return cuda_fail(e, "matvec launch");
    }
    return TSRC_OK;
}

int tsrc_mvm(tsrc_ctx* ctx, const tsrc_weight* w, const int8_t* q, const float* d, const int16_t* bs, uint32_t T, float* y,
             uint32_t y_stride, const float* add, uint32_t add_stride, uint32_t flags, float s0, float s1, void* stream) {
    if (!ctx || !w || !q || !d || !y) return fail(TSRC_E_ARG, "tsrc_mvm: NULL argument");
    if (w->ctx != ctx) return fail(TSRC_E_ARG, "tsrc_mvm: the weight belongs to another context");
    if (w->fmt == TSRC_FMT_Q4_K && !bs) return fail(TSRC_E_ARG, "tsrc_mvm: Q4_K needs bs");
    if (T == 0) return TSRC_OK;
    if (T > tsrc::kMvMaxT) return fail(TSRC_E_ARG, "tsrc_mvm: T %u > %u", T, tsrc::kMvMaxT);
    if (tsrc::mv_smem_bytes(w->fmt, w->K, T) > kSmemBudget) return fail(TSRC_E_SHAPE, "tsrc_mvm: T x K too large for one launch");
    if (flags & ~(TSRC_MM_ADD | TSRC_MM_SCALE | TSRC_MM_SOFTCAP)) return fail(TSRC_E_ARG, "tsrc_mvm: undefined flag bits 0x%x", flags);
    if ((flags & TSRC_MM_ADD) && ((flags & (TSRC_MM_SCALE | TSRC_MM_SOFTCAP)) || !add))
        return fail(TSRC_E_ARG, "tsrc_mvm: ADD needs an addend and excludes SCALE / SOFTCAP");
    if ((flags & TSRC_MM_SCALE) && (flags & TSRC_MM_SOFTCAP)) return fail(TSRC_E_ARG, "tsrc_mvm: SCALE and SOFTCAP are exclusive");
    if (y_stride == 0) y_stride = w->n_rows;
    int rc = use_device(ctx);
    if (rc) return rc;
    tsrc::MvArgs a{};
    a.qs = w->qs;
    a.meta = w->meta;
    a.n_rows = w->n_rows;
    a.K = w->K;
    a.qx = q;
    a.dx = d;
    a.bsx = bs;
    a.T = T;
    a.y = y;
    a.y_stride = y_stride;
    a.add = (flags & TSRC_MM_ADD) ? add : nullptr;
    a.add_stride = add_stride;
    a.flags = flags;
    a.s0 = daz_host(s0);
    a.s1 = daz_host(s1);
    cudaError_t e = tsrc::launch_matvec(w->fmt, a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "matvec launch");
    return TSRC_OK;
}

int tsrc_mul_mat(tsrc_ctx* ctx, const tsrc_weight* w, const float* x, uint32_t T, uint32_t x_stride, float* y, uint32_t y_stride,
                 const float* add, uint32_t add_stride, uint32_t flags, float s0, float s1, void* stream) {
    return mul_mat_impl(ctx, w, x, T, x_stride, y, y_stride, add, add_stride, flags, s0, s1, nullptr, stream);
}

int tsrc_dev_alloc(tsrc_ctx* ctx, size_t bytes, void** out) {
    if (!ctx || !out) return fail(TSRC_E_ARG, "tsrc_dev_alloc: NULL argument");
    *out = nullptr;
    int rc = use_device(ctx);
    if (rc) return rc;
    if (bytes == 0) return TSRC_OK;
    const cudaError_t e = cudaMalloc(out, bytes);
    if (e != cudaSuccess) return fail(TSRC_E_NOMEM, "tsrc_dev_alloc: %zu bytes: %s", bytes, cudaGetErrorString(e));
    return TSRC_OK;
}

int tsrc_dev_free(tsrc_ctx* ctx, void* p) {
    if (!ctx) return fail(TSRC_E_ARG, "tsrc_dev_free: NULL context");
    if (!p) return TSRC_OK;
    int rc = use_device(ctx);
    if (rc) return rc;
    const cudaError_t e = cudaFree(p);
    return e == cudaSuccess ? TSRC_OK : cuda_fail(e, "tsrc_dev_free");
}

int tsrc_copy(tsrc_ctx* ctx, void* dst, const void* src, size_t bytes, uint32_t to_device, void* stream) {
    if (!ctx || (bytes && (!dst || !src))) return fail(TSRC_E_ARG, "tsrc_copy: NULL argument");
    if (bytes == 0) return TSRC_OK;
    int rc = use_device(ctx);
    if (rc) return rc;
    const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, to_device ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToHost,
                                          static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? TSRC_OK : cuda_fail(e, "tsrc_copy");
}

int tsrc_mul_mat_id(tsrc_ctx* ctx, const tsrc_weight* w, uint32_t n_exp, const float* x, uint32_t x_slots, uint32_t x_slot_stride,
                    uint32_t x_tok_stride, const int32_t* ids, uint32_t ids_stride, uint32_t n_used, uint32_t T, float* y,
                    uint32_t y_slot_stride, uint32_t y_tok_stride, void* stream) {
    return mul_mat_id_impl(ctx, w, n_exp, x, x_slots, x_slot_stride, x_tok_stride, ids, ids_stride, n_used, T, y, y_slot_stride,
                           y_tok_stride, stream);
}

int tsrc_mul_mat_isums(tsrc_ctx* ctx, const tsrc_weight* w, const float* x, float* y, int32_t* isum, void* stream) {
    if (!isum) return fail(TSRC_E_ARG, "tsrc_mul_mat_isums: NULL isum");
    return mul_mat_impl(ctx, w, x, 1, 0, y, 0, nullptr, 0, 0, 1.0f, 1.0f, isum, stream);
}

int tsrc_qact(tsrc_ctx* ctx, uint32_t kind, const float* x, uint32_t K, uint32_t T, uint32_t x_stride, int8_t* q, float* d,
              int16_t* bs, void* stream) {
    if (!ctx || !x || !q || !d) return fail(TSRC_E_ARG, "tsrc_qact: NULL argument");
    if (kind > TSRC_QA_A256) return fail(TSRC_E_ARG, "tsrc_qact: kind %u", kind);
    const uint32_t bsz = kind == TSRC_QA_A32 ? 32u : 256u;
    if (K == 0 || K % bsz) return fail(TSRC_E_SHAPE, "tsrc_qact: K %u is not a positive multiple of %u", K, bsz);
    if (kind == TSRC_QA_A256 && !bs) return fail(TSRC_E_ARG, "tsrc_qact: A256 needs bs");
    if (x_stride == 0) x_stride = K;
    if (x_stride < K) return fail(TSRC_E_ARG, "tsrc_qact: x_stride < K");
    int rc = use_device(ctx);
    if (rc) return rc;
    cudaError_t e = tsrc::launch_qact(kind, x, K, T, x_stride, q, d, bs, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "QACT launch");
    return TSRC_OK;
}

// ---- KV cache and flash attention -------------------------------------------------------------

int tsrc_kv_create(tsrc_ctx* ctx, uint32_t n_head_kv, uint32_t D, uint32_t n_cells, tsrc_kv** out) {
    if (!ctx || !out) return fail(TSRC_E_ARG, "tsrc_kv_create: NULL argument");
    *out = nullptr;
    if (!kv_geometry_ok(n_head_kv, D)) return fail(TSRC_E_SHAPE, "tsrc_kv_create: head_dim must be 64/128/256/512, E / 64 <= 511");
    if (n_cells == 0 || n_cells > (1u << 30)) return fail(TSRC_E_SHAPE, "tsrc_kv_create: n_cells must be 1..2^30");
    int rc = use_device(ctx);
    if (rc) return rc;
    const uint32_t n_alloc = (n_cells + 15u) & ~15u;
    const size_t qb = align256((size_t)n_head_kv * n_alloc * D), db = align256((size_t)n_head_kv * n_alloc * (D / 32u) * 2u);
    const size_t bytes = 2u * (qb + db);
    uint8_t* mem = nullptr;
    cudaError_t e = cudaMalloc(&mem, bytes);
    if (e != cudaSuccess) return fail(TSRC_E_NOMEM, "cudaMalloc of %zu KV bytes: %s", bytes, cudaGetErrorString(e));
    e = cudaMemset(mem, 0, bytes);
    if (e != cudaSuccess) {
        cudaFree(mem);
        return cuda_fail(e, "cudaMemset");
    }
    tsrc_kv* kv = new tsrc_kv{};
    kv->ctx = ctx;
    kv->n_head_kv = n_head_kv;
    kv->D = D;
    kv->n_cells = n_cells;
    kv->n_alloc = n_alloc;
    kv->mem = mem;
    kv->bytes = bytes;
    for (int w = 0; w < 2; ++w) {
        kv->q[w] = reinterpret_cast<int8_t*>(mem + (size_t)w * (qb + db));
        kv->d[w] = reinterpret_cast<uint16_t*>(mem + (size_t)w * (qb + db) + qb);
    }
    ctx->kvs.insert(kv);
    *out = kv;
    return TSRC_OK;
}

int tsrc_kv_free(tsrc_kv* kv) {
    if (!kv) return fail(TSRC_E_ARG, "tsrc_kv_free: NULL cache");
    use_device(kv->ctx);
    cudaDeviceSynchronize();
    drop_kv(kv);
    return TSRC_OK;
}

int tsrc_kv_set_rows(tsrc_ctx* ctx, tsrc_kv* kv, uint32_t which, const float* rows, uint32_t n, uint32_t row_stride,
                     const int64_t* cells, uint32_t cell0, void* stream) {
    if (!ctx || !kv || !rows) return fail(TSRC_E_ARG, "tsrc_kv_set_rows: NULL argument");
    if (kv->ctx != ctx) return fail(TSRC_E_ARG, "tsrc_kv_set_rows: the cache belongs to another context");
    if (which > TSRC_KV_V) return fail(TSRC_E_ARG, "tsrc_kv_set_rows: which must be TSRC_KV_K or TSRC_KV_V");
    const uint32_t E = kv->n_head_kv * kv->D;
    if (row_stride == 0) row_stride = E;
    if (row_stride < E) return fail(TSRC_E_ARG, "tsrc_kv_set_rows: row_stride < E");
    if (!cells && (uint64_t)cell0 + n > kv->n_cells) return fail(TSRC_E_ARG, "tsrc_kv_set_rows: cells [%u, %u+%u) outside the cache", cell0, cell0, n);
    if (n == 0) return TSRC_OK;
    int rc = use_device(ctx);
    if (rc) return rc;
    cudaError_t e = tsrc::launch_kv_store(rows, n, row_stride, cells, cell0, kv->n_head_kv, kv->D, kv->n_alloc,
                                          which == TSRC_KV_V, kv->q[which], kv->d[which], static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "KVST launch");
    return TSRC_OK;
}

static int kv_bytes_io(tsrc_kv* kv, uint32_t which, void* host, uint32_t cell0, uint32_t n, bool to_device) {
    if (!kv || !host) return fail(TSRC_E_ARG, "tsrc_kv_%s_bytes: NULL argument", to_device ? "set" : "get");
    if (which > TSRC_KV_V) return fail(TSRC_E_ARG, "tsrc_kv_*_bytes: which must be TSRC_KV_K or TSRC_KV_V");
    if ((uint64_t)cell0 + n > kv->n_cells) return fail(TSRC_E_ARG, "tsrc_kv_*_bytes: cells outside the cache");
    if (n == 0) return TSRC_OK;
    int rc = use_device(kv->ctx);
    if (rc) return rc;
    const size_t bytes = (size_t)n * (kv->n_head_kv * kv->D / 32u) * 34u;
    uint8_t* stage = nullptr;
    cudaError_t e = cudaMalloc(&stage, bytes);
    if (e != cudaSuccess) return fail(TSRC_E_NOMEM, "cudaMalloc of %zu staging bytes", bytes);
    if (to_device) {
        e = cudaMemcpy(stage, host, bytes, cudaMemcpyHostToDevice);
        if (e == cudaSuccess)
            e = tsrc::launch_kv_from_ggml(stage, n, cell0, kv->n_head_kv, kv->D, kv->n_alloc, which == TSRC_KV_V, kv->q[which],
                                          kv->d[which], 0);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
    } else {
        e = cudaDeviceSynchronize();
        if (e == cudaSuccess)
            e = tsrc::launch_kv_to_ggml(kv->q[which], kv->d[which], n, cell0, kv->n_head_kv, kv->D, kv->n_alloc,
                                        which == TSRC_KV_V, stage, 0);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e == cudaSuccess) e = cudaMemcpy(host, stage, bytes, cudaMemcpyDeviceToHost);
    }
    cudaFree(stage);
    if (e != cudaSuccess) return cuda_fail(e, to_device ? "KV upload" : "KV download");
    return TSRC_OK;
}

int tsrc_kv_set_bytes(tsrc_kv* kv, uint32_t which, const void* ggml_rows, uint32_t cell0, uint32_t n) {
    return kv_bytes_io(kv, which, const_cast<void*>(ggml_rows), cell0, n, true);
}

int tsrc_kv_get_bytes(const tsrc_kv* kv, uint32_t which, void* ggml_rows, uint32_t cell0, uint32_t n) {
    return kv_bytes_io(const_cast<tsrc_kv*>(kv), which, ggml_rows, cell0, n, false);
}

}  // extern "C"

namespace tsrc {
// Everything of one FLASH_ATTN_EXT call up to the kernel launches: checks, the plan, the scratch
// layout, the H2D copies of a large plan or a GENERAL mask (queued on st); *la receives the launch
// arguments and *n_max_groups the chunk size bound the launch needs.
int fa_setup(tsrc_ctx* ctx, const tsrc_kv* kv, const float* q, uint32_t T, uint32_t n_head, uint32_t n_kv,
             const uint16_t* mask, uint32_t mask_stride, float scale, uint32_t new_lo, uint32_t new_hi,
             const tsrc_fa_cfg* cfg, float* out, cudaStream_t st, FaLaunch* la, uint32_t* n_max_groups) {
    if (!ctx || !kv || !q || !out) return fail(TSRC_E_ARG, "tsrc_flash_attn: NULL argument");
    if (kv->ctx != ctx) return fail(TSRC_E_ARG, "tsrc_flash_attn: the cache belongs to another context");
    if (n_kv > kv->n_cells) return fail(TSRC_E_ARG, "tsrc_flash_attn: n_kv %u exceeds the cache's %u cells", n_kv, kv->n_cells);
    if (mask && mask_stride < n_kv) return fail(TSRC_E_ARG, "tsrc_flash_attn: mask_stride < n_kv");
    uint32_t sb;
    std::memcpy(&sb, &scale, 4);
    if ((sb & 0x80000000u) || (sb & 0x7F800000u) == 0 || (sb & 0x7F800000u) == 0x7F800000u)
        return fail(TSRC_E_SHAPE, "FLASH_ATTN: scale must be finite, normal and > 0");
    const tsrc_fa_cfg def{4, 4, 9344, 32768, 0};
    const tsrc_fa_cfg& c = cfg ? *cfg : def;
    tsrc::FaPlanIn in{};
    in.C = c.C;
    in.t_max = c.t_max;
    in.pcap = c.pcap;
    in.k_max = c.k_max;
    if (c.plan_n_head_kv && (c.plan_n_head_kv < kv->n_head_kv || c.plan_n_head_kv % kv->n_head_kv))
        return fail(TSRC_E_ARG, "tsrc_flash_attn: plan_n_head_kv %u is not a multiple of the cache's %u KV heads",
                    c.plan_n_head_kv, kv->n_head_kv);
    in.plan_n_head_kv = c.plan_n_head_kv ? c.plan_n_head_kv : kv->n_head_kv;
    in.T = T;
    in.D = kv->D;
    in.n_head = n_head;
    in.n_head_kv = kv->n_head_kv;
    in.n_kv = n_kv;
    in.mask = mask;
    in.mask_stride = mask_stride;
    in.new_lo = new_lo;
    in.new_hi = new_hi;
    tsrc::FaPlanOut po{};
    tsrc::FaItem* items = nullptr;
    uint32_t* tiles = nullptr;
    uint32_t n_items = 0;
    const char* why = nullptr;
    int rc = tsrc::fa_plan(in, &po, &items, &n_items, &tiles, &why);
    if (rc != TSRC_OK) return fail(rc, "%s", why ? why : "FLASH_ATTN: planning failed");
    if (tsrc::fa_smem_bytes(kv->D, po.n_max_groups, c.C) > 227u * 1024u) {
        tsrc::fa_plan_free(items, tiles);
        return fail(TSRC_E_SHAPE, "FLASH_ATTN: a chunk needs more shared memory than a CTA has");
    }
    rc = use_device(ctx);
    if (rc) {
        tsrc::fa_plan_free(items, tiles);
        return rc;
    }
    const uint32_t rows_max = po.Tq0 * po.G;
    const size_t b_items = align256((size_t)n_items * sizeof(tsrc::FaItem));
    const size_t b_tiles = align256((size_t)(po.n_tiles + 1u) * 4u);
    const size_t b_oc = align256((size_t)n_items * kv->n_head_kv * c.C * rows_max * kv->D * 4u);
    const size_t b_lc = align256((size_t)n_items * kv->n_head_kv * c.C * rows_max * 4u);
    const size_t b_mk = align256((size_t)n_items * kv->n_head_kv * rows_max * 4u);
    const size_t b_m16 = po.general ? align256((size_t)T * mask_stride * 2u) : 0u;
    const size_t b_mf = po.general ? align256((size_t)T * n_kv * 4u) : 0u;
    rc = ensure_fa_scratch(ctx, b_items + b_tiles + b_oc + b_lc + b_mk + b_m16 + b_mf);
    if (rc) {
        tsrc::fa_plan_free(items, tiles);
        return rc;
    }
    uint8_t* p = ctx->fa_scratch;
    tsrc::FaLaunch& a = *la;
    a = tsrc::FaLaunch{};
    a.items = reinterpret_cast<const tsrc::FaItem*>(p);
    a.tile_items = reinterpret_cast<const uint32_t*>(p + b_items);
    a.ok = reinterpret_cast<float*>(p + b_items + b_tiles);
    a.lk = reinterpret_cast<float*>(p + b_items + b_tiles + b_oc);
    a.mk = reinterpret_cast<float*>(p + b_items + b_tiles + b_oc + b_lc);
    uint16_t* m16 = reinterpret_cast<uint16_t*>(p + b_items + b_tiles + b_oc + b_lc + b_mk);
    float* mf = reinterpret_cast<float*>(p + b_items + b_tiles + b_oc + b_lc + b_mk + b_m16);
    cudaError_t e = cudaSuccess;
    if (n_items <= tsrc::kFaInlineItems) {
        // a small plan travels in the kernel parameters (no copy: the call can be graph-captured)
        std::memcpy(a.inl_items, items, (size_t)n_items * sizeof(tsrc::FaItem));
        std::memcpy(a.inl_tiles, tiles, (size_t)(po.n_tiles + 1u) * 4u);
    } else {
        // host -> device copies of the plan: the sources are staged before cudaMemcpyAsync
        // returns, so they may be released right after
        e = cudaMemcpyAsync(const_cast<tsrc::FaItem*>(a.items), items, (size_t)n_items * sizeof(tsrc::FaItem),
                            cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(const_cast<uint32_t*>(a.tile_items), tiles, (size_t)(po.n_tiles + 1u) * 4u,
                                cudaMemcpyHostToDevice, st);
    }
    tsrc::fa_plan_free(items, tiles);
    if (e == cudaSuccess && po.general) {
        e = cudaMemcpyAsync(m16, mask, (size_t)T * mask_stride * 2u, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = tsrc::launch_fa_maskf(m16, mask_stride, T, n_kv, scale, mf, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, "FLASH_ATTN setup");
    a.q = q;
    a.T = T;
    a.n_head = n_head;
    a.n_head_kv = kv->n_head_kv;
    a.D = kv->D;
    a.G = po.G;
    a.C = c.C;
    a.n_kv = n_kv;
    a.n_cells = kv->n_alloc;
    a.kq = kv->q[0];
    a.kd = kv->d[0];
    a.vq = kv->q[1];
    a.vd = kv->d[1];
    a.maskf = po.general ? mf : nullptr;
    a.maskf_stride = n_kv;
    a.scale = scale;
    a.n_items = n_items;
    a.n_tiles = po.n_tiles;
    a.Tq0 = po.Tq0;
    a.out = out;
    *n_max_groups = po.n_max_groups;
    return TSRC_OK;
}
}  // namespace tsrc

extern "C" {

int tsrc_flash_attn(tsrc_ctx* ctx, const tsrc_kv* kv, const float* q, uint32_t T, uint32_t n_head, uint32_t n_kv,
                    const uint16_t* mask, uint32_t mask_stride, float scale, uint32_t new_lo, uint32_t new_hi,
                    const tsrc_fa_cfg* cfg, float* out, void* stream) {
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    tsrc::FaLaunch a;
    uint32_t n_max_groups = 0;
    int rc = tsrc::fa_setup(ctx, kv, q, T, n_head, n_kv, mask, mask_stride, scale, new_lo, new_hi, cfg, out, st, &a, &n_max_groups);
    if (rc) return rc;
    cudaError_t e = tsrc::launch_fa(a, n_max_groups, st);
    if (e != cudaSuccess) return cuda_fail(e, "FLASH_ATTN launch");
    return TSRC_OK;
}

}  // extern "C"
