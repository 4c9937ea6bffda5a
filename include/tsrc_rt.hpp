// tsrc_rt.hpp -- the ggml-free runtime front end over the C ABI: weight upload and y = x . W^T, as the
// reference's tsr::rt::device (jwkim04/tesseract-npu sw/rt/tsr_rt.h:66-288; its PyTorch QuantLinear binds
// it) offers them, for hosts that do not go through ggml.
//
// Numerics are the MUL_MAT path's: f32 / f16 / bf16 weights become Q8_0 at upload (to_float, then
// quantize_row_q8_0_ref), Q8_0 / Q4_K blocks are kept as they are, activations are quantized by QACT on
// the device, results are f32, every value the reference's bit for bit. K parts follow the reference
// (tsr_rt.h:30-37): a weight with K above K_MAX (32768, the release configuration; weight_options can
// force smaller parts) is stored as column ranges of at most K_MAX, and linear() accumulates the parts in
// order with one f32 add each, y = ((y_0 + y_1) + y_2) ..., each y_j the MUL_MAT row result over part j.
// N parts do not change any value (rows are independent) and are not made.
//
// Not carried over: linear_ref (the reference computes it on the host with its own simulator library;
// here that is test infrastructure, oracle/), the whole-graph API (graph_*), and the device counters of
// the FPGA transport. Thread safety: every member function takes the device's mutex.
//
// Errors: tsrc::rt::error (a std::runtime_error carrying tsrc_last_error()); invalid arguments:
// std::invalid_argument.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "tsrc.h"

namespace tsrc::rt {

class error : public std::runtime_error {
public:
    using std::runtime_error::runtime_error;
};

// Host types a weight can be uploaded from (the reference's values). Row-major [N, K], any row stride.
enum class dtype : uint32_t {
    f32 = 0,    // float32                          -> Q8_0
    f16 = 1,    // IEEE binary16 bits               -> f32 (exact) -> Q8_0
    bf16 = 2,   // bfloat16 bits                    -> f32 (exact) -> Q8_0
    q8_0 = 3,   // ggml block_q8_0, 34 B per 32     -> Q8_0 as is
    q4_k = 4,   // ggml block_q4_K, 144 B per 256   -> Q4_K as is
};

inline const char* dtype_name(dtype t) {
    switch (t) {
        case dtype::f32: return "f32";
        case dtype::f16: return "f16";
        case dtype::bf16: return "bf16";
        case dtype::q8_0: return "q8_0";
        case dtype::q4_k: return "q4_k";
    }
    return "?";
}
// TSRC_FMT_Q4_K for q4_k, TSRC_FMT_Q8_0 otherwise
inline uint32_t dtype_device_format(dtype t) { return t == dtype::q4_k ? TSRC_FMT_Q4_K : TSRC_FMT_Q8_0; }
// ggml.h's type value of a host type
inline uint32_t dtype_ggml_type(dtype t) {
    switch (t) {
        case dtype::f32: return 0u;
        case dtype::f16: return 1u;
        case dtype::bf16: return 30u;
        case dtype::q8_0: return 8u;
        case dtype::q4_k: return 12u;
    }
    return 0xFFFFFFFFu;
}
// Bytes of one packed row of K elements; 0 if K is not a whole number of blocks or t is unknown.
inline size_t dtype_row_bytes(dtype t, uint32_t K) {
    uint32_t be = 0, bb = 0, fmt = 0;
    if (tsrc_ggml_type_info(dtype_ggml_type(t), &be, &bb, &fmt) != TSRC_OK || K == 0 || K % be) return 0;
    if (K % (fmt == TSRC_FMT_Q4_K ? 256u : 32u)) return 0;
    return (size_t)(K / be) * bb;
}

struct open_options {
    int device = 0;                 // CUDA device index
};

struct weight_options {
    uint32_t max_part_rows = 0;     // accepted for compatibility; rows are never split (no value depends on it)
    uint32_t max_part_k = 0;        // 0: K parts of K_MAX; else at most this K per part (a multiple of the block)
};

struct weight_info {
    uint32_t N, K;
    dtype src;                      // host type given at upload
    uint32_t fmt;                   // TSRC_FMT_Q8_0 / TSRC_FMT_Q4_K
    uint32_t n_parts, n_part;       // always 1, N
    uint32_t k_parts;               // K parts: columns [j k_part, min((j + 1) k_part, K)), added in order
    uint32_t k_part;
    uint64_t dev_bytes;             // device memory of every part
};

struct counters {
    uint64_t linears = 0;           // linear() calls with T >= 1
    uint64_t tokens = 0;            // the sum of their T
    uint64_t launches = 0;          // MUL_MAT calls they made (one per K part)
};

using weight_handle = uint64_t;     // 0 is never a valid handle

constexpr uint32_t kKMax = 32768;   // the release configuration's K_MAX

class device {
public:
    explicit device(const open_options& o = open_options()) {
        if (tsrc_open(o.device, &ctx_) != TSRC_OK) throw error(std::string("tsrc::rt::device: ") + tsrc_last_error());
        desc_ = std::string("tsrc on CUDA device ") + std::to_string(o.device) + " (" + tsrc_version() + ")";
    }
    ~device() {
        for (auto& kv : weights_)
            for (tsrc_weight* w : kv.second.parts) tsrc_weight_free(w);
        for (void* p : {xd_, ya_, yb_})
            if (p) tsrc_dev_free(ctx_, p);
        tsrc_close(ctx_);
    }
    device(const device&) = delete;
    device& operator=(const device&) = delete;

    const char* description() const { return desc_.c_str(); }
    tsrc_ctx* context() const { return ctx_; }     // the C ABI context (MUL_MAT, KV caches, ... on device data)

    // nullptr if a weight of this type and shape can be uploaded, else the reason (a static string)
    const char* unsupported_reason(dtype t, uint32_t N, uint32_t K, const weight_options& o = weight_options()) const {
        if (dtype_ggml_type(t) == 0xFFFFFFFFu) return "unknown dtype";
        if (N == 0) return "N must be at least 1";
        if (dtype_row_bytes(t, K) == 0) return "K is not a whole number of the format's blocks";
        const uint32_t kp = k_part_of(t, K, o);
        if (kp == 0) return "max_part_k is not a multiple of the format's block";
        return tsrc_mul_mat_unsupported(dtype_device_format(t), N, kp, 1);
    }

    // Upload W [N, K] (row r at data + r * row_stride_bytes; 0 = packed rows). Returns a handle (never 0).
    weight_handle upload(dtype t, const void* data, uint32_t N, uint32_t K, size_t row_stride_bytes = 0,
                         const weight_options& o = weight_options()) {
        std::lock_guard<std::mutex> lk(mu_);
        if (!data) throw std::invalid_argument("tsrc::rt::device::upload: NULL data");
        if (const char* why = unsupported_reason(t, N, K, o))
            throw std::invalid_argument(std::string("tsrc::rt::device::upload: ") + why);
        const size_t rb = dtype_row_bytes(t, K);
        if (row_stride_bytes == 0) row_stride_bytes = rb;
        if (row_stride_bytes < rb) throw std::invalid_argument("tsrc::rt::device::upload: row stride shorter than a row");
        uint32_t be = 0, bb = 0, fmt = 0;
        tsrc_ggml_type_info(dtype_ggml_type(t), &be, &bb, &fmt);
        Weight w;
        w.info = weight_info{N, K, t, fmt, 1u, N, 0u, k_part_of(t, K, o), 0u};
        const uint32_t kp = w.info.k_part;
        w.info.k_parts = (K + kp - 1u) / kp;
        const uint8_t* src = static_cast<const uint8_t*>(data);
        std::vector<uint8_t> part;
        for (uint32_t j = 0; j < w.info.k_parts; ++j) {
            const uint32_t k0 = j * kp, k1 = K - k0 < kp ? K : k0 + kp;
            const size_t off = (size_t)(k0 / be) * bb, len = (size_t)((k1 - k0) / be) * bb;
            part.resize(len * N);
            for (uint32_t r = 0; r < N; ++r) std::memcpy(part.data() + (size_t)r * len, src + (size_t)r * row_stride_bytes + off, len);
            tsrc_weight* h = nullptr;
            if (tsrc_weight_upload_ggml(ctx_, dtype_ggml_type(t), part.data(), N, k1 - k0, 0, N, &h) != TSRC_OK) {
                for (tsrc_weight* p : w.parts) tsrc_weight_free(p);
                throw error(std::string("tsrc::rt::device::upload: ") + tsrc_last_error());
            }
            uint64_t bytes = 0;
            tsrc_weight_info(h, nullptr, nullptr, nullptr, nullptr, nullptr, &bytes);
            w.info.dev_bytes += bytes;
            w.parts.push_back(h);
        }
        const weight_handle id = ++next_;
        weights_.emplace(id, std::move(w));
        return id;
    }

    void free_weight(weight_handle h) {
        std::lock_guard<std::mutex> lk(mu_);
        auto it = weights_.find(h);
        if (it == weights_.end()) throw std::invalid_argument("tsrc::rt::device::free_weight: unknown handle");
        for (tsrc_weight* w : it->second.parts) tsrc_weight_free(w);
        weights_.erase(it);
    }

    weight_info info(weight_handle h) const {
        std::lock_guard<std::mutex> lk(mu_);
        return find(h).info;
    }

    // Rows [r0, r1) as stored on the device, in ggml blocks of the device format (Q8_0: K/32 x 34 B, Q4_K:
    // K/256 x 144 B per row, rows packed at dst): for f32 / f16 / bf16 weights the bytes of the load-time
    // conversion, for q8_0 / q4_k the uploaded bytes.
    void read_blocks(weight_handle h, uint32_t r0, uint32_t r1, void* dst) const {
        std::lock_guard<std::mutex> lk(mu_);
        const Weight& w = find(h);
        if (r0 > r1 || r1 > w.info.N || (!dst && r1 > r0)) throw std::invalid_argument("tsrc::rt::device::read_blocks: bad rows");
        const uint32_t bs = w.info.fmt == TSRC_FMT_Q4_K ? 256u : 32u, bb = w.info.fmt == TSRC_FMT_Q4_K ? 144u : 34u;
        const size_t row = (size_t)(w.info.K / bs) * bb;
        std::vector<uint8_t> all;
        size_t off = 0;
        for (uint32_t j = 0; j < w.info.k_parts; ++j) {
            const uint32_t k0 = j * w.info.k_part, kn = w.info.K - k0 < w.info.k_part ? w.info.K - k0 : w.info.k_part;
            const size_t len = (size_t)(kn / bs) * bb;
            all.resize(len * w.info.N);
            if (tsrc_weight_download(w.parts[j], all.data()) != TSRC_OK)
                throw error(std::string("tsrc::rt::device::read_blocks: ") + tsrc_last_error());
            for (uint32_t r = r0; r < r1; ++r)
                std::memcpy(static_cast<uint8_t*>(dst) + (size_t)(r - r0) * row + off, all.data() + (size_t)r * len, len);
            off += len;
        }
    }

    // y[t, n] = sum_k W[n, k] x[t, k] for t < T (host memory): x row t at x + t * x_stride floats (0 = K),
    // y row t at y + t * y_stride floats (0 = N); only y[t, 0..N) is written. T = 0: no-op. Synchronous.
    void linear(weight_handle h, const float* x, uint32_t T, float* y, size_t x_stride = 0, size_t y_stride = 0) {
        std::lock_guard<std::mutex> lk(mu_);
        const Weight& w = find(h);
        if (T == 0) return;
        if (!x || !y) throw std::invalid_argument("tsrc::rt::device::linear: NULL x or y");
        const uint32_t N = w.info.N, K = w.info.K;
        if (x_stride == 0) x_stride = K;
        if (y_stride == 0) y_stride = N;
        if (x_stride < K || y_stride < N) throw std::invalid_argument("tsrc::rt::device::linear: a stride is shorter than its row");
        reserve((size_t)T * K, (size_t)T * N);
        // x rows packed on the device
        if (x_stride == K) {
            check(tsrc_copy(ctx_, xd_, x, (size_t)T * K * sizeof(float), 1u, nullptr), "copy of x");
        } else {
            std::vector<float> xp((size_t)T * K);
            for (uint32_t t = 0; t < T; ++t) std::memcpy(xp.data() + (size_t)t * K, x + (size_t)t * x_stride, (size_t)K * sizeof(float));
            check(tsrc_copy(ctx_, xd_, xp.data(), xp.size() * sizeof(float), 1u, nullptr), "copy of x");
        }
        // the K parts in order: y_0, then y = y_j + y (one f32 add each, the MUL_MAT addend epilogue)
        float* cur = static_cast<float*>(ya_);
        float* other = static_cast<float*>(yb_);
        for (uint32_t j = 0; j < w.info.k_parts; ++j) {
            const float* xj = static_cast<const float*>(xd_) + (size_t)j * w.info.k_part;
            float* out = j == 0 ? cur : other;
            check(tsrc_mul_mat(ctx_, w.parts[j], xj, T, K, out, N, j == 0 ? nullptr : cur, N, j == 0 ? 0u : TSRC_MM_ADD, 1.0f, 1.0f,
                               nullptr),
                  "MUL_MAT");
            if (j) std::swap(cur, other);
            ++counters_.launches;
        }
        std::vector<float> yh((size_t)T * N);
        check(tsrc_copy(ctx_, yh.data(), cur, yh.size() * sizeof(float), 0u, nullptr), "copy of y");
        check(tsrc_sync(ctx_, nullptr), "linear");
        for (uint32_t t = 0; t < T; ++t) std::memcpy(y + (size_t)t * y_stride, yh.data() + (size_t)t * N, (size_t)N * sizeof(float));
        ++counters_.linears;
        counters_.tokens += T;
    }

    counters get_counters() const {
        std::lock_guard<std::mutex> lk(mu_);
        return counters_;
    }

private:
    struct Weight {
        weight_info info;
        std::vector<tsrc_weight*> parts;
    };

    static uint32_t k_part_of(dtype t, uint32_t K, const weight_options& o) {
        const uint32_t bs = dtype_device_format(t) == TSRC_FMT_Q4_K ? 256u : 32u;
        const uint32_t lim = o.max_part_k ? o.max_part_k : kKMax;
        if (lim % bs) return 0;
        return K < lim ? K : lim;
    }
    const Weight& find(weight_handle h) const {
        auto it = weights_.find(h);
        if (it == weights_.end()) throw std::invalid_argument("tsrc::rt::device: unknown weight handle");
        return it->second;
    }
    void check(int rc, const char* what) const {
        if (rc != TSRC_OK) throw error(std::string("tsrc::rt::device: ") + what + ": " + tsrc_last_error());
    }
    void reserve(size_t xn, size_t yn) {
        if (xn > xcap_) {
            if (xd_) tsrc_dev_free(ctx_, xd_);
            xd_ = nullptr;
            check(tsrc_dev_alloc(ctx_, xn * sizeof(float), &xd_), "x buffer");
            xcap_ = xn;
        }
        if (yn > ycap_) {
            for (void** p : {&ya_, &yb_}) {
                if (*p) tsrc_dev_free(ctx_, *p);
                *p = nullptr;
                check(tsrc_dev_alloc(ctx_, yn * sizeof(float), p), "y buffer");
            }
            ycap_ = yn;
        }
    }

    tsrc_ctx* ctx_ = nullptr;
    std::string desc_;
    mutable std::mutex mu_;
    std::map<weight_handle, Weight> weights_;
    weight_handle next_ = 0;
    void *xd_ = nullptr, *ya_ = nullptr, *yb_ = nullptr;
    size_t xcap_ = 0, ycap_ = 0;
    counters counters_;
};

}  // namespace tsrc::rt
