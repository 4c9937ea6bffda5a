// tsrc_ggml.cu -- ggml tensor types at load time (host code): which types load, their block
// geometry, and the conversion of non-native rows to Q8_0 blocks.
//
// The reference's device stores Q8_0 and Q4_K only (sw/ggml-tesseract/tsr-weights.h:1-30): Q8_0 and
// Q4_K tensors keep their ggml blocks (bit-identical, repacked on the device), and every other type
// that ggml can turn into f32 is converted when it is loaded: ggml's to_float of the type, then
// quantize_row_q8_0_ref. The to_float rules below follow ggml's published block formats
// (dequantize_row_q4_0 / q4_1 / q5_0 / q5_1 / q5_K / q6_K, fp16 and bf16 widening) operation by
// operation, each f32 product and sum rounded separately (the host code is built for baseline
// x86-64, which has no fused multiply-add to contract them into); quantize_row_q8_0_ref is: amax = MAX(amax, |x|) over the block
// (MAX(a, b) = a > b ? a : b), d = amax / 127, id = d ? 1 / d : 0, the block scale fp16(d) rounded
// to nearest even, q = roundf(x * id) (half away from zero).
#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

#include "tsrc_internal.h"
#include "../../include/tsrc.h"

namespace {

// ggml_type values (ggml.h) of the types this loader knows
constexpr uint32_t kF32 = 0, kF16 = 1, kQ4_0 = 2, kQ4_1 = 3, kQ5_0 = 6, kQ5_1 = 7, kQ8_0 = 8, kQ4_K = 12, kQ5_K = 13,
                   kQ6_K = 14, kBF16 = 30;

struct TypeInfo {
    uint32_t type, block_elems, block_bytes;
};
constexpr TypeInfo kTypes[] = {
    {kF32, 1, 4},     {kF16, 1, 2},      {kQ4_0, 32, 18},  {kQ4_1, 32, 20},  {kQ5_0, 32, 22},  {kQ5_1, 32, 24},
    {kQ8_0, 32, 34},  {kQ4_K, 256, 144}, {kQ5_K, 256, 176}, {kQ6_K, 256, 210}, {kBF16, 1, 2},
};

const TypeInfo* type_info(uint32_t t) {
    for (const TypeInfo& i : kTypes)
        if (i.type == t) return &i;
    return nullptr;
}

// IEEE binary16 -> binary32 (exact)
float h2f_host(uint16_t h) {
    const uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    uint32_t u;
    if (e == 0) {
        if (m == 0) {
            u = s;
        } else {                                  // subnormal: normalise
            uint32_t mm = m, ee = 113;            // 127 - 15 + 1
            while (!(mm & 0x400u)) {
                mm <<= 1;
                --ee;
            }
            u = s | (ee << 23) | ((mm & 0x3FFu) << 13);
        }
    } else if (e == 31) {
        u = s | 0x7F800000u | (m << 13);
    } else {
        u = s | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// binary32 -> binary16, round to nearest even (overflow to infinity, NaN stays a quiet NaN)
uint16_t f2h_host(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    const uint16_t s = (uint16_t)((u >> 16) & 0x8000u);
    const uint32_t a = u & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return (uint16_t)(s | 0x7E00u | ((a >> 13) & 0x3FFu));
    if (a >= 0x477FF000u) return (uint16_t)(s | 0x7C00u);       // rounds to >= 2^16: infinity
    if (a < 0x38800000u) {                                        // below 2^-14: subnormal or zero
        if (a < 0x33000000u) return s;                            // below 2^-25: rounds to zero
        const uint32_t e = a >> 23, m = (a & 0x7FFFFFu) | 0x800000u;
        const uint32_t sh = 126u - e;                             // 14..24 bits to drop
        uint32_t r = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1u);
        if (rem > half || (rem == half && (r & 1u))) ++r;
        return (uint16_t)(s | r);
    }
    uint32_t r = ((a - 0x38000000u) >> 13);                       // rebias 127 -> 15
    const uint32_t rem = a & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;
    return (uint16_t)(s | r);
}

float bf2f_host(uint16_t h) {
    const uint32_t u = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

int failf(int code, const char* fmt, ...) {
    char buf[256];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    return tsrc::api_fail(code, buf);
}

uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// the 6-bit scale and min j of a K-quant superblock's 12 scale bytes (ggml's get_scale_min_k4 format)
void scale_min_k4(uint32_t j, const uint8_t* q, uint8_t* d, uint8_t* m) {
    if (j < 4) {
        *d = q[j] & 63u;
        *m = q[j + 4] & 63u;
    } else {
        *d = (uint8_t)((q[j + 4] & 0xFu) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

// to_float of one row of K values
void row_to_f32(uint32_t type, const uint8_t* src, uint32_t K, float* y) {
    switch (type) {
        case kF32:
            std::memcpy(y, src, (size_t)K * 4u);
            return;
        case kF16:
            for (uint32_t i = 0; i < K; ++i) y[i] = h2f_host(rd16(src + 2u * i));
            return;
        case kBF16:
            for (uint32_t i = 0; i < K; ++i) y[i] = bf2f_host(rd16(src + 2u * i));
            return;
        case kQ4_0:
            for (uint32_t b = 0; b < K / 32u; ++b, src += 18, y += 32) {
                const float d = h2f_host(rd16(src));
                for (uint32_t j = 0; j < 16; ++j) {
                    const int x0 = (src[2 + j] & 0x0F) - 8, x1 = (src[2 + j] >> 4) - 8;
                    y[j] = (float)x0 * d;
                    y[j + 16] = (float)x1 * d;
                }
            }
            return;
        case kQ4_1:
            for (uint32_t b = 0; b < K / 32u; ++b, src += 20, y += 32) {
                const float d = h2f_host(rd16(src)), m = h2f_host(rd16(src + 2));
                for (uint32_t j = 0; j < 16; ++j) {
                    const int x0 = src[4 + j] & 0x0F, x1 = src[4 + j] >> 4;
                    y[j] = (float)x0 * d + m;
                    y[j + 16] = (float)x1 * d + m;
                }
            }
            return;
        case kQ5_0:
            for (uint32_t b = 0; b < K / 32u; ++b, src += 22, y += 32) {
                const float d = h2f_host(rd16(src));
                uint32_t qh;
                std::memcpy(&qh, src + 2, 4);
                for (uint32_t j = 0; j < 16; ++j) {
                    const uint8_t xh0 = (uint8_t)(((qh >> j) << 4) & 0x10u), xh1 = (uint8_t)((qh >> (j + 12)) & 0x10u);
                    const int x0 = ((src[6 + j] & 0x0F) | xh0) - 16, x1 = ((src[6 + j] >> 4) | xh1) - 16;
                    y[j] = (float)x0 * d;
                    y[j + 16] = (float)x1 * d;
                }
            }
            return;
        case kQ5_1:
            for (uint32_t b = 0; b < K / 32u; ++b, src += 24, y += 32) {
                const float d = h2f_host(rd16(src)), m = h2f_host(rd16(src + 2));
                uint32_t qh;
                std::memcpy(&qh, src + 4, 4);
                for (uint32_t j = 0; j < 16; ++j) {
                    const uint8_t xh0 = (uint8_t)(((qh >> j) << 4) & 0x10u), xh1 = (uint8_t)((qh >> (j + 12)) & 0x10u);
                    const int x0 = (src[8 + j] & 0x0F) | xh0, x1 = (src[8 + j] >> 4) | xh1;
                    y[j] = (float)x0 * d + m;
                    y[j + 16] = (float)x1 * d + m;
                }
            }
            return;
        case kQ5_K:
            for (uint32_t b = 0; b < K / 256u; ++b, src += 176) {
                const float d = h2f_host(rd16(src)), mn = h2f_host(rd16(src + 2));
                const uint8_t* sc = src + 4;
                const uint8_t* qh = src + 16;
                const uint8_t* ql = src + 48;
                uint8_t u1 = 1, u2 = 2;
                for (uint32_t j = 0, is = 0; j < 256; j += 64, is += 2, ql += 32) {
                    uint8_t s, m;
                    scale_min_k4(is, sc, &s, &m);
                    const float d1 = d * (float)s, m1 = mn * (float)m;
                    scale_min_k4(is + 1, sc, &s, &m);
                    const float d2 = d * (float)s, m2 = mn * (float)m;
                    for (uint32_t l = 0; l < 32; ++l) *y++ = d1 * (float)((ql[l] & 0xF) + ((qh[l] & u1) ? 16 : 0)) - m1;
                    for (uint32_t l = 0; l < 32; ++l) *y++ = d2 * (float)((ql[l] >> 4) + ((qh[l] & u2) ? 16 : 0)) - m2;
                    u1 = (uint8_t)(u1 << 2);
                    u2 = (uint8_t)(u2 << 2);
                }
            }
            return;
        case kQ6_K:
            for (uint32_t b = 0; b < K / 256u; ++b, src += 210) {
                const uint8_t* ql = src;
                const uint8_t* qh = src + 128;
                const int8_t* sc = reinterpret_cast<const int8_t*>(src + 192);
                const float d = h2f_host(rd16(src + 208));
                for (uint32_t n = 0; n < 256; n += 128, y += 128, ql += 64, qh += 32, sc += 8) {
                    for (uint32_t l = 0; l < 32; ++l) {
                        const uint32_t is = l / 16u;
                        const int q1 = (int8_t)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                        const int q2 = (int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                        const int q3 = (int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                        const int q4 = (int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                        y[l] = d * (float)sc[is] * (float)q1;
                        y[l + 32] = d * (float)sc[is + 2] * (float)q2;
                        y[l + 64] = d * (float)sc[is + 4] * (float)q3;
                        y[l + 96] = d * (float)sc[is + 6] * (float)q4;
                    }
                }
            }
            return;
        default:
            return;
    }
}

// quantize_row_q8_0_ref of one row of K values into K / 32 blocks of 34 bytes
void row_to_q8_0(const float* x, uint32_t K, uint8_t* dst) {
    for (uint32_t b = 0; b < K / 32u; ++b, x += 32, dst += 34) {
        float amax = 0.0f;
        for (uint32_t j = 0; j < 32; ++j) {
            const float a = std::fabs(x[j]);
            amax = amax > a ? amax : a;
        }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        const uint16_t h = f2h_host(d);
        dst[0] = (uint8_t)(h & 0xFFu);
        dst[1] = (uint8_t)(h >> 8);
        for (uint32_t j = 0; j < 32; ++j) {
            const float r = std::roundf(x[j] * id);
            // the C conversion of roundf's value to int8_t as x86 performs it (cvttss2si, low byte);
            // a NaN or out-of-range value gives INT32_MIN, whose low byte is 0
            const int32_t v = (r != r || r >= 2147483648.0f || r < -2147483648.0f) ? INT32_MIN : (int32_t)r;
            dst[2 + j] = (uint8_t)(v & 0xFF);
        }
    }
}

}  // namespace

extern "C" {

int tsrc_ggml_type_info(uint32_t ggml_type, uint32_t* block_elems, uint32_t* block_bytes, uint32_t* dev_fmt) {
    const TypeInfo* t = type_info(ggml_type);
    if (!t) return failf(TSRC_E_SHAPE, "tsrc_ggml_type_info: ggml type %u is not loadable", ggml_type);
    if (block_elems) *block_elems = t->block_elems;
    if (block_bytes) *block_bytes = t->block_bytes;
    if (dev_fmt) *dev_fmt = ggml_type == kQ4_K ? TSRC_FMT_Q4_K : TSRC_FMT_Q8_0;
    return TSRC_OK;
}

int tsrc_ggml_rows_to_dev(uint32_t ggml_type, const void* src, uint32_t n_rows, uint32_t K, void* dst) {
    const TypeInfo* t = type_info(ggml_type);
    if (!t) return failf(TSRC_E_SHAPE, "tsrc_ggml_rows_to_dev: ggml type %u is not loadable", ggml_type);
    if (!src || !dst) return failf(TSRC_E_ARG, "tsrc_ggml_rows_to_dev: NULL argument");
    const uint32_t fmt = ggml_type == kQ4_K ? TSRC_FMT_Q4_K : TSRC_FMT_Q8_0;
    if (K == 0 || K % (fmt == TSRC_FMT_Q4_K ? 256u : 32u) || K % t->block_elems)
        return failf(TSRC_E_SHAPE, "tsrc_ggml_rows_to_dev: K = %u is not a whole number of blocks", K);
    const size_t src_row = (size_t)K / t->block_elems * t->block_bytes;
    const size_t dst_row = fmt == TSRC_FMT_Q4_K ? (size_t)K / 256u * 144u : (size_t)K / 32u * 34u;
    const uint8_t* s = static_cast<const uint8_t*>(src);
    uint8_t* d = static_cast<uint8_t*>(dst);
    if (ggml_type == kQ8_0 || ggml_type == kQ4_K) {           // native: the blocks as they are
        std::memcpy(d, s, src_row * n_rows);
        return TSRC_OK;
    }
    // rows are independent: split them over the host's threads for large tensors (the reference
    // converts with TSR_LOAD_THREADS load threads)
    const uint64_t work = (uint64_t)n_rows * K;
    const uint32_t hw = std::max(1u, std::thread::hardware_concurrency());
    const uint32_t n_thr = work < (1u << 20) ? 1u : std::min<uint32_t>(std::min(hw, 32u), n_rows);
    auto run = [&](uint32_t r0, uint32_t r1) {
        std::vector<float> tmp(K);
        for (uint32_t r = r0; r < r1; ++r) {
            row_to_f32(ggml_type, s + (size_t)r * src_row, K, tmp.data());
            row_to_q8_0(tmp.data(), K, d + (size_t)r * dst_row);
        }
    };
    if (n_thr == 1) {
        run(0, n_rows);
    } else {
        std::vector<std::thread> th;
        const uint32_t per = (n_rows + n_thr - 1u) / n_thr;
        for (uint32_t i = 0; i < n_thr; ++i) {
            const uint32_t r0 = std::min(n_rows, i * per), r1 = std::min(n_rows, r0 + per);
            if (r0 < r1) th.emplace_back(run, r0, r1);
        }
        for (auto& x : th) x.join();
    }
    return TSRC_OK;
}

int tsrc_weight_upload_ggml(tsrc_ctx* ctx, uint32_t ggml_type, const void* rows, uint32_t N, uint32_t K, uint32_t row0,
                            uint32_t n_rows, tsrc_weight** out) {
    uint32_t fmt = 0;
    int rc = tsrc_ggml_type_info(ggml_type, nullptr, nullptr, &fmt);
    if (rc) return rc;
    if (ggml_type == kQ8_0 || ggml_type == kQ4_K) return tsrc_weight_upload(ctx, fmt, rows, N, K, row0, n_rows, out);
    const size_t dst_row = (size_t)K / 32u * 34u;
    std::vector<uint8_t> conv;
    try {
        conv.resize(dst_row * n_rows);
    } catch (...) {
        return failf(TSRC_E_NOMEM, "tsrc_weight_upload_ggml: host buffer of %zu bytes", dst_row * n_rows);
    }
    rc = tsrc_ggml_rows_to_dev(ggml_type, rows, n_rows, K, conv.data());
    if (rc) return rc;
    return tsrc_weight_upload(ctx, fmt, conv.data(), N, K, row0, n_rows, out);
}

}  // extern "C"
