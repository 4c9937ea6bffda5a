// tsrc_internal.h -- declarations shared by the library's translation units (not part of the ABI).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

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
    uint32_t T;
    float* y;                 // y [t * y_stride + n]
    uint32_t y_stride;
    const float* add;         // addend [t * add_stride + n] (kMmAdd)
    uint32_t add_stride;
    uint32_t flags;
    float s0, s1;
    int32_t* isum_out;        // optional: the kernel's exact block sums of token 0
};

cudaError_t launch_qact(uint32_t kind, const float* x, uint32_t K, uint32_t T, uint32_t x_stride, int8_t* q, float* d,
                        int16_t* bs, cudaStream_t st);
cudaError_t launch_matvec(uint32_t fmt, const MvArgs& a, cudaStream_t st);
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

}  // namespace tsrc
