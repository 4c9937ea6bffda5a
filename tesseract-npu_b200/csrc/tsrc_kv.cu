// tsrc_kv.cu -- the q8_0 KV cache planes on the device.
//
// The reference keeps K and V in FPGA planes (token-major K, slice-major V, 16-cell groups
// interleaved over channels; jwkim04/tesseract-npu sw/sim/tsr_ref_at.c:91-212) and converts
// ggml's q8_0 cache rows into them in the backend's set_tensor. Here a plane is split per KV
// head, head-major, so that a 16-cell group of one head is one contiguous run of bytes:
//   K quants  q[head][cell][D]                  (cell-major: a cell's D values contiguous, the
//                                                row operand of the QK products)
//   V quants  q[head][group][D][16]             (value-major inside a 16-cell group: 16 cells of
//                                                one value contiguous, the tensor-core A operand
//                                                of the P.V products)
//   scales    d[head][cell][D / 32]             (the ggml block's fp16 d, K and V alike)
// The planes hold exactly the bytes of the ggml image (get / set round-trip them); the cell count
// is padded to a multiple of 16 with zeros so that a group never runs past the allocation.
//
// KVST (tsr_ref_at.c:244-264): a new f32 row of E = n_head_kv * D values is quantized with QACT
// A32 per 32 values and stored as {fp16(d), q} -- the same bytes as ggml's quantize_row_q8_0 for
// finite rows, which is what SET_ROWS into a q8_0 cache writes.
#include "tsrc_internal.h"
#include "tsrc_numerics.cuh"

namespace tsrc {

namespace {

__device__ __forceinline__ size_t qoff(bool vt, uint32_t g, uint32_t n_cells, uint32_t D, size_t cell, uint32_t k) {
    return kv_qoff(vt, g, n_cells, D, cell, k);
}

// one warp per 32-value block of a row
__global__ void kv_store_kernel(const float* rows, uint32_t n, uint32_t row_stride, const int64_t* cells, uint32_t cell0,
                                uint32_t n_head_kv, uint32_t D, uint32_t n_cells, bool vt, int8_t* q, uint16_t* d,
                                unsigned int* err) {
    const uint32_t nb = n_head_kv * D / 32u;
    const size_t wi = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint32_t lane = threadIdx.x & 31u;
    if (wi >= (size_t)n * nb) return;
    const uint32_t i = (uint32_t)(wi / nb), b = (uint32_t)(wi - (size_t)i * nb);
    const int64_t cell = cells ? cells[i] : (int64_t)cell0 + i;
    if (cell < 0 || cell >= (int64_t)n_cells) {
        if (lane == 0) atomicCAS(err, 0u, 1u);          // a row index outside the cache: not stored
        return;
    }
    const float v = rows[(size_t)i * row_stride + 32u * b + lane];
    const uint32_t amax = __reduce_max_sync(0xFFFFFFFFu, amax_key(v));
    const float db = fdiv(ffrom(amax), 127.0f);
    const float id = (fbits(db) & ~kSign) ? frecip(db) : 0.0f;
    const uint32_t g = 32u * b / D, k = 32u * b - g * D;
    const size_t hc = (size_t)g * n_cells + (size_t)cell;
    q[qoff(vt, g, n_cells, D, (size_t)cell, k + lane)] = (int8_t)round_away_sat8(fmul(daz(v), id));
    if (lane == 0) d[hc * (D / 32u) + k / 32u] = f2h(db);
}

// one thread per (cell, block): ggml block {fp16 d; int8 qs[32]} (34 bytes) <-> planes
__global__ void kv_from_ggml_kernel(const uint8_t* ggml, uint32_t n, uint32_t cell0, uint32_t n_head_kv, uint32_t D,
                                    uint32_t n_cells, bool vt, int8_t* q, uint16_t* d) {
    const uint32_t nb = n_head_kv * D / 32u;
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (size_t)n * nb) return;
    const uint32_t i = (uint32_t)(t / nb), b = (uint32_t)(t - (size_t)i * nb);
    const uint8_t* src = ggml + ((size_t)i * nb + b) * 34u;
    const uint32_t g = 32u * b / D, k = 32u * b - g * D;
    const size_t hc = (size_t)g * n_cells + cell0 + i;
    d[hc * (D / 32u) + k / 32u] = (uint16_t)(src[0] | (src[1] << 8));
    if (vt) {
        for (uint32_t j = 0; j < 32; ++j) q[qoff(true, g, n_cells, D, (size_t)cell0 + i, k + j)] = (int8_t)src[2 + j];
        return;
    }
    uint32_t w[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
        w[j] = (uint32_t)src[2 + 4 * j] | ((uint32_t)src[3 + 4 * j] << 8) | ((uint32_t)src[4 + 4 * j] << 16) |
               ((uint32_t)src[5 + 4 * j] << 24);
    uint4* dst = reinterpret_cast<uint4*>(q + hc * D + k);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

__global__ void kv_to_ggml_kernel(const int8_t* q, const uint16_t* d, uint32_t n, uint32_t cell0, uint32_t n_head_kv, uint32_t D,
                                  uint32_t n_cells, bool vt, uint8_t* ggml) {
    const uint32_t nb = n_head_kv * D / 32u;
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (size_t)n * nb) return;
    const uint32_t i = (uint32_t)(t / nb), b = (uint32_t)(t - (size_t)i * nb);
    uint8_t* dst = ggml + ((size_t)i * nb + b) * 34u;
    const uint32_t g = 32u * b / D, k = 32u * b - g * D;
    const size_t hc = (size_t)g * n_cells + cell0 + i;
    const uint16_t h = d[hc * (D / 32u) + k / 32u];
    dst[0] = (uint8_t)(h & 0xFFu);
    dst[1] = (uint8_t)(h >> 8);
    if (vt) {
        for (uint32_t j = 0; j < 32; ++j) dst[2 + j] = (uint8_t)q[qoff(true, g, n_cells, D, (size_t)cell0 + i, k + j)];
        return;
    }
    const uint4* src = reinterpret_cast<const uint4*>(q + hc * D + k);
    const uint4 a = src[0], c = src[1];
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) dst[2 + 4 * j + e] = (uint8_t)(w[j] >> (8 * e));
}

__device__ unsigned int g_kv_error;

}  // namespace

cudaError_t kv_error_flag(unsigned int** err) { return cudaGetSymbolAddress(reinterpret_cast<void**>(err), g_kv_error); }

cudaError_t launch_kv_store(const float* rows, uint32_t n, uint32_t row_stride, const int64_t* cells, uint32_t cell0,
                            uint32_t n_head_kv, uint32_t D, uint32_t n_cells, bool vt, int8_t* q, uint16_t* d, cudaStream_t st) {
    const size_t threads = (size_t)n * (n_head_kv * D / 32u) * 32u;
    if (threads == 0) return cudaSuccess;
    unsigned int* err = nullptr;
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_kv_error);
    if (e != cudaSuccess) return e;
    kv_store_kernel<<<(unsigned)((threads + 255u) / 256u), 256, 0, st>>>(rows, n, row_stride, cells, cell0, n_head_kv, D, n_cells,
                                                                         vt, q, d, err);
    return cudaGetLastError();
}

// The first error any KVST launch recorded on the current device (0 = none; 1 = a cell index
// outside the cache), cleared when read with clear = true.
cudaError_t kv_error(uint32_t* code, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(code, g_kv_error, sizeof(uint32_t));
    if (e == cudaSuccess && clear && *code) {
        const uint32_t zero = 0;
        e = cudaMemcpyToSymbol(g_kv_error, &zero, sizeof(uint32_t));
    }
    return e;
}

cudaError_t launch_kv_from_ggml(const uint8_t* ggml, uint32_t n, uint32_t cell0, uint32_t n_head_kv, uint32_t D,
                                uint32_t n_cells, bool vt, int8_t* q, uint16_t* d, cudaStream_t st) {
    const size_t t = (size_t)n * (n_head_kv * D / 32u);
    if (t == 0) return cudaSuccess;
    kv_from_ggml_kernel<<<(unsigned)((t + 255u) / 256u), 256, 0, st>>>(ggml, n, cell0, n_head_kv, D, n_cells, vt, q, d);
    return cudaGetLastError();
}

cudaError_t launch_kv_to_ggml(const int8_t* q, const uint16_t* d, uint32_t n, uint32_t cell0, uint32_t n_head_kv, uint32_t D,
                              uint32_t n_cells, bool vt, uint8_t* ggml, cudaStream_t st) {
    const size_t t = (size_t)n * (n_head_kv * D / 32u);
    if (t == 0) return cudaSuccess;
    kv_to_ggml_kernel<<<(unsigned)((t + 255u) / 256u), 256, 0, st>>>(q, d, n, cell0, n_head_kv, D, n_cells, vt, ggml);
    return cudaGetLastError();
}

}  // namespace tsrc
