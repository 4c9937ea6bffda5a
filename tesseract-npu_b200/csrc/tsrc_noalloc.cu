// tsrc_noalloc.cu -- MUL_MAT for callers that cannot allocate device memory.
//
// tsrc_mul_mat quantizes the activations of a multi-token call into a scratch image that the
// context allocates (cudaMalloc) the first time it needs one of that size. Some callers cannot let
// a library do that: a host that has planned all of the device's memory up front (llama.cpp's ggml
// allocator reserves its compute buffers before the first graph and expects backends not to grow
// behind it), a latency-bound decode loop in which a cudaMalloc / cudaFree would synchronise the
// whole device, or code that runs while a stream is being captured. tsrc_mul_mat_noalloc does the
// same work with its scratch in a fixed array that is part of this library's device image
// (kNoAllocScratchBytes on every device that loads the library, held until the process exits),
// so a call allocates nothing.
//
// Host code cannot use the array's name as a device address (it names a host-side shadow): the
// device address is fetched once per device with cudaGetSymbolAddress, with that device current,
// and passed to the kernels. That set-up happens in the first call on each device, so make the
// first call before starting any stream capture.
//
// Every call uses the same array. Calls queued on one stream are ordered, so they do not clash;
// calls that can run at the same time on one device (several streams, or several contexts on the
// device) race on the array and must be serialised by the caller. Nothing in the array needs to
// start at zero: each call writes the whole quantized image before the matvec reads it.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <mutex>

#include "../../include/tsrc.h"
#include "tsrc_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = 1u << 20;     // 1 MiB: the quantized image of up to 8 tokens of K <= 65536
constexpr uint32_t kKMax = 65536;                     // the matvec's own bound on K (its shared-memory image)
// The image of a full tile of 8 tokens at the largest K the matvec accepts fits the array (Q8_0, the
// larger image: q 8 K + d 8 K / 32 * 4 + bs 8 K / 16 * 2 bytes, each rounded up to 256), so the
// TSRC_E_SHAPE branch below is a defensive check that valid weights never reach.
static_assert(8u * kKMax + 8u * (kKMax / 32u) * 4u + 8u * (kKMax / 16u) * 2u <= kNoAllocScratchBytes,
              "the array must hold 8 tokens of the largest K");

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
uint8_t* g_noalloc_ptr[64];          // device address of the array, per device (set once)

size_t a256(size_t n) { return (n + 255u) & ~(size_t)255u; }

// The array's device address on the current device, or NULL with *err set.
uint8_t* scratch_for_current_device(cudaError_t* err) {
    int dev = 0;
    *err = cudaGetDevice(&dev);
    if (*err != cudaSuccess) return nullptr;
    if (dev < 0 || dev >= 64) {
        *err = cudaErrorInvalidDevice;
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        *err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (*err != cudaSuccess) return nullptr;
        g_noalloc_ptr[dev] = static_cast<uint8_t*>(p);
    }
    return g_noalloc_ptr[dev];
}

}  // namespace

// Defined in tsrc_api.cu: the argument checks of tsrc_mul_mat, the weight fields, errors.
namespace tsrc {
int mm_check(tsrc_ctx* ctx, const tsrc_weight* w, const float* x, uint32_t T, uint32_t* x_stride, float* y, uint32_t* y_stride,
             const float* add, uint32_t add_stride, uint32_t flags, float s0, float s1, MvArgs* base, uint32_t* fmt,
             const char* who);
int set_error(int code, const char* msg);
}  // namespace tsrc

extern "C" TSRC_API int tsrc_mul_mat_noalloc(tsrc_ctx* ctx, const tsrc_weight* w, const float* x, uint32_t T,
                                             uint32_t x_stride, float* y, uint32_t y_stride, const float* add,
                                             uint32_t add_stride, uint32_t flags, float s0, float s1, void* stream) {
    tsrc::MvArgs base{};
    uint32_t fmt = 0;
    int rc = tsrc::mm_check(ctx, w, x, T, &x_stride, y, &y_stride, add, add_stride, flags, s0, s1, &base, &fmt,
                            "tsrc_mul_mat_noalloc");
    if (rc != TSRC_OK || T == 0) return rc;
    const uint32_t K = base.K;
    const uint32_t bsz = fmt == 0 ? 32u : 256u;
    // tokens per launch: as many as one matvec launch takes (<= 8) and the array holds
    uint32_t tt = std::min<uint32_t>(T, tsrc::kMvMaxT);
    auto image_bytes = [&](uint32_t n) {
        return a256((size_t)n * K) + a256((size_t)n * (K / bsz) * 4u) + a256((size_t)n * (K / 16u) * 2u);
    };
    while (tt > 1 && (image_bytes(tt) > kNoAllocScratchBytes || tsrc::mv_smem_bytes(fmt, K, tt) > 200u * 1024u)) --tt;
    if (image_bytes(tt) > kNoAllocScratchBytes) {
        char msg[200];
        snprintf(msg, sizeof msg,
                 "tsrc_mul_mat_noalloc: one token of K = %u needs %zu scratch bytes; the fixed array holds %zu (use tsrc_mul_mat)",
                 K, image_bytes(1), kNoAllocScratchBytes);
        return tsrc::set_error(TSRC_E_SHAPE, msg);
    }
    cudaError_t e = cudaSuccess;
    uint8_t* scratch = scratch_for_current_device(&e);
    if (!scratch) {
        char msg[200];
        snprintf(msg, sizeof msg, "tsrc_mul_mat_noalloc: cudaGetSymbolAddress of the scratch array: %s", cudaGetErrorString(e));
        return tsrc::set_error(TSRC_E_CUDA, msg);
    }
    int8_t* q = reinterpret_cast<int8_t*>(scratch);
    float* d = reinterpret_cast<float*>(scratch + a256((size_t)tt * K));
    int16_t* bs = reinterpret_cast<int16_t*>(scratch + a256((size_t)tt * K) + a256((size_t)tt * (K / bsz) * 4u));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    for (uint32_t t0 = 0; t0 < T; t0 += tt) {
        const uint32_t n = std::min(tt, T - t0);
        e = tsrc::launch_qact(fmt, x + (size_t)t0 * x_stride, K, n, x_stride, q, d, bs, st);
        if (e == cudaSuccess) {
            tsrc::MvArgs a = base;
            a.bsx = bs;
            a.qx = q;
            a.dx = d;
            a.x = nullptr;
            a.T = n;
            a.y = y + (size_t)t0 * y_stride;
            a.add = (flags & TSRC_MM_ADD) ? add + (size_t)t0 * add_stride : nullptr;
            e = tsrc::launch_matvec(fmt, a, st);
        }
        if (e != cudaSuccess) {
            char msg[200];
            snprintf(msg, sizeof msg, "tsrc_mul_mat_noalloc: launch: %s", cudaGetErrorString(e));
            return tsrc::set_error(TSRC_E_CUDA, msg);
        }
    }
    return TSRC_OK;
}
