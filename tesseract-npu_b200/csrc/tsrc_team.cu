// tsrc_team.cu -- MUL_MAT with the all-gather of its rows fused in, over the GPUs of one box.
//
// Tensor parallelism splits a weight's rows over the ranks (the reference's symmetric row split,
// jwkim04/tesseract-npu sw/sim/tsr_ref.c:335-357); every rank then needs every row of y for the
// next layer. Instead of a matvec followed by a collective, the matvec kernel itself stores each
// finished row into every rank's staging buffer over NVLink (CUDA IPC mappings of the peers'
// buffers: plain P2P stores, no multicast) as one 64-bit word {value, step + 1}, and each CTA
// copies its share of the gathered vector out once every word of the share carries the step's tag
// (a bounded wait). The reference has no counterpart (its channels live on one card).
//
// A team's buffer on each rank: staging [2][n_max] tagged u64 words (double-buffered by step
// parity) | state [2] u32 (this rank's steps, CTAs finished in the current launch). All start at
// zero; every rank must run the same sequence of tsrc_mul_mat_allgather calls (one step each).
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>

#include "../../include/tsrc.h"
#include "tsrc_internal.h"

namespace tsrc {
int set_error(int code, const char* msg);
int mm_check(tsrc_ctx* ctx, const tsrc_weight* w, const float* x, uint32_t T, uint32_t* x_stride, float* y, uint32_t* y_stride,
             const float* add, uint32_t add_stride, uint32_t flags, float s0, float s1, MvArgs* base, uint32_t* fmt,
             const char* who);
int weight_rows(const tsrc_weight* w, uint32_t* N, uint32_t* row0, uint32_t* n_rows);
int ctx_device(const tsrc_ctx* ctx, int* dev);
}  // namespace tsrc

struct tsrc_team {
    tsrc_ctx* ctx;
    int device;
    uint32_t rank, world, n_max;
    size_t staging_bytes, bytes;
    uint8_t* local;             // this rank's buffer
    uint8_t* peer[64];          // every rank's buffer (this rank's is `local`)
    bool opened[64];
    bool connected;
    unsigned long long** dev_y;  // device array of every rank's staging pointer
};

namespace {

size_t a256(size_t n) { return (n + 255u) & ~(size_t)255u; }

int cuda_err(cudaError_t e, const char* what) {
    char msg[256];
    snprintf(msg, sizeof msg, "%s: %s", what, cudaGetErrorString(e));
    return tsrc::set_error(TSRC_E_CUDA, msg);
}

}  // namespace

extern "C" {

int tsrc_team_create(tsrc_ctx* ctx, uint32_t rank, uint32_t world, uint32_t n_max, void* handle_out, tsrc_team** out) {
    if (!ctx || !handle_out || !out) return tsrc::set_error(TSRC_E_ARG, "tsrc_team_create: NULL argument");
    *out = nullptr;
    if (world < 1 || world > 64 || rank >= world) return tsrc::set_error(TSRC_E_ARG, "tsrc_team_create: rank / world out of range");
    if (n_max == 0) return tsrc::set_error(TSRC_E_ARG, "tsrc_team_create: n_max is 0");
    int dev = 0;
    int rc = tsrc::ctx_device(ctx, &dev);      // the buffers live on the context's device
    if (rc != TSRC_OK) return rc;
    tsrc_team* t = new tsrc_team{};
    t->ctx = ctx;
    t->device = dev;
    t->rank = rank;
    t->world = world;
    t->n_max = n_max;
    t->staging_bytes = a256((size_t)2 * n_max * 8u);
    t->bytes = t->staging_bytes + 256u;
    cudaError_t e = cudaMalloc(&t->local, t->bytes);
    if (e == cudaSuccess) e = cudaMemset(t->local, 0, t->bytes);
    if (e == cudaSuccess) e = cudaMalloc(&t->dev_y, sizeof(unsigned long long*) * world);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, t->local);
    if (e != cudaSuccess) {
        cudaFree(t->local);
        cudaFree(t->dev_y);
        delete t;
        return cuda_err(e, "tsrc_team_create");
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == TSRC_TEAM_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle_out, &h, sizeof h);
    t->peer[rank] = t->local;
    *out = t;
    return TSRC_OK;
}

int tsrc_team_connect(tsrc_team* t, const void* handles) {
    if (!t || !handles) return tsrc::set_error(TSRC_E_ARG, "tsrc_team_connect: NULL argument");
    if (t->connected) return tsrc::set_error(TSRC_E_ARG, "tsrc_team_connect: already connected");
    int dev = 0;
    int rc = tsrc::ctx_device(t->ctx, &dev);   // the peers' buffers are mapped into the team's device
    if (rc != TSRC_OK) return rc;
    for (uint32_t r = 0; r < t->world; ++r) {
        if (r == t->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)r * TSRC_TEAM_HANDLE_BYTES, sizeof h);
        void* p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            char msg[160];
            snprintf(msg, sizeof msg, "tsrc_team_connect: opening rank %u's buffer", r);
            return cuda_err(e, msg);
        }
        t->peer[r] = static_cast<uint8_t*>(p);
        t->opened[r] = true;
    }
    unsigned long long* ys[64];
    for (uint32_t r = 0; r < t->world; ++r) ys[r] = reinterpret_cast<unsigned long long*>(t->peer[r]);
    cudaError_t e = cudaMemcpy(t->dev_y, ys, sizeof(unsigned long long*) * t->world, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_err(e, "tsrc_team_connect");
    t->connected = true;
    return TSRC_OK;
}

int tsrc_team_connect_local(tsrc_team* t, const tsrc_team* const* members) {
    if (!t || !members) return tsrc::set_error(TSRC_E_ARG, "tsrc_team_connect_local: NULL argument");
    if (t->connected) return tsrc::set_error(TSRC_E_ARG, "tsrc_team_connect_local: already connected");
    unsigned long long* ys[64];
    for (uint32_t r = 0; r < t->world; ++r) {
        const tsrc_team* m = members[r];
        if (!m || m->world != t->world || m->rank != r || m->n_max != t->n_max)
            return tsrc::set_error(TSRC_E_ARG, "tsrc_team_connect_local: members must be ranks 0..world-1 of equal teams");
        // the kernels store through these pointers with no peer mapping: members on other GPUs
        // must connect through tsrc_team_connect (IPC handles, which enable peer access)
        if (m->device != t->device)
            return tsrc::set_error(TSRC_E_ARG, "tsrc_team_connect_local: every member must be on the team's device");
        t->peer[r] = m->local;
        ys[r] = reinterpret_cast<unsigned long long*>(m->local);
    }
    cudaError_t e = cudaMemcpy(t->dev_y, ys, sizeof(unsigned long long*) * t->world, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_err(e, "tsrc_team_connect_local");
    t->connected = true;
    return TSRC_OK;
}

int tsrc_team_free(tsrc_team* t) {
    if (!t) return tsrc::set_error(TSRC_E_ARG, "tsrc_team_free: NULL team");
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != t->device) cudaSetDevice(t->device);     // the team's device, not the caller's current one
    cudaDeviceSynchronize();
    for (uint32_t r = 0; r < t->world; ++r)
        if (t->opened[r]) cudaIpcCloseMemHandle(t->peer[r]);
    cudaFree(t->local);
    cudaFree(t->dev_y);
    delete t;
    return TSRC_OK;
}

int tsrc_mul_mat_allgather(tsrc_ctx* ctx, tsrc_team* t, const tsrc_weight* w, const float* x, float* y, void* stream) {
    if (!t || !t->connected) return tsrc::set_error(TSRC_E_ARG, "tsrc_mul_mat_allgather: team missing or not connected");
    tsrc::MvArgs a{};
    uint32_t fmt = 0, x_stride = 0, y_stride = 0;
    int rc = tsrc::mm_check(ctx, w, x, 1, &x_stride, y, &y_stride, nullptr, 0, 0, 1.0f, 1.0f, &a, &fmt,
                            "tsrc_mul_mat_allgather");
    if (rc != TSRC_OK) return rc;
    uint32_t N = 0, row0 = 0, n_rows = 0;
    tsrc::weight_rows(w, &N, &row0, &n_rows);
    if (N > t->n_max) return tsrc::set_error(TSRC_E_ARG, "tsrc_mul_mat_allgather: N exceeds the team's n_max");
    a.x = x;
    a.x_stride = x_stride;
    a.T = 1;
    a.y = y;
    a.team_y = t->dev_y;
    a.team_state = reinterpret_cast<uint32_t*>(t->local + t->staging_bytes);
    a.team_world = t->world;
    a.team_rank = t->rank;
    a.team_row0 = row0;
    a.team_n = N;
    a.team_half = t->n_max;
    cudaError_t e = tsrc::launch_matvec(fmt, a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_err(e, "tsrc_mul_mat_allgather launch");
    return TSRC_OK;
}

}  // extern "C"

namespace tsrc {

int team_info(const tsrc_team* t, uint32_t* rank, uint32_t* world, uint32_t* n_max) {
    if (!t || !t->connected) return set_error(TSRC_E_ARG, "team missing or not connected");
    *rank = t->rank;
    *world = t->world;
    *n_max = t->n_max;
    return TSRC_OK;
}

// The fused MUL_MAT + all-gather with the options the model runner needs: the residual addend (the
// full vector; row n of the shard adds add[row0 + n]) and RMS_NORM + MUL of x in front.
int team_mul_mat(tsrc_ctx* ctx, tsrc_team* t, const tsrc_weight* w, const float* x, float* y, const float* add,
                 const float* rms_w, float eps, float inv_n, bool rms, void* stream) {
    if (!t || !t->connected) return set_error(TSRC_E_ARG, "team_mul_mat: team missing or not connected");
    MvArgs a{};
    uint32_t fmt = 0, x_stride = 0, y_stride = 0;
    int rc = mm_check(ctx, w, x, 1, &x_stride, y, &y_stride, add, 0, add ? TSRC_MM_ADD : 0u, 1.0f, 1.0f, &a, &fmt,
                      "team_mul_mat");
    if (rc != TSRC_OK) return rc;
    uint32_t N = 0, row0 = 0, n_rows = 0;
    weight_rows(w, &N, &row0, &n_rows);
    if (N > t->n_max) return set_error(TSRC_E_ARG, "team_mul_mat: N exceeds the team's n_max");
    a.x = x;
    a.x_stride = x_stride;
    a.T = 1;
    a.y = y;
    a.add = add ? add + row0 : nullptr;
    a.rms = rms ? 1u : 0u;
    a.rms_w = rms_w;
    a.rms_eps = eps;
    a.rms_inv_n = inv_n;
    a.team_y = t->dev_y;
    a.team_state = reinterpret_cast<uint32_t*>(t->local + t->staging_bytes);
    a.team_world = t->world;
    a.team_rank = t->rank;
    a.team_row0 = row0;
    a.team_n = N;
    a.team_half = t->n_max;
    cudaError_t e = launch_matvec(fmt, a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_err(e, "team_mul_mat launch");
    return TSRC_OK;
}

int team_mul_mat_swiglu(tsrc_ctx* ctx, tsrc_team* t, const tsrc_weight* w, const float* x, float* y, uint32_t out0,
                        uint32_t out_n, const float* rms_w, float eps, float inv_n, void* stream) {
    if (!t || !t->connected) return set_error(TSRC_E_ARG, "team_mul_mat_swiglu: team missing or not connected");
    MvArgs a{};
    uint32_t fmt = 0, x_stride = 0, y_stride = 0;
    int rc = mm_check(ctx, w, x, 1, &x_stride, y, &y_stride, nullptr, 0, 0u, 1.0f, 1.0f, &a, &fmt, "team_mul_mat_swiglu");
    if (rc != TSRC_OK) return rc;
    uint32_t N = 0, row0 = 0, n_rows = 0;
    weight_rows(w, &N, &row0, &n_rows);
    if ((n_rows & 1u) || out_n > t->n_max || out0 + n_rows / 2u > out_n)
        return set_error(TSRC_E_ARG, "team_mul_mat_swiglu: rows and output range do not fit");
    a.x = x;
    a.x_stride = x_stride;
    a.T = 1;
    a.y = y;
    a.rms = 1u;
    a.rms_w = rms_w;
    a.rms_eps = eps;
    a.rms_inv_n = inv_n;
    a.swiglu_pairs = 1u;
    a.team_y = t->dev_y;
    a.team_state = reinterpret_cast<uint32_t*>(t->local + t->staging_bytes);
    a.team_world = t->world;
    a.team_rank = t->rank;
    a.team_row0 = out0;
    a.team_n = out_n;
    a.team_half = t->n_max;
    cudaError_t e = launch_matvec(fmt, a, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_err(e, "team_mul_mat_swiglu launch");
    return TSRC_OK;
}

// dst[offset .. offset + n_local) = src on every rank (dst holds n values)
int team_gather(tsrc_team* t, const float* src, uint32_t n_local, uint32_t offset, float* dst, uint32_t n, void* stream) {
    return team_gather_rows(t, src, n_local, n_local, offset, dst, n, n, 1u, stream);
}

// T token rows: dst[t dst_stride + offset .. + n_local) = src[t src_stride ..] on every rank (a row
// of dst holds n values); as many rows per launch (one team step each) as the staging half holds
int team_gather_rows(tsrc_team* t, const float* src, uint32_t src_stride, uint32_t n_local, uint32_t offset, float* dst,
                     uint32_t dst_stride, uint32_t n, uint32_t T, void* stream) {
    if (!t || !t->connected) return set_error(TSRC_E_ARG, "team_gather: team missing or not connected");
    if (n == 0 || n > t->n_max || offset + n_local > n || src_stride < n_local || dst_stride < n)
        return set_error(TSRC_E_ARG, "team_gather: sizes exceed the team's n_max");
    const uint32_t per = t->n_max / n;                   // token rows per step
    for (uint32_t t0 = 0; t0 < T; t0 += per) {
        TeamGather g{};
        g.team_y = t->dev_y;
        g.team_state = reinterpret_cast<uint32_t*>(t->local + t->staging_bytes);
        g.world = t->world;
        g.rank = t->rank;
        g.half = t->n_max;
        g.src = src + (size_t)t0 * src_stride;
        g.n_local = n_local;
        g.offset = offset;
        g.n = n;
        g.dst = dst + (size_t)t0 * dst_stride;
        g.T = T - t0 < per ? T - t0 : per;
        g.src_stride = src_stride;
        g.dst_stride = dst_stride;
        cudaError_t e = launch_team_gather(g, static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) return cuda_err(e, "team_gather launch");
    }
    return TSRC_OK;
}

}  // namespace tsrc
