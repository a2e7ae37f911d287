// Multi-GPU long-context split-KV decode: the one exchange step of the path.
//
// The reference is single-GPU (CudaPagedTransformerRunner.cs:108).  Sequence partitioning
// (one pool per GPU) needs no collective; only a sequence too long for one GPU's share is
// split by contiguous block range across ranks.  Each rank then decodes its range into a
// normalised output plus the log-sum-exp of its softmax denominator, the ranks all-gather
// those (rows * (dv + 1) floats each) with NCCL over NVLink, and every rank merges them:
// out = sum_r exp(lse_r - LSE) * out_r, LSE = ln(sum_r exp(lse_r) [+ exp(sink)]).
//
// Every NCCL wait is bounded: the communicator is created non-blocking and polled against a
// host timeout, and a timeout aborts it (ncclCommAbort) and returns GKV_ETIMEDOUT.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cmath>
#include <cstring>
#include <new>
#include <mutex>
#include <thread>
#include <type_traits>

#include "gkv_internal.h"

struct gkv_comm {
    ncclComm_t comm = nullptr;
    int32_t n_ranks = 0, rank = 0, device = 0, timeout_ms = 0;
    float* d_send = nullptr;
    float* d_recv = nullptr;
    size_t cap_floats = 0;  // per rank
    bool aborted = false;
};

namespace {

using gkv::set_error;

// NCCL is loaded on first use (dlopen), not linked: a process that already loaded an NCCL
// (e.g. through PyTorch) keeps that one, and hosts that never split sequences never load it.
struct Nccl {
    decltype(&ncclGetUniqueId) GetUniqueId = nullptr;
    decltype(&ncclCommInitRankConfig) CommInitRankConfig = nullptr;
    decltype(&ncclCommGetAsyncError) CommGetAsyncError = nullptr;
    decltype(&ncclCommAbort) CommAbort = nullptr;
    decltype(&ncclCommFinalize) CommFinalize = nullptr;
    decltype(&ncclCommDestroy) CommDestroy = nullptr;
    decltype(&ncclAllGather) AllGather = nullptr;
    decltype(&ncclGetErrorString) GetErrorString = nullptr;
    bool ok = false;
};

const Nccl& nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        auto sym = [&](auto& fn, const char* name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            return fn != nullptr;
        };
        n.ok = sym(n.GetUniqueId, "ncclGetUniqueId") && sym(n.CommInitRankConfig, "ncclCommInitRankConfig") &&
               sym(n.CommGetAsyncError, "ncclCommGetAsyncError") && sym(n.CommAbort, "ncclCommAbort") &&
               sym(n.CommFinalize, "ncclCommFinalize") && sym(n.CommDestroy, "ncclCommDestroy") &&
               sym(n.AllGather, "ncclAllGather") && sym(n.GetErrorString, "ncclGetErrorString");
    });
    return n;
}

int nccl_missing() { return set_error(GKV_ENCCL, "libnccl.so.2 could not be loaded"); }

int nccl_fail(ncclResult_t r, const char* what) {
    return set_error(GKV_ENCCL, "%s: %s (%d)", what, nccl().GetErrorString(r), static_cast<int>(r));
}

// Polls a non-blocking communicator until its pending operation settles.
int nccl_wait(gkv_comm* c, const char* what) {
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = nccl().CommGetAsyncError(c->comm, &st);
        if (r != ncclSuccess) return nccl_fail(r, what);
        if (st == ncclSuccess) return GKV_OK;
        if (st != ncclInProgress) return nccl_fail(st, what);
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                            std::chrono::steady_clock::now() - t0).count();
        if (c->timeout_ms >= 0 && ms >= c->timeout_ms) {
            nccl().CommAbort(c->comm);
            c->comm = nullptr;
            c->aborted = true;
            return set_error(GKV_ETIMEDOUT, "%s: no progress after %d ms; communicator aborted", what,
                             c->timeout_ms);
        }
        // A data-path call finishes enqueueing within microseconds: poll without sleeping
        // first (a sleep here delays every later launch of the step), then back off.
        if (ms >= 2) std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

}  // namespace

extern "C" {

int gkv_comm_unique_id(uint8_t* out_id) {
    if (!out_id) return set_error(GKV_EINVAL, "out_id is NULL");
    if (!nccl().ok) return nccl_missing();
    ncclUniqueId id;
    ncclResult_t r = nccl().GetUniqueId(&id);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    static_assert(sizeof(id.internal) == 128, "ncclUniqueId is 128 bytes");
    memcpy(out_id, id.internal, 128);
    return GKV_OK;
}

int gkv_comm_init(const uint8_t* unique_id, int32_t n_ranks, int32_t rank, int32_t device,
                  int32_t timeout_ms, gkv_comm** out_comm) {
    if (!unique_id || !out_comm) return set_error(GKV_EINVAL, "unique_id/out_comm is NULL");
    if (n_ranks < 1 || rank < 0 || rank >= n_ranks || device < 0)
        return set_error(GKV_EINVAL, "n_ranks=%d rank=%d device=%d", n_ranks, rank, device);
    *out_comm = nullptr;
    if (!nccl().ok) return nccl_missing();
    gkv::DeviceGuard guard(device);
    if (!guard.ok()) return set_error(GKV_ECUDA, "cudaSetDevice(%d) failed", device);
    gkv_comm* c = new (std::nothrow) gkv_comm();
    if (!c) return set_error(GKV_ENOMEM, "host allocation failed");
    c->n_ranks = n_ranks;
    c->rank = rank;
    c->device = device;
    c->timeout_ms = timeout_ms;
    ncclUniqueId id;
    memcpy(id.internal, unique_id, 128);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = nccl().CommInitRankConfig(&c->comm, n_ranks, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        delete c;
        return nccl_fail(r, "ncclCommInitRankConfig");
    }
    const int rc = nccl_wait(c, "ncclCommInitRankConfig");
    if (rc != GKV_OK) {
        if (c->comm) nccl().CommAbort(c->comm);
        delete c;
        return rc;
    }
    *out_comm = c;
    return GKV_OK;
}

int gkv_comm_abort(gkv_comm* c) {
    if (!c) return GKV_OK;
    if (c->comm) nccl().CommAbort(c->comm);
    c->comm = nullptr;
    c->aborted = true;
    return GKV_OK;
}

int gkv_comm_destroy(gkv_comm* c) {
    if (!c) return GKV_OK;
    gkv::DeviceGuard guard(c->device);
    if (c->comm) {
        nccl().CommFinalize(c->comm);
        nccl_wait(c, "ncclCommFinalize");
        if (c->comm) nccl().CommDestroy(c->comm);
    }
    if (c->d_send) cudaFree(c->d_send);
    if (c->d_recv) cudaFree(c->d_recv);
    delete c;
    return GKV_OK;
}

int gkv_paged_decode_lse(gkv_pool* pool, int32_t layer, const float* d_q, float* d_out,
                         float* d_lse, int32_t n_heads, float scale, const float* d_sinks,
                         void* stream) {
    if (!pool) return set_error(GKV_EINVAL, "pool handle is NULL");
    if (!pool->impl.has_arena) return set_error(GKV_ESTATE, "pool has no device arena (metadata-only pool)");
    if (!d_lse) return set_error(GKV_EINVAL, "lse is NULL");
    gkv::DeviceGuard guard(pool->impl.desc.device);
    pool->impl.last_launches = 0;
    return gkv::step_decode_lse(&pool->impl, layer, d_q, d_out, d_lse, n_heads, scale, d_sinks,
                                static_cast<cudaStream_t>(stream));
}

int gkv_lse_merge(const float* d_parts, int32_t n_parts, int32_t rows, int32_t dv,
                  const float* d_sinks, int32_t n_heads, float* d_out, void* stream) {
    if (n_parts < 1 || rows < 0 || dv < 1 || (d_sinks && n_heads < 1))
        return set_error(GKV_EINVAL, "n_parts=%d rows=%d dv=%d n_heads=%d", n_parts, rows, dv, n_heads);
    if (rows > 0 && (!d_parts || !d_out)) return set_error(GKV_EINVAL, "parts/out is NULL");
    cudaError_t e = gkv::launch_lse_merge(d_parts, n_parts, rows, dv, d_sinks, n_heads > 0 ? n_heads : 1,
                                          d_out, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return gkv::cuda_fail(e, "lse_merge launch");
    return GKV_OK;
}

int gkv_paged_decode_splitkv_dist(gkv_pool* pool, gkv_comm* c, int32_t layer, const float* d_q,
                                  float* d_out, int32_t n_heads, float scale,
                                  const float* d_sinks, void* stream) {
    if (!pool || !c) return set_error(GKV_EINVAL, "pool/comm is NULL");
    gkv::Pool& P = pool->impl;
    if (!P.has_arena) return set_error(GKV_ESTATE, "pool has no device arena (metadata-only pool)");
    if (c->aborted || !c->comm) return set_error(GKV_ESTATE, "communicator was aborted");
    if (c->device != P.desc.device)
        return set_error(GKV_EINVAL, "communicator device %d != pool device %d", c->device, P.desc.device);
    if (!P.ws.uploaded) return set_error(GKV_ESTATE, "no step uploaded (call gkv_upload_step first)");
    gkv::DeviceGuard guard(P.desc.device);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int32_t dv = P.desc.v_head_dim;
    const int64_t rows = static_cast<int64_t>(P.ws.batch) * n_heads;
    const size_t per = static_cast<size_t>(rows) * (dv + 1);
    if (per > c->cap_floats) {
        cudaDeviceSynchronize();
        if (c->d_send) cudaFree(c->d_send);
        if (c->d_recv) cudaFree(c->d_recv);
        c->d_send = c->d_recv = nullptr;
        c->cap_floats = 0;
        cudaError_t e = cudaMalloc(&c->d_send, per * sizeof(float));
        if (e == cudaSuccess) e = cudaMalloc(&c->d_recv, per * sizeof(float) * c->n_ranks);
        if (e != cudaSuccess) return gkv::cuda_fail(e, "cudaMalloc(split-KV exchange)");
        c->cap_floats = per;
    }
    float* send_out = c->d_send;
    float* send_lse = c->d_send + rows * dv;
    P.last_launches = 0;
    // rows this rank holds no tokens of keep lse = -inf (weight 0 in the merge)
    cudaError_t e = gkv::launch_fill(send_lse, rows, -INFINITY, st);
    if (e != cudaSuccess) return gkv::cuda_fail(e, "fill launch");
    int rc = gkv::step_decode_lse(&P, layer, d_q, send_out, send_lse, n_heads, scale, nullptr, st);
    if (rc != GKV_OK) return rc;
    const int launches = P.last_launches + 1;
    ncclResult_t r = nccl().AllGather(c->d_send, c->d_recv, per, ncclFloat, c->comm, st);
    if (r == ncclInProgress) {
        rc = nccl_wait(c, "ncclAllGather");
        if (rc != GKV_OK) return rc;
    } else if (r != ncclSuccess) {
        return nccl_fail(r, "ncclAllGather");
    }
    e = gkv::launch_lse_merge(c->d_recv, c->n_ranks, static_cast<int>(rows), dv, d_sinks, n_heads, d_out, st);
    if (e != cudaSuccess) return gkv::cuda_fail(e, "lse_merge launch");
    P.last_launches = launches + 1;
    return GKV_OK;
}

}  // extern "C"
