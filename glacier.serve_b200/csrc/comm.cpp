// Multi-GPU long-context split-KV decode: the one exchange step of the path.
//
// The reference is single-GPU (CudaPagedTransformerRunner.cs:108).  Sequence partitioning
// (one pool per GPU) needs no collective; only a sequence too long for one GPU's share is
// split by contiguous block range across ranks.  Each rank then decodes its range into a
// normalised output plus the log-sum-exp of its softmax denominator, the ranks all-gather
// those (rows * (dv + 1) floats each) with NCCL over NVLink, and every rank merges them:
// out = sum_r exp(lse_r - LSE) * out_r, LSE = ln(sum_r exp(lse_r) [+ exp(sink)]).
//
// The exchange itself goes through peer memory when the ranks can map each other's HBM (CUDA
// IPC over NVLink, set up once with two small NCCL all-gathers): each rank's decode writes its
// block into its own mailbox, and one kernel publishes an epoch flag to every rank, waits for
// every rank's flag and merges all blocks with plain loads over NVLink (exchange.cu).  That
// replaces a ring all-gather whose N-1 latency-bound steps cost more than the decode itself
// at 8 ranks.  Without peer mappings the ranks agree to use ncclAllGather instead.
//
// Every NCCL wait is bounded: the communicator is created non-blocking and polled against a
// host timeout, and a timeout aborts it (ncclCommAbort) and returns GKV_ETIMEDOUT.  The merge
// kernel's wait on peer flags is bounded too (kErrWaitTimeout in the pool's error word).
#include <algorithm>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cmath>
#include <cstring>
#include <new>
#include <mutex>
#include <thread>
#include <type_traits>
#include <vector>

#include "gkv_internal.h"

struct gkv_comm {
    ncclComm_t comm = nullptr;
    int32_t n_ranks = 0, rank = 0, device = 0, timeout_ms = 0;
    float* d_send = nullptr;
    float* d_recv = nullptr;
    size_t cap_floats = 0;  // per rank
    bool aborted = false;
    // peer-memory exchange: 0 = not set up yet, 1 = NCCL all-gather, 2 = peer mailboxes
    int kind = 0;
    void* d_mbox = nullptr;                     // this rank's mailbox (floats, then flags)
    void* peer_base[gkv::kMaxExchangeRanks] = {};  // IPC mappings of the other ranks' mailboxes
    gkv::ExchangePeers peers{};
    unsigned epoch = 0;
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

// NCCL all-gather of `bytes` per rank through device buffers, completed before returning.
int allgather_host(gkv_comm* c, const void* mine, void* all, size_t bytes, cudaStream_t st) {
    void* d = nullptr;
    cudaError_t e = cudaMalloc(&d, bytes * (c->n_ranks + 1));
    if (e != cudaSuccess) return gkv::cuda_fail(e, "cudaMalloc(exchange set-up)");
    char* send = static_cast<char*>(d) + bytes * c->n_ranks;
    int rc = GKV_OK;
    e = cudaMemcpyAsync(send, mine, bytes, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) rc = gkv::cuda_fail(e, "cudaMemcpyAsync(exchange set-up)");
    if (rc == GKV_OK) {
        ncclResult_t r = nccl().AllGather(send, d, bytes, ncclChar, c->comm, st);
        if (r == ncclInProgress) rc = nccl_wait(c, "ncclAllGather(exchange set-up)");
        else if (r != ncclSuccess) rc = nccl_fail(r, "ncclAllGather(exchange set-up)");
    }
    if (rc == GKV_OK) {
        e = cudaMemcpyAsync(all, d, bytes * c->n_ranks, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) rc = gkv::cuda_fail(e, "exchange set-up copy");
    }
    cudaFree(d);
    return rc;
}

void release_p2p(gkv_comm* c) {
    for (int r = 0; r < gkv::kMaxExchangeRanks; ++r)
        if (c->peer_base[r]) {
            cudaIpcCloseMemHandle(c->peer_base[r]);
            c->peer_base[r] = nullptr;
        }
    if (c->d_mbox) cudaFree(c->d_mbox);
    c->d_mbox = nullptr;
}

// Collective: every rank calls it on its first split-KV decode with the same slot size.
// Sets c->kind to 2 when every rank mapped every other rank's mailbox, else to 1.
int setup_exchange(gkv_comm* c, int64_t per, cudaStream_t st) {
    const int n = c->n_ranks;
    const int64_t slot = (per + 3) / 4 * 4 * 2;  // room for twice the first call's rows
    const size_t floats_bytes = static_cast<size_t>(2) * n * slot * sizeof(float);
    const size_t bytes = floats_bytes + static_cast<size_t>(2) * n * sizeof(unsigned);
    struct Entry {
        cudaIpcMemHandle_t handle;
        int32_t ok;
    } mine{};
    mine.ok = n <= gkv::kMaxExchangeRanks;
    if (mine.ok && cudaMalloc(&c->d_mbox, bytes) != cudaSuccess) mine.ok = 0;
    if (mine.ok && cudaMemset(c->d_mbox, 0, bytes) != cudaSuccess) mine.ok = 0;
    if (mine.ok && cudaIpcGetMemHandle(&mine.handle, c->d_mbox) != cudaSuccess) mine.ok = 0;
    cudaGetLastError();
    std::vector<Entry> all(static_cast<size_t>(n));
    int rc = allgather_host(c, &mine, all.data(), sizeof(Entry), st);
    if (rc != GKV_OK) return rc;
    int32_t ok = 1;
    for (const Entry& en : all) ok &= en.ok;
    if (ok) {
        for (int r = 0; r < n; ++r) {
            if (r == c->rank) continue;
            if (cudaIpcOpenMemHandle(&c->peer_base[r], all[static_cast<size_t>(r)].handle,
                                     cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                c->peer_base[r] = nullptr;
                ok = 0;
                break;
            }
        }
        cudaGetLastError();
    }
    // every rank must take the same path
    std::vector<int32_t> oks(static_cast<size_t>(n));
    rc = allgather_host(c, &ok, oks.data(), sizeof(int32_t), st);
    if (rc != GKV_OK) return rc;
    for (int32_t v : oks) ok &= v;
    if (!ok) {
        release_p2p(c);
        c->kind = 1;
        return GKV_OK;
    }
    c->peers.n_ranks = n;
    c->peers.slot = slot;
    for (int r = 0; r < n; ++r) {
        char* base = static_cast<char*>(r == c->rank ? c->d_mbox : c->peer_base[r]);
        c->peers.mbox[r] = reinterpret_cast<float*>(base);
        c->peers.flags[r] = reinterpret_cast<unsigned*>(base + floats_bytes);
    }
    c->kind = 2;
    return GKV_OK;
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
    cudaDeviceSynchronize();  // the last merge has read every peer's block
    release_p2p(c);
    if (c->d_send) cudaFree(c->d_send);
    if (c->d_recv) cudaFree(c->d_recv);
    delete c;
    return GKV_OK;
}

int gkv_comm_exchange_kind(const gkv_comm* c) { return c ? c->kind : 0; }

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
    const size_t per4 = (per + 3) / 4 * 4;  // mailbox slots hold whole float4s
    if (per4 > c->cap_floats) {
        cudaDeviceSynchronize();
        if (c->d_send) cudaFree(c->d_send);
        if (c->d_recv) cudaFree(c->d_recv);
        c->d_send = c->d_recv = nullptr;
        c->cap_floats = 0;
        cudaError_t e = cudaMalloc(&c->d_send, per4 * sizeof(float));
        if (e == cudaSuccess) e = cudaMalloc(&c->d_recv, per4 * sizeof(float) * c->n_ranks);
        if (e != cudaSuccess) return gkv::cuda_fail(e, "cudaMalloc(split-KV exchange)");
        c->cap_floats = per4;
    }
    if (c->kind == 0) {  // first call: map the mailboxes (or agree on the NCCL fallback)
        int rc = setup_exchange(c, static_cast<int64_t>(per), st);
        if (rc != GKV_OK) return rc;
    }
    // the slot size is fixed at set-up; every rank sees the same rows, so all take the same path
    const bool p2p = c->kind == 2 && static_cast<int64_t>(per4) <= c->peers.slot && dv % 4 == 0;
    unsigned ep = 0;
    int parity = 0;
    float* send_out = c->d_send;
    if (p2p) {  // the decode writes straight into this rank's own mailbox slot
        ep = ++c->epoch;
        parity = static_cast<int>(ep & 1u);
        send_out = gkv::exchange_slot(c->peers, c->rank, parity);
    }
    float* send_lse = send_out + rows * dv;
    P.last_launches = 0;
    // rows this rank holds no tokens of keep lse = -inf (weight 0 in the merge); when every
    // sequence has tokens here the decode writes every row and the fill launch is skipped
    cudaError_t e = cudaSuccess;
    int fills = 0;
    if (std::find(P.ws.h_ctx.begin(), P.ws.h_ctx.end(), 0) != P.ws.h_ctx.end()) {
        e = gkv::launch_fill(send_lse, rows, -INFINITY, st);
        if (e != cudaSuccess) return gkv::cuda_fail(e, "fill launch");
        fills = 1;
    }
    int rc = gkv::step_decode_lse(&P, layer, d_q, send_out, send_lse, n_heads, scale, nullptr, st);
    if (rc != GKV_OK) return rc;
    const int launches = P.last_launches + fills;
    if (p2p) {
        e = gkv::launch_exchange_pull_merge(c->peers, c->rank, parity, ep, static_cast<int>(rows), dv, d_sinks, n_heads,
                                            d_out, P.ws.d_err, st);
        if (e != cudaSuccess) return gkv::cuda_fail(e, "exchange merge launch");
        P.last_launches = launches + 1;
        return GKV_OK;
    }
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
