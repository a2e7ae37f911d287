// Host mirror of PagedBlockPool / BlockTable and the device block arena.
//
// Reference: src/Glacier.Serve/Inference/PagedAttention/PagedBlockPool.cs and BlockTable.cs.
// The allocator of record stays on the host (block ids only ever reach the device inside
// uploaded block tables and slot mappings); this file keeps the reference's semantics:
// LIFO free list popped 0..N-1 first, atomic reference counts starting at 1, idempotent
// release, prefix map with hash re-validation, copy-on-write forks.  What changes is that
// the K/V arena lives in HBM and CoW copies become batched device block copies.
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "gkv_internal.h"

namespace gkv {

// ---- errors ---------------------------------------------------------------------------

static thread_local std::string t_last_error;

int set_error(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    t_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    cudaGetLastError();  // clear the sticky-free error state of the runtime
    return set_error(e == cudaErrorMemoryAllocation ? GKV_ENOMEM : GKV_ECUDA, "%s: %s (%d)", what,
                     cudaGetErrorString(e), static_cast<int>(e));
}

DeviceGuard::DeviceGuard(int device) {
    if (cudaGetDevice(&prev_) != cudaSuccess) {
        cudaGetLastError();
        prev_ = -1;
    }
    if (prev_ == device) {
        ok_ = true;
        return;
    }
    ok_ = cudaSetDevice(device) == cudaSuccess;
    if (!ok_) cudaGetLastError();
}

DeviceGuard::~DeviceGuard() {
    int cur = -1;
    if (prev_ >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev_) cudaSetDevice(prev_);
}

// ---- free list ---------------------------------------------------------------------------

void FreeStack::init(int32_t n) {
    next_.reset(new std::atomic<int32_t>[static_cast<size_t>(n)]);
    head_.store(0, std::memory_order_relaxed);
    count_.store(0, std::memory_order_relaxed);
    // PagedBlockPool.cs:117-120 pushes N-1 down to 0, so block 0 is popped first.
    for (int32_t i = n - 1; i >= 0; --i) push(i);
}

void FreeStack::push(int32_t idx) {
    uint64_t old = head_.load(std::memory_order_acquire);
    for (;;) {
        const uint32_t top = static_cast<uint32_t>(old);  // index + 1, 0 = empty
        next_[idx].store(static_cast<int32_t>(top) - 1, std::memory_order_relaxed);
        const uint64_t tag = (old >> 32) + 1;
        const uint64_t nw = (tag << 32) | static_cast<uint32_t>(idx + 1);
        if (head_.compare_exchange_weak(old, nw, std::memory_order_acq_rel,
                                        std::memory_order_acquire))
            break;
    }
    count_.fetch_add(1, std::memory_order_acq_rel);
}

int32_t FreeStack::pop() {
    uint64_t old = head_.load(std::memory_order_acquire);
    for (;;) {
        const uint32_t top = static_cast<uint32_t>(old);
        if (top == 0) return -1;
        const int32_t idx = static_cast<int32_t>(top) - 1;
        const int32_t nxt = next_[idx].load(std::memory_order_relaxed);
        const uint64_t tag = (old >> 32) + 1;
        const uint64_t nw = (tag << 32) | static_cast<uint32_t>(nxt + 1);
        if (head_.compare_exchange_weak(old, nw, std::memory_order_acq_rel,
                                        std::memory_order_acquire)) {
            count_.fetch_sub(1, std::memory_order_acq_rel);
            return idx;
        }
    }
}

// ---- prefix map ----------------------------------------------------------------------------

bool PrefixMap::find(uint64_t h, int32_t* out) const {
    const Shard& s = shards_[shard_of(h)];
    std::lock_guard<std::mutex> lk(s.mu);
    auto it = s.map.find(h);
    if (it == s.map.end()) return false;
    *out = it->second;
    return true;
}

void PrefixMap::set(uint64_t h, int32_t id) {
    Shard& s = shards_[shard_of(h)];
    std::lock_guard<std::mutex> lk(s.mu);
    s.map[h] = id;
}

void PrefixMap::remove_if(uint64_t h, int32_t id) {
    Shard& s = shards_[shard_of(h)];
    std::lock_guard<std::mutex> lk(s.mu);
    auto it = s.map.find(h);
    if (it != s.map.end() && it->second == id) s.map.erase(it);
}

// ---- allocator primitives -----------------------------------------------------------------

int32_t Pool::try_allocate() {
    // TryAllocateBlock, PagedBlockPool.cs:178-189
    const int32_t id = free_stack.pop();
    if (id < 0) return -1;
    allocated[id].store(1, std::memory_order_release);
    refcount[id].store(1, std::memory_order_release);
    prefix_hash[id].store(0, std::memory_order_release);
    return id;
}

int Pool::release(int32_t b) {
    // ReleaseBlock, PagedBlockPool.cs:251-279
    if (!in_range(b)) return 0;
    const int remaining = refcount[b].fetch_sub(1, std::memory_order_acq_rel) - 1;
    if (remaining < 0) {
        refcount[b].store(0, std::memory_order_release);
        return 0;
    }
    if (remaining == 0) {
        const uint64_t h = prefix_hash[b].load(std::memory_order_acquire);
        if (h != 0) {
            prefix_map.remove_if(h, b);
            prefix_hash[b].store(0, std::memory_order_release);
        }
        int32_t one = 1;
        if (allocated[b].compare_exchange_strong(one, 0, std::memory_order_acq_rel))
            free_stack.push(b);
    }
    return remaining;
}

int Pool::retain(int32_t b) {
    // RetainBlock, PagedBlockPool.cs:240-245
    if (!in_range(b)) return set_error(GKV_EINVAL, "block id %d outside [0, %d)", b, desc.total_blocks);
    return refcount[b].fetch_add(1, std::memory_order_acq_rel) + 1;
}

int Pool::refs(int32_t b) const {
    // GetRefCount, PagedBlockPool.cs:285-289
    if (!in_range(b)) return 0;
    return refcount[b].load(std::memory_order_acquire);
}

bool Pool::try_find_prefix(uint64_t h, int32_t* out) {
    // TryFindPrefixBlock, PagedBlockPool.cs:194-220
    *out = -1;
    int32_t id = -1;
    if (h == 0 || !prefix_map.find(h, &id) || !in_range(id)) return false;
    for (;;) {
        int cur = refcount[id].load(std::memory_order_acquire);
        if (cur <= 0) return false;
        if (refcount[id].compare_exchange_weak(cur, cur + 1, std::memory_order_acq_rel)) {
            if (prefix_hash[id].load(std::memory_order_acquire) != h) {
                release(id);
                return false;
            }
            *out = id;
            return true;
        }
    }
}

bool Pool::try_fork(int32_t src, int32_t valid, int32_t* out) {
    // TryForkBlock, PagedBlockPool.cs:332-342; the data copy is queued for the device.
    const int32_t id = try_allocate();
    *out = id;
    if (id < 0) return false;
    if (has_arena && valid > 0 && in_range(src)) {
        std::lock_guard<std::mutex> lk(pending_mu);
        pending.push_back(src);
        pending.push_back(id);
        pending.push_back(valid);
    }
    return true;
}

int Pool::launch_copies(const int32_t* h_ops, int n, cudaStream_t st) {
    if (n <= 0) return GKV_OK;
    const size_t bytes = static_cast<size_t>(n) * 3 * sizeof(int32_t);
    if (bytes > copy_ops_cap) {
        if (copy_ops_copied) cudaEventSynchronize(copy_ops_copied);
        if (d_copy_ops) cudaFree(d_copy_ops);
        if (h_copy_ops) cudaFreeHost(h_copy_ops);
        d_copy_ops = nullptr;
        h_copy_ops = nullptr;
        copy_ops_cap = 0;
        size_t cap = 4096;
        while (cap < bytes) cap <<= 1;
        cudaError_t e = cudaMalloc(&d_copy_ops, cap);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(block copy ops)");
        e = cudaMallocHost(&h_copy_ops, cap);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMallocHost(block copy ops)");
        copy_ops_cap = cap;
        if (!copy_ops_copied) {
            e = cudaEventCreateWithFlags(&copy_ops_copied, cudaEventDisableTiming);
            if (e != cudaSuccess) return cuda_fail(e, "cudaEventCreate");
        }
    } else if (copy_ops_copied) {
        cudaError_t e = cudaEventSynchronize(copy_ops_copied);
        if (e != cudaSuccess) return cuda_fail(e, "cudaEventSynchronize(block copy ops)");
    }
    memcpy(h_copy_ops, h_ops, bytes);
    cudaError_t e = cudaMemcpyAsync(d_copy_ops, h_copy_ops, bytes, cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync(block copy ops)");
    e = cudaEventRecord(copy_ops_copied, st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
    e = launch_block_copy(geom, d_copy_ops, n, ws.d_err, st);
    if (e != cudaSuccess) return cuda_fail(e, "block_copy launch");
    return GKV_OK;
}

int Pool::flush_copies(cudaStream_t st) {
    std::vector<int32_t> ops;
    {
        std::lock_guard<std::mutex> lk(pending_mu);
        ops.swap(pending);
    }
    if (ops.empty()) return GKV_OK;
    const int rc = launch_copies(ops.data(), static_cast<int>(ops.size() / 3), st);
    if (rc == GKV_OK) last_launches += 1;
    return rc;
}

}  // namespace gkv

using gkv::Pool;
using gkv::set_error;

#define GKV_CHECK_POOL(p)                                                  \
    do {                                                                   \
        if (!(p)) return set_error(GKV_EINVAL, "pool handle is NULL");     \
    } while (0)

extern "C" {

const char* gkv_last_error(void) { return gkv::t_last_error.c_str(); }

const char* gkv_version(void) { return "glacier_kv 0.1 sm_100a"; }

int gkv_pool_create(const gkv_pool_desc* desc, gkv_pool** out_pool) {
    if (!desc || !out_pool) return set_error(GKV_EINVAL, "desc/out_pool is NULL");
    *out_pool = nullptr;
    gkv_pool_desc d = *desc;
    if (d.block_size == 0) d.block_size = 16;
    if (d.v_head_dim <= 0) d.v_head_dim = d.head_dim;
    // PagedBlockPool.cs:63-67
    if (d.total_blocks < 1) return set_error(GKV_EINVAL, "totalBlocks must be >= 1 (got %d)", d.total_blocks);
    if (d.layers < 1) return set_error(GKV_EINVAL, "layers must be >= 1 (got %d)", d.layers);
    if (d.heads_kv < 1) return set_error(GKV_EINVAL, "headsKv must be >= 1 (got %d)", d.heads_kv);
    if (d.head_dim < 1) return set_error(GKV_EINVAL, "headDim must be >= 1 (got %d)", d.head_dim);
    if (d.block_size < 1) return set_error(GKV_EINVAL, "blockSize must be >= 1 (got %d)", d.block_size);
    if (!gkv::valid_kv_dtype(d.dtype))
        return set_error(GKV_EINVAL, "dtype %d is not GKV_DTYPE_F32, _BF16, _F16 or _FP8_E4M3", d.dtype);
    // FP8 rows are whole 16-byte vectors (appends store 4 elements a lane, block copies move
    // 2 bytes a lane at least, decode copies 8-token spans in 16-byte units)
    if (d.dtype == GKV_DTYPE_FP8_E4M3 && (d.head_dim % 16 != 0 || d.v_head_dim % 16 != 0))
        return set_error(GKV_EINVAL, "FP8 storage needs head dims that are multiples of 16 (got %d / %d)",
                         d.head_dim, d.v_head_dim);
    if (d.allocate_device_arena && d.device < 0) return set_error(GKV_EINVAL, "device %d < 0", d.device);

    gkv_pool* p = new (std::nothrow) gkv_pool();
    if (!p) return set_error(GKV_ENOMEM, "host allocation failed");
    Pool& P = p->impl;
    P.desc = d;
    P.elem_bytes = static_cast<size_t>(gkv::elem_bytes_of(d.dtype));
    // strides, PagedBlockPool.cs:77-83
    gkv::ArenaGeom& g = P.geom;
    g.k_head_stride = static_cast<int64_t>(d.block_size) * d.head_dim;
    g.k_layer_stride = static_cast<int64_t>(d.heads_kv) * g.k_head_stride;
    g.k_block_stride = static_cast<int64_t>(d.layers) * g.k_layer_stride;
    g.v_head_stride = static_cast<int64_t>(d.block_size) * d.v_head_dim;
    g.v_layer_stride = static_cast<int64_t>(d.heads_kv) * g.v_head_stride;
    g.v_block_stride = static_cast<int64_t>(d.layers) * g.v_layer_stride;
    g.total_blocks = d.total_blocks;
    g.layers = d.layers;
    g.heads_kv = d.heads_kv;
    g.head_dim = d.head_dim;
    g.v_head_dim = d.v_head_dim;
    g.block_size = d.block_size;
    g.dtype = d.dtype;
    P.k_bytes = static_cast<int64_t>(d.total_blocks) * g.k_block_stride * static_cast<int64_t>(P.elem_bytes);
    P.v_bytes = static_cast<int64_t>(d.total_blocks) * g.v_block_stride * static_cast<int64_t>(P.elem_bytes);
    if (static_cast<int64_t>(d.total_blocks) * d.block_size > INT32_MAX) {
        delete p;
        return set_error(GKV_EINVAL, "totalBlocks * blockSize overflows int32 token slots");
    }

    P.allocated.reset(new std::atomic<int32_t>[static_cast<size_t>(d.total_blocks)]);
    P.refcount.reset(new std::atomic<int32_t>[static_cast<size_t>(d.total_blocks)]);
    P.prefix_hash.reset(new std::atomic<uint64_t>[static_cast<size_t>(d.total_blocks)]);
    for (int32_t i = 0; i < d.total_blocks; ++i) {
        P.allocated[i].store(0, std::memory_order_relaxed);
        P.refcount[i].store(0, std::memory_order_relaxed);
        P.prefix_hash[i].store(0, std::memory_order_relaxed);
    }
    P.free_stack.init(d.total_blocks);

    if (d.allocate_device_arena) {
        gkv::DeviceGuard guard(d.device);
        if (!guard.ok()) {
            delete p;
            return set_error(GKV_ECUDA, "cudaSetDevice(%d) failed", d.device);
        }
        void* k = nullptr;
        void* v = nullptr;
        cudaError_t e = cudaMalloc(&k, static_cast<size_t>(P.k_bytes));
        if (e == cudaSuccess) e = cudaMalloc(&v, static_cast<size_t>(P.v_bytes));
        if (e == cudaSuccess) e = cudaMemset(k, 0, static_cast<size_t>(P.k_bytes));
        if (e == cudaSuccess) e = cudaMemset(v, 0, static_cast<size_t>(P.v_bytes));
        if (e == cudaSuccess) e = cudaMalloc(&P.ws.d_err, sizeof(int));
        if (e == cudaSuccess) e = cudaMemset(P.ws.d_err, 0, sizeof(int));
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) {
            const int rc = gkv::cuda_fail(e, "device arena allocation");
            if (k) cudaFree(k);
            if (v) cudaFree(v);
            if (P.ws.d_err) cudaFree(P.ws.d_err);
            delete p;
            return rc;
        }
        g.k = k;
        g.v = v;
        P.has_arena = true;
        if (d.dtype == GKV_DTYPE_FP8_E4M3) {
            // scales and reciprocals start at 1
            const size_t n = static_cast<size_t>(d.layers) * d.heads_kv;
            std::vector<float> ones(4 * n, 1.f);
            e = cudaMalloc(&P.d_scales, 4 * n * sizeof(float));
            if (e == cudaSuccess) e = cudaMemcpy(P.d_scales, ones.data(), 4 * n * sizeof(float), cudaMemcpyHostToDevice);
            if (e != cudaSuccess) {
                const int rc = gkv::cuda_fail(e, "fp8 scale allocation");
                if (P.d_scales) cudaFree(P.d_scales);
                cudaFree(k);
                cudaFree(v);
                cudaFree(P.ws.d_err);
                delete p;
                return rc;
            }
            g.k_scale = P.d_scales;
            g.v_scale = P.d_scales + n;
            g.k_inv = P.d_scales + 2 * n;
            g.v_inv = P.d_scales + 3 * n;
        }
        // TMA maps for the tensor-core kernels (16-bit or FP8 storage, d = dv = 128,
        // 8-token-aligned blocks); 16-bit copies move 2-byte elements, whichever format
        int rank = 0;
        if (d.dtype != GKV_DTYPE_F32 && d.head_dim == 128 && d.v_head_dim == 128 && d.block_size % 8 == 0)
            rank = gkv::encode_decode_tmaps(g, P.tmap_k, P.tmap_v);
        if (rank > 0) {
            g.tmap_k = P.tmap_k;
            g.tmap_v = P.tmap_v;
            g.tmap_rank = rank;
        }
        if (rank > 0 && d.dtype != GKV_DTYPE_FP8_E4M3) {
            // whole-page boxes (16 slots) for the prefill kernel when the block size allows
            if (d.block_size % 16 == 0 && gkv::encode_arena_map(P.tmap_pk, g.k, g, 128, 16) &&
                gkv::encode_arena_map(P.tmap_pv, g.v, g, 128, 16)) {
                g.tmap_pk = P.tmap_pk;
                g.tmap_pv = P.tmap_pv;
            }
        }
    }
    *out_pool = p;
    return GKV_OK;
}

int gkv_pool_destroy(gkv_pool* pool) {
    if (!pool) return GKV_OK;
    Pool& P = pool->impl;
    if (P.has_arena) {
        gkv::DeviceGuard guard(P.desc.device);
        cudaDeviceSynchronize();
        gkv::step_free(&P);
        if (P.d_copy_ops) cudaFree(P.d_copy_ops);
        if (P.h_copy_ops) cudaFreeHost(P.h_copy_ops);
        if (P.copy_ops_copied) cudaEventDestroy(P.copy_ops_copied);
        if (P.ws.d_err) cudaFree(P.ws.d_err);
        if (P.d_scales) cudaFree(P.d_scales);
        cudaFree(P.geom.k);
        cudaFree(P.geom.v);
    }
    delete pool;
    return GKV_OK;
}

int gkv_pool_set_kv_scales(gkv_pool* pool, const float* h_k_scales, const float* h_v_scales) {
    GKV_CHECK_POOL(pool);
    Pool& P = pool->impl;
    if (P.desc.dtype != GKV_DTYPE_FP8_E4M3) return set_error(GKV_ESTATE, "KV scales belong to FP8 pools");
    if (!h_k_scales || !h_v_scales) return set_error(GKV_EINVAL, "scales are NULL");
    const size_t n = static_cast<size_t>(P.desc.layers) * P.desc.heads_kv;
    std::vector<float> all(4 * n);
    for (size_t i = 0; i < n; ++i) {
        const float ks = h_k_scales[i], vs = h_v_scales[i];
        if (!(ks > 0.f) || !(vs > 0.f) || !std::isfinite(ks) || !std::isfinite(vs))
            return set_error(GKV_EINVAL, "scale %zu (%g, %g) is not positive and finite", i, static_cast<double>(ks),
                             static_cast<double>(vs));
        all[i] = ks;
        all[n + i] = vs;
        all[2 * n + i] = 1.f / ks;
        all[3 * n + i] = 1.f / vs;
    }
    if (!P.has_arena) return GKV_OK;
    gkv::DeviceGuard guard(P.desc.device);
    cudaError_t e = cudaMemcpy(P.d_scales, all.data(), 4 * n * sizeof(float), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return gkv::cuda_fail(e, "cudaMemcpy(fp8 scales)");
    return GKV_OK;
}

int gkv_pool_stats_get(const gkv_pool* pool, gkv_pool_stats* s) {
    GKV_CHECK_POOL(pool);
    if (!s) return set_error(GKV_EINVAL, "stats is NULL");
    const Pool& P = pool->impl;
    const int32_t free_n = P.free_stack.count();
    s->total_blocks = P.desc.total_blocks;
    s->free_blocks = free_n;
    s->allocated_blocks = P.desc.total_blocks - free_n;
    s->capacity_tokens = P.desc.total_blocks * P.desc.block_size;
    s->active_tokens = s->allocated_blocks * P.desc.block_size;
    s->block_size = P.desc.block_size;
    {
        std::lock_guard<std::mutex> lk(const_cast<Pool&>(P).pending_mu);
        s->pending_copies = static_cast<int32_t>(P.pending.size() / 3);
    }
    s->has_device_arena = P.has_arena ? 1 : 0;
    s->total_memory_bytes = P.has_arena ? P.k_bytes + P.v_bytes : 0;
    return GKV_OK;
}

int gkv_pool_kv_ptrs(const gkv_pool* pool, void** d_k, void** d_v) {
    GKV_CHECK_POOL(pool);
    if (d_k) *d_k = pool->impl.geom.k;
    if (d_v) *d_v = pool->impl.geom.v;
    return GKV_OK;
}

int gkv_pool_element_offset(const gkv_pool* pool, int32_t which, int32_t block, int32_t layer,
                            int32_t head_kv, int32_t slot, int64_t* out_offset) {
    GKV_CHECK_POOL(pool);
    const Pool& P = pool->impl;
    if (!out_offset) return set_error(GKV_EINVAL, "out_offset is NULL");
    if (!P.in_range(block) || layer < 0 || layer >= P.desc.layers || head_kv < 0 ||
        head_kv >= P.desc.heads_kv || slot < 0 || slot >= P.desc.block_size)
        return set_error(GKV_EINVAL, "(block %d, layer %d, head %d, slot %d) outside the arena",
                         block, layer, head_kv, slot);
    const gkv::ArenaGeom& g = P.geom;
    if (which == 0)
        *out_offset = block * g.k_block_stride + layer * g.k_layer_stride +
                      head_kv * g.k_head_stride + static_cast<int64_t>(slot) * g.head_dim;
    else
        *out_offset = block * g.v_block_stride + layer * g.v_layer_stride +
                      head_kv * g.v_head_stride + static_cast<int64_t>(slot) * g.v_head_dim;
    return GKV_OK;
}

int gkv_pool_try_allocate_block(gkv_pool* pool, int32_t* out_block) {
    GKV_CHECK_POOL(pool);
    const int32_t id = pool->impl.try_allocate();
    if (out_block) *out_block = id;
    return id >= 0 ? 1 : 0;
}

int gkv_pool_release_block(gkv_pool* pool, int32_t block) {
    GKV_CHECK_POOL(pool);
    return pool->impl.release(block);
}

int gkv_pool_free_block(gkv_pool* pool, int32_t block) {
    GKV_CHECK_POOL(pool);
    pool->impl.release(block);
    return GKV_OK;
}

int gkv_pool_free_blocks(gkv_pool* pool, const int32_t* blocks, int32_t n) {
    GKV_CHECK_POOL(pool);
    if (n > 0 && !blocks) return set_error(GKV_EINVAL, "blocks is NULL");
    for (int32_t i = 0; i < n; ++i) pool->impl.release(blocks[i]);
    return GKV_OK;
}

int gkv_pool_retain_block(gkv_pool* pool, int32_t block) {
    GKV_CHECK_POOL(pool);
    return pool->impl.retain(block);
}

int gkv_pool_get_ref_count(const gkv_pool* pool, int32_t block) {
    GKV_CHECK_POOL(pool);
    return pool->impl.refs(block);
}

int gkv_pool_try_find_prefix_block(gkv_pool* pool, uint64_t prefix_hash, int32_t* out_block) {
    GKV_CHECK_POOL(pool);
    int32_t id = -1;
    const bool ok = pool->impl.try_find_prefix(prefix_hash, &id);
    if (out_block) *out_block = id;
    return ok ? 1 : 0;
}

int gkv_pool_bind_prefix_block(gkv_pool* pool, uint64_t prefix_hash, int32_t block) {
    GKV_CHECK_POOL(pool);
    Pool& P = pool->impl;
    // BindPrefixBlock, PagedBlockPool.cs:225-234
    if (!P.in_range(block)) return set_error(GKV_EINVAL, "block id %d outside [0, %d)", block, P.desc.total_blocks);
    if (prefix_hash == 0) return set_error(GKV_EINVAL, "Prefix hash cannot be 0.");
    P.prefix_hash[block].store(prefix_hash, std::memory_order_release);
    P.prefix_map.set(prefix_hash, block);
    return GKV_OK;
}

int gkv_pool_try_fork_block(gkv_pool* pool, int32_t src_block, int32_t valid_tokens,
                            int32_t* out_block) {
    GKV_CHECK_POOL(pool);
    int32_t id = -1;
    const bool ok = pool->impl.try_fork(src_block, valid_tokens, &id);
    if (out_block) *out_block = id;
    return ok ? 1 : 0;
}

int gkv_pool_flush_copies(gkv_pool* pool, void* stream) {
    GKV_CHECK_POOL(pool);
    Pool& P = pool->impl;
    if (!P.has_arena) return GKV_OK;
    gkv::DeviceGuard guard(P.desc.device);
    P.last_launches = 0;
    return P.flush_copies(static_cast<cudaStream_t>(stream));
}

int gkv_block_copy(gkv_pool* pool, const int32_t* h_src, const int32_t* h_dst,
                   const int32_t* h_valid, int32_t n, void* stream) {
    GKV_CHECK_POOL(pool);
    Pool& P = pool->impl;
    if (!P.has_arena) return set_error(GKV_ESTATE, "Host KV buffers were omitted.");
    if (n < 0 || (n > 0 && (!h_src || !h_dst || !h_valid)))
        return set_error(GKV_EINVAL, "bad block copy list (n=%d)", n);
    std::vector<int32_t> ops;
    ops.reserve(static_cast<size_t>(n) * 3);
    for (int32_t i = 0; i < n; ++i) {
        if (h_valid[i] <= 0) continue;  // CopyBlockData returns early, PagedBlockPool.cs:308
        if (!P.in_range(h_src[i]) || !P.in_range(h_dst[i]))
            return set_error(GKV_EINVAL, "block copy %d: (%d -> %d) outside [0, %d)", i, h_src[i],
                             h_dst[i], P.desc.total_blocks);
        ops.push_back(h_src[i]);
        ops.push_back(h_dst[i]);
        ops.push_back(h_valid[i] < P.desc.block_size ? h_valid[i] : P.desc.block_size);
    }
    gkv::DeviceGuard guard(P.desc.device);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    P.last_launches = 0;
    int rc = P.flush_copies(st);
    if (rc != GKV_OK) return rc;
    rc = P.launch_copies(ops.data(), static_cast<int>(ops.size() / 3), st);
    if (rc == GKV_OK && !ops.empty()) P.last_launches += 1;
    return rc;
}

int gkv_pool_store(gkv_pool* pool, int32_t block, int32_t layer, int32_t slot, const float* d_k,
                   const float* d_v, void* stream) {
    GKV_CHECK_POOL(pool);
    Pool& P = pool->impl;
    if (!P.has_arena)
        return set_error(GKV_ESTATE, "Host KV buffers were omitted because KV pages reside exclusively in GPU VRAM.");
    if (!P.in_range(block) || layer < 0 || layer >= P.desc.layers || slot < 0 || slot >= P.desc.block_size)
        return set_error(GKV_EINVAL, "store target (block %d, layer %d, slot %d) outside the arena", block, layer, slot);
    if (!d_k || !d_v) return set_error(GKV_EINVAL, "k/v source is NULL");
    gkv::DeviceGuard guard(P.desc.device);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    P.last_launches = 0;
    int rc = P.flush_copies(st);
    if (rc != GKV_OK) return rc;
    const int64_t s = static_cast<int64_t>(block) * P.desc.block_size + slot;
    cudaError_t e = gkv::launch_kv_append(P.geom, layer, d_k, d_v, 0, 0, nullptr, s, 1, P.ws.d_err, st);
    if (e != cudaSuccess) return gkv::cuda_fail(e, "kv_append launch");
    P.last_launches += 1;
    return GKV_OK;
}

int gkv_pool_last_launch_count(const gkv_pool* pool) {
    GKV_CHECK_POOL(pool);
    return pool->impl.last_launches;
}

// ---- BlockTable -------------------------------------------------------------------------

int gkv_table_create(gkv_pool* pool, gkv_table** out_table) {
    if (!pool) return set_error(GKV_EINVAL, "pool is NULL (ArgumentNullException)");
    if (!out_table) return set_error(GKV_EINVAL, "out_table is NULL");
    gkv_table* t = new (std::nothrow) gkv_table();
    if (!t) return set_error(GKV_ENOMEM, "host allocation failed");
    t->impl.pool = &pool->impl;
    t->impl.ids.reserve(16);
    *out_table = t;
    return GKV_OK;
}

int gkv_table_destroy(gkv_table* table) {
    delete table;
    return GKV_OK;
}

int gkv_table_attach_prefix_blocks(gkv_table* table, const int32_t* blocks, int32_t n,
                                   int32_t token_count) {
    if (!table) return set_error(GKV_EINVAL, "table is NULL");
    // AttachPrefixBlocks, BlockTable.cs:31-39
    if (token_count < 0) return set_error(GKV_EINVAL, "tokenCount must be >= 0 (got %d)", token_count);
    if (n > 0 && !blocks) return set_error(GKV_EINVAL, "blocks is NULL");
    for (int32_t i = 0; i < n; ++i) table->impl.ids.push_back(blocks[i]);
    table->impl.token_count = token_count;
    return GKV_OK;
}

int gkv_table_append_token(gkv_table* table, int32_t* out_block, int32_t* out_offset) {
    if (!table) return set_error(GKV_EINVAL, "table is NULL");
    gkv::Table& T = table->impl;
    Pool& P = *T.pool;
    const int32_t bs = P.desc.block_size;
    auto fail = [&]() {
        if (out_block) *out_block = -1;
        if (out_offset) *out_offset = -1;
        return 0;
    };
    // AppendToken, BlockTable.cs:46-80
    if (T.token_count % bs == 0) {
        const int32_t id = P.try_allocate();
        if (id < 0) return fail();
        T.ids.push_back(id);
    } else {
        if (T.ids.empty())
            return set_error(GKV_ESTATE, "table has %d tokens but no blocks", T.token_count);
        const int32_t last = T.ids.back();
        if (P.refs(last) > 1) {
            int32_t forked = -1;
            if (!P.try_fork(last, T.token_count % bs, &forked)) return fail();
            P.release(last);
            T.ids.back() = forked;
        }
    }
    if (out_block) *out_block = T.ids.back();
    if (out_offset) *out_offset = T.token_count % bs;
    T.token_count += 1;
    return 1;
}

int gkv_table_get_token_location(const gkv_table* table, int32_t token_index, int32_t* out_block,
                                 int32_t* out_offset) {
    if (!table) return set_error(GKV_EINVAL, "table is NULL");
    const gkv::Table& T = table->impl;
    const int32_t bs = T.pool->desc.block_size;
    // GetTokenLocation, BlockTable.cs:86-91 (List indexer throws out of range)
    const int32_t bi = token_index / bs;
    if (token_index < 0 || bi >= static_cast<int32_t>(T.ids.size()))
        return set_error(GKV_EINVAL, "token index %d has no block (BlockCount %zu)", token_index, T.ids.size());
    if (out_block) *out_block = T.ids[static_cast<size_t>(bi)];
    if (out_offset) *out_offset = token_index % bs;
    return GKV_OK;
}

int gkv_table_get_block_id(const gkv_table* table, int32_t block_index) {
    if (!table) return set_error(GKV_EINVAL, "table is NULL");
    const gkv::Table& T = table->impl;
    if (block_index < 0 || block_index >= static_cast<int32_t>(T.ids.size()))
        return set_error(GKV_EINVAL, "block index %d outside [0, %zu)", block_index, T.ids.size());
    return T.ids[static_cast<size_t>(block_index)];
}

int gkv_table_token_count(const gkv_table* table) {
    if (!table) return set_error(GKV_EINVAL, "table is NULL");
    return table->impl.token_count;
}

int gkv_table_block_count(const gkv_table* table) {
    if (!table) return set_error(GKV_EINVAL, "table is NULL");
    return static_cast<int>(table->impl.ids.size());
}

int gkv_table_block_ids(const gkv_table* table, int32_t* out, int32_t cap) {
    if (!table) return set_error(GKV_EINVAL, "table is NULL");
    const gkv::Table& T = table->impl;
    const int32_t n = static_cast<int32_t>(T.ids.size());
    for (int32_t i = 0; i < n && i < cap && out; ++i) out[i] = T.ids[static_cast<size_t>(i)];
    return n;
}

int gkv_table_release_all(gkv_table* table) {
    if (!table) return set_error(GKV_EINVAL, "table is NULL");
    gkv::Table& T = table->impl;
    // ReleaseAll, BlockTable.cs:108-116
    for (int32_t id : T.ids) T.pool->release(id);
    T.ids.clear();
    T.token_count = 0;
    return GKV_OK;
}

}  // extern "C"
