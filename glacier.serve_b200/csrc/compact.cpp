// Compaction of the block arena after evictions.
//
// The reference recycles a finished or cancelled sequence's blocks in the engine's eviction
// loop (ContinuousBatchEngine.cs:498-512 -> BlockTable.ReleaseAll, BlockTable.cs:108-116) and
// never moves a live block, so after admit/evict churn the live blocks are scattered over the
// whole pool.  On the device that costs page-granular gathers spread over the arena and keeps a
// fragmented free list.  This file turns a fragmented pool into a compact one:
//
//  * plan: a block may move only if every reference to it is accounted for by the tables the
//    caller passes (its reference count equals its number of occurrences in them) -- a block
//    also held elsewhere (a prefix-cache lookup in flight, a table not passed) stays put.
//    Free ids are taken from the bottom, movable blocks from the top (two fingers), until they
//    meet or max_moves is reached, so the number of moves is the least that fills the holes
//    below the live blocks;
//  * device: ONE batched block-copy launch (the CopyBlockData kernel, PagedBlockPool.cs:
//    304-327) copies each moved block's every (layer, head) page, K and V, on the caller's
//    stream, after the pool's queued copy-on-write copies;
//  * host: reference counts and prefix-cache bindings (the hash -> id map and the per-block
//    hash, PagedBlockPool.cs:168-234) move with their blocks, every passed table is rewritten,
//    and the free list is rebuilt so that the lowest free id pops first (the pool's initial
//    order, PagedBlockPool.cs:116-120).
#include <algorithm>
#include <memory>
#include <vector>

#include "gkv_internal.h"

namespace gkv {

void FreeStack::rebuild(const std::vector<int32_t>& pop_order) {
    head_.store(0, std::memory_order_relaxed);
    count_.store(0, std::memory_order_relaxed);
    for (auto it = pop_order.rbegin(); it != pop_order.rend(); ++it) push(*it);
}

int Pool::compact(Table* const* tables, int32_t n_tables, int32_t max_moves, std::vector<int32_t>* src,
                  std::vector<int32_t>* dst, cudaStream_t st) {
    const int32_t N = desc.total_blocks;
    src->clear();
    dst->clear();
    // references the passed tables hold, per block
    std::vector<int32_t> occ(static_cast<size_t>(N), 0);
    for (int32_t t = 0; t < n_tables; ++t)
        for (int32_t id : tables[t]->ids)
            if (in_range(id)) ++occ[static_cast<size_t>(id)];
    auto is_free = [&](int32_t b) { return allocated[b].load(std::memory_order_acquire) == 0; };
    auto movable = [&](int32_t b) {
        return !is_free(b) && occ[static_cast<size_t>(b)] > 0 &&
               refcount[b].load(std::memory_order_acquire) == occ[static_cast<size_t>(b)];
    };
    int32_t lo = 0, hi = N - 1;
    for (;;) {
        while (lo < N && !is_free(lo)) ++lo;
        while (hi >= 0 && !movable(hi)) --hi;
        if (lo >= hi || (max_moves > 0 && static_cast<int32_t>(src->size()) >= max_moves)) break;
        src->push_back(hi);
        dst->push_back(lo);
        ++lo;
        --hi;
    }
    if (src->empty()) return 0;
    // the queued forks name ids of the old layout: they go first, then the moves
    if (has_arena) {
        int rc = flush_copies(st);
        if (rc != GKV_OK) return rc;
        std::vector<int32_t> ops;
        ops.reserve(src->size() * 3);
        for (size_t i = 0; i < src->size(); ++i) {
            ops.push_back((*src)[i]);
            ops.push_back((*dst)[i]);
            ops.push_back(desc.block_size);
        }
        rc = launch_copies(ops.data(), static_cast<int>(src->size()), st);
        if (rc != GKV_OK) return rc;
        last_launches += 1;
    }
    // host state follows the data
    std::vector<int32_t> remap(static_cast<size_t>(N), -1);
    for (size_t i = 0; i < src->size(); ++i) {
        const int32_t s = (*src)[i], d = (*dst)[i];
        remap[static_cast<size_t>(s)] = d;
        const uint64_t h = prefix_hash[s].load(std::memory_order_acquire);
        refcount[d].store(refcount[s].load(std::memory_order_acquire), std::memory_order_release);
        prefix_hash[d].store(h, std::memory_order_release);
        allocated[d].store(1, std::memory_order_release);
        if (h != 0) {
            int32_t cur = -1;
            if (prefix_map.find(h, &cur) && cur == s) prefix_map.set(h, d);
        }
        refcount[s].store(0, std::memory_order_release);
        prefix_hash[s].store(0, std::memory_order_release);
        allocated[s].store(0, std::memory_order_release);
    }
    for (int32_t t = 0; t < n_tables; ++t)
        for (int32_t& id : tables[t]->ids)
            if (in_range(id) && remap[static_cast<size_t>(id)] >= 0) id = remap[static_cast<size_t>(id)];
    std::vector<int32_t> free_ids;
    free_ids.reserve(static_cast<size_t>(free_stack.count()));
    for (int32_t b = 0; b < N; ++b)
        if (is_free(b)) free_ids.push_back(b);
    free_stack.rebuild(free_ids);
    return static_cast<int>(src->size());
}

}  // namespace gkv

using gkv::set_error;

extern "C" int gkv_pool_compact(gkv_pool* pool, gkv_table* const* tables, int32_t n_tables, int32_t max_moves,
                                int32_t* out_src, int32_t* out_dst, int32_t cap, void* stream) {
    if (!pool) return set_error(GKV_EINVAL, "pool handle is NULL");
    gkv::Pool& P = pool->impl;
    if (n_tables < 0 || (n_tables > 0 && !tables)) return set_error(GKV_EINVAL, "tables is NULL");
    std::vector<gkv::Table*> ts(static_cast<size_t>(n_tables));
    for (int32_t t = 0; t < n_tables; ++t) {
        if (!tables[t] || tables[t]->impl.pool != &P)
            return set_error(GKV_EINVAL, "table %d is NULL or belongs to another pool", t);
        ts[static_cast<size_t>(t)] = &tables[t]->impl;
    }
    if (out_src || out_dst) {  // the move list must fit the caller's arrays
        if (cap < 0) return set_error(GKV_EINVAL, "cap %d < 0", cap);
        if (cap == 0) return 0;
        if (max_moves <= 0 || max_moves > cap) max_moves = cap;
    }
    std::vector<int32_t> src, dst;
    std::unique_ptr<gkv::DeviceGuard> guard;
    if (P.has_arena) guard.reset(new gkv::DeviceGuard(P.desc.device));
    P.last_launches = 0;
    const int n = P.compact(ts.data(), n_tables, max_moves, &src, &dst, static_cast<cudaStream_t>(stream));
    if (n < 0) return n;
    if (out_src || out_dst) {
        for (int32_t i = 0; i < n; ++i) {
            if (out_src) out_src[i] = src[static_cast<size_t>(i)];
            if (out_dst) out_dst[i] = dst[static_cast<size_t>(i)];
        }
    }
    return n;
}
