// Multi-GPU host logic: sequence partitioning over per-GPU pools and block-range splits.
//
// The reference is single-GPU (one GpuContext(0), src/Glacier.Serve/Inference/
// PagedAttention/CudaPagedTransformerRunner.cs:108).  Decode work shards naturally by
// sequence: each GPU owns its own pool and tables, so the only host decision is which GPU a
// sequence lives on.  Decode cost is proportional to context length, so sequences are
// placed longest-first onto the least-loaded rank (LPT), which keeps the slowest rank
// within 4/3 of optimal.
#include <algorithm>
#include <numeric>
#include <vector>

#include "gkv_internal.h"

using gkv::set_error;

extern "C" {

int gkv_partition_lpt(const int32_t* ctx_lens, int32_t n, int32_t n_ranks, int32_t* out_rank) {
    if (n < 0 || n_ranks < 1) return set_error(GKV_EINVAL, "n=%d n_ranks=%d", n, n_ranks);
    if (n > 0 && (!ctx_lens || !out_rank)) return set_error(GKV_EINVAL, "NULL argument");
    std::vector<int32_t> order(static_cast<size_t>(n));
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(),
                     [&](int32_t a, int32_t b) { return ctx_lens[a] > ctx_lens[b]; });
    std::vector<int64_t> load(static_cast<size_t>(n_ranks), 0);
    for (int32_t i : order) {
        int32_t best = 0;
        for (int32_t r = 1; r < n_ranks; ++r)
            if (load[static_cast<size_t>(r)] < load[static_cast<size_t>(best)]) best = r;
        out_rank[i] = best;
        load[static_cast<size_t>(best)] += ctx_lens[i] > 0 ? ctx_lens[i] : 0;
    }
    return GKV_OK;
}

int gkv_split_block_range(int32_t n_blocks, int32_t n_ranks, int32_t rank, int32_t* out_begin,
                          int32_t* out_end) {
    if (n_blocks < 0 || n_ranks < 1 || rank < 0 || rank >= n_ranks)
        return set_error(GKV_EINVAL, "n_blocks=%d n_ranks=%d rank=%d", n_blocks, n_ranks, rank);
    const int32_t base = n_blocks / n_ranks;
    const int32_t extra = n_blocks % n_ranks;
    const int32_t begin = rank * base + (rank < extra ? rank : extra);
    const int32_t end = begin + base + (rank < extra ? 1 : 0);
    if (out_begin) *out_begin = begin;
    if (out_end) *out_end = end;
    return GKV_OK;
}

}  // extern "C"
