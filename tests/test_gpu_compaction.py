"""gkv_pool_compact on the device: one batched block copy moves the live blocks, and the decode of
the rewritten tables gives the same bits as before the move (and the oracle's result)."""
import math

import numpy as np
import pytest

import glacier_kv as G
from gpu_helpers import TOL, arena_to_host, geom_of, random_arena
from oracle import pyoracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_decode_unchanged_after_compaction(cuda, dtype):
    import torch

    rng = np.random.default_rng(41)
    nb, nKv, d, bs = 400, 4, 128, 16
    pool = G.PagedBlockPool(nb, 2, nKv, d, bs, dtype=dtype)
    random_arena(pool, rng)
    # churn: admit 30 sequences, evict every other one, admit 6 more (they take the holes and the
    # top of the free list), with one shared prefix block and a copy-on-write fork queued
    tables = []
    for i in range(30):
        t = G.BlockTable(pool)
        for _ in range(int(rng.integers(5, 200))):
            assert t.append_token()[0]
        tables.append(t)
    for t in tables[::2]:
        t.release_all()
    tables = tables[1::2]
    shared = tables[0].get_block_id(0)
    for _ in range(6):
        t = G.BlockTable(pool)
        pool.retain_block(shared)
        t.attach_prefix_blocks([shared], 10)  # a partial shared block: the next append forks it
        for _ in range(int(rng.integers(1, 150))):
            assert t.append_token()[0]
        tables.append(t)
    ctx = np.array([t.token_count for t in tables], np.int32)
    q = torch.from_numpy(rng.standard_normal((len(tables), 28, d)).astype(np.float32)).to(cuda)
    out0 = torch.zeros((len(tables), 28, d), device=cuda)
    out1 = torch.zeros_like(out0)
    scale = 1 / math.sqrt(d)
    pool.upload_step_tables(tables)
    pool.paged_decode(1, q, out0, 28, scale)
    pool.sync()
    K0, V0 = arena_to_host(pool)
    src, dst = pool.compact(tables)
    assert len(src) > 0 and pool.last_launch_count == 1
    after = [t.as_span() for t in tables]
    assert max(int(r.max()) for r in after) < pool.allocated_blocks_count
    pool.upload_step_tables(tables)
    pool.paged_decode(1, q, out1, 28, scale)
    pool.sync()
    assert torch.equal(out0, out1)  # same values in the same order: the same bits
    K, V = arena_to_host(pool)
    # every moved block holds its source's data, all layers, heads and slots
    assert np.array_equal(K[dst], K0[src]) and np.array_equal(V[dst], V0[src])
    g = geom_of(pool)
    width = max(len(r) for r in after)
    tab = np.full((len(tables), width), -1, np.int32)
    for i, r in enumerate(after):
        tab[i, :len(r)] = r
    ref = O.decode_batch(K, V, g, 1, tab, ctx, q.cpu().numpy(), 28, scale)
    np.testing.assert_allclose(out1.cpu().numpy(), ref, atol=TOL[dtype], rtol=0)
    for t in tables:
        t.release_all()
    assert pool.free_blocks_count == nb
    pool.close()
