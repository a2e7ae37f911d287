"""gkv_pool_compact on the host (metadata-only pools, no GPU): after a seeded admit/evict churn
the planner moves the live blocks into the lowest ids with no block lost or duplicated, the
reference counts and prefix-cache bindings follow the blocks, blocks held outside the passed tables
stay put, and the free list pops the lowest free id first afterwards (PagedBlockPool.cs:116-120,
178-299; the reference's evict loop, ContinuousBatchEngine.cs:498-512, never moves a block)."""
import numpy as np
import pytest

import glacier_kv as G


def _churn(pool, rng, n_seq=40, rounds=300):
    """Admit/evict on real BlockTables, with prefix sharing and copy-on-write forks."""
    live = []
    for _ in range(rounds):
        if live and rng.random() < 0.45:
            t = live.pop(int(rng.integers(len(live))))
            t.release_all()
            continue
        t = G.BlockTable(pool)
        if live and rng.random() < 0.3:  # share a full prefix block of a live table
            donor = live[int(rng.integers(len(live)))]
            if donor.block_count > 1:
                b = donor.get_block_id(0)
                pool.retain_block(b)
                t.attach_prefix_blocks([b], 16)
        for _ in range(int(rng.integers(1, 120))):
            ok, _, _ = t.append_token()
            if not ok:
                break
        live.append(t)
        if len(live) > n_seq:
            live.pop(0).release_all()
    return live


def _snapshot(pool, tables):
    """Per logical block reference: (table index, block index) -> id, and id -> refcount."""
    ids = [t.as_span().tolist() for t in tables]
    refs = {b: pool.get_ref_count(b) for row in ids for b in row}
    return ids, refs


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_compaction_moves_blocks_down_and_keeps_every_reference(seed):
    rng = np.random.default_rng(seed)
    pool = G.PagedBlockPool(600, 2, 2, 32, 16, allocate_device_arena=False)
    tables = _churn(pool, rng)
    h = 0xABCD0000 + seed
    bound = tables[0].get_block_id(0)
    pool.bind_prefix_block(h, bound)
    ids0, refs0 = _snapshot(pool, tables)
    allocated0 = pool.allocated_blocks_count
    live0 = sorted({b for row in ids0 for b in row})
    assert len(live0) == allocated0  # every allocated block belongs to a passed table
    src, dst = pool.compact(tables)
    ids1, refs1 = _snapshot(pool, tables)
    # the moves: distinct sources (live, high) onto distinct destinations (free, low)
    assert len(set(src.tolist())) == len(src) and len(set(dst.tolist())) == len(dst)
    assert set(src.tolist()) <= set(live0) and not set(dst.tolist()) & set(live0)
    assert all(d < s for s, d in zip(src, dst))
    remap = dict(zip(src.tolist(), dst.tolist()))
    # every table is the old one with moved ids renamed; shared blocks stay shared
    for r0, r1 in zip(ids0, ids1):
        assert r1 == [remap.get(b, b) for b in r0]
    # reference counts followed their blocks; nothing was allocated or freed
    for b, c in refs0.items():
        assert refs1[remap.get(b, b)] == c
    assert pool.allocated_blocks_count == allocated0
    assert pool.free_blocks_count == 600 - allocated0
    # compact: the live blocks are exactly ids 0 .. n-1
    assert sorted({b for row in ids1 for b in row}) == list(range(allocated0))
    for b in src:
        assert pool.get_ref_count(int(b)) == 0
    # the prefix binding moved with its block
    ok, found = pool.try_find_prefix_block(h)
    assert ok and found == remap.get(bound, bound)
    pool.release_block(found)
    # the lowest free id pops first; a second compaction has nothing to do
    ok, nxt = pool.try_allocate_block()
    assert ok and nxt == allocated0
    pool.release_block(nxt)
    assert pool.compact(tables)[0].size == 0
    for t in tables:
        t.release_all()
    assert pool.free_blocks_count == 600
    pool.close()


def test_blocks_held_outside_the_passed_tables_stay_put():
    pool = G.PagedBlockPool(64, 1, 1, 32, 16, allocate_device_arena=False)
    a, b = G.BlockTable(pool), G.BlockTable(pool)
    for t, n in ((a, 40), (b, 40)):
        for _ in range(n):
            assert t.append_token()[0]
    held = G.BlockTable(pool)  # not passed: its blocks must not move
    for _ in range(20):
        assert held.append_token()[0]
    a.release_all()  # holes at the bottom
    pinned = held.as_span().tolist()
    extra = b.get_block_id(1)
    pool.retain_block(extra)  # a reference the tables do not account for
    src, dst = pool.compact([b])
    assert not set(src.tolist()) & (set(pinned) | {extra})
    assert held.as_span().tolist() == pinned
    assert extra in b.as_span().tolist()
    # max_moves bounds the work of one call
    pool.release_block(extra)
    b2 = G.BlockTable(pool)
    for _ in range(70):
        assert b2.append_token()[0]
    b.release_all()
    src, _ = pool.compact([b2, held], max_moves=2)
    assert len(src) <= 2
    pool.close()


def test_compaction_rejects_foreign_tables():
    p1 = G.PagedBlockPool(8, 1, 1, 32, 16, allocate_device_arena=False)
    p2 = G.PagedBlockPool(8, 1, 1, 32, 16, allocate_device_arena=False)
    t = G.BlockTable(p2)
    with pytest.raises(G.ArgumentOutOfRangeError):
        p1.compact([t])
    p1.close()
    p2.close()
