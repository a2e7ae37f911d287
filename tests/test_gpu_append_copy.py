"""KV append (bit-exact) and block copy / copy-on-write on the device, through the C ABI."""
import json
import os
import threading

import numpy as np
import pytest

import glacier_kv as G
from conftest import ROOT
from gpu_helpers import ODT, arena_to_host, geom_of, random_arena
from oracle import pyoracle as O

pytestmark = pytest.mark.gpu


def test_store_and_retrieve_exact_vectors(cuda):
    """PagedAttentionTests.cs:82-109 (block size 4, layer 1, slot 2)."""
    import torch

    s = json.load(open(os.path.join(ROOT, "tests", "golden", "store_retrieve.json")))
    pool = G.PagedBlockPool(s["total_blocks"], s["layers"], s["heads_kv"], s["head_dim"], s["block_size"])
    ok, blk = pool.try_allocate_block()
    assert ok
    k = torch.tensor(s["k"], dtype=torch.float32, device=cuda)
    v = torch.tensor(s["v"], dtype=torch.float32, device=cuda)
    pool.store(blk, s["layer"], s["slot"], k, v)
    pool.sync()
    K, V = pool.key_view(), pool.value_view()
    assert K[blk, 1, 0, 2].tolist() == s["k"][:4] and K[blk, 1, 1, 2].tolist() == s["k"][4:]
    assert V[blk, 1, 0, 2].tolist() == s["v"][:4] and V[blk, 1, 1, 2].tolist() == s["v"][4:]
    assert float(K.sum()) == sum(s["k"]) and float(V.sum()) == sum(s["v"])
    pool.free_block(blk)


def test_arena_is_zeroed_and_aligned(cuda):
    pool = G.PagedBlockPool(8, 2, 2, 32, 16)
    assert pool.key_buffer_address % 256 == 0 and pool.value_buffer_address % 256 == 0  # >= 64 (:69-75)
    assert float(pool.key_view().abs().sum()) == 0 and float(pool.value_view().abs().sum()) == 0
    assert pool.total_memory_bytes == 2 * 8 * 2 * 2 * 16 * 32 * 4


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
def test_batched_append_bit_exact(cuda, dtype):
    """cfg2 shape: 64 tokens (one per sequence) scattered into a 16384-block pool, plus
    padding slots; every appended row matches the oracle's Store bit for bit and nothing
    else in the arena changes."""
    import torch

    from glacier_kv import workloads as W

    w = W.cfg2()
    pool = G.PagedBlockPool(w.total_blocks, 1, w.heads_kv, w.head_dim, 16, dtype=dtype)
    rng = np.random.default_rng(21)
    slots = np.concatenate([w.slot_mapping, [-1, -1]]).astype(np.int64)
    n = slots.size
    k = rng.standard_normal((n, w.heads_kv, w.head_dim)).astype(np.float32)
    v = rng.standard_normal((n, w.heads_kv, w.v_head_dim)).astype(np.float32)
    k[0, 0, :4] = [np.inf, -np.inf, -0.0, 1e-42]  # specials and a subnormal survive the copy
    # fp16 edges: past the largest finite value (-> inf), just under the rounding threshold, an
    # fp16 subnormal, a value that rounds to the smallest normal
    k[1, 0, :5] = [1e5, 65519.0, 3e-6, 6.1033e-05, -65520.0]
    before_k = pool.key_view().clone()
    pool.upload_step(w.tables, w.ctx_lens, slots)
    pool.kv_append(0, torch.from_numpy(k).to(cuda), torch.from_numpy(v).to(cuda))
    pool.sync()
    K, V = pool.key_view(), pool.value_view()
    for i, s in enumerate(slots):
        if s < 0:
            continue
        blk, off = divmod(int(s), 16)
        for h in range(w.heads_kv):
            gk, gv = K[blk, 0, h, off], V[blk, 0, h, off]
            if dtype == "f32":
                assert np.array_equal(gk.cpu().numpy().view(np.uint32), k[i, h].view(np.uint32))
                assert np.array_equal(gv.cpu().numpy().view(np.uint32), v[i, h].view(np.uint32))
            else:
                bits = lambda x: O.to_storage_bits(x, ODT[dtype])  # noqa: E731
                assert np.array_equal(gk.view(torch.int16).cpu().numpy().view(np.uint16), bits(k[i, h]))
                assert np.array_equal(gv.view(torch.int16).cpu().numpy().view(np.uint16), bits(v[i, h]))
    changed = (K != before_k).reshape(w.total_blocks, -1).any(1).nonzero().flatten().cpu().numpy()
    assert set(changed.tolist()) <= {int(s) // 16 for s in slots if s >= 0}
    assert pool.last_launch_count == 1


def test_append_matches_oracle_store_random_slots(cuda):
    import torch

    rng = np.random.default_rng(22)
    pool = G.PagedBlockPool(30, 2, 3, 64, 8, v_head_dim=32)
    K, V = arena_to_host(pool)
    g = geom_of(pool)
    slots = rng.choice(30 * 8, size=50, replace=False).astype(np.int64)
    k = rng.standard_normal((50, 3, 64)).astype(np.float32)
    v = rng.standard_normal((50, 3, 32)).astype(np.float32)
    pool.upload_step(np.zeros((1, 1), np.int32), np.zeros(1, np.int32), slots)
    pool.kv_append(1, torch.from_numpy(k).to(cuda), torch.from_numpy(v).to(cuda))
    pool.sync()
    for i, s in enumerate(slots):
        O.store(K, V, g, int(s) // 8, 1, int(s) % 8, k[i].ravel(), v[i].ravel())
    Kg, Vg = arena_to_host(pool)
    assert np.array_equal(Kg.view(np.uint32), K.view(np.uint32))
    assert np.array_equal(Vg.view(np.uint32), V.view(np.uint32))


@pytest.mark.parametrize("heads,d,dv,dtype", [(3, 128, 128, "f32"), (3, 128, 64, "bf16"), (1, 30, 18, "f32"),
                                              (3, 128, 128, "f16"), (1, 30, 18, "f16")])
def test_large_append_matches_oracle_store_loop(cuda, heads, d, dv, dtype):
    """An odd number of (token, head) rows, more than one pass of the grid-stride loop, with
    padding slots; the scalar path (d not a multiple of 4) included.  Bit-exact against the
    runner's per-token Store loop."""
    import torch

    rng = np.random.default_rng(24)
    bs, nb, n = 16, 1400, 20001
    pool = G.PagedBlockPool(nb, 1, heads, d, bs, v_head_dim=dv, dtype=dtype)
    K, V = random_arena(pool, rng)
    g = geom_of(pool)
    slots = rng.choice(nb * bs, size=n, replace=False).astype(np.int64)
    slots[rng.choice(n, 37, replace=False)] = -1
    k = rng.standard_normal((n, heads, d)).astype(np.float32)
    v = rng.standard_normal((n, heads, dv)).astype(np.float32)
    pool.reserve_step(1, 1, n, heads)
    pool.upload_step(np.zeros((1, 1), np.int32), np.zeros(1, np.int32), slots)
    pool.kv_append(0, torch.from_numpy(k).to(cuda), torch.from_numpy(v).to(cuda))
    pool.sync()
    assert O.store_many(K, V, g, 0, slots, k, v) == 0
    Kg, Vg = arena_to_host(pool)
    assert np.array_equal(Kg, K) and np.array_equal(Vg, V)


@pytest.mark.parametrize("d,dv", [(128, 128), (30, 18)])
@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
def test_large_block_copy_matches_oracle(cuda, dtype, d, dv):
    """More 2 KB chunks than one pass of the grid-stride loop; ragged valid counts; spans that
    end in a tail shorter than 16 bytes (d 30 / dv 18)."""
    rng = np.random.default_rng(25)
    nb, n = 3000, 1400
    pool = G.PagedBlockPool(nb, 1, 4, d, 16, v_head_dim=dv, dtype=dtype)
    K, V = random_arena(pool, rng)
    g = geom_of(pool)
    perm = rng.permutation(nb)
    src, dst = perm[:n], perm[n:2 * n]
    valid = rng.integers(-2, 20, n).astype(np.int32)
    pool.block_copy(src, dst, valid)
    pool.sync()
    assert O.copy_many(K, V, g, src, dst, valid) == 0
    Kg, Vg = arena_to_host(pool)
    assert np.array_equal(Kg, K) and np.array_equal(Vg, V)


def test_cow_fork_preserves_data(cuda):
    """PrefixHashKvCacheTests.cs:134-181 with the arena on the device."""
    pool = G.PagedBlockPool(16, 2, 2, 32, 16)
    a = G.BlockTable(pool)
    for _ in range(10):
        assert a.append_token()[0]
    shared = a.get_block_id(0)
    K = pool.key_view()
    K[shared, 0, 0, 0, 0] = 42.0
    b = G.BlockTable(pool)
    pool.retain_block(shared)
    b.attach_prefix_blocks([shared], 10)
    ok, forked, off = a.append_token()
    assert ok and off == 10 and forked != shared
    assert pool.get_ref_count(shared) == 1 and pool.get_ref_count(forked) == 1
    assert pool.pending_copies == 1
    pool.flush_copies()
    pool.sync()
    assert pool.pending_copies == 0
    assert float(K[forked, 0, 0, 0, 0]) == 42.0
    K[forked, 0, 0, 0, 0] = 999.0
    assert float(K[shared, 0, 0, 0, 0]) == 42.0
    a.release_all()
    b.release_all()
    assert pool.free_blocks_count == 16


def test_cow_16_concurrent_sequences_preserve_data(cuda):
    """PrefixHashKvCacheAdversarialTests.cs:43-107 with the arena on the device."""
    n = 16
    pool = G.PagedBlockPool(64, 1, 1, 16, 16)
    shared = pool.try_allocate_block()[1]
    K = pool.key_view()
    for t in range(8):
        K[shared, 0, 0, t, 0] = 100.0 + t
    for _ in range(1, n):
        pool.retain_block(shared)
    tables = [G.BlockTable(pool) for _ in range(n)]
    for t in tables:
        t.attach_prefix_blocks([shared], 8)
    res = [None] * n
    ths = [threading.Thread(target=lambda i=i: res.__setitem__(i, tables[i].append_token())) for i in range(n)]
    [t.start() for t in ths]
    [t.join() for t in ths]
    pool.flush_copies()
    pool.sync()
    for i, (ok, blk, off) in enumerate(res):
        assert ok and off == 8
        K[blk, 0, 0, 8, 0] = 1000.0 + i
    for i, t in enumerate(tables):
        blk = t.get_block_id(0)
        assert K[blk, 0, 0, :8, 0].tolist() == [100.0 + j for j in range(8)]
        assert float(K[blk, 0, 0, 8, 0]) == 1000.0 + i
    for t in tables:
        t.release_all()
    assert pool.free_blocks_count == 64


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
def test_batched_block_copy_matches_oracle(cuda, dtype):
    rng = np.random.default_rng(23)
    pool = G.PagedBlockPool(40, 3, 2, 64, 16, v_head_dim=32, dtype=dtype)
    K, V = random_arena(pool, rng)
    g = geom_of(pool)
    src = rng.choice(20, 12, replace=False)
    dst = 20 + rng.choice(20, 12, replace=False)
    valid = np.array([1, 2, 7, 8, 9, 15, 16, 20, 0, -3, 5, 11])
    pool.block_copy(src, dst, valid)
    pool.sync()
    assert pool.last_launch_count == 1
    for s, d, n in zip(src, dst, valid):
        O.copy_block_data(K, V, g, int(s), int(d), int(n))
    Kg, Vg = arena_to_host(pool)
    assert np.array_equal(Kg, K) and np.array_equal(Vg, V)
    with pytest.raises(G.ArgumentOutOfRangeError):
        pool.block_copy([0], [40], [4])


def test_queued_forks_run_before_the_next_append(cuda):
    """A fork queued on the host is issued (one launch) ahead of the append that writes the
    forked block, so the append lands on top of the copied prefix."""
    import torch

    pool = G.PagedBlockPool(8, 1, 1, 32, 16)
    a = G.BlockTable(pool)
    for _ in range(5):
        assert a.append_token()[0]
    shared = a.get_block_id(0)
    pool.key_view()[shared, 0, 0, :5] = torch.arange(5, dtype=torch.float32, device=cuda)[:, None]
    pool.retain_block(shared)
    b = G.BlockTable(pool)
    b.attach_prefix_blocks([shared], 5)
    ok, blk, off = a.append_token()
    assert ok and off == 5 and blk != shared
    k = torch.full((1, 1, 32), 55.0, device=cuda)
    pool.upload_step(np.array([[blk]], np.int32), np.array([6], np.int32), np.array([blk * 16 + off], np.int64))
    pool.kv_append(0, k, k.clone())
    pool.sync()
    assert pool.last_launch_count == 2  # the flushed fork + the append
    col = pool.key_view()[blk, 0, 0, :6, 0].tolist()
    assert col == [0.0, 1.0, 2.0, 3.0, 4.0, 55.0]
