"""Host allocator semantics of the shim, ported from the reference's own tests.

Metadata-only pools (the reference's allocateHostBuffers:false) so these run without a GPU;
the same C++ allocator backs device pools.  Sources:
  tests/Glacier.Serve.Tests/PagedAttentionTests.cs, PrefixHashKvCacheTests.cs,
  PrefixHashKvCacheAdversarialTests.cs, PhaseCServeRemediationTests.cs.
The prefix hash itself (XXH3, System.IO.Hashing) stays in the C# host; tests here feed the
pool fixed or stand-in 64-bit hashes.
"""
import hashlib
import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

from glacier_kv import ArgumentOutOfRangeError, BlockTable, InvalidOperationError, PagedBlockPool


def pool(total, layers=1, heads_kv=1, head_dim=16, block_size=16):
    return PagedBlockPool(total, layers, heads_kv, head_dim, block_size, allocate_device_arena=False)


def h64(parent, tokens):
    """Stand-in chained 64-bit prefix hash (the real one is computed by the C# host)."""
    d = hashlib.blake2b(int(parent).to_bytes(8, "little") + np.asarray(tokens, np.int32).tobytes(),
                        digest_size=8).digest()
    return int.from_bytes(d, "little") or 1


# ---- PagedAttentionTests.cs -------------------------------------------------------------

def test_allocates_and_recycles_blocks_in_constant_time():  # :11-34
    p = pool(64, layers=4, heads_kv=2, head_dim=64)
    assert (p.total_blocks, p.free_blocks_count, p.allocated_blocks_count) == (64, 64, 0)
    assert p.capacity_tokens == 1024
    got = [p.try_allocate_block() for _ in range(10)]
    assert all(ok for ok, _ in got)
    assert (p.free_blocks_count, p.allocated_blocks_count, p.active_tokens) == (54, 10, 160)
    p.free_blocks([b for _, b in got])
    assert (p.free_blocks_count, p.allocated_blocks_count) == (64, 0)


def test_block_table_expands_across_token_boundaries():  # :37-79
    p = pool(16, layers=2, heads_kv=2, head_dim=32)
    t = BlockTable(p)
    assert (t.token_count, t.block_count) == (0, 0)
    for i in range(35):
        ok, blk, off = t.append_token()
        assert ok and blk >= 0 and off == i % 16
    assert (t.token_count, t.block_count, p.free_blocks_count) == (35, 3, 13)
    assert t.get_token_location(0) == (t.get_block_id(0), 0)
    assert t.get_token_location(15) == (t.get_block_id(0), 15)
    assert t.get_token_location(16) == (t.get_block_id(1), 0)
    assert t.get_token_location(34) == (t.get_block_id(2), 2)
    t.release_all()
    assert (t.token_count, t.block_count, p.free_blocks_count) == (0, 0, 16)


def test_free_list_pops_zero_first_and_is_lifo():
    p = pool(8)
    ids = [p.try_allocate_block()[1] for _ in range(8)]
    assert ids == list(range(8))  # PagedBlockPool.cs:117-120
    assert p.try_allocate_block() == (False, -1)
    p.release_block(5)
    p.release_block(2)
    assert p.try_allocate_block() == (True, 2)
    assert p.try_allocate_block() == (True, 5)


# ---- PrefixHashKvCacheTests.cs ------------------------------------------------------------

def test_refcount_initializes_to_one():  # :53-63
    p = pool(8, layers=2, heads_kv=2, head_dim=32)
    ok, b = p.try_allocate_block()
    assert ok and p.get_ref_count(b) == 1
    p.release_block(b)
    assert p.get_ref_count(b) == 0 and p.free_blocks_count == 8


def test_retain_and_release_count_accurately():  # :65-84
    p = pool(8, layers=2, heads_kv=2, head_dim=32)
    _, b = p.try_allocate_block()
    assert p.retain_block(b) == 2 and p.retain_block(b) == 3 and p.get_ref_count(b) == 3
    assert p.release_block(b) == 2 and p.release_block(b) == 1
    assert p.free_blocks_count == 7
    assert p.release_block(b) == 0 and p.free_blocks_count == 8


def test_concurrent_retain_release_no_leak_or_double_free():  # :86-104
    p = pool(32, layers=2, heads_kv=2, head_dim=32)

    def work(_):
        ok, b = p.try_allocate_block()
        if ok:
            p.retain_block(b)
            p.release_block(b)
            p.release_block(b)

    with ThreadPoolExecutor(16) as ex:
        list(ex.map(work, range(10_000)))
    assert p.free_blocks_count == 32 and p.allocated_blocks_count == 0


def test_prefix_bind_find_and_recycle():  # :106-132
    p = pool(16, layers=2, heads_kv=2, head_dim=32)
    h = h64(0, range(1, 17))
    _, b = p.try_allocate_block()
    p.bind_prefix_block(h, b)
    ok, found = p.try_find_prefix_block(h)
    assert ok and found == b and p.get_ref_count(b) == 2
    p.release_block(b)
    assert p.get_ref_count(b) == 1
    p.release_block(found)
    assert p.get_ref_count(b) == 0
    assert p.try_find_prefix_block(h) == (False, -1)
    assert p.free_blocks_count == 16


def test_cow_append_on_shared_block_forks_and_queues_copy():  # :134-181 (bookkeeping half)
    p = pool(16, layers=2, heads_kv=2, head_dim=32)
    a = BlockTable(p)
    for _ in range(10):
        assert a.append_token()[0]
    shared = a.get_block_id(0)
    assert p.get_ref_count(shared) == 1
    b = BlockTable(p)
    p.retain_block(shared)
    b.attach_prefix_blocks([shared], token_count=10)
    assert p.get_ref_count(shared) == 2
    ok, blk, off = a.append_token()
    assert ok and off == 10 and blk != shared
    assert p.get_ref_count(shared) == 1 and p.get_ref_count(blk) == 1
    # a metadata-only pool queues no device copy (TryForkBlock copies only with buffers)
    assert p.pending_copies == 0
    a.release_all()
    b.release_all()
    assert p.free_blocks_count == 16


def test_attach_prefix_blocks():  # :183-200
    p = pool(16, layers=2, heads_kv=2, head_dim=32)
    b0 = p.try_allocate_block()[1]
    b1 = p.try_allocate_block()[1]
    t = BlockTable(p)
    t.attach_prefix_blocks([b0, b1], token_count=32)
    assert (t.token_count, t.block_count, t.get_block_id(0), t.get_block_id(1)) == (32, 2, b0, b1)
    assert list(t.as_span()) == [b0, b1]
    t.release_all()
    assert p.free_blocks_count == 16
    with pytest.raises(ArgumentOutOfRangeError):
        t.attach_prefix_blocks([], token_count=-1)


# ---- PrefixHashKvCacheAdversarialTests.cs ----------------------------------------------

def test_bind_overwrite_release_first_keeps_second():  # :13-41
    p = pool(16, layers=2, heads_kv=2, head_dim=32)
    h = 0xABCD1234EF567890
    a = p.try_allocate_block()[1]
    b = p.try_allocate_block()[1]
    p.bind_prefix_block(h, a)
    p.bind_prefix_block(h, b)
    p.release_block(a)
    ok, found = p.try_find_prefix_block(h)
    assert ok and found == b
    p.release_block(b)
    p.release_block(b)


def test_cow_16_concurrent_sequences_get_private_blocks():  # :43-107 (bookkeeping half)
    n = 16
    p = pool(64)
    shared = p.try_allocate_block()[1]
    for _ in range(1, n):
        p.retain_block(shared)
    assert p.get_ref_count(shared) == n
    tables = [BlockTable(p) for _ in range(n)]
    for t in tables:
        t.attach_prefix_blocks([shared], token_count=8)
    results = [None] * n

    def work(i):
        results[i] = tables[i].append_token()

    with ThreadPoolExecutor(n) as ex:
        list(ex.map(work, range(n)))
    assert all(ok and off == 8 for ok, _, off in results)
    blocks = {blk for _, blk, _ in results}
    # every sequence but the last one standing forked; the original keeps one owner
    assert len(blocks) == n
    assert sum(p.get_ref_count(b) for b in blocks) == n
    for t in tables:
        t.release_all()
    assert p.free_blocks_count == 64


def test_cow_out_of_memory_leaves_state_consistent():  # :109-141
    p = pool(1)
    b0 = p.try_allocate_block()[1]
    p.retain_block(b0)
    a, b = BlockTable(p), BlockTable(p)
    a.attach_prefix_blocks([b0], token_count=4)
    b.attach_prefix_blocks([b0], token_count=4)
    assert a.append_token() == (False, -1, -1)
    assert (a.token_count, a.block_count, a.get_block_id(0), p.get_ref_count(b0)) == (4, 1, b0, 2)
    a.release_all()
    assert p.get_ref_count(b0) == 1
    b.release_all()
    assert p.get_ref_count(b0) == 0 and p.free_blocks_count == 1


def test_concurrent_find_and_release_stress_no_negative_refcount():  # :179-207
    p = pool(32)
    base = 0x1234567890ABCDEF

    def work(i):
        ok, b = p.try_allocate_block()
        if ok:
            p.bind_prefix_block(base + (i % 8), b)
            okf, f = p.try_find_prefix_block(base + (i % 8))
            if okf:
                p.release_block(f)
            p.release_block(b)

    with ThreadPoolExecutor(16) as ex:
        list(ex.map(work, range(5000)))
    assert all(p.get_ref_count(b) >= 0 for b in range(32))


def test_aba_race_never_returns_dead_block():  # :209-265
    p = pool(4)
    ha, hb = 0xAAAAAAAAAAAAAAAA, 0xBBBBBBBBBBBBBBBB
    violations = []

    def work(i):
        if i % 2 == 0:
            ok, b = p.try_allocate_block()
            if ok:
                p.bind_prefix_block(ha, b)
                p.release_block(b)
                ok2, b2 = p.try_allocate_block()
                if ok2:
                    p.bind_prefix_block(hb, b2)
                    p.release_block(b2)
        else:
            ok, f = p.try_find_prefix_block(ha)
            if ok:
                if p.get_ref_count(f) <= 0:
                    violations.append(f)
                p.release_block(f)

    with ThreadPoolExecutor(16) as ex:
        list(ex.map(work, range(10_000)))
    assert not violations
    assert all(p.get_ref_count(b) >= 0 for b in range(4))


def test_multi_block_overwrite_eviction_isolation():  # :267-309
    p = pool(8)
    h = 0xFEEDFACECAFEBABE
    ids = [p.try_allocate_block()[1] for _ in range(8)]
    for b in ids:
        p.bind_prefix_block(h, b)
    ok, f = p.try_find_prefix_block(h)
    assert ok and f == ids[-1]
    p.release_block(f)
    for b in ids[:-1]:
        p.release_block(b)
    ok, f = p.try_find_prefix_block(h)
    assert ok and f == ids[-1]
    p.release_block(f)
    p.release_block(ids[-1])
    assert p.try_find_prefix_block(h) == (False, -1)
    assert p.free_blocks_count == 8


def test_zero_hash_rejected_and_not_found():  # :311-323
    p = pool(4)
    b = p.try_allocate_block()[1]
    with pytest.raises(ArgumentOutOfRangeError):
        p.bind_prefix_block(0, b)
    assert p.try_find_prefix_block(0) == (False, -1)
    p.release_block(b)
    assert p.free_blocks_count == 4


def test_double_free_is_idempotent():  # :325-350
    p = pool(4)
    b = p.try_allocate_block()[1]
    assert p.free_blocks_count == 3
    assert p.release_block(b) == 0 and p.free_blocks_count == 4
    assert p.release_block(b) == 0 and p.free_blocks_count == 4
    p.free_block(b)
    assert p.free_blocks_count == 4
    for _ in range(4):
        assert p.try_allocate_block()[0]
    assert p.free_blocks_count == 0


def test_out_of_range_ids_handled_safely():  # :352-366
    p = pool(4)
    assert p.release_block(-1) == 0 and p.release_block(100) == 0
    assert p.get_ref_count(-1) == 0 and p.get_ref_count(100) == 0
    for bad in (-1, 100):
        with pytest.raises(ArgumentOutOfRangeError):
            p.retain_block(bad)
        with pytest.raises(ArgumentOutOfRangeError):
            p.bind_prefix_block(0x1234, bad)


def test_multi_turn_prefix_branching_isolation():  # :368-437
    p = pool(16)
    h0 = h64(0, range(1, 17))
    h1 = h64(h0, range(17, 33))
    s0, s1 = p.try_allocate_block()[1], p.try_allocate_block()[1]
    p.bind_prefix_block(h0, s0)
    p.bind_prefix_block(h1, s1)
    a = BlockTable(p)
    p.retain_block(s0)
    p.retain_block(s1)
    a.attach_prefix_blocks([s0, s1], token_count=32)
    for _ in range(5):
        assert a.append_token()[0]
    assert (a.token_count, a.block_count) == (37, 3)
    b = BlockTable(p)
    p.retain_block(s0)
    p.retain_block(s1)
    b.attach_prefix_blocks([s0, s1], token_count=32)
    for _ in range(10):
        assert b.append_token()[0]
    assert (b.token_count, b.block_count) == (42, 3)
    assert p.get_ref_count(s0) == 3 and p.get_ref_count(s1) == 3
    a.release_all()
    assert p.get_ref_count(s0) == 2 and b.token_count == 42
    b.release_all()
    assert p.get_ref_count(s0) == 1 and p.get_ref_count(s1) == 1
    p.release_block(s0)
    p.release_block(s1)
    assert p.try_find_prefix_block(h0) == (False, -1)
    assert p.try_find_prefix_block(h1) == (False, -1)
    assert p.free_blocks_count == 16


def test_32_thread_prefix_churn_stress():  # :439-467
    p = pool(64)

    def work(i):
        h = 0xAA000000 + (i % 16)
        ok, b = p.try_allocate_block()
        if ok:
            p.bind_prefix_block(h, b)
            okf, f = p.try_find_prefix_block(h)
            if okf:
                assert 0 <= f < 64
                p.release_block(f)
            p.release_block(b)

    with ThreadPoolExecutor(32) as ex:
        list(ex.map(work, range(10_000)))
    assert all(p.get_ref_count(b) >= 0 for b in range(64))


# ---- PhaseCServeRemediationTests.cs ------------------------------------------------------

def test_double_free_and_unallocated_free_never_corrupt_stack():  # :69-112
    p = pool(8, layers=2, heads_kv=2, head_dim=32)
    b0 = p.try_allocate_block()[1]
    b1 = p.try_allocate_block()[1]
    assert b0 != b1 and p.free_blocks_count == 6
    p.free_block(b0)
    assert p.free_blocks_count == 7
    p.free_block(b0)
    assert p.free_blocks_count == 7
    for c in range(8):
        if c != b1:
            p.free_block(c)
    assert p.free_blocks_count == 7
    seen = {b1}
    for _ in range(7):
        ok, n = p.try_allocate_block()
        assert ok and n not in seen
        seen.add(n)
    assert p.free_blocks_count == 0
    assert p.try_allocate_block() == (False, -1)


def test_metadata_only_pool():  # :1081-1097
    p = PagedBlockPool(32, 4, 2, 64, allocate_device_arena=False)
    assert not p.has_device_arena and p.total_memory_bytes == 0
    assert p.key_buffer_address == 0 and p.value_buffer_address == 0
    ok, b = p.try_allocate_block()
    assert ok and b >= 0 and p.free_blocks_count == 31
    p.free_block(b)
    assert p.free_blocks_count == 32
    # device operations are refused like GetKeyPtr's InvalidOperationException (:126-127)
    with pytest.raises(InvalidOperationError):
        p.copy_block_data(0, 1, 4)
    with pytest.raises(InvalidOperationError):
        p.store(0, 0, 0, None, None)


@pytest.mark.parametrize("kw", [dict(total=0), dict(layers=0), dict(heads_kv=0), dict(head_dim=0),
                                dict(block_size=-1)])
def test_constructor_rejects_sizes_below_one(kw):  # PagedBlockPool.cs:63-67
    args = dict(total=4, layers=1, heads_kv=1, head_dim=16, block_size=16)
    args.update(kw)
    with pytest.raises(ArgumentOutOfRangeError):
        PagedBlockPool(args["total"], args["layers"], args["heads_kv"], args["head_dim"], args["block_size"],
                       allocate_device_arena=False)


def test_element_offsets_follow_reference_strides():  # PagedBlockPool.cs:77-83,124-145
    p = PagedBlockPool(4, 2, 2, 4, block_size=4, v_head_dim=8, allocate_device_arena=False)
    # K: head stride 4*4=16, layer stride 2*16=32, block stride 2*32=64
    assert p.element_offset(0, 3, 1, 1, 2) == 3 * 64 + 32 + 16 + 2 * 4
    # V: head stride 4*8=32, layer stride 64, block stride 128
    assert p.element_offset(1, 3, 1, 1, 2) == 3 * 128 + 64 + 32 + 2 * 8
    with pytest.raises(ArgumentOutOfRangeError):
        p.element_offset(0, 4, 0, 0, 0)


def test_table_edges():
    p = pool(2, block_size=4)
    t = BlockTable(p)
    with pytest.raises(ArgumentOutOfRangeError):
        t.get_token_location(0)
    with pytest.raises(ArgumentOutOfRangeError):
        t.get_block_id(0)
    for _ in range(8):
        assert t.append_token()[0]
    assert t.append_token() == (False, -1, -1)  # pool exhausted at a block boundary
    assert t.token_count == 8


# ---- FP8 E4M3 storage (no reference counterpart) ---------------------------------------

def test_fp8_pool_checks_head_dims_and_scales():
    """An FP8 pool needs head dims that are multiples of 16 and positive, finite scales, one
    K and one V scale per (layer, kv head); scales belong to FP8 pools only."""
    with pytest.raises(ArgumentOutOfRangeError):
        PagedBlockPool(8, 1, 2, 24, 16, allocate_device_arena=False, dtype="fp8")
    p = PagedBlockPool(8, 2, 2, 64, 16, allocate_device_arena=False, dtype="fp8")
    p.set_kv_scales(np.full((2, 2), 0.5), np.full((2, 2), 2.0))
    for bad in (0.0, -1.0, np.inf, np.nan):
        ks = np.ones((2, 2), np.float32)
        ks[1, 0] = bad
        with pytest.raises(ArgumentOutOfRangeError):
            p.set_kv_scales(ks, np.ones((2, 2)))
    with pytest.raises(ArgumentOutOfRangeError):
        p.set_kv_scales(np.ones(3), np.ones(4))
    f = PagedBlockPool(8, 2, 2, 64, 16, allocate_device_arena=False, dtype="bf16")
    with pytest.raises(InvalidOperationError):
        f.set_kv_scales(np.ones((2, 2)), np.ones((2, 2)))


def test_static_step_layout_needs_a_device_arena():
    """gkv_step_set_static fixes device metadata for CUDA-graph capture: a metadata-only pool
    (no device arena) refuses it, as it refuses every device call."""
    p = PagedBlockPool(8, 1, 2, 64, 16, allocate_device_arena=False)
    with pytest.raises(InvalidOperationError):
        p.set_static_step(True)
    with pytest.raises(InvalidOperationError):
        p.set_static_step(False)
