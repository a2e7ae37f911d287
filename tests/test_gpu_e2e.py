"""Whole append+decode iterations at the BASELINE sizes: host-buffer path vs device path,
oracle parity on every sequence, and size-independent properties."""
import numpy as np
import pytest

import glacier_kv as G
from glacier_kv import workloads as W
from gpu_helpers import TOL, compact, gpu_decode
from oracle import pyoracle as O

pytestmark = pytest.mark.gpu


def _cfg2_pool():
    w = W.cfg2()
    pool = W.make_pool(w)
    W.fill_arena_randn(pool, seed=w.seed)
    return w, pool


def test_cfg2_full_iteration_parity_and_host_path(cuda):
    import torch

    w, pool = _cfg2_pool()
    rng = np.random.default_rng(w.seed + 1)
    q = rng.standard_normal((w.batch, w.n_heads, w.head_dim)).astype(np.float32)
    kn = rng.standard_normal((w.batch, w.heads_kv, w.head_dim)).astype(np.float32)
    vn = rng.standard_normal((w.batch, w.heads_kv, w.v_head_dim)).astype(np.float32)
    # host-buffer iteration (pinned), the path a P/Invoke caller takes
    hq, hk, hv = (torch.from_numpy(x).pin_memory() for x in (q, kn, vn))
    hout = torch.zeros((w.batch, w.n_heads, w.v_head_dim), dtype=torch.float32).pin_memory()
    pool.decode_step_host(0, w.tables, w.ctx_lens, w.slot_mapping, hk, hv, hq, hout, w.n_heads, w.scale)
    pool.sync()
    assert pool.last_launch_count in (2, 3)
    host_out = hout.numpy().copy()
    # the appended rows are in place, bit for bit
    K = pool.key_view()
    for b in range(w.batch):
        blk, off = divmod(int(w.slot_mapping[b]), 16)
        assert np.array_equal(K[blk, 0, :, off].cpu().numpy().view(np.uint32), kn[b].view(np.uint32))
    # the device path on the same state gives the same bits
    dev_out = gpu_decode(pool, 0, w.tables, w.ctx_lens, q, w.n_heads, w.scale)
    assert np.array_equal(dev_out, host_out)
    # oracle on every sequence (compacted per group of rows to bound host memory)
    for rows in np.array_split(np.arange(w.batch), 4):
        g, Kh, Vh, sub = compact(pool, w.tables, w.ctx_lens, rows)
        ref = O.decode_batch(Kh, Vh, g, 0, sub, w.ctx_lens[rows], q[rows], w.n_heads, w.scale)
        np.testing.assert_allclose(host_out[rows], ref, atol=TOL["f32"], rtol=0)
    pool.close()


def test_cfg2_properties_linearity_and_permutation(cuda):
    """Size-independent checks at full size: scaling every V by c scales the output by c;
    permuting the batch permutes the output; a constant-V arena returns the constant."""
    w, pool = _cfg2_pool()
    rng = np.random.default_rng(w.seed + 2)
    q = rng.standard_normal((w.batch, w.n_heads, w.head_dim)).astype(np.float32)
    base = gpu_decode(pool, 0, w.tables, w.ctx_lens, q, w.n_heads, w.scale)
    perm = rng.permutation(w.batch)
    permuted = gpu_decode(pool, 0, w.tables[perm], w.ctx_lens[perm], q[perm], w.n_heads, w.scale)
    np.testing.assert_allclose(permuted, base[perm], atol=1e-6, rtol=0)
    pool.value_view().mul_(2.0)  # exact in fp32
    doubled = gpu_decode(pool, 0, w.tables, w.ctx_lens, q, w.n_heads, w.scale)
    np.testing.assert_allclose(doubled, 2 * base, atol=1e-6, rtol=0)
    pool.value_view().fill_(0.25)
    const = gpu_decode(pool, 0, w.tables, w.ctx_lens, q, w.n_heads, w.scale)
    np.testing.assert_allclose(const, 0.25, atol=1e-6, rtol=0)
    pool.close()


def test_cfg1_parity(cuda):
    w = W.cfg1()
    pool = W.make_pool(w)
    W.fill_arena_randn(pool, seed=w.seed)
    rng = np.random.default_rng(w.seed + 3)
    q = rng.standard_normal((w.batch, w.n_heads, w.head_dim)).astype(np.float32)
    out = gpu_decode(pool, 0, w.tables, w.ctx_lens, q, w.n_heads, w.scale)
    g, K, V, sub = compact(pool, w.tables, w.ctx_lens, np.arange(w.batch))
    ref = O.decode_batch(K, V, g, 0, sub, w.ctx_lens, q, w.n_heads, w.scale)
    np.testing.assert_allclose(out, ref, atol=TOL["f32"], rtol=0)
    pool.close()


def test_cfg5_local_shard_parity(cuda):
    """One GPU's block range of the long-context config (bf16, group 8)."""
    w = W.cfg5_local(0, 8)
    pool = W.make_pool(w)
    W.fill_arena_randn(pool, seed=w.seed)
    rng = np.random.default_rng(w.seed + 4)
    q = rng.standard_normal((w.batch, w.n_heads, w.head_dim)).astype(np.float32)
    out = gpu_decode(pool, 0, w.tables, w.ctx_lens, q, w.n_heads, w.scale)
    g, K, V, sub = compact(pool, w.tables, w.ctx_lens, np.arange(2))
    ref = O.decode_batch(K, V, g, 0, sub, w.ctx_lens[:2], q[:2], w.n_heads, w.scale)
    np.testing.assert_allclose(out[:2], ref, atol=TOL["bf16"], rtol=0)
    pool.close()


def test_consecutive_host_steps_overlap_and_stay_exact(cuda):
    """Back-to-back host-buffer calls (copies of one call overlap the neighbours' compute):
    every call's output equals the device path for its own q, bit for bit."""
    import torch

    w, pool = _cfg2_pool()
    rng = np.random.default_rng(w.seed + 3)
    kn = torch.from_numpy(rng.standard_normal((w.batch, w.heads_kv, w.head_dim)).astype(np.float32)).pin_memory()
    vn = torch.from_numpy(rng.standard_normal((w.batch, w.heads_kv, w.v_head_dim)).astype(np.float32)).pin_memory()
    qs = [rng.standard_normal((w.batch, w.n_heads, w.head_dim)).astype(np.float32) for _ in range(5)]
    hqs = [torch.from_numpy(q).pin_memory() for q in qs]
    houts = [torch.full((w.batch, w.n_heads, w.v_head_dim), np.nan, dtype=torch.float32).pin_memory() for _ in qs]
    for hq, hout in zip(hqs, houts):  # no sync between the calls
        pool.decode_step_host(0, w.tables, w.ctx_lens, w.slot_mapping, kn, vn, hq, hout, w.n_heads, w.scale)
    pool.sync()
    for q, hout in zip(qs, houts):
        dev = gpu_decode(pool, 0, w.tables, w.ctx_lens, q, w.n_heads, w.scale)
        assert np.array_equal(hout.numpy(), dev)
    pool.close()
