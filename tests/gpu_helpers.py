"""Shared helpers of the GPU parity tests (device arena <-> host oracle arrays)."""
import math

import numpy as np

from oracle import pyoracle as O

# max-abs parity bars: fp32 KV; 16-bit KV storage (the tensor-core decode rounds q and p);
# fp8 KV (the CUDA-core decode computes in fp32 on the same stored values)
TOL = {"f32": 1e-4, "bf16": 2e-2, "f16": 2e-2, "fp8": 1e-4}
ODT = {"f32": O.F32, "bf16": O.BF16, "f16": O.F16, "fp8": O.FP8}


def torch():
    import torch as _t

    return _t


def geom_of(pool, total_blocks=None):
    g = O.geom(pool.total_blocks if total_blocks is None else total_blocks, pool.layers, pool.heads_kv,
               pool.head_dim, pool.value_head_dim, pool.block_size, ODT[pool.dtype])
    if pool.dtype == "fp8":
        g.set_scales(*pool.kv_scales)
    return g


def arena_to_host(pool):
    """Host copies of the K and V arenas in the oracle's representation."""
    t = torch()
    k, v = pool.key_view(), pool.value_view()
    if pool.dtype == "fp8":
        return k.cpu().numpy(), v.cpu().numpy()
    if pool.dtype != "f32":
        return (k.view(t.int16).cpu().numpy().view(np.uint16), v.view(t.int16).cpu().numpy().view(np.uint16))
    return k.cpu().numpy(), v.cpu().numpy()


def host_to_arena(pool, K, V):
    t = torch()
    for view, arr in ((pool.key_view(), K), (pool.value_view(), V)):
        if pool.dtype == "fp8":
            view.copy_(t.from_numpy(np.ascontiguousarray(arr, np.uint8)))
        elif pool.dtype != "f32":
            view.view(t.int16).copy_(t.from_numpy(np.ascontiguousarray(arr).view(np.int16)))
        else:
            view.copy_(t.from_numpy(np.ascontiguousarray(arr)))


def random_arena(pool, rng):
    g = geom_of(pool)
    K, V = O.new_arena(g)
    kf = rng.standard_normal(K.shape).astype(np.float32)
    vf = rng.standard_normal(V.shape).astype(np.float32)
    K[...] = O.to_storage_bits(kf, g.dtype)
    V[...] = O.to_storage_bits(vf, g.dtype)
    host_to_arena(pool, K, V)
    return K, V


def random_tables(rng, ctx, bs, total_blocks):
    mb = max(1, max((int(c) + bs - 1) // bs for c in ctx))
    need = sum((int(c) + bs - 1) // bs for c in ctx)
    assert need <= total_blocks
    perm = rng.permutation(total_blocks).astype(np.int32)
    tables = np.full((len(ctx), mb), -1, np.int32)
    at = 0
    for i, c in enumerate(ctx):
        n = (int(c) + bs - 1) // bs
        tables[i, :n] = perm[at: at + n]
        at += n
    return tables


def gpu_decode(pool, layer, tables, ctx, q_np, n_heads, scale, sinks=None, out_init=0.0):
    t = torch()
    dev = f"cuda:{pool.device}"
    q = t.from_numpy(np.ascontiguousarray(q_np, np.float32)).to(dev)
    out = t.full((len(ctx), n_heads, pool.value_head_dim), out_init, dtype=t.float32, device=dev)
    pool.upload_step(tables, np.asarray(ctx, np.int32))
    pool.paged_decode(layer, q, out, n_heads, scale,
                      None if sinks is None else t.from_numpy(np.asarray(sinks, np.float32)).to(dev))
    pool.sync()
    return out.cpu().numpy()


def compact(pool, tables, ctx, rows):
    """Device-side gather of the blocks `rows` use into a small host arena + renumbered tables,
    so the oracle can check sampled sequences of a multi-GB pool."""
    t = torch()
    sub = tables[rows]
    ids = sorted({int(b) for r, c in zip(sub, np.asarray(ctx)[rows]) for b in r[: (int(c) + pool.block_size - 1) // pool.block_size]})
    remap = {b: i for i, b in enumerate(ids)}
    idx = t.tensor(ids, dtype=t.long, device=f"cuda:{pool.device}")
    k = pool.key_view().index_select(0, idx)
    v = pool.value_view().index_select(0, idx)
    if pool.dtype == "fp8":
        K, V = k.cpu().numpy(), v.cpu().numpy()
    elif pool.dtype != "f32":
        K = k.view(t.int16).cpu().numpy().view(np.uint16)
        V = v.view(t.int16).cpu().numpy().view(np.uint16)
    else:
        K, V = k.cpu().numpy(), v.cpu().numpy()
    new = np.full_like(sub, -1)
    for i, (r, c) in enumerate(zip(sub, np.asarray(ctx)[rows])):
        n = (int(c) + pool.block_size - 1) // pool.block_size
        new[i, :n] = [remap[int(b)] for b in r[:n]]
    g = geom_of(pool, len(ids))
    return g, np.ascontiguousarray(K), np.ascontiguousarray(V), new


def scale_of(d):
    return 1.0 / math.sqrt(d)
