"""Seeded synthetic workloads of the BASELINE configs (shapes, pools, value distributions).

The reference publishes no dataset for this path; every input here is generated from a seed:
context lengths, block tables (drawn from a LIFO free list with the allocator's semantics, so
their fragmentation is what the pool's free list produces), and N(0,1) values for Q, K and V.

Table generation is numpy only: importing this module maps no native code (the benchmark's CPU
reference arm uses it).  ``churn_tables`` replays the same churn on a real pool's allocator, and
a CPU test checks that both give identical tables.

    cfg1  decode, 20 seqs, ctx ~ U{128..1024}, 28q/4kv, d 128, fp32, pool 1024 (permuted)
    cfg2  append + decode, 64 seqs x (2048 cached + 1 new), 32q/8kv, d 128, fp32, pool 16384
    cfg3  decode, 256 seqs, ctx ~ lognormal(ln 1500, 1) in [16, 32768], 28q/4kv, d 128,
          fp32 or bf16, pool 65536 after a 10k-op admit/evict churn
    cfg4  chunked causal prefill, 8 seqs x (prefix ~ U{0..4096} + 2048-token chunk),
          28q/4kv, d 128, bf16
    cfg5  long-context decode, 4 seqs x 131072, 64q/8kv, d 128, bf16, split by block range
"""
from __future__ import annotations

import dataclasses
import math
from typing import List, Optional

import numpy as np

SEED = 0x61AC1E5


@dataclasses.dataclass
class DecodeWorkload:
    name: str
    n_heads: int
    heads_kv: int
    head_dim: int
    v_head_dim: int
    block_size: int
    total_blocks: int
    dtype: str
    ctx_lens: np.ndarray          # [B] tokens attended (after the append, if any)
    tables: np.ndarray            # [B, max_blocks] int32, -1 padded
    slot_mapping: np.ndarray      # [n_tok] int64 slots of appended tokens (may be empty)
    append_rows: np.ndarray       # [n_tok] batch row of each appended token
    scale: float
    seed: int

    @property
    def batch(self) -> int:
        return int(self.ctx_lens.shape[0])

    @property
    def elem_bytes(self) -> int:
        return {"f32": 4, "bf16": 2, "f16": 2, "fp8": 1}[self.dtype]

    def kv_bytes(self) -> int:
        """Algorithmic KV bytes one decode step reads (each K/V row once)."""
        return int(self.ctx_lens.astype(np.int64).sum()) * self.heads_kv * (self.head_dim + self.v_head_dim) * self.elem_bytes

    def qo_bytes(self) -> int:
        return self.batch * self.n_heads * (self.head_dim + self.v_head_dim) * 4

    def append_bytes(self) -> int:
        """Bytes the append writes (fp32 source rows are read once more)."""
        n = int(self.slot_mapping.shape[0])
        return n * self.heads_kv * (self.head_dim + self.v_head_dim) * self.elem_bytes

    def flops(self) -> int:
        return 2 * int(self.ctx_lens.astype(np.int64).sum()) * self.n_heads * (self.head_dim + self.v_head_dim)


def _pack(tables: List[List[int]]) -> np.ndarray:
    mb = max(1, max(len(t) for t in tables))
    out = np.full((len(tables), mb), -1, np.int32)
    for i, t in enumerate(tables):
        out[i, : len(t)] = t
    return out


def cfg1(seed: int = SEED) -> DecodeWorkload:
    rng = np.random.default_rng(seed)
    B, bs, pool_blocks = 20, 16, 1024
    ctx = rng.integers(128, 1024, size=B, endpoint=True).astype(np.int32)
    perm = rng.permutation(pool_blocks).astype(np.int32)
    tables, at = [], 0
    for c in ctx:
        n = (int(c) + bs - 1) // bs
        tables.append(perm[at: at + n].tolist())
        at += n
    return DecodeWorkload("cfg1", 28, 4, 128, 128, bs, pool_blocks, "f32", ctx, _pack(tables),
                          np.zeros(0, np.int64), np.zeros(0, np.int32), 1.0 / math.sqrt(128), seed)


def cfg2(seed: int = SEED, batch: int = 64, cached: int = 2048) -> DecodeWorkload:
    """64 sequences x 2048 cached tokens; one new token each lands at offset 0 of a fresh
    block (2048 / 16 = block index 128), then every sequence attends 2049 tokens."""
    rng = np.random.default_rng(seed)
    bs, pool_blocks = 16, 16384
    perm = rng.permutation(pool_blocks).astype(np.int32)
    n_blocks = cached // bs + 1
    assert batch * n_blocks <= pool_blocks
    tables = perm[: batch * n_blocks].reshape(batch, n_blocks)
    ctx = np.full(batch, cached + 1, np.int32)
    slots = (tables[:, cached // bs].astype(np.int64) * bs + (cached % bs)).astype(np.int64)
    return DecodeWorkload("cfg2", 32, 8, 128, 128, bs, pool_blocks, "f32", ctx, np.ascontiguousarray(tables),
                          slots, np.arange(batch, dtype=np.int32), 1.0 / math.sqrt(128), seed)


class LifoFreeList:
    """The pool's free-list semantics in plain Python: block 0 is popped first
    (PagedBlockPool.cs:116-120), pops take the most recently released block (ConcurrentStack,
    PagedBlockPool.cs:39,178-189), and a block released with one reference returns to the top
    (ReleaseBlock, :251-279).  Enough to replay an admit/evict trace without a pool."""

    def __init__(self, total_blocks: int, block_size: int = 16):
        self.total_blocks = total_blocks
        self.block_size = block_size
        self._stack = list(range(total_blocks - 1, -1, -1))

    def try_allocate_block(self):
        if not self._stack:
            return False, -1
        return True, self._stack.pop()

    def release_block(self, block: int) -> int:
        self._stack.append(block)
        return 0


def churn_tables(pool, ctx_lens: np.ndarray, rng: np.random.Generator, ops: int = 10_000,
                 max_live_frac: float = 0.4) -> np.ndarray:
    """Admit/evict churn on `pool`'s free list (a PagedBlockPool or a LifoFreeList), then
    allocate one table per ctx."""
    bs = pool.block_size
    total = pool.total_blocks
    live: List[List[int]] = []
    live_blocks = 0
    for _ in range(ops):
        admit = rng.random() < 0.55 or not live
        if admit:
            need = int(rng.integers(1, 256))
            if live_blocks + need > max_live_frac * total:
                admit = False
        if admit:
            ids = []
            for _b in range(need):
                ok, b = pool.try_allocate_block()
                assert ok
                ids.append(b)
            live.append(ids)
            live_blocks += need
        else:
            ids = live.pop(int(rng.integers(0, len(live))))
            live_blocks -= len(ids)
            for b in ids:
                pool.release_block(b)
    for ids in live:
        for b in ids:
            pool.release_block(b)
    tables = []
    for c in ctx_lens:
        n = (int(c) + bs - 1) // bs
        ids = []
        for _ in range(n):
            ok, b = pool.try_allocate_block()
            assert ok, "pool too small for the workload"
            ids.append(b)
        tables.append(ids)
    return _pack(tables)


def cfg3_ctx(rng: np.random.Generator, batch: int = 256) -> np.ndarray:
    return np.clip(np.round(rng.lognormal(math.log(1500.0), 1.0, size=batch)), 16, 32768).astype(np.int32)


def cfg3(seed: int = SEED, dtype: str = "f32", batch: int = 256, total_blocks: int = 65536,
         ops: int = 10_000) -> DecodeWorkload:
    rng = np.random.default_rng(seed)
    ctx = cfg3_ctx(rng, batch)
    bs = 16
    tables = churn_tables(LifoFreeList(total_blocks, bs), ctx, rng, ops=ops)
    return DecodeWorkload("cfg3", 28, 4, 128, 128, bs, total_blocks, dtype, ctx, tables,
                          np.zeros(0, np.int64), np.zeros(0, np.int32), 1.0 / math.sqrt(128), seed)


def lpt_share(w: DecodeWorkload, rank: int, world: int) -> DecodeWorkload:
    """This rank's sequences of `w` under longest-first partitioning (gkv_partition_lpt): the
    same global batch split over `world` GPUs, each with the whole pool geometry."""
    from . import partition_lpt

    rows = np.nonzero(partition_lpt(w.ctx_lens, world) == rank)[0]
    ctx = w.ctx_lens[rows]
    nb = max(1, max((int(c) + w.block_size - 1) // w.block_size for c in ctx)) if rows.size else 1
    tables = np.ascontiguousarray(w.tables[rows, :nb])
    return dataclasses.replace(w, ctx_lens=ctx, tables=tables)


def cfg5_local(rank: int, world: int, seed: int = SEED, batch: int = 4, ctx: int = 131072) -> DecodeWorkload:
    """Rank `rank`'s contiguous block range of each long sequence (split-KV across GPUs)."""
    bs = 16
    n_blocks = ctx // bs
    if world == 1:  # the whole sequences (no native call: the CPU reference arm uses this case)
        b0, b1 = 0, n_blocks
    else:
        from . import split_block_range

        b0, b1 = split_block_range(n_blocks, world, rank)
    per = b1 - b0
    rng = np.random.default_rng(seed + 7919 * rank)
    total_blocks = batch * per
    perm = rng.permutation(total_blocks).astype(np.int32)
    tables = perm.reshape(batch, per)
    ctx_local = np.full(batch, per * bs, np.int32)
    return DecodeWorkload("cfg5", 64, 8, 128, 128, bs, total_blocks, "bf16", ctx_local, np.ascontiguousarray(tables),
                          np.zeros(0, np.int64), np.zeros(0, np.int32), 1.0 / math.sqrt(128), seed)


@dataclasses.dataclass
class PrefillWorkload:
    """Chunked causal prefill: every sequence has `prefix[b]` cached tokens, `chunk` new tokens
    are appended after them and attend causally over prefix + chunk."""
    name: str
    n_heads: int
    heads_kv: int
    head_dim: int
    v_head_dim: int
    block_size: int
    total_blocks: int
    dtype: str
    prefix: np.ndarray            # [B] cached tokens before the chunk
    chunk: int                    # queries (= appended tokens) per sequence
    tables: np.ndarray            # [B, max_blocks] int32, -1 padded
    slot_mapping: np.ndarray      # [B * chunk] int64 slots of the chunk tokens, sequence-major
    scale: float
    seed: int

    @property
    def batch(self) -> int:
        return int(self.prefix.shape[0])

    @property
    def token_counts(self) -> np.ndarray:
        return (self.prefix + self.chunk).astype(np.int32)

    @property
    def q_lens(self) -> np.ndarray:
        return np.full(self.batch, self.chunk, np.int32)

    @property
    def n_queries(self) -> int:
        return self.batch * self.chunk

    def flops(self) -> int:
        """Causal-only count: 2 * (d + dv) * n_heads per visible (query, key) pair."""
        pairs = sum(self.chunk * (int(p) + 1) + self.chunk * (self.chunk - 1) // 2 for p in self.prefix)
        return 2 * (self.head_dim + self.v_head_dim) * self.n_heads * pairs

    def append_bytes(self) -> int:
        eb = 2 if self.dtype == "bf16" else 4
        return self.n_queries * self.heads_kv * (self.head_dim + self.v_head_dim) * eb


def cfg4(seed: int = SEED, batch: int = 8, chunk: int = 2048, max_prefix: int = 4096) -> PrefillWorkload:
    """8 sequences, prefix ~ U{0..4096}, a 2048-token chunk each; 28q/4kv, d 128, bf16."""
    rng = np.random.default_rng(seed)
    bs = 16
    prefix = rng.integers(0, max_prefix, size=batch, endpoint=True).astype(np.int32)
    n_blocks = [(int(p) + chunk + bs - 1) // bs for p in prefix]
    total_blocks = sum(n_blocks) + 64
    perm = rng.permutation(total_blocks).astype(np.int32)
    tables, at = [], 0
    for n in n_blocks:
        tables.append(perm[at: at + n].tolist())
        at += n
    packed = _pack(tables)
    slots = []
    for b, p in enumerate(prefix):
        pos = np.arange(int(p), int(p) + chunk)
        slots.append(packed[b, pos // bs].astype(np.int64) * bs + pos % bs)
    return PrefillWorkload("cfg4", 28, 4, 128, 128, bs, total_blocks, "bf16", prefix, chunk, packed,
                           np.concatenate(slots).astype(np.int64), 1.0 / math.sqrt(128), seed)


def make_pool(w: DecodeWorkload, device: int = 0, layers: int = 1):
    from . import PagedBlockPool

    return PagedBlockPool(w.total_blocks, layers, w.heads_kv, w.head_dim, w.block_size, w.v_head_dim,
                          allocate_device_arena=True, device=device, dtype=w.dtype)


def fill_arena_randn(pool, seed: int, blocks: Optional[np.ndarray] = None) -> None:
    """N(0,1) K and V (rounded to the storage type) written straight into the device arena."""
    import torch

    g = torch.Generator(device=f"cuda:{pool.device}")
    g.manual_seed(seed)
    for view in (pool.key_view(), pool.value_view()):
        flat = view.reshape(view.shape[0], -1)
        step = max(1, (1 << 26) // flat.shape[1])
        for i in range(0, flat.shape[0], step):
            chunk = torch.randn(flat[i: i + step].shape, generator=g, device=view.device, dtype=torch.float32)
            if view.dtype == torch.uint8:  # FP8 arena: e4m3 bytes (|x| << 448, scale 1)
                flat[i: i + step].copy_(chunk.to(torch.float8_e4m3fn).view(torch.uint8))
            else:
                flat[i: i + step].copy_(chunk.to(view.dtype))


def randn(shape, seed: int, device: str = "cpu"):
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randn(shape, generator=g, device=device, dtype=torch.float32)
