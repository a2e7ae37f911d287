"""Host-side planning logic: the split-KV work list and the multi-GPU partitioners (no GPU)."""
import numpy as np
import pytest

import glacier_kv as G
from glacier_kv import workloads as W


def chunks(ctx, bs):
    if ctx <= 0:
        return 0
    cpp = -(-bs // 8)
    full, rem = divmod(ctx, bs)
    return full * cpp + -(-rem // 8)


@pytest.mark.parametrize("ctx,heads,bs,workers", [
    ([2049] * 64, 8, 16, 1184),
    ([1, 15, 16, 17, 0, 300], 2, 16, 7),
    ([5, 9, 0], 2, 4, 3),
    ([100], 1, 12, 64),
    ([131072] * 4, 8, 16, 1184),
    ([0, 0], 4, 16, 8),
])
def test_work_list_covers_every_chunk_once_and_balances(ctx, heads, bs, workers):
    plan = G.plan_decode(ctx, heads, bs, workers)
    total = sum(chunks(c, bs) for c in ctx) * heads
    assert plan["total_chunks"] == total
    seen = {}
    for s, c0, c1 in zip(plan["piece_seg"], plan["piece_c0"], plan["piece_c1"]):
        assert 0 <= c0 < c1 <= chunks(ctx[s // heads], bs)
        for c in range(c0, c1):
            assert (s, c) not in seen
            seen[(s, c)] = 1
    assert len(seen) == total
    wb = plan["worker_begin"]
    assert wb[0] == 0 and wb[-1] == plan["n_pieces"] and np.all(np.diff(wb) >= 0)
    # equal contiguous ranges of the charged stream: a worker's chunks plus segment_cost for
    # every segment it starts agree to within one chunk plus the charge of a segment whose
    # start another worker's range cut
    cost = plan["segment_cost"]
    assert cost >= 0
    load = []
    for w in range(workers):
        c0 = plan["piece_c0"][wb[w]:wb[w + 1]]
        c1 = plan["piece_c1"][wb[w]:wb[w + 1]]
        load.append(int((c1 - c0).sum()) + cost * int((c0 == 0).sum()))
    assert max(load) - min(load) <= 1 + 2 * cost
    # a segment split over several workers gets contiguous partial slots
    slots = plan["piece_slot"]
    split = [s for s in set(plan["piece_seg"].tolist()) if (plan["piece_seg"] == s).sum() > 1]
    assert plan["n_merge"] == len(split)
    assert plan["n_slots"] == int((slots >= 0).sum())
    for s in split:
        ss = slots[plan["piece_seg"] == s]
        assert np.all(np.diff(ss) == 1)
    assert np.all(slots[[(plan["piece_seg"] == s).sum() == 1 for s in plan["piece_seg"]]] == -1)


def test_plan_rejects_bad_arguments():
    with pytest.raises(G.ArgumentOutOfRangeError):
        G.plan_decode([1], 0, 16, 4)
    with pytest.raises(G.ArgumentOutOfRangeError):
        G.plan_decode([1], 1, 16, 0)


def test_lpt_partition_balances_context():
    rng = np.random.default_rng(1)
    ctx = np.clip(np.round(rng.lognormal(np.log(1500), 1.0, 256)), 16, 32768).astype(np.int32)
    for ranks in (1, 2, 4, 8):
        r = G.partition_lpt(ctx, ranks)
        assert r.min() >= 0 and r.max() < ranks
        loads = np.bincount(r, weights=ctx, minlength=ranks)
        # LPT bound: max load <= 4/3 optimum; the optimum >= max(mean, longest job)
        assert loads.max() <= 4 / 3 * max(loads.mean(), ctx.max()) + 1
        assert np.array_equal(r, G.partition_lpt(ctx, ranks))  # deterministic on every rank


def test_split_block_range_tiles_the_table():
    for n, r in [(8192, 8), (10, 3), (3, 8), (0, 2)]:
        rs = [G.split_block_range(n, r, i) for i in range(r)]
        assert rs[0][0] == 0 and rs[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
        sizes = [e - b for b, e in rs]
        assert max(sizes) - min(sizes) <= 1
    with pytest.raises(G.ArgumentOutOfRangeError):
        G.split_block_range(8, 2, 2)


def test_workload_generators_match_the_configs():
    w1 = W.cfg1()
    assert w1.batch == 20 and 128 <= w1.ctx_lens.min() and w1.ctx_lens.max() <= 1024
    used = w1.tables[w1.tables >= 0]
    assert len(set(used.tolist())) == used.size and used.max() < 1024
    w2 = W.cfg2()
    assert w2.batch == 64 and np.all(w2.ctx_lens == 2049)
    assert w2.kv_bytes() == 1_074_266_112  # the algorithmic figure of the config
    assert np.all(w2.slot_mapping == w2.tables[:, 128].astype(np.int64) * 16)
    used = w2.tables[w2.tables >= 0]
    assert len(set(used.tolist())) == used.size
    w3 = W.cfg3(ops=2000)
    assert w3.batch == 256 and w3.ctx_lens.min() >= 16 and w3.ctx_lens.max() <= 32768
    used = w3.tables[w3.tables >= 0]
    assert len(set(used.tolist())) == used.size and used.max() < 65536
    # churn leaves the pages non-contiguous
    first = w3.tables[:, :2]
    assert np.mean(first[:, 1] - first[:, 0] != 1) > 0.2
    w5 = W.cfg5_local(3, 8)
    assert w5.batch == 4 and np.all(w5.ctx_lens == 131072 // 8)


def test_lpt_shares_cover_the_global_batch_once():
    w = W.cfg3(ops=2000)
    for world in (1, 2, 8):
        shares = [W.lpt_share(w, r, world) for r in range(world)]
        assert sum(s.batch for s in shares) == w.batch
        assert sum(int(s.ctx_lens.sum()) for s in shares) == int(w.ctx_lens.sum())
        # every share keeps its sequences' own table rows
        rank = G.partition_lpt(w.ctx_lens, world)
        for r, s in enumerate(shares):
            rows = np.nonzero(rank == r)[0]
            assert np.array_equal(s.ctx_lens, w.ctx_lens[rows])
            assert np.array_equal(s.tables, w.tables[rows, : s.tables.shape[1]])
            assert np.all(w.tables[rows, s.tables.shape[1]:] < 0)
        loads = [int(s.ctx_lens.sum()) for s in shares]
        assert max(loads) <= int(w.ctx_lens.sum()) / world + int(w.ctx_lens.max())
