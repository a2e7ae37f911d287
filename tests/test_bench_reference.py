"""The reference arm of bench.py (`--impl reference`): it times the CPU restatement of the
reference's code for the same metric and prints one JSON line with the contract's keys; under a
multi-rank launch only rank 0 runs it.  CPU only."""
import json
import os
import subprocess
import sys

import pytest

from conftest import ROOT

BENCH = os.path.join(ROOT, "bench.py")


def run_reference(config: str, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    r = subprocess.run([sys.executable, BENCH, "--impl", "reference", "--config", config, "--steps", "1",
                        "--warmup", "3"], capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    return [json.loads(l) for l in r.stdout.splitlines() if l.startswith("{")]


@pytest.mark.parametrize("config,unit", [("cfg3", "tokens/s"), ("cfg2", "tokens/s"), ("cfg1", "tokens/s"),
                                         ("append", "GB/s"), ("copy", "GB/s")])
def test_reference_arm_prints_one_contract_line(config, unit):
    lines = run_reference(config)
    assert len(lines) == 1
    d = lines[0]
    assert d["impl"] == "reference" and d["unit"] == unit and d["value"] > 0
    assert d["higher_is_better"] is True and d["steps"] == 1 and d["warmup"] == 3
    assert d["e2e"] == {"value": d["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"]
    assert d["config"]["workload"]


def test_reference_arm_runs_on_rank_zero_only():
    assert run_reference("cfg2", {"RANK": "1", "WORLD_SIZE": "2"}) == []


def test_reference_arm_maps_no_product_library_and_uses_every_core():
    """The arm a torchrun launch starts (OMP_NUM_THREADS=1 in its environment) still times the
    restatement on all the host cores it may use, and maps only the oracle's library."""
    from oracle import pyoracle as O

    (d,) = run_reference("cfg3", {"OMP_NUM_THREADS": "1"})
    assert d["native_so_loaded"] == ["oracle/lib/libgkv_oracle.so"]
    assert d["cpu_baseline"]["cores"] == O.host_cores() == d["host_cores"]
    assert d["scaling"] == "strong" and d["kv_dtype"] == "f32"
    assert d["config"]["workload"].startswith("cfg3: decode, 256 seqs")


def test_numpy_churn_gives_the_pool_allocators_tables():
    """cfg3's block tables come from a plain-Python LIFO free list; replaying the same seeded
    admit/evict trace on the shim's allocator (metadata-only pool, no GPU) gives the same tables."""
    import numpy as np

    import glacier_kv as G
    from glacier_kv import workloads as W

    rng = np.random.default_rng(W.SEED)
    ctx = W.cfg3_ctx(rng, 256)
    state = rng.bit_generator.state
    t_np = W.churn_tables(W.LifoFreeList(65536, 16), ctx, rng)
    rng.bit_generator.state = state
    meta = G.PagedBlockPool(65536, 1, 4, 128, 16, allocate_device_arena=False)
    try:
        t_pool = W.churn_tables(meta, ctx, rng)
    finally:
        meta.close()
    assert np.array_equal(t_np, t_pool)
    assert np.array_equal(W.cfg3(W.SEED).tables, t_np)
