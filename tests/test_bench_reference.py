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


@pytest.mark.parametrize("config,unit", [("cfg2", "tokens/s"), ("cfg1", "tokens/s"), ("append", "GB/s"),
                                         ("copy", "GB/s")])
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
