"""bench.py's reference arm (the CPU oracle timed on the host cores): one JSON
line with the contract's keys, printed by rank 0 only under torchrun."""

from __future__ import annotations

import json
import os
import subprocess
import sys
import time

import pytest

from tests.conftest import ROOT

KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
        "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


def _json_lines(out: str) -> list[dict]:
    return [json.loads(ln) for ln in out.splitlines() if ln.startswith("{")]


def _env():
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", OMP_NUM_THREADS="4")
    env.pop("CUDA_VISIBLE_DEVICES", None)
    return env


@pytest.mark.parametrize("workload", ["dit", "block"])
def test_reference_arm_json(workload):
    t0 = time.perf_counter()
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--workload", workload,
                        "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=600, env=_env(),
                       cwd=ROOT)
    wall = time.perf_counter() - t0
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1
    d = lines[0]
    assert KEYS <= set(d)
    assert d["impl"] == "reference" and d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 3
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["unit"] == d["unit"]
    # the line claims only the work it timed: steps x ms_per_step fits inside the run
    assert d["steps"] * d["ms_per_step"] / 1e3 <= wall


def test_reference_arm_two_ranks_prints_once():
    """Under torchrun (gloo on this CPU box) rank 0 alone runs and prints; the
    other rank exits 0 without work."""
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", "29613", str(ROOT / "bench.py"), "--impl", "reference",
           "--workload", "block", "--gpus", "2", "--steps", "1", "--warmup", "3"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=_env(), cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = _json_lines(r.stdout)
    assert len(lines) == 1 and lines[0]["n_gpus"] == 2 and lines[0]["impl"] == "reference"
