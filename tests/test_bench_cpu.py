"""CPU tests of bench.py's contract pieces that run without a GPU.

* the CPU-baseline harness (per-pass timing with min/median/p95/max, one
  thread and all cores, as in the reference's sw/board_performance.py:195-204,
  321-331);
* the reference arm (``--impl reference``): one JSON line with the metric,
  unit, ``cpu_baseline`` and a zero-transfer ``e2e`` object.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
import oracle  # noqa: E402


def test_pass_stats():
    st = bench.pass_stats([0.4, 0.1, 0.3, 0.2, 0.5])
    assert st["repeats"] == 5
    assert st["min_s"] == 0.1 and st["max_s"] == 0.5 and st["median_s"] == 0.3
    assert 0.3 < st["p95_s"] <= 0.5


def test_cpu_baseline_runs_small():
    rng = np.random.default_rng(0)
    q = oracle.fp32_to_bf16_u16(rng.standard_normal((2, 8, 64), dtype=np.float32))
    k = oracle.fp32_to_bf16_u16(rng.standard_normal((2, 2, 96, 64), dtype=np.float32))
    v = oracle.fp32_to_bf16_u16(rng.standard_normal((2, 2, 96, 64), dtype=np.float32))
    lens = np.array([96, 40], np.int32)
    pairs = [(b, h) for b in range(2) for h in range(2)]
    gbs, st_all, gbs1, st_one, n1 = bench.cpu_baseline_runs(q, k, v, lens, pairs, 2, 0.0, one_thread_pass_s=0.01)
    assert gbs > 0 and gbs1 > 0
    assert st_all["repeats"] >= 5 and st_one["repeats"] >= 5
    assert 1 <= n1 <= len(pairs)
    # bytes per pass: sum of the pairs' lengths x 2 (K, V) x 2 B x head_dim
    nbytes, times = bench.cpu_pass_times(q, k, v, lens, pairs[:1], 1, 1)
    assert nbytes == 96 * 64 * 4 and len(times) == 1


def test_reference_arm_json_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1", "--batch", "2", "--seq-len", "256"],
                         capture_output=True, text=True, env=env, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["unit"] == "GB/s" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["metric"] == bench.METRIC
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"]
    assert cb["single_thread"]["cores"] == 1 and cb["pass_seconds"]["repeats"] == 1
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
