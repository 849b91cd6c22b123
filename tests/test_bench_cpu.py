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


def test_reference_arm_config_matches_our_arm():
    """Both arms quote the same workload dict (same keys and values)."""
    from lara_b200.workloads import CONFIGS

    cfg = CONFIGS[2]
    ours = bench.workload_config(2, cfg.batch, cfg.seq_len)
    assert ours == {"workload": "llama3_8b_decode", "global_batch": 64, "seq_len": 4096, "n_q_heads": 32,
                    "n_kv_heads": 8, "head_dim": 128}
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1", "--batch", "2", "--seq-len", "256"],
                         capture_output=True, text=True, env=env, timeout=300)
    d = json.loads([ln for ln in out.stdout.splitlines() if ln.startswith("{")][0])
    assert d["config"] == bench.workload_config(2, 2, 256)
    assert d["scaling"] == "strong"


def test_rotation_count_covers_four_l2():
    assert bench.rotation_count(2 << 30) == 1
    r = bench.rotation_count(134_217_728)  # config 2 at 8 GPUs: 8 sequences per rank
    assert r * 134_217_728 >= 4 * bench.L2_BYTES and (r - 1) * 134_217_728 < 4 * bench.L2_BYTES


def test_prefill_units_partition_every_unit_once():
    from lara_b200.workloads import PREFILL, prefill_launch_groups, prefill_units

    for world in range(1, 9):
        seen = []
        for rank in range(world):
            for b, h0, nh in prefill_units(PREFILL, world, rank):
                assert 0 <= h0 and h0 + nh <= PREFILL.n_kv_heads and nh > 0
                seen += [(b, h) for h in range(h0, h0 + nh)]
        assert sorted(seen) == [(b, h) for b in range(PREFILL.batch) for h in range(PREFILL.n_kv_heads)]
    # whole sequences of a rank share one batched launch; a split sequence is a launch of its own
    assert prefill_launch_groups(PREFILL, prefill_units(PREFILL, 1, 0)) == [(0, 4, 0, 8)]
    assert prefill_launch_groups(PREFILL, prefill_units(PREFILL, 8, 3)) == [(1, 1, 4, 4)]
    assert prefill_launch_groups(PREFILL, prefill_units(PREFILL, 3, 1)) == [(1, 1, 3, 5), (2, 1, 0, 6)]


def test_decode_shard_is_rank_independent(monkeypatch):
    """A token range drawn by a split-KV rank equals the same range of the
    whole-sequence draw, across token-block boundaries; a sequence's words do
    not depend on which other sequences a rank holds."""
    import torch

    from lara_b200 import workloads

    monkeypatch.setattr(workloads, "TOKEN_BLOCK", 16)
    cfg = workloads.DecodeConfig("t", 3, 4, 2, 8, 50, 0.5, 11, k_boost_channels=(0,), k_boost=20.0)
    lens = np.array([50, 37, 50], np.int32)
    q, k, v, ln = workloads.decode_shard(cfg, "cpu", [0, 1, 2], lens)
    assert ln.tolist() == [50, 37, 50]
    assert torch.all(k[1, :, 37:] == 0)
    for start, cnt in ((0, 13), (13, 20), (33, 17)):
        qs, ks, vs, ls = workloads.decode_shard(cfg, "cpu", [0, 2], lens, token_start=start, token_count=cnt)
        assert ls.tolist() == [cnt, cnt]
        assert torch.equal(ks[0, :, :cnt], k[0, :, start:start + cnt])
        assert torch.equal(vs[1, :, :cnt], v[2, :, start:start + cnt])
        assert torch.equal(qs[1], q[2])
    q1, k1, _, _ = workloads.decode_shard(cfg, "cpu", [2], lens)
    assert torch.equal(k1[0], k[2]) and torch.equal(q1[0], q[2])
    # the boosted channel carries the x20 scale
    assert float(k[..., 0].float().abs().mean()) > 10 * float(k[..., 1].float().abs().mean())


def test_prefill_shard_heads_slice_the_whole_draw():
    import torch

    from lara_b200 import workloads

    cfg = workloads.PrefillConfig(batch=2, n_q_heads=8, n_kv_heads=4, head_dim=8, cached=20, new=6, std=0.5, seed=3)
    q, k, v, kn, vn, l0 = workloads.prefill_shard(cfg, "cpu", 1, 0, 4)
    qa, ka, va, kna, vna, _ = workloads.prefill_shard(cfg, "cpu", 1, 1, 2)
    assert torch.equal(qa[0], q[0, :, 2:6]) and torch.equal(ka[0], k[0, 1:3]) and torch.equal(vna[0], vn[0, 1:3])
    assert l0.tolist() == [20] and torch.all(k[0, :, 20:] == 0)
