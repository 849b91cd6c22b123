"""GPU parity of the balanced decode schedule (CUDA-core kernel, contiguous cache).

For uniform batches too small to fill the SM slots evenly with whole splits,
``lara_decode_plan`` returns a balanced plan (``chunk_tokens < 0``): the
(sequence, kv head) units' tiles are laid end to end and cut into equal runs,
one per CTA, so a CTA may finish one unit and start the next.  These tests
check it against the CPU oracle with both parity criteria of
``tests/parity.py``, and against the per-split schedule on the same inputs:
the planner's choice at the batch sizes the benchmark runs per GPU, forced
plans with many short runs per unit and with runs that span several units,
ragged and zero lengths (runs that fall past a sequence's end), the
partial-output mode used by split-KV across GPUs, and repeat determinism with
the arrival counters back at zero.
"""

from __future__ import annotations

import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from parity import assert_bf16_parity, words_of  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture
def dev(monkeypatch):
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    monkeypatch.setenv("LARA_DECODE_PATH", "simt")
    return torch.device("cuda:0")


def _inputs(dev, B, Hq, Hkv, D, L, seed, std=0.5):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    q = (torch.randn((B, Hq, D), generator=g, device=dev) * std).to(torch.bfloat16)
    k = (torch.randn((B, Hkv, L, D), generator=g, device=dev) * std).to(torch.bfloat16)
    v = (torch.randn((B, Hkv, L, D), generator=g, device=dev) * std).to(torch.bfloat16)
    return q, k, v


def _check(o, q, k, v, lens, pairs, what, tensor_core=False):
    G = q.shape[1] // k.shape[1]
    qw, ow = words_of(q), words_of(o)
    for b, h in pairs:
        n = int(lens[b])
        kw, vw = words_of(k[b:b + 1, h:h + 1, :n]), words_of(v[b:b + 1, h:h + 1, :n])
        qs = qw[b:b + 1, h * G:(h + 1) * G]
        gold = oracle.decode_attention(qs, kw, vw, np.array([n]))
        g64 = oracle.decode_attention_fp64(qs, kw, vw, np.array([n]))
        assert_bf16_parity(ow[b, h * G:(h + 1) * G], gold[0], g64[0], what=f"{what} b={b} kvh={h}",
                           tensor_core=tensor_core)


@pytest.mark.parametrize("B", [8, 10, 16, 20])
def test_planner_picks_balanced_for_small_uniform_batches(dev, B):
    from lara_b200 import ops

    Hq, Hkv, D, L = 32, 8, 128, 4096
    plan = ops.decode_plan(B, Hq, Hkv, D, L, np.full(B, L, np.int32))
    assert plan.chunk_tokens < 0, plan  # balanced
    q, k, v = _inputs(dev, B, Hq, Hkv, D, L, seed=B)
    lens = torch.full((B,), L, dtype=torch.int32, device=dev)
    dec = ops.Decoder(B, Hq, Hkv, D, L, dev, lens=np.full(B, L))
    assert dec.plan.chunk_tokens < 0
    o = dec(q, k, v, lens)
    torch.cuda.synchronize()
    assert ops.workspace_status(dec.workspace) == 0
    ref = ops.Decoder(B, Hq, Hkv, D, L, dev, num_splits=4, chunk_tokens=1024)(q, k, v, lens)
    e = oracle.bf16_parity_error(words_of(o), oracle.bf16_u16_to_fp32(words_of(ref)))
    assert e["max_ulp"] <= oracle.PARITY_ULPS, e
    rng = np.random.default_rng(B)
    pairs = sorted({(int(b), int(h)) for b, h in zip(rng.integers(0, B, 5), rng.integers(0, Hkv, 5))} | {(B - 1, 7)})
    _check(o, q, k, v, np.full(B, L), pairs, f"balanced B={B} plan={dec.plan}")


@pytest.mark.parametrize("geom,per_tiles", [
    ((8, 32, 8, 128, 4096), 3),      # 64 tiles per unit in runs of 3: up to 23 segments per unit
    ((8, 32, 8, 128, 4096), 200),    # runs of 200 tiles span up to 5 units
    ((5, 8, 2, 64, 700), 4),         # head_dim 64, a ragged last tile per unit
    ((6, 16, 8, 128, 1000), 5),      # groups of 2
    ((4, 8, 8, 128, 513), 2),        # groups of 1
])
def test_forced_balanced_plans_ragged_lengths(dev, geom, per_tiles):
    """Forced balanced plans over ragged lengths: runs past a sequence's end
    (empty segments) and zero-length sequences still merge correctly."""
    from lara_b200 import _native, ops

    B, Hq, Hkv, D, L = geom
    tile = 64  # the CUDA-core kernel's tile for these groups (1, 2, 4)
    tpu = math.ceil(L / tile)
    chunk = per_tiles * tile
    slots = math.ceil(tpu / per_tiles) + 1
    rng = np.random.default_rng(B * 7 + per_tiles)
    lens_np = rng.integers(0, L + 1, B).astype(np.int32)
    lens_np[0] = L
    lens_np[-1] = 0
    q, k, v = _inputs(dev, B, Hq, Hkv, D, L, seed=B + per_tiles)
    lens = torch.tensor(lens_np, device=dev)
    ws = ops.new_workspace(int(_native.lib.lara_decode_workspace_bytes(B, Hq, Hkv, D, slots)), dev)
    o = torch.full_like(q, float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # twice: the arrival counters must be back at zero
        rc = _native.lib.lara_gqa_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), lens.data_ptr(), o.data_ptr(), B,
                                         Hq, Hkv, D, L, 1.0 / math.sqrt(D), slots, -chunk, ws.data_ptr(), ws.numel(),
                                         stream)
        assert rc == 0, _native.last_error()
        torch.cuda.synchronize()
        assert ops.workspace_status(ws) == 0
        ctr = ws[256:256 + 4 * B * Hkv].view(torch.int32)
        assert int(ctr.abs().sum()) == 0
    assert not np.any(words_of(o)[-1])  # zero-length sequence -> zeros
    qw, kw, vw = words_of(q), words_of(k), words_of(v)
    gold = oracle.decode_attention(qw, kw, vw, lens_np)
    g64 = oracle.decode_attention_fp64(qw, kw, vw, lens_np)
    assert_bf16_parity(words_of(o), gold, g64, what=f"forced balanced {geom} per={per_tiles}")
    # too few partial slots, and runs that span more units than a CTA tracks, are rejected
    assert _native.lib.lara_gqa_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), lens.data_ptr(), o.data_ptr(), B,
                                       Hq, Hkv, D, L, 1.0 / math.sqrt(D), slots - 1, -chunk, ws.data_ptr(),
                                       ws.numel(), stream) == _native.LARA_ERR_BAD_CFG
    assert _native.lib.lara_gqa_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), lens.data_ptr(), o.data_ptr(), B,
                                       Hq, Hkv, D, L, 1.0 / math.sqrt(D), 64, -(8 * tpu * tile), ws.data_ptr(),
                                       ws.numel(), stream) == _native.LARA_ERR_BAD_CFG


def test_balanced_partial_output_and_combine(dev):
    """Partial-output mode (split-KV across GPUs) under a balanced plan: four
    token ranges decoded as partials and merged by the LSE combine."""
    from lara_b200 import ops

    B, Hq, Hkv, D, L, P = 8, 32, 8, 128, 16384, 4
    q, k, v = _inputs(dev, B, Hq, Hkv, D, L, seed=99)
    shard = L // P
    mls, accs = [], []
    for i in range(P):
        ks = k[:, :, i * shard:(i + 1) * shard].contiguous()
        vs = v[:, :, i * shard:(i + 1) * shard].contiguous()
        dec = ops.Decoder(B, Hq, Hkv, D, shard, dev, lens=np.full(B, shard))
        assert dec.plan.chunk_tokens < 0, dec.plan
        ml, acc = dec.partial(q, ks, vs, torch.full((B,), shard, dtype=torch.int32, device=dev))
        mls.append(ml)
        accs.append(acc)
    o = ops.lse_combine(torch.stack(mls), torch.stack(accs)).view(B, Hq, D)
    _check(o, q, k, v, np.full(B, L), [(0, 0), (3, 5), (7, 7)], "balanced partial + combine")


def test_balanced_plan_on_the_tensor_core_path_runs_as_splits(dev, monkeypatch):
    """A balanced plan handed to a path without the balanced kernel (the
    tensor-core kernel here) runs as equal splits of the same length and still
    meets the oracle."""
    from lara_b200 import ops

    B, Hq, Hkv, D, L = 8, 32, 8, 128, 4096
    plan = ops.decode_plan(B, Hq, Hkv, D, L, np.full(B, L, np.int32))
    assert plan.chunk_tokens < 0
    q, k, v = _inputs(dev, B, Hq, Hkv, D, L, seed=5)
    lens = torch.full((B,), L, dtype=torch.int32, device=dev)
    monkeypatch.setenv("LARA_DECODE_PATH", "tc")
    dec = ops.Decoder(B, Hq, Hkv, D, L, dev, num_splits=plan.num_splits, chunk_tokens=plan.chunk_tokens)
    o = dec(q, k, v, lens)
    torch.cuda.synchronize()
    assert ops.workspace_status(dec.workspace) == 0
    _check(o, q, k, v, np.full(B, L), [(0, 0), (7, 3)], "tensor-core path", tensor_core=True)
