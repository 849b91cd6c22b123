"""Layer prologue (RMSNorm -> QKV projection -> RoPE): oracle pins and GPU parity.

The reference's ``run_layer`` (sw/attn_driver.py:552-586) imports its host
helpers from ``host_attention.py``, which the reference does not ship; the
contract is restated in ``oracle/prologue.py``.  Pins: the RoPE frequencies
equal ``hw/data/rope_theta.hex`` word for word (SHA-256 below; compared with
the file when the reference tree is present); RoPE is a rotation (pair norms
kept) whose scores depend only on the position difference.  GPU: the fused
tcgen05 kernel (``lara_layer_prologue``) is within 2 bf16 ulp (floored ulp,
the tolerance of ``oracle.attention``) of the oracle, from single tokens to the
Llama-3-8B projection (hidden 4096 -> 32 q + 8 k + 8 v heads of 128).
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest

import oracle
from oracle import prologue
from conftest import REFERENCE

REF_THETA = (REFERENCE / "hw" / "data" / "rope_theta.hex") if REFERENCE else Path("/nonexistent-lara-reference")
# SHA-256 of hw/data/rope_theta.hex's 64 words (little-endian uint32)
THETA_SHA256 = "517d37a3dd07d63acf7d03dc05ff2e4f3a778c2783e9541d86ef1cd37bb5b968"


def test_rope_theta_pinned():
    t = prologue.rope_theta()
    assert hashlib.sha256(t.view("<u4").tobytes()).hexdigest() == THETA_SHA256
    assert t[0] == 1.0 and t.dtype == np.float32 and np.all(np.diff(t) < 0)


@pytest.mark.skipif(not REF_THETA.exists(), reason="reference tree not present")
def test_rope_theta_equals_reference_hex():
    ref = np.array([int(w, 16) for w in REF_THETA.read_text().split()], dtype="<u4")
    np.testing.assert_array_equal(prologue.rope_theta().view("<u4"), ref)


def test_rope_is_a_relative_rotation():
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, 8, 128)).astype(np.float32)
    k = rng.standard_normal((1, 8, 128)).astype(np.float32)
    r = prologue.apply_rope(q, 100)
    np.testing.assert_allclose(np.hypot(r[..., 0::2], r[..., 1::2]), np.hypot(q[..., 0::2], q[..., 1::2]),
                               rtol=1e-5)
    # q at position p, k at position p': the score depends on p - p' only
    s1 = np.einsum("hd,hd->h", prologue.apply_rope(q, 37)[0, :1], prologue.apply_rope(k, 30)[0, :1])
    s2 = np.einsum("hd,hd->h", prologue.apply_rope(q, 1007)[0, :1], prologue.apply_rope(k, 1000)[0, :1])
    np.testing.assert_allclose(s1, s2, rtol=2e-3, atol=2e-3)


def _words(a):
    return oracle.fp32_to_bf16_u16(np.asarray(a, np.float32))


def _case(seed, L, hidden, hq, hkv, scale_w):
    rng = np.random.default_rng(seed)
    x = _words(rng.standard_normal((L, hidden)))
    w = _words(rng.standard_normal((hidden, (hq + 2 * hkv) * 128)) * scale_w)
    g = _words(1.0 + 0.1 * rng.standard_normal(hidden))
    return x, w, g


CASES = [
    # (L, hidden, Hq, Hkv, rms, q_pos_base, kv_pos_base)
    (1, 64, 4, 2, True, 0, 0),
    (77, 256, 8, 2, True, 31, 7),
    (128, 512, 4, 4, False, 0, 0),
    (300, 4096, 32, 8, True, 3, 3),        # Llama-3-8B projection, 3 token tiles (last ragged)
    (16, 4096, 32, 8, True, 65000, 65000),  # large positions (angles up to ~6.5e4 rad)
    (40, 128, 1, 1, True, 5, 9),            # 3 heads: a ragged 128-column last tile
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=lambda c: f"L{c[0]}_H{c[1]}_q{c[2]}kv{c[3]}_{'rms' if c[4] else 'raw'}_p{c[5]}")
def test_prologue_parity(case):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    from lara_b200 import ops
    from parity import assert_bf16_parity, words_of

    L, hidden, hq, hkv, rms, qb, kb = case
    x, w, g = _case(L * 7 + hidden, L, hidden, hq, hkv, 1.0 / np.sqrt(hidden))
    dev = torch.device("cuda:0")
    t = lambda a: torch.from_numpy(a.view(np.int16)).to(dev)  # noqa: E731
    q, k, v = ops.layer_prologue(t(x), t(w), t(g) if rms else None, n_q_heads=hq, n_kv_heads=hkv,
                                 q_pos_base=qb, kv_pos_base=kb)
    torch.cuda.synchronize()
    gq, gk, gv = prologue.layer_prologue(x, w, g if rms else None, n_q_heads=hq, n_kv_heads=hkv, q_pos_base=qb,
                                         kv_pos_base=kb)
    for name, got, gold in (("q", q, gq), ("k", k, gk), ("v", v, gv)):
        assert_bf16_parity(words_of(got), gold, what=f"{name} {case}")


@pytest.mark.gpu
def test_rmsnorm_words_bit_exact():
    """x_n (the workspace's bf16 RMSNorm output, after the 256-byte status
    block) equals the oracle's words exactly: the fp64 statistic makes the
    fp32 inverse RMS reproducible."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    from lara_b200 import _native, ops
    from parity import words_of

    L, hidden = 200, 4096
    x, w, g = _case(5, L, hidden, 4, 2, 1.0 / 64)
    dev = torch.device("cuda:0")
    t = lambda a: torch.from_numpy(a.view(np.int16)).to(dev)  # noqa: E731
    xd, wd, gd = t(x), t(w), t(g)
    q = torch.empty((4, L, 128), dtype=torch.int16, device=dev)
    k = torch.empty((2, L, 128), dtype=torch.int16, device=dev)
    v = torch.empty_like(k)
    nb = int(_native.lib.lara_layer_prologue_workspace_bytes(1, L, hidden))
    ws = ops.new_workspace(nb, dev)
    _native.check(_native.lib.lara_layer_prologue(xd.data_ptr(), gd.data_ptr(), wd.data_ptr(), q.data_ptr(),
                                                  k.data_ptr(), v.data_ptr(), 1, L, hidden, 4, 2, 128, 0, 0, 1e-5,
                                                  10000.0, ws.data_ptr(), ws.numel(),
                                                  torch.cuda.current_stream().cuda_stream), "prologue")
    torch.cuda.synchronize()
    assert ops.workspace_status(ws) == 0
    xn = words_of(ws[256:256 + L * hidden * 2].view(torch.int16)).reshape(L, hidden)
    np.testing.assert_array_equal(xn, prologue.rms_norm(x, g, 1e-5))


@pytest.mark.gpu
def test_prologue_batched_equals_per_sequence():
    """batch = 3 in one launch gives each sequence's single-sequence words."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    from lara_b200 import ops
    from parity import words_of

    L, hidden = 150, 256
    rng = np.random.default_rng(8)
    xs = _words(rng.standard_normal((3, L, hidden)))
    _, w, g = _case(9, L, hidden, 8, 2, 1.0 / 16)
    dev = torch.device("cuda:0")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev)  # noqa: E731
    qb, kb, vb = ops.layer_prologue(t(xs), t(w), t(g), n_q_heads=8, n_kv_heads=2, q_pos_base=100, kv_pos_base=90)
    for b in range(3):
        q1, k1, v1 = ops.layer_prologue(t(xs[b]), t(w), t(g), n_q_heads=8, n_kv_heads=2, q_pos_base=100,
                                        kv_pos_base=90)
        for got, want in ((qb[b], q1), (kb[b], k1), (vb[b], v1)):
            np.testing.assert_array_equal(words_of(got), words_of(want))
