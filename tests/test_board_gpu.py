"""GPU: the board-arithmetic kernel is bit-exact with the board oracle.

``lara_attention_dense_board`` (lara_b200/csrc/board.cu) must reproduce the
bf16 words of ``oracle/board_arith.c`` -- the C restatement of LARA's
synthesized datapath -- on every case: the reference's transaction matrix
(L in {1, 16, 32, 64, 128, 512} x causal x position bases, as in
sw/run_board_full_validation.py and sw/board_matrix.py), ragged lengths that
end mid-block, softmax stress (large logits, so exp inputs fall below -8 and
corrections are tiny), and inputs salted with zeros, bf16 denormals and huge
values so that every slow path of the primitives (signed zeros, flushed
denormals, exponent overflow with the RTL's 8-bit wraparound) is exercised.
The bar is bit equality.  For L >= 128 the oracle checks a head subset (the
kernel always runs all 32 heads).
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from oracle import board  # noqa: E402
from parity import words_of  # noqa: E402

pytestmark = pytest.mark.gpu

HQ, HKV = 32, 8


def _dev():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    return torch.device("cuda:0")


def _inputs(seed, L, scale=0.5, stress=False, salt=False):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((HQ, L, 128)).astype(np.float32) * scale
    k = rng.standard_normal((HKV, L, 128)).astype(np.float32) * scale
    v = rng.standard_normal((HKV, L, 128)).astype(np.float32) * scale
    if stress:
        k[:, :, :4] *= 20.0  # large logits: exp arguments far below -8
    w = [oracle.fp32_to_bf16_u16(a) for a in (q, k, v)]
    if salt:
        specials = np.array([0x0000, 0x8000, 0x0001, 0x8003, 0x7F00, 0xFE80, 0x0080, 0x3F80], np.uint16)
        for a in w:
            m = rng.random(a.shape) < 0.02
            a[m] = rng.choice(specials, int(m.sum()))
    return w


def _run(dev, q, k, v, causal, qb, kb):
    from lara_b200 import ops

    t = lambda a: torch.from_numpy(a.view(np.int16)).to(dev)  # noqa: E731
    o = ops.attention_dense_board(t(q), t(k), t(v), causal=causal, q_pos_base=qb, kv_pos_base=kb)
    torch.cuda.synchronize()
    return words_of(o)


def _check(o, q, k, v, causal, qb, kb, heads=None):
    if heads is None:
        want = board.attention_board(q, k, v, causal=causal, q_pos_base=qb, kv_pos_base=kb)
        np.testing.assert_array_equal(o, want)
        return
    g = HQ // HKV
    for grp in heads:  # whole groups: q heads grp*G .. grp*G+G-1 read kv group grp
        hs = slice(grp * g, grp * g + g)
        want = board.attention_board(q[hs], k[grp:grp + 1], v[grp:grp + 1], causal=causal, q_pos_base=qb,
                                     kv_pos_base=kb)
        np.testing.assert_array_equal(o[hs], want, err_msg=f"group {grp}")


MATRIX = [(L, c, qb, kb) for L in (1, 16, 32, 64) for c in (True, False) for qb, kb in ((0, 0), (31, 7))]


@pytest.mark.parametrize("case", MATRIX, ids=lambda c: f"L{c[0]}_{'c' if c[1] else 'nc'}_q{c[2]}kv{c[3]}")
def test_board_matrix_bit_exact(case):
    L, causal, qb, kb = case
    dev = _dev()
    q, k, v = _inputs(1000 + L, L)
    _check(_run(dev, q, k, v, causal, qb, kb), q, k, v, causal, qb, kb)


@pytest.mark.parametrize("L,causal,qb,kb", [(128, True, 0, 0), (128, False, 31, 7), (512, True, 31, 7),
                                            (97, True, 7, 31), (200, True, 0, 100)])
def test_board_long_and_ragged(L, causal, qb, kb):
    dev = _dev()
    q, k, v = _inputs(2000 + L, L)
    o = _run(dev, q, k, v, causal, qb, kb)
    _check(o, q, k, v, causal, qb, kb, heads=[0, 7] if L >= 128 else None)


def test_board_softmax_stress():
    dev = _dev()
    q, k, v = _inputs(31, 96, scale=1.0, stress=True)
    _check(_run(dev, q, k, v, True, 0, 0), q, k, v, True, 0, 0)


@pytest.mark.parametrize("seed", [41, 42])
def test_board_special_values_take_the_rtl_paths(seed):
    dev = _dev()
    q, k, v = _inputs(seed, 48, scale=2.0, salt=True)
    _check(_run(dev, q, k, v, True, 3, 0), q, k, v, True, 3, 0)
    _check(_run(dev, q, k, v, False, 0, 0), q, k, v, False, 0, 0)


def test_zero_and_identity():
    dev = _dev()
    z = np.zeros((HQ, 16, 128), np.uint16)
    zk = np.zeros((HKV, 16, 128), np.uint16)
    assert not np.any(_run(dev, z, zk, zk, True, 0, 0))
    q, k, v = _inputs(5, 1)
    np.testing.assert_array_equal(_run(dev, q, k, v, True, 0, 0), np.repeat(v, HQ // HKV, axis=0))


def test_driver_board_arithmetic(tmp_path):
    """The harness route: a deployment descriptor with arithmetic 'board' makes
    AttentionAccelerator.run_attention return the oracle's words."""
    from lara_b200 import deploy
    from lara_b200.attn_driver import AttentionAccelerator

    bit, _, _ = deploy.write_descriptors(tmp_path, arithmetic="board")
    q, k, v = _inputs(77, 64)
    with AttentionAccelerator(str(bit)) as acc:
        assert acc.arithmetic == "board"
        o = acc.run_attention(q, k, v, seq_len=64, causal=True, q_pos_base=31, kv_pos_base=7)
        perf = acc.read_perf()
        assert 0 <= perf["mac_cycles"] <= perf["cycles"]
        acc.set_arithmetic("ieee")
        o_ieee = acc.run_attention(q, k, v, seq_len=64, causal=True, q_pos_base=31, kv_pos_base=7)
    np.testing.assert_array_equal(o, board.attention_board(q, k, v, causal=True, q_pos_base=31, kv_pos_base=7))
    gold = oracle.cpu_attention_numpy(q, k, v, causal=True, q_pos_base=31, kv_pos_base=7)
    from parity import assert_bf16_parity, prefill_on_tensor_cores

    g64 = oracle.dense_attention_fp64(q, k, v, causal=True, q_pos_base=31, kv_pos_base=7)
    assert_bf16_parity(o_ieee, gold, g64, what="ieee after board", tensor_core=prefill_on_tensor_cores(32, 8, 128))
