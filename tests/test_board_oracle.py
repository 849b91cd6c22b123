"""Board-arithmetic oracle (``oracle/board_arith.c``): pins and properties.

What pins the restatement of LARA's synthesized arithmetic:

* the exp and reciprocal tables equal the reference's ``hw/data/exp_lut.hex``
  / ``recip_lut.hex`` (SHA-256 of the words; compared with the files directly
  when the reference tree is present), and the product library's compiled
  tables (``lara_b200/csrc/board_luts.inc``) equal them too;
* the RTL's fp32 adder and multiplier (hw/rtl/pkg/attn_pkg.sv:404-544) round to
  nearest even exactly as IEEE-754 on normal operands with normal results, and
  bf16_mul_to_fp32 (:546-597) is the exact product -- checked against NumPy
  float32 on random and cancellation-heavy operands;
* the RTL's special-value rules (signed zeros, NaN, infinities) follow the
  Verilog, checked on hand-derived cases;
* transaction-level properties: zero in -> zero out (sw/board_test.py:45-79),
  one visible key -> the V row exactly, fully masked rows -> zeros, and the
  board result stays close to the exact-exp golden model.

The transaction as a whole has no board vectors to pin it (the reference ships
no case files): parity of the model with the FPGA is unpinned.
"""

from __future__ import annotations

import re
from pathlib import Path

import numpy as np
import pytest

import oracle
from oracle import board, board_luts
from conftest import REFERENCE

REF = (REFERENCE / "hw" / "data") if REFERENCE else Path("/nonexistent-lara-reference")
ROOT = Path(__file__).resolve().parents[1]


def _hex_words(path: Path) -> np.ndarray:
    return np.array([int(t, 16) for t in path.read_text().split()], dtype="<u4")


def test_tables_pinned():
    e, r = board_luts.load()
    assert e.shape == (1024,) and r.shape == (256,)
    assert board_luts.sha256_words(board_luts.make_recip_lut()) == board_luts.RECIP_LUT_SHA256
    assert e[1023] == 0x3F800000 and e[0] == np.float32(np.exp(np.float32(-8.0))).view(np.uint32)


@pytest.mark.skipif(not REF.exists(), reason="reference tree not present")
def test_tables_equal_reference_hex():
    e, r = board_luts.load()
    np.testing.assert_array_equal(e, _hex_words(REF / "exp_lut.hex"))
    np.testing.assert_array_equal(r, _hex_words(REF / "recip_lut.hex"))


def test_product_tables_equal_oracle_tables():
    text = (ROOT / "lara_b200" / "csrc" / "board_luts.inc").read_text()
    blocks = re.findall(r"\{([^}]*)\}", text)
    exp = np.array([int(t.rstrip("u"), 16) for t in re.findall(r"0x[0-9a-f]+u", blocks[0])], dtype="<u4")
    rec = np.array([int(t.rstrip("u"), 16) for t in re.findall(r"0x[0-9a-f]+u", blocks[1])], dtype="<u4")
    e, r = board_luts.load()
    np.testing.assert_array_equal(exp, e)
    np.testing.assert_array_equal(rec, r)


def _random_normal_words(rng, n, emin=64, emax=190):
    e = rng.integers(emin, emax, n).astype(np.uint32)
    m = rng.integers(0, 1 << 23, n).astype(np.uint32)
    s = rng.integers(0, 2, n).astype(np.uint32)
    return (s << 31) | (e << 23) | m


def test_fp32_add_is_ieee_rne_on_normals():
    rng = np.random.default_rng(11)
    n = 300_000
    a, b = _random_normal_words(rng, n), _random_normal_words(rng, n)
    # half the pairs within 3 binades of each other: alignment, carries and cancellation
    h = n // 2
    shift = rng.integers(-3, 4, h)
    eb = (((a[:h] >> 23) & 0xFF).astype(np.int64) + shift).astype(np.uint32)
    b[:h] = (b[:h] & 0x807FFFFF) | (eb << 23)
    b[: n // 8] = a[: n // 8] ^ 0x80000000 ^ rng.integers(0, 4, n // 8).astype(np.uint32)  # near-exact cancellation
    got = board.fp32_add(a, b)
    ref = (a.view(np.float32) + b.view(np.float32)).view(np.uint32)
    normal_or_zero = (((ref >> 23) & 0xFF) != 0) | ((ref & 0x7FFFFFFF) == 0)
    np.testing.assert_array_equal(got[normal_or_zero], ref[normal_or_zero])
    assert normal_or_zero.mean() > 0.99


def test_fp32_mul_and_bf16_mul_are_ieee_on_normals():
    rng = np.random.default_rng(12)
    n = 300_000
    a, b = _random_normal_words(rng, n), _random_normal_words(rng, n)
    with np.errstate(over="ignore", under="ignore"):
        ref = (a.view(np.float32) * b.view(np.float32)).view(np.uint32)
    ok = ((ref >> 23) & 0xFF) - 1 < 254
    np.testing.assert_array_equal(board.fp32_mul(a, b)[ok], ref[ok])
    qa = rng.integers(0, 1 << 16, n).astype(np.uint16)
    qb = rng.integers(0, 1 << 16, n).astype(np.uint16)
    with np.errstate(all="ignore"):
        fa = (qa.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
        fb = (qb.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
        exact = (fa * fb).astype(np.float32).view(np.uint32)
    ea, eb, er = (qa >> 7) & 0xFF, (qb >> 7) & 0xFF, (exact >> 23) & 0xFF
    ok = (ea - 1 < 254) & (eb - 1 < 254) & (er - 1 < 254)
    np.testing.assert_array_equal(board.bf16_mul(qa, qb)[ok], exact[ok])


def test_special_values_follow_the_rtl():
    u = np.uint32
    # fp32_add returns the other operand when one is +-0 (attn_pkg.sv:426-427),
    # so +0 + -0 is -0 (IEEE would give +0); exact cancellation gives +0
    assert board.fp32_add(u(0), u(0x80000000))[()] == 0x80000000
    assert board.fp32_add(u(0x3F800000), u(0xBF800000))[()] == 0
    assert board.fp32_add(u(0x7FC00001), u(0x3F800000))[()] == 0x7FC00000
    # -inf - -inf cancels to +0 in the RTL adder (no infinity rule)
    assert board.fp32_add(u(0xFF800000), u(0x7F800000))[()] == 0
    # fp32_mul tests zero before infinity: inf * 0 = 0 (attn_pkg.sv:514-516)
    assert board.fp32_mul(u(0x7F800000), u(0))[()] == 0
    assert board.fp32_mul(u(0x80000000), u(0x3F800000))[()] == 0x80000000
    # bf16 exponent 0 is zero (denormals flush): sign is the xor of the signs
    assert board.bf16_mul(np.uint16(0x0001), np.uint16(0xBF80))[()] == 0x80000000
    assert board.bf16_mul(np.uint16(0x7F80), np.uint16(0x0000))[()] == 0x7FC00000


def test_exp_lookup_properties():
    e, _ = board.tables()
    u = np.uint32
    assert board.exp_lookup(u(0))[()] == 0x3F800000
    assert board.exp_lookup(u(0x80000000))[()] == 0x3F800000
    assert board.exp_lookup(u(0x3F000000))[()] == 0x3F800000      # x > 0 -> 1
    assert board.exp_lookup(u(0xC1000000))[()] == e[0]            # x = -8 -> first entry
    assert board.exp_lookup(u(0xC1000001))[()] == 0               # x < -8 -> 0
    assert board.exp_lookup(u(0xFF800000))[()] == 0               # -inf -> 0
    x = np.linspace(-8.0, 0.0, 200_001, dtype=np.float32)
    y = board.exp_lookup(x).view(np.float32)
    assert np.all(np.diff(y) >= 0), "interpolated exp must be monotone"
    rel = np.abs(y.astype(np.float64) / np.exp(x.astype(np.float64)) - 1.0)
    assert rel.max() < 1.0e-5, rel.max()  # linear interpolation over 8/1023 spacing


def test_recip_lut_properties():
    rng = np.random.default_rng(3)
    x = (rng.random(100_000) * 1000 + 1e-3).astype(np.float32)
    r = board.recip_lut_bits(x).view(np.float32)
    rel = np.abs(r.astype(np.float64) * x - 1.0)
    assert rel.max() <= 1.0 / 512 + 1e-7  # bucket-midpoint reciprocal of the top 8 fraction bits
    p2 = np.array([0.5, 1.0, 2.0, 4096.0], np.float32)
    np.testing.assert_array_equal(board.recip_lut_bits(p2).view(np.float32), 1.0 / p2)


def _pk(x):
    return oracle.fp32_to_bf16_u16(np.asarray(x, np.float32))


def test_zero_and_identity_transactions():
    z = np.zeros((32, 16, 128), np.uint16)
    assert not np.any(board.attention_board(z, np.zeros((8, 16, 128), np.uint16), np.zeros((8, 16, 128), np.uint16)))
    rng = np.random.default_rng(5)
    q, k, v = _pk(rng.standard_normal((32, 1, 128))), _pk(rng.standard_normal((8, 1, 128))), \
        _pk(rng.standard_normal((8, 1, 128)))
    np.testing.assert_array_equal(board.attention_board(q, k, v), np.repeat(v, 4, axis=0))


def test_dead_causal_rows_are_zero():
    rng = np.random.default_rng(6)
    q, k, v = (_pk(rng.standard_normal(s) * 0.5) for s in ((32, 40, 128), (8, 40, 128), (8, 40, 128)))
    o = board.attention_board(q, k, v, causal=True, q_pos_base=0, kv_pos_base=8)
    assert not np.any(o[:, :8]) and np.all(np.any(o[:, 8:], axis=2))


@pytest.mark.parametrize("L,causal,qb,kb", [(64, True, 0, 0), (77, False, 0, 0), (50, True, 31, 7)])
def test_board_result_tracks_golden_model(L, causal, qb, kb):
    """Board arithmetic differs from exact-exp fp32 by P's bf16 truncation and the
    LUT exp; the result stays within a few bf16 ulp of the golden model."""
    rng = np.random.default_rng(L)
    q, k, v = (_pk(rng.standard_normal(s) * 0.5) for s in ((32, L, 128), (8, L, 128), (8, L, 128)))
    ob = oracle.bf16_u16_to_fp32(board.attention_board(q, k, v, causal=causal, q_pos_base=qb, kv_pos_base=kb))
    gold = oracle.cpu_attention_numpy(q, k, v, causal=causal, q_pos_base=qb, kv_pos_base=kb)
    scale = np.abs(gold).max(axis=2, keepdims=True)
    err = np.abs(ob - gold) / np.maximum(scale, 1e-30)
    assert err.max() < 2.0 ** -5, err.max()
    assert err.mean() < 2.0 ** -9, err.mean()
