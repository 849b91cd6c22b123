"""Pin the CPU oracle to the reference's own outputs (golden fixtures).

The fixtures in ``tests/golden`` were produced by importing the reference's
``sw/attn_driver.py`` and ``sw/board_performance.py`` / ``sw/benchmark.py``
(``tests/golden/make_golden.py``).  These tests need no GPU.
"""

from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest

import make_golden as mg
import oracle
from oracle import attention as oa


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_bf16_pack_known_answers(golden_dir):
    kat = np.load(golden_dir / "kat_bf16.npz")
    got = oracle.fp32_to_bf16_u16(kat["fp32_bits"].view(np.float32))
    np.testing.assert_array_equal(got, kat["bf16_words"])


def test_bf16_unpack_all_words(golden_dir):
    kat = np.load(golden_dir / "kat_bf16.npz")
    words = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    got = oracle.bf16_u16_to_fp32(words)
    assert _sha(got.view(np.uint32)) == str(kat["unpack_sha256"])


def test_bf16_pack_uint16_passthrough():
    w = np.array([1, 2, 0xFFFF], dtype=np.uint16)
    assert oracle.fp32_to_bf16_u16(w) is not None
    np.testing.assert_array_equal(oracle.fp32_to_bf16_u16(w), w)


def test_counts_match_reference(golden_dir):
    for row in json.loads((golden_dir / "counts.json").read_text()):
        args = (row["L"], row["causal"], row["q_pos_base"], row["kv_pos_base"])
        assert oracle.valid_pairs(*args) == row["valid_pairs"], row
        assert oracle.tile_pairs_per_head(*args) == row["tile_pairs_per_head"], row


@pytest.mark.parametrize("case", mg.BOARD_CASES, ids=lambda c: f"L{c[0]}_{'c' if c[1] else 'nc'}_q{c[2]}kv{c[3]}")
def test_board_attention_bit_exact(golden_dir, case):
    L, causal, qb, kb = case
    name = f"board_L{L}_{'causal' if causal else 'noncausal'}_q{qb}_kv{kb}"
    fx = np.load(golden_dir / f"{name}.npz")
    q, k, v = mg.board_inputs(int(fx["seed"]), L, oracle.fp32_to_bf16_u16)
    assert _sha(q) + _sha(k) + _sha(v) == str(fx["input_sha256"]), "NumPy generator stream changed"
    o = oracle.cpu_attention_numpy(q, k, v, causal=causal, q_pos_base=qb, kv_pos_base=kb)
    rows = fx["rows"]
    np.testing.assert_array_equal(o[:, rows, :], fx["o_rows"])
    assert _sha(o) == str(fx["o_sha256"]), "oracle is not bit-identical to the reference output"
    assert _sha(oracle.fp32_to_bf16_u16(o)) == str(fx["o_bf16_sha256"])


def test_decode_cfg1_matches_reference(golden_dir):
    fx = np.load(golden_dir / "decode_cfg1.npz")
    q, kc, vc, kn, vn = mg.decode_cfg1_inputs(oracle.fp32_to_bf16_u16)
    for a, key in ((q, "q"), (kc, "k_cache"), (vc, "v_cache"), (kn, "k_new"), (vn, "v_new")):
        np.testing.assert_array_equal(a, fx[key])
    k_all = np.concatenate([kc, kn[:, :, None, :]], axis=2)
    v_all = np.concatenate([vc, vn[:, :, None, :]], axis=2)
    o = oracle.decode_attention(q, k_all, v_all, np.array([513]))
    # Same math; BLAS may block a [G,D]x[D,n] product differently from the
    # reference's [G,n,D]x[D,n], so fp32 agreement is to a few ulp.
    np.testing.assert_allclose(o, fx["o_fp32"], rtol=0, atol=1e-6 * np.abs(fx["o_fp32"]).max())
    assert np.max(oa.ulp_distance(oracle.fp32_to_bf16_u16(o), fx["o_bf16"])) <= 1.0


def test_prefill_cfg1_matches_reference(golden_dir):
    fx = np.load(golden_dir / "decode_cfg1.npz")
    q, kc, vc, kn, vn = mg.decode_cfg1_inputs(oracle.fp32_to_bf16_u16)
    k_all = np.concatenate([kc, kn[:, :, None, :]], axis=2)
    v_all = np.concatenate([vc, vn[:, :, None, :]], axis=2)
    n = k_all.shape[2]
    rng = np.random.default_rng(int(fx["prefill_seed"]))
    q_pref = oracle.fp32_to_bf16_u16(rng.standard_normal((8, n, 64), dtype=np.float32))
    o = oracle.prefill_attention(q_pref[None], k_all, v_all, np.array([n]), 0, causal=True)[0]
    rows = fx["prefill_rows"]
    ref = fx["o_prefill_rows"]
    np.testing.assert_allclose(o[:, rows, :], ref, rtol=0, atol=1e-6 * np.abs(ref).max())


def test_cpu_attention_raises_on_dead_causal_row():
    q = np.zeros((32, 4, 128), np.uint16)
    k = np.zeros((8, 4, 128), np.uint16)
    with pytest.raises(ValueError):
        oracle.cpu_attention_numpy(q, k, k, causal=True, q_pos_base=0, kv_pos_base=10)


def test_zero_in_zero_out():
    # sw/board_test.py:78-79: all-zero inputs give an all-zero output
    q = np.zeros((32, 16, 128), np.uint16)
    k = np.zeros((8, 16, 128), np.uint16)
    o = oracle.cpu_attention_numpy(q, k, k, causal=True, q_pos_base=0, kv_pos_base=0)
    assert not np.any(oracle.fp32_to_bf16_u16(o))


def test_decode_dead_row_is_zero():
    q = np.ones((2, 4, 64), np.uint16)
    kc = np.ones((2, 1, 8, 64), np.uint16)
    o = oracle.decode_attention(q, kc, kc, np.array([0, 3]))
    assert np.all(o[0] == 0) and np.all(np.isfinite(o[1]))


def test_ulp_helpers():
    w = oracle.fp32_to_bf16_u16(np.array([1.0, 2.0, 0.0], np.float32))
    np.testing.assert_allclose(oracle.bf16_ulp(w), [2.0**-7, 2.0**-6, 2.0**-133])
    nxt = (w + 1).astype(np.uint16)
    np.testing.assert_allclose(oracle.ulp_distance(nxt, w)[:2], [1.0, 1.0])


def test_numeric_error_keys():
    e = oracle.numeric_error(np.array([1.0, 2.0]), np.array([1.0, 2.5]))
    assert set(e) == {"max_abs", "mean_abs", "rmse", "normalized_rmse", "max_relative_floor_1e-6"}
    assert e["max_abs"] == 0.5
