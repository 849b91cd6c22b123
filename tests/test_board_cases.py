"""Board case files (``tests/golden/make_board_cases.py``) and the board-matrix replay.

CPU: the generated directories have the reference's case format and pass its
own loader (``discover_cases`` / ``load_case``, sw/board_performance.py:99-156)
when the reference tree is present.  GPU: the loop of ``sw/board_matrix.py``
(:110-160) -- one ``AttentionAccelerator(bitstream)`` per case, ``run_attention``
with the case's registers, ``np.argwhere(actual != expected)`` must be empty --
passes on every case of both case sets, with the bitstream being a
``lara_b200.deploy`` descriptor that selects board arithmetic.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

import make_board_cases as mbc
from conftest import REFERENCE

REF_SW = (REFERENCE / "sw") if REFERENCE else Path("/nonexistent-lara-reference")


def _load(path: Path):
    with np.load(path) as d:
        return {k: np.asarray(d[k]) for k in d.files}


def test_generated_case_format(tmp_path):
    paths = mbc.generate(tmp_path, sets=("q31kv7",), lengths=(1, 16), extended=False)
    assert sorted(p.name for p in paths) == ["case_L001_causal.npz", "case_L001_noncausal.npz",
                                             "case_L016_causal.npz", "case_L016_noncausal.npz"]
    d = _load(paths[0])
    assert set(d) == {"q_heads", "k_heads", "v_heads", "expected_o", "seq_len", "causal", "q_pos_base",
                      "kv_pos_base"}
    assert d["q_heads"].dtype == np.uint16 and d["q_heads"].shape == (32, 1, 128)
    assert d["k_heads"].shape == (8, 1, 128) and d["expected_o"].shape == (32, 1, 128)
    assert int(d["q_pos_base"]) == 31 and int(d["kv_pos_base"]) == 7
    # one visible key: the expected words are the group's V row (board arithmetic keeps it exactly)
    np.testing.assert_array_equal(d["expected_o"], np.repeat(d["v_heads"], 4, axis=0))
    # deterministic inputs
    np.testing.assert_array_equal(_load(paths[2])["q_heads"], mbc.case_inputs("q31kv7", 16, True)[0])


@pytest.mark.skipif(not (REF_SW / "board_performance.py").exists(), reason="reference tree not present")
def test_reference_loader_accepts_generated_cases(tmp_path):
    mbc.generate(tmp_path, lengths=(1, 16, 32), extended=False)
    saved = {k: sys.modules.pop(k) for k in ("attn_driver", "board_performance") if k in sys.modules}
    sys.path.insert(0, str(REF_SW))
    try:
        import board_performance as bp

        sets = [(label, tmp_path / d) for label, (d, _, _) in mbc.CASE_SETS.items()]
        cases = bp.discover_cases(sets, lengths=(1, 16, 32))
        assert len(cases) == 12
        assert {(c.q_pos_base, c.kv_pos_base) for c in cases} == {(3, 3), (31, 7)}
    finally:
        sys.path.remove(str(REF_SW))
        for k in ("attn_driver", "board_performance"):
            sys.modules.pop(k, None)
        sys.modules.update(saved)


@pytest.mark.gpu
def test_board_matrix_replay(tmp_path):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    from lara_b200 import deploy
    from lara_b200.attn_driver import AttentionAccelerator

    bit, _, _ = deploy.write_descriptors(tmp_path / "deploy", arithmetic="board")
    paths = mbc.generate(tmp_path / "cases")
    assert len(paths) == 21
    failures = []
    for path in sorted(paths):
        d = _load(path)
        accel = AttentionAccelerator(str(bit))
        try:
            actual = accel.run_attention(d["q_heads"], d["k_heads"], d["v_heads"], seq_len=int(d["seq_len"]),
                                         causal=bool(int(d["causal"])), q_pos_base=int(d["q_pos_base"]),
                                         kv_pos_base=int(d["kv_pos_base"]))
            perf = accel.read_perf()
        finally:
            accel.close()
        mismatch = np.argwhere(actual != d["expected_o"])
        if mismatch.size:
            failures.append(f"{path.parent.name}/{path.name}: {len(mismatch)} words, first at {tuple(mismatch[0])}")
        assert perf["cycles"] > 0 and 0 <= perf["mac_cycles"] <= perf["cycles"]
    assert not failures, failures
