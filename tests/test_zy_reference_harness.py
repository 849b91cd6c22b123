"""LARA's own harness scripts, unmodified, driving this library on the GPU.

The drop-in contract of the attention path is that the reference's harnesses
(``sw/board_test.py``, ``sw/board_matrix.py``, ``sw/board_performance.py``,
``sw/run_board_full_validation.py``; ``sw/benchmark.py`` beside them) run
unchanged with ``sw/attn_driver.py`` replaced by the one-file shim of
INTEGRATION.md.  The scripts are staged from a LARA source tree by
``tests/ref_harness/stage.py`` into ``baseline/_ref/sw/`` and checked here
against the pinned SHA-256 digests before anything runs.

The test lays out a ``sw/`` directory the way a LARA checkout has it: the five
scripts, the shim as ``attn_driver.py``, the deployment descriptor trio written
with board arithmetic (``python -m lara_b200.deploy descriptors --arithmetic
board``), the environment report (``deploy environment``) and both board case
sets (``tests/golden/make_board_cases.py``; their ``expected_o`` words are the
board-arithmetic oracle's).  Then each script runs as a subprocess with its
usual command line and must exit 0:

* ``board_test.py``: the zero-input smoke (sw/board_test.py:68-92);
* ``board_matrix.py``: both case sets, bit for bit (sw/board_matrix.py:115-155);
* ``board_performance.py --repeats 2``: FPGA-path timing beside the CPU
  baseline, every case bit-exact (sw/board_performance.py:281-473, 634-656);
* ``run_board_full_validation.py``: the whole orchestration, whose
  consolidated report must show 10 + 10 functional and 20 performance passes
  (sw/run_board_full_validation.py:116-144, 300-347);
* ``benchmark.py``: the analytical cycle model (it never imports the driver).
"""

from __future__ import annotations

import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tests" / "ref_harness"))

import stage  # noqa: E402

pytestmark = pytest.mark.gpu

SHIM = '''# sw/attn_driver.py -- B200 backend for the LARA harnesses
from lara_b200.attn_driver import *            # noqa: F401,F403  constants, helpers, classes
from lara_b200.attn_driver import _self_test    # noqa: F401
if __name__ == "__main__":
    _self_test()
'''


def _run(cmd, cwd, env, timeout=900):
    res = subprocess.run(cmd, cwd=cwd, env=env, capture_output=True, text=True, timeout=timeout)
    tail = (res.stdout[-3000:] + "\n" + res.stderr[-3000:]).strip()
    return res.returncode, res.stdout, tail


@pytest.fixture(scope="module")
def sw_dir(tmp_path_factory):
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    ok, why = stage.staged_ok()
    if not ok:
        pytest.skip(f"reference harness scripts not staged: {why}")
    sw = tmp_path_factory.mktemp("lara") / "sw"
    sw.mkdir()
    for name in stage.expected_digests():
        shutil.copyfile(stage.STAGE / name, sw / name)
        assert stage.sha256(sw / name) == stage.expected_digests()[name]
    (sw / "attn_driver.py").write_text(SHIM)
    env = dict(os.environ, PYTHONPATH=str(ROOT) + os.pathsep + os.environ.get("PYTHONPATH", ""))
    py = sys.executable
    for cmd in ([py, "-m", "lara_b200.deploy", "descriptors", "--out", ".", "--arithmetic", "board"],
                [py, "-m", "lara_b200.deploy", "environment", "--bitstream", "./lara_attention.bit"],
                [py, str(ROOT / "tests" / "golden" / "make_board_cases.py"), "--out", "."]):
        rc, _, tail = _run(cmd, sw, env)
        assert rc == 0, f"{cmd}: {tail}"
    report = json.loads((sw / "board_environment.json").read_text())
    assert report["overall_status"] == "PASS", report
    return sw, env


def test_board_test_zero_smoke(sw_dir):
    sw, env = sw_dir
    rc, out, tail = _run([sys.executable, "board_test.py", "--bitstream", "lara_attention.bit"], sw, env)
    assert rc == 0, tail
    assert "LARA KV260 smoke test PASS" in out


def test_board_matrix_both_case_sets_bit_exact(sw_dir):
    sw, env = sw_dir
    for cases, n in (("board_cases_rtl_contract_v2.6_fixed", 10), ("board_cases_rtl_contract_v2.6_q31_kv7", 11)):
        rc, out, tail = _run([sys.executable, "board_matrix.py", "--bitstream", "lara_attention.bit", "--cases",
                              cases, "--output-dir", f"matrix_{cases}"], sw, env)
        assert rc == 0, tail
        assert f"board matrix: {n}/{n} PASS" in out, tail
        rows = json.loads((sw / f"matrix_{cases}" / "summary.json").read_text())
        assert len(rows) == n and all(r["status"] == "PASS" for r in rows)


def test_board_performance_repeats_2(sw_dir):
    sw, env = sw_dir
    rc, out, tail = _run([sys.executable, "board_performance.py", "--bitstream", "lara_attention.bit",
                          "--warmup", "1", "--repeats", "2", "--output-dir", "perf",
                          "--lengths", "1", "16", "32", "64", "128"], sw, env)
    assert rc == 0, tail
    assert "bit-exact matrix: 20/20 PASS" in out, tail
    report = json.loads((sw / "perf" / "performance.json").read_text())
    assert not report["benchmark_errors"] and len(report["results"]) == 20
    for row in report["results"]:
        assert row["correctness"]["fpga_bit_exact_expected"] is True


def test_run_board_full_validation_end_to_end(sw_dir):
    sw, env = sw_dir
    rc, out, tail = _run([sys.executable, "run_board_full_validation.py", "--bitstream", "./lara_attention.bit",
                          "--output-dir", "./board_full_results"], sw, env)
    assert rc == 0, tail
    assert "FULL VALIDATION STATUS: PASS" in out, tail
    cons = json.loads((sw / "board_full_results" / "consolidated_results.json").read_text())
    assert cons["overall_status"] == "PASS"
    for label in ("q3kv3", "q31kv7"):
        f = cons["functional"][label]
        assert (f["passed"], f["total"]) == (10, 10)
    p = cons["performance"]["cpu1"]
    assert (p["passed"], p["total"]) == (20, 20) and not p["benchmark_errors"]
    # the extended maximum-length run as well
    rc, out, tail = _run([sys.executable, "run_board_full_validation.py", "--bitstream", "./lara_attention.bit",
                          "--output-dir", "./board_l512_results", "--extended-q31kv7-l512"], sw, env)
    assert rc == 0, tail
    assert "FULL VALIDATION STATUS: PASS" in out, tail


def test_benchmark_cycle_model_runs(sw_dir):
    sw, env = sw_dir
    for extra in ([], ["--seq-len", "128", "--non-causal"], ["--seq-len", "64", "--q-pos-base", "31",
                                                             "--kv-pos-base", "7"]):
        rc, out, tail = _run([sys.executable, "benchmark.py", *extra], sw, env)
        assert rc == 0, tail
        json.loads(out)
