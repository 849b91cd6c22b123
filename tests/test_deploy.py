"""Deployment descriptors and the environment report (``lara_b200.deploy``).

The reference harnesses require a ``.bit/.hwh/.xsa`` trio
(sw/board_performance.py:634-639, sw/run_board_full_validation.py:245-256)
and a ``board_environment.json`` whose ``overall_status`` is PASS
(sw/run_board_full_validation.py:258-271).  CPU tests cover the descriptor
trio, the stale-build check and the FAIL report without a device; the GPU
test checks that a B200 passes the report, self-checks included.
"""

from __future__ import annotations

import json

import pytest

from lara_b200 import deploy


def test_descriptor_trio(tmp_path):
    bit, hwh, xsa = deploy.write_descriptors(tmp_path)
    assert [p.suffix for p in (bit, hwh, xsa)] == [".bit", ".hwh", ".xsa"]
    assert bit.name == "lara_attention.bit"
    doc = json.loads(bit.read_text())
    assert doc["kind"] == "bitstream" and len(doc["library_sha256"]) == 64 and doc["abi_version"] >= 1
    assert json.loads(hwh.read_text())["driver_defaults"]["head_dim"] == 128
    assert json.loads(xsa.read_text())["arch"] == "sm_100a"


def test_stale_and_missing_artifacts_are_issues(tmp_path):
    bit, hwh, _ = deploy.write_descriptors(tmp_path)
    doc = json.loads(bit.read_text())
    doc["library_sha256"] = "0" * 64
    bit.write_text(json.dumps(doc))
    hwh.unlink()
    issues: list[str] = []
    arts, manifest = deploy._check_artifacts(bit, issues)
    assert any("stale deployment" in i for i in issues)
    assert any("missing" in i and i.endswith(".hwh") for i in issues)
    assert arts["lara_attention.hwh"]["exists"] is False
    assert manifest[-1].endswith("liblara_b200.so")


def test_environment_cli_writes_reports(tmp_path, monkeypatch):
    torch = pytest.importorskip("torch")
    deploy.write_descriptors(tmp_path)
    env_json, env_txt, sha = tmp_path / "env.json", tmp_path / "env.txt", tmp_path / "sha.txt"
    rc = deploy.main(["environment", "--bitstream", str(tmp_path / "lara_attention.bit"),
                      "--environment-json", str(env_json), "--environment-output", str(env_txt),
                      "--hardware-sha256-output", str(sha)])
    rep = json.loads(env_json.read_text())
    assert rc == (0 if rep["overall_status"] == "PASS" else 1)
    assert env_txt.read_text().splitlines()[1] == f"overall_status: {rep['overall_status']}"
    assert len(sha.read_text().splitlines()) == 4
    if not torch.cuda.is_available():
        assert rep["overall_status"] == "FAIL"
        assert any("no CUDA device" in i for i in rep["issues"])


@pytest.mark.gpu
def test_environment_passes_on_b200(tmp_path):
    bit, _, _ = deploy.write_descriptors(tmp_path)
    rep = deploy.environment_report(bit, device=0)
    assert rep["issues"] == [] and rep["overall_status"] == "PASS"
    dev = rep["device"]
    assert dev["compute_capability"].startswith("10.") and dev["kernel_image_ok"]
    assert dev["self_checks"] == {"zero_transaction": True, "one_token_identity": True, "perf_valid": True}
