"""Deployment descriptors and the environment report for the LARA harnesses.

The reference deploys its FPGA image as a file trio -- ``.bit`` (bitstream),
``.hwh`` (hardware handoff) and ``.xsa`` (platform archive) -- that the
harnesses require and hash (sw/board_performance.py:634-639,
sw/run_board_full_validation.py:175-180,245-256).  Every full-validation run
is gated on ``board_environment.json`` with ``overall_status == "PASS"``
(sw/run_board_full_validation.py:258-271), which sw/clear_pynq_cache.py
writes after checking the board (cache state, device-tree overlay, ``xbutil
examine`` reporting a ready device; :147-339).

On B200 the deployed artefact is ``liblara_b200.so``:

* ``write_descriptors`` writes the trio as small JSON documents describing
  that library: the ``.bit`` pins the library's SHA-256 and ABI version, the
  ``.hwh`` lists the compiled kernel geometries and the driver's limits, the
  ``.xsa`` names the target architecture and build flags.
* ``environment_report`` replaces the board bring-up: the deployment files
  exist and the ``.bit`` matches the library now on disk (the analogue of the
  stale-PYNQ-cache check, sw/clear_pynq_cache.py:24-51), a CUDA device of
  compute capability 10.x is visible, the library's sm_100a image loads on it,
  and two self-checks pass through the driver: a zero transaction returns zero
  words (sw/board_test.py:45-79), and a one-token transaction returns each
  group's V row exactly (softmax over one key is 1, so O = V bit for bit).

Command line::

    python -m lara_b200.deploy descriptors --out DIR [--name lara_attention]
        [--arithmetic ieee|board]
    python -m lara_b200.deploy environment [--bitstream DIR/lara_attention.bit]
        [--environment-output board_environment.txt]
        [--environment-json board_environment.json]
        [--hardware-sha256-output deployed_hardware_sha256.txt]

``environment`` exits 0 only when the report's ``overall_status`` is PASS, as
sw/clear_pynq_cache.py:339 does.
"""

from __future__ import annotations

import argparse
import ctypes
import hashlib
import json
import os
import platform
import sys
from datetime import datetime, timezone
from pathlib import Path
from typing import Any

import numpy as np

SCHEMA_DEPLOY = "lara-b200-deployment-v1"
SCHEMA_ENV = "lara-b200-environment-v1"
DEFAULT_NAME = "lara_attention"  # sw/run_board_full_validation.py default --bitstream ./lara_attention.bit

# Kernel geometries compiled into the library (lara_b200/csrc/decode.cu,
# decode_tc.cu and prefill_tc.cu instantiate exactly these).
DECODE_HEAD_DIMS = (64, 128)
DECODE_GROUP_SIZES = (1, 2, 4, 8)
TENSOR_CORE_DECODE_GROUP_SIZES = (1, 2, 4, 8, 16)
TENSOR_CORE_HEAD_DIMS = (128,)


def _sha256(path: Path) -> str:
    digest = hashlib.sha256()
    with path.open("rb") as stream:
        for chunk in iter(lambda: stream.read(1 << 20), b""):
            digest.update(chunk)
    return digest.hexdigest()


def _library():
    from . import _native

    return _native


def descriptor_paths(bitstream: Path) -> tuple[Path, Path, Path]:
    return bitstream, bitstream.with_suffix(".hwh"), bitstream.with_suffix(".xsa")


def write_descriptors(out_dir: str | Path, name: str = DEFAULT_NAME, arithmetic: str = "ieee") -> tuple[Path, Path, Path]:
    """Write ``<name>.bit/.hwh/.xsa`` describing the built library; returns their paths.

    ``arithmetic`` ("ieee" or "board") is recorded in the ``.bit`` descriptor;
    an ``AttentionAccelerator`` opened with that descriptor as its
    ``bitstream_path`` computes ``run_attention`` in that arithmetic.
    """
    if arithmetic not in ("ieee", "board"):
        raise ValueError("arithmetic must be 'ieee' or 'board'")
    from . import attn_driver as drv
    from . import build as bld

    nat = _library()
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    lib_path = Path(nat.LIB_PATH)
    bit, hwh, xsa = descriptor_paths(out / f"{name}.bit")
    common = {"schema": SCHEMA_DEPLOY, "created_utc": datetime.now(timezone.utc).isoformat()}
    docs = {
        bit: {**common, "kind": "bitstream", "library": lib_path.name, "library_path": str(lib_path),
              "library_sha256": _sha256(lib_path), "library_size_bytes": lib_path.stat().st_size,
              "abi_version": int(nat.lib.lara_abi_version()), "arithmetic": arithmetic},
        hwh: {**common, "kind": "hardware_handoff",
              "decode_kernel": {"head_dims": list(DECODE_HEAD_DIMS), "group_sizes": list(DECODE_GROUP_SIZES)},
              "tensor_core_kernel": {"head_dims": list(TENSOR_CORE_HEAD_DIMS),
                                     "decode_group_sizes": list(TENSOR_CORE_DECODE_GROUP_SIZES)},
              "driver_defaults": {"n_q_heads": drv.N_Q_HEADS, "n_kv_heads": drv.N_KV_HEADS,
                                  "head_dim": drv.HEAD_DIM, "max_seq_len": drv.MAX_SEQ_LEN,
                                  "absolute_position_limit": drv.ABSOLUTE_POSITION_LIMIT,
                                  "clock_mhz": drv.DEVICE_CLOCK_MHZ}},
        xsa: {**common, "kind": "platform", "target": "NVIDIA B200", "arch": "sm_100a",
              "compute_capability": "10.0", "nvcc_flags": [*bld.ARCH_FLAGS, "-O3", "-lineinfo"],
              "cudart": "static"},
    }
    for path, doc in docs.items():
        path.write_text(json.dumps(doc, indent=2) + "\n", encoding="utf-8")
    return bit, hwh, xsa


def _check_artifacts(bitstream: Path, issues: list[str]) -> tuple[dict[str, Any], list[str]]:
    nat = _library()
    artifacts: dict[str, Any] = {}
    manifest: list[str] = []
    for path in descriptor_paths(bitstream):
        details: dict[str, Any] = {"path": str(path), "exists": path.is_file()}
        if path.is_file():
            details["size_bytes"] = path.stat().st_size
            details["sha256"] = _sha256(path)
            manifest.append(f"{details['sha256']}  {path}")
        else:
            issues.append(f"deployment artifact is missing: {path}")
        artifacts[path.name] = details
    if bitstream.is_file():
        try:
            doc = json.loads(bitstream.read_text(encoding="utf-8"))
        except (OSError, UnicodeError, json.JSONDecodeError) as exc:
            issues.append(f"{bitstream} is not a lara_b200 deployment descriptor: {exc}")
        else:
            lib_hash = _sha256(Path(nat.LIB_PATH))
            if doc.get("schema") != SCHEMA_DEPLOY or doc.get("kind") != "bitstream":
                issues.append(f"{bitstream} is not a lara_b200 bitstream descriptor")
            elif doc.get("library_sha256") != lib_hash:
                issues.append(f"{bitstream} describes a different build of {Path(nat.LIB_PATH).name} "
                              "(stale deployment; rerun `python -m lara_b200.deploy descriptors`)")
            if doc.get("abi_version") not in (None, int(nat.lib.lara_abi_version())):
                issues.append("descriptor ABI version differs from the loaded library")
    manifest.append(f"{_sha256(Path(nat.LIB_PATH))}  {nat.LIB_PATH}")
    return artifacts, manifest


def _self_checks(device: int, issues: list[str]) -> dict[str, Any]:
    """Zero transaction and one-token identity transaction through the driver."""
    from .attn_driver import (GQA_GROUP_SIZE, HEAD_DIM, N_KV_HEADS, N_Q_HEADS, AttentionAccelerator,
                              fp32_to_bf16_u16)

    out: dict[str, Any] = {}
    try:
        with AttentionAccelerator(device=device) as acc:
            z_q = np.zeros((N_Q_HEADS, 16, HEAD_DIM), np.uint16)
            z_kv = np.zeros((N_KV_HEADS, 16, HEAD_DIM), np.uint16)
            zero = acc.run_attention(z_q, z_kv, z_kv, seq_len=16)
            out["zero_transaction"] = bool(not np.any(zero))
            if not out["zero_transaction"]:
                issues.append("zero transaction returned non-zero words")
            rng = np.random.default_rng(0)
            q = rng.standard_normal((N_Q_HEADS, 1, HEAD_DIM)).astype(np.float32)
            k = rng.standard_normal((N_KV_HEADS, 1, HEAD_DIM)).astype(np.float32)
            v = rng.standard_normal((N_KV_HEADS, 1, HEAD_DIM)).astype(np.float32)
            o = acc.run_attention(q, k, v, seq_len=1)
            # head h reads group h // G (sw/board_performance.py:182-184)
            want = np.repeat(fp32_to_bf16_u16(v), GQA_GROUP_SIZE, axis=0)
            ident = bool(np.array_equal(o, want))
            out["one_token_identity"] = ident
            if not ident:
                issues.append("one-token transaction did not return the V rows")
            perf = acc.read_perf()
            out["perf_valid"] = bool(perf["cycles"] > 0 and 0 <= perf["mac_cycles"] <= perf["cycles"])
    except Exception as exc:  # the report records every failure instead of raising
        issues.append(f"driver self-check failed: {type(exc).__name__}: {exc}")
    return out


def environment_report(bitstream: str | Path | None = None, device: int | None = None) -> dict[str, Any]:
    """Collect the environment facts; ``overall_status`` is PASS when ``issues`` is empty."""
    issues: list[str] = []
    software: dict[str, Any] = {"python": sys.version.split()[0], "numpy": np.__version__}
    device_report: dict[str, Any] = {}
    artifacts: dict[str, Any] = {}
    manifest: list[str] = []
    try:
        nat = _library()
    except ImportError as exc:
        nat = None
        issues.append(f"liblara_b200.so cannot be loaded: {exc}")
    if nat is not None:
        software.update({"library": str(nat.LIB_PATH), "abi_version": int(nat.lib.lara_abi_version())})
        if bitstream is not None:
            artifacts, manifest = _check_artifacts(Path(bitstream).expanduser().resolve(), issues)
        else:
            issues.append("--bitstream was not provided; deployment artifacts were not verified")
        if device is None:
            device = int(os.environ.get("LARA_DEVICE", os.environ.get("LOCAL_RANK", "0")))
        count = ctypes.c_int(0)
        rc = nat.lib.lara_device_count(ctypes.byref(count))
        device_report["visible_devices"] = int(count.value)
        if rc != 0 or count.value == 0:
            issues.append(f"no CUDA device visible ({nat.last_error() or 'count is 0'})")
        else:
            info = nat.LaraDeviceInfo()
            rc = nat.lib.lara_device_query(int(device), ctypes.byref(info))
            if rc != 0:
                issues.append(f"device {device}: {nat.last_error()}")
            else:
                device_report.update({
                    "index": int(device), "name": info.name.decode(errors="replace"),
                    "pci_bus_id": info.pci_bus_id.decode(errors="replace"),
                    "compute_capability": f"{info.cc_major}.{info.cc_minor}", "sm_count": info.sm_count,
                    "total_mem_bytes": int(info.total_mem_bytes), "driver_version": info.driver_version,
                    "runtime_version": info.runtime_version, "kernel_image_ok": bool(info.kernel_image_ok)})
                if info.cc_major != 10:
                    issues.append(f"device {device} has compute capability {info.cc_major}.{info.cc_minor}; "
                                  "the library is built for sm_100a")
                elif not info.kernel_image_ok:
                    issues.append(f"the library's sm_100a image does not load on device {device}")
                else:
                    device_report["self_checks"] = _self_checks(int(device), issues)
    return {
        "schema": SCHEMA_ENV,
        "overall_status": "PASS" if not issues else "FAIL",
        "timestamp_utc": datetime.now(timezone.utc).isoformat(),
        "system": {"hostname": platform.node(), "platform": platform.platform(), "uname": list(platform.uname()),
                   "cpu_count": len(os.sched_getaffinity(0))},
        "software": software,
        "device": device_report,
        "deployment_artifacts": artifacts,
        "hardware_manifest": manifest,
        "issues": issues,
    }


def render_text(report: dict[str, Any]) -> str:
    dev = report["device"]
    lines = [
        "LARA B200 environment report",
        f"overall_status: {report['overall_status']}",
        f"timestamp_utc: {report['timestamp_utc']}",
        f"hostname: {report['system']['hostname']}",
        f"platform: {report['system']['platform']}",
        f"python: {report['software'].get('python')}",
        f"numpy: {report['software'].get('numpy')}",
        f"library: {report['software'].get('library')}",
        f"device: {dev.get('name')} ({dev.get('pci_bus_id')}, cc {dev.get('compute_capability')}, "
        f"{dev.get('sm_count')} SMs)",
        f"kernel_image_ok: {dev.get('kernel_image_ok')}",
        f"self_checks: {dev.get('self_checks')}",
        "",
        "deployment_artifacts:",
    ]
    for name, details in report["deployment_artifacts"].items():
        lines.append(f"  {name}: {details}")
    lines.extend(["", "issues:"])
    lines.extend([f"  - {issue}" for issue in report["issues"]] or ["  none"])
    return "\n".join(lines).rstrip() + "\n"


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="cmd", required=True)
    d = sub.add_parser("descriptors", help="write the .bit/.hwh/.xsa descriptor trio")
    d.add_argument("--out", type=Path, default=Path("."))
    d.add_argument("--name", default=DEFAULT_NAME)
    d.add_argument("--arithmetic", choices=("ieee", "board"), default="ieee",
                   help="run_attention arithmetic: IEEE fp32 (default) or the FPGA's output words bit for bit")
    e = sub.add_parser("environment", help="check the device and write board_environment.{txt,json}")
    e.add_argument("--bitstream", type=Path)
    e.add_argument("--device", type=int)
    e.add_argument("--environment-output", type=Path, default=Path("board_environment.txt"))
    e.add_argument("--environment-json", type=Path, default=Path("board_environment.json"))
    e.add_argument("--hardware-sha256-output", type=Path, default=Path("deployed_hardware_sha256.txt"))
    args = ap.parse_args(argv)
    if args.cmd == "descriptors":
        for p in write_descriptors(args.out, args.name, args.arithmetic):
            print(p)
        return 0
    report = environment_report(args.bitstream, args.device)
    text = render_text(report)
    args.environment_output.write_text(text, encoding="utf-8")
    args.environment_json.write_text(json.dumps(report, indent=2) + "\n", encoding="utf-8")
    manifest = report["hardware_manifest"]
    args.hardware_sha256_output.write_text("\n".join(manifest) + ("\n" if manifest else ""), encoding="utf-8")
    print(text, end="")
    return 0 if report["overall_status"] == "PASS" else 1


if __name__ == "__main__":
    raise SystemExit(main())
