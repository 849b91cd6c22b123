"""Stage LARA's own harness scripts, unmodified, for the harness GPU test.

The reference's host harnesses (``sw/board_test.py``, ``sw/board_matrix.py``,
``sw/board_performance.py``, ``sw/benchmark.py``,
``sw/run_board_full_validation.py``) are the acceptance test of the drop-in
boundary: they must run unchanged against this library's ``attn_driver``
shim.  Their sources are not part of this repository.  This script copies them
from a LARA source tree into ``baseline/_ref/sw/`` -- the reference's install
location, which git ignores and which travels to the GPU box with the rest of
the working tree -- and refuses any file whose SHA-256 differs from
``SHA256SUMS`` beside this script (the digests of the reference revision the
shim was written against).

Usage: ``python tests/ref_harness/stage.py [--reference DIR]`` (default:
``$LARA_REFERENCE``).  ``tests/test_zy_reference_harness.py`` checks the same
digests again before it runs anything.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
STAGE = ROOT / "baseline" / "_ref" / "sw"


def expected_digests() -> dict[str, str]:
    out = {}
    for line in (HERE / "SHA256SUMS").read_text().splitlines():
        if line.strip():
            digest, name = line.split()
            out[name] = digest
    return out


def sha256(path: Path) -> str:
    return hashlib.sha256(path.read_bytes()).hexdigest()


def staged_ok(stage: Path = STAGE) -> tuple[bool, str]:
    """(True, "") when every harness script is staged with its pinned digest."""
    for name, digest in expected_digests().items():
        p = stage / name
        if not p.is_file():
            return False, f"{p} is missing (run tests/ref_harness/stage.py with LARA_REFERENCE set)"
        if sha256(p) != digest:
            return False, f"{p} differs from the pinned reference revision"
    return True, ""


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--reference", default=os.environ.get("LARA_REFERENCE"), help="LARA source tree")
    args = ap.parse_args(argv)
    if not args.reference:
        ap.error("give --reference or set LARA_REFERENCE to the LARA source tree")
    src = Path(args.reference) / "sw"
    STAGE.mkdir(parents=True, exist_ok=True)
    for name, digest in expected_digests().items():
        got = sha256(src / name)
        if got != digest:
            print(f"{src / name}: SHA-256 {got} differs from the pinned {digest}", file=sys.stderr)
            return 1
        shutil.copyfile(src / name, STAGE / name)
    ok, why = staged_ok()
    if not ok:
        print(why, file=sys.stderr)
        return 1
    print(f"staged {len(expected_digests())} harness scripts in {STAGE}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
