"""TEST INFRASTRUCTURE ONLY -- lookup tables of the board-arithmetic oracle.

LARA's softmax evaluates exp with a 1024-entry fp32 table over [-8, 0]
(hw/rtl/core/softmax_engine.sv:570-705, hw/rtl/pkg/attn_pkg.sv:230-235) and
the output buffer normalises with a 256-entry reciprocal-mantissa table
(hw/rtl/mem/output_buffer.sv:192-224).  The tables ship as
``hw/data/exp_lut.hex`` and ``hw/data/recip_lut.hex``; this module rebuilds
them from their definitions (it does not read those files):

* ``exp_lut[i]  = float32 exp(float32(-8 + 8 i / 1023))`` with NumPy's float32
  ``exp`` as evaluated on AVX-512 x86 hosts (it is within 2 ulp of the
  correctly rounded value, and the reference table carries exactly those
  roundings);
* ``recip_lut[i] = round(2^23 * (2 / (1 + (2 i + 1) / 512) - 1))``: the
  mantissa of 2 / (1 + f) at the midpoint of bucket ``i`` of the top eight
  fraction bits (exact integer arithmetic; no ties can occur).

``python -m oracle.board_luts`` regenerates ``board_luts.npz`` and refuses to
write a table whose SHA-256 differs from the pinned digest of the reference
table (the digests below are of the reference files' words as little-endian
uint32; ``tests/test_board_oracle.py`` also compares against the hex files
directly whenever the reference tree is present).
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
NPZ = HERE / "board_luts.npz"

EXP_LUT_SHA256 = "5bb7b38e5c092f53f1e1cda7882f187acbd98d17bfed640558007409d2258d86"
RECIP_LUT_SHA256 = "ece13472fc6fcee75ee95ac9448006705883957a68170311fc76cc3440214498"


def sha256_words(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a, dtype="<u4").tobytes()).hexdigest()


def make_exp_lut() -> np.ndarray:
    x = np.array([-8.0 + 8.0 * i / 1023.0 for i in range(1024)], dtype=np.float64).astype(np.float32)
    return np.exp(x).view(np.uint32).astype("<u4")


def make_recip_lut() -> np.ndarray:
    # 2^23 * (511 - 2i) / (513 + 2i), rounded to nearest (odd denominator: no ties)
    out = [((1 << 24) * (511 - 2 * i) + (513 + 2 * i)) // (2 * (513 + 2 * i)) for i in range(256)]
    return np.array(out, dtype="<u4")


def load() -> tuple[np.ndarray, np.ndarray]:
    """(exp_lut[1024], recip_lut[256]) as uint32, checked against the pinned digests."""
    with np.load(NPZ) as z:
        e, r = z["exp_lut"].astype("<u4"), z["recip_lut"].astype("<u4")
    if sha256_words(e) != EXP_LUT_SHA256 or sha256_words(r) != RECIP_LUT_SHA256:
        raise RuntimeError(f"{NPZ} does not hold the pinned board tables")
    return e, r


def main() -> int:
    e, r = make_exp_lut(), make_recip_lut()
    if sha256_words(r) != RECIP_LUT_SHA256:
        raise SystemExit("reciprocal table does not match the pinned digest")
    if sha256_words(e) != EXP_LUT_SHA256:
        raise SystemExit("this host's NumPy float32 exp does not reproduce the pinned exp table "
                         "(regenerate on an AVX-512 x86 host)")
    np.savez(NPZ, exp_lut=e, recip_lut=r)
    print(NPZ)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
