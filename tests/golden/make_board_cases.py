"""Generate board case files (``case_*.npz``) for LARA's board harnesses.

``sw/board_matrix.py``, ``sw/board_performance.py`` and
``sw/run_board_full_validation.py`` read case directories of ``case_*.npz``
files with the keys ``q_heads`` (uint16 ``[32, L, 128]``), ``k_heads`` /
``v_heads`` (uint16 ``[8, L, 128]``), ``expected_o`` (uint16 ``[32, L, 128]``)
and the scalars ``seq_len``, ``causal``, ``q_pos_base``, ``kv_pos_base``
(sw/board_performance.py:99-116); one case per (L, causal) per directory
(:119-156).  The reference's generator and its case directories are not in
the repository, so this script writes them:

* the two case sets the harnesses name (sw/run_board_full_validation.py:20-24):
  ``board_cases_rtl_contract_v2.6_fixed`` (label q3kv3: q_pos_base = kv_pos_base
  = 3) and ``board_cases_rtl_contract_v2.6_q31_kv7`` (q_pos_base 31,
  kv_pos_base 7);
* L in (1, 16, 32, 64, 128), causal and non-causal (REQUIRED_LENGTHS x
  REQUIRED_MODES, sw/board_performance.py:47-48), plus the L = 512 causal
  case of the q31kv7 set (``--extended-q31kv7-l512``,
  sw/run_board_full_validation.py:229-234) unless ``--no-extended``;
* inputs: bf16 (round to nearest even) of N(0, 1) * 0.5, NumPy
  ``default_rng`` seeded per (set, L, causal);
* ``expected_o``: the board-arithmetic oracle (``oracle/board_arith.c``), i.e.
  the words the FPGA datapath produces, so ``board_matrix.py``'s bit-for-bit
  comparison holds for a backend that runs board arithmetic.

Usage: ``python tests/golden/make_board_cases.py --out DIR [--sets q3kv3 q31kv7]
[--lengths 1 16 ...] [--no-extended]``; directories are created under DIR.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402
from oracle import board  # noqa: E402

CASE_SETS = {  # label -> (directory, q_pos_base, kv_pos_base)
    "q3kv3": ("board_cases_rtl_contract_v2.6_fixed", 3, 3),
    "q31kv7": ("board_cases_rtl_contract_v2.6_q31_kv7", 31, 7),
}
LENGTHS = (1, 16, 32, 64, 128)
EXTENDED = ("q31kv7", 512)
N_Q_HEADS, N_KV_HEADS, HEAD_DIM = 32, 8, 128


def case_seed(label: str, L: int, causal: bool) -> int:
    return 7_000_000 + 10_000 * list(CASE_SETS).index(label) + 2 * L + (1 if causal else 0)


def case_inputs(label: str, L: int, causal: bool) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    rng = np.random.default_rng(case_seed(label, L, causal))
    q = rng.standard_normal((N_Q_HEADS, L, HEAD_DIM)).astype(np.float32) * 0.5
    k = rng.standard_normal((N_KV_HEADS, L, HEAD_DIM)).astype(np.float32) * 0.5
    v = rng.standard_normal((N_KV_HEADS, L, HEAD_DIM)).astype(np.float32) * 0.5
    return tuple(oracle.fp32_to_bf16_u16(a) for a in (q, k, v))


def case_name(L: int, causal: bool) -> str:
    return f"case_L{L:03d}_{'causal' if causal else 'noncausal'}.npz"


def write_case(directory: Path, label: str, L: int, causal: bool) -> Path:
    _, qb, kb = CASE_SETS[label]
    q, k, v = case_inputs(label, L, causal)
    expected = board.attention_board(q, k, v, causal=causal, q_pos_base=qb, kv_pos_base=kb)
    path = directory / case_name(L, causal)
    np.savez(path, q_heads=q, k_heads=k, v_heads=v, expected_o=expected, seq_len=np.int64(L),
             causal=np.int64(int(causal)), q_pos_base=np.int64(qb), kv_pos_base=np.int64(kb))
    return path


def generate(out: Path, sets=tuple(CASE_SETS), lengths=LENGTHS, extended: bool = True) -> list[Path]:
    paths = []
    for label in sets:
        directory = out / CASE_SETS[label][0]
        directory.mkdir(parents=True, exist_ok=True)
        for L in lengths:
            for causal in (True, False):
                paths.append(write_case(directory, label, L, causal))
        if extended and label == EXTENDED[0]:
            paths.append(write_case(directory, label, EXTENDED[1], True))
    return paths


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--out", type=Path, default=Path("."))
    ap.add_argument("--sets", nargs="+", choices=tuple(CASE_SETS), default=list(CASE_SETS))
    ap.add_argument("--lengths", nargs="+", type=int, default=list(LENGTHS))
    ap.add_argument("--no-extended", action="store_true", help="skip the q31kv7 L=512 causal case")
    args = ap.parse_args()
    for p in generate(args.out, args.sets, args.lengths, not args.no_extended):
        print(p)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
