#!/usr/bin/env python3
"""Generate the golden fixtures that pin the CPU oracle to the LARA reference.

Run where the LARA sources are available (the ``--reference`` flag names
the source tree).  The script imports the reference's own Python code and
records its outputs:

* ``sw/attn_driver.py:88-103`` ``fp32_to_bf16_u16`` / ``bf16_u16_to_fp32`` on a
  known-answer set of fp32 bit patterns (ties, carries, subnormals, inf, NaN)
  and on all 65536 bf16 words;
* ``sw/board_performance.py:158-192`` ``cpu_attention_numpy`` on the board case
  matrix (L in {1,16,32,64,128} x causal/non-causal x position bases (3,3) and
  (31,7), plus L=512 causal at (31,7)) with seeded N(0,1)*0.5 inputs;
* the same function with its module geometry set to the decode config (8 Q
  heads, 2 KV heads, head_dim 64) to give the single decode step over 512
  cached + 1 appended tokens (seed 0, N(0,1));
* ``sw/board_performance.py:222-227`` ``_valid_pairs`` and
  ``sw/benchmark.py:36-57`` ``tile_pairs_per_head`` on a grid of workloads.

Inputs are regenerated from their seed by the tests; each fixture stores the
SHA-256 of the input words so a change in NumPy's generator stream is caught.
Outputs are stored in full for small cases, and as SHA-256 digests plus
sampled query rows for the larger ones, to keep the fixtures small.
"""

from __future__ import annotations

import argparse
import os
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def board_inputs(seed: int, L: int, pack):
    """Seeded board-shaped inputs: q[32,L,128], k/v[8,L,128] bf16 words."""
    rng = np.random.default_rng(seed)
    q = pack(rng.standard_normal((32, L, 128), dtype=np.float32) * np.float32(0.5))
    k = pack(rng.standard_normal((8, L, 128), dtype=np.float32) * np.float32(0.5))
    v = pack(rng.standard_normal((8, L, 128), dtype=np.float32) * np.float32(0.5))
    return q, k, v


def decode_cfg1_inputs(pack):
    """Config 1: B=1, 8 Q heads, 2 KV heads, D=64, 512 cached + 1 appended; seed 0, N(0,1)."""
    rng = np.random.default_rng(0)
    q = pack(rng.standard_normal((1, 8, 64), dtype=np.float32))
    k_cache = pack(rng.standard_normal((1, 2, 512, 64), dtype=np.float32))
    v_cache = pack(rng.standard_normal((1, 2, 512, 64), dtype=np.float32))
    k_new = pack(rng.standard_normal((1, 2, 64), dtype=np.float32))
    v_new = pack(rng.standard_normal((1, 2, 64), dtype=np.float32))
    return q, k_cache, v_cache, k_new, v_new


BOARD_CASES = [(L, causal, qb, kb) for (qb, kb) in ((3, 3), (31, 7))
               for L in (1, 16, 32, 64, 128) for causal in (True, False)] + [(512, True, 31, 7)]


def case_seed(L, causal, qb, kb) -> int:
    return 1000 + L * 10 + (1 if causal else 0) + (100000 if qb == 31 else 0)


def sample_rows(L: int) -> np.ndarray:
    return np.unique(np.array([0, L // 2, L - 1]))


def kat_bits() -> np.ndarray:
    """fp32 bit patterns that exercise every branch of the RNE pack."""
    pats = [0x00000000, 0x80000000, 0x3F800000, 0xBF800000, 0x7F7FFFFF, 0xFF7FFFFF,
            0x7F800000, 0xFF800000, 0x7FC00000, 0xFFC00000, 0x7F800001, 0x7FFFFFFF,
            0x00000001, 0x007FFFFF, 0x00800000, 0x0000FFFF, 0x00008000, 0x00018000,
            0x3F808000, 0x3F818000, 0x3F808001, 0x3F807FFF, 0x3F80FFFF, 0x7F7F8000,
            0x7F7F7FFF, 0x7F7FC000, 0xC0490FDB, 0x3DB504F3]
    rng = np.random.default_rng(7)
    rnd = rng.integers(0, 2**32, size=4096, dtype=np.uint64).astype(np.uint32)
    # force a slice of random words onto exact ties
    rnd[:512] = (rnd[:512] & np.uint32(0xFFFF0000)) | np.uint32(0x8000)
    return np.concatenate([np.array(pats, dtype=np.uint32), rnd])


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", default=os.environ.get("LARA_REFERENCE"),
                    help="LARA source tree (default: $LARA_REFERENCE)")
    ap.add_argument("--out", default=str(HERE))
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set LARA_REFERENCE to the LARA source tree")
    sw = Path(args.reference) / "sw"
    sys.path.insert(0, str(sw))
    import attn_driver as ref_driver  # noqa: E402  (reference code, read-only)
    import benchmark as ref_bench  # noqa: E402
    import board_performance as ref_perf  # noqa: E402

    out = Path(args.out)
    out.mkdir(parents=True, exist_ok=True)
    pack = ref_driver.fp32_to_bf16_u16

    # --- a1: bf16 pack/unpack known answers --------------------------------
    bits = kat_bits()
    packed = ref_driver.fp32_to_bf16_u16(bits.view(np.float32))
    all_words = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    unpacked = ref_driver.bf16_u16_to_fp32(all_words)
    np.savez_compressed(out / "kat_bf16.npz", fp32_bits=bits, bf16_words=packed,
                        unpack_sha256=np.array(sha(unpacked.view(np.uint32))))

    # --- a13 / harness counts ------------------------------------------------
    counts = []
    for L in (1, 2, 15, 16, 17, 31, 32, 33, 63, 64, 65, 128, 200, 511, 512):
        for causal in (True, False):
            for qb, kb in ((0, 0), (3, 3), (31, 7), (7, 31), (0, 100)):
                Case = ref_perf.BoardCase
                case = Case("x", Path("."), None, None, None, None, L, causal, qb, kb)
                counts.append({
                    "L": L, "causal": causal, "q_pos_base": qb, "kv_pos_base": kb,
                    "valid_pairs": int(ref_perf._valid_pairs(case)),
                    "tile_pairs_per_head": int(ref_bench.tile_pairs_per_head(L, causal, qb, kb)),
                })
    (out / "counts.json").write_text(json.dumps(counts, indent=1) + "\n")

    # --- a3-a12: board-geometry attention (32/8/128) -------------------------
    manifest = []
    for (L, causal, qb, kb) in BOARD_CASES:
        seed = case_seed(L, causal, qb, kb)
        q, k, v = board_inputs(seed, L, pack)
        o = ref_perf.cpu_attention_numpy(q, k, v, causal=causal, q_pos_base=qb, kv_pos_base=kb)
        rows = sample_rows(L)
        name = f"board_L{L}_{'causal' if causal else 'noncausal'}_q{qb}_kv{kb}"
        np.savez_compressed(
            out / f"{name}.npz", seed=seed, seq_len=L, causal=int(causal), q_pos_base=qb,
            kv_pos_base=kb, rows=rows, o_rows=o[:, rows, :],
            input_sha256=np.array(sha(q) + sha(k) + sha(v)),
            o_sha256=np.array(sha(o)), o_bf16_sha256=np.array(sha(pack(o))))
        manifest.append(name)

    # --- config 1: golden single decode step ---------------------------------
    q, kc, vc, kn, vn = decode_cfg1_inputs(pack)
    k_all = np.concatenate([kc, kn[:, :, None, :]], axis=2)  # [1,2,513,64]
    v_all = np.concatenate([vc, vn[:, :, None, :]], axis=2)
    saved = (ref_perf.N_Q_HEADS, ref_perf.N_KV_HEADS, ref_perf.HEAD_DIM, ref_perf.GQA_GROUP_SIZE)
    ref_perf.N_Q_HEADS, ref_perf.N_KV_HEADS, ref_perf.HEAD_DIM, ref_perf.GQA_GROUP_SIZE = 8, 2, 64, 4
    try:
        n = k_all.shape[2]
        # The reference needs Lq == Lkv; every query row is the decode query,
        # non-causal, so each row attends to all 513 tokens.
        q_rows = np.repeat(q[0][:, None, :], n, axis=1)
        o_full = ref_perf.cpu_attention_numpy(q_rows, k_all[0], v_all[0], causal=False,
                                              q_pos_base=0, kv_pos_base=0)
        # causal prefill of the same 513 tokens (rows differ per position)
        rng = np.random.default_rng(10)
        q_pref = pack(rng.standard_normal((8, n, 64), dtype=np.float32))
        o_pref = ref_perf.cpu_attention_numpy(q_pref, k_all[0], v_all[0], causal=True,
                                              q_pos_base=0, kv_pos_base=0)
    finally:
        ref_perf.N_Q_HEADS, ref_perf.N_KV_HEADS, ref_perf.HEAD_DIM, ref_perf.GQA_GROUP_SIZE = saved
    np.savez_compressed(out / "decode_cfg1.npz", q=q, k_cache=kc, v_cache=vc, k_new=kn, v_new=vn,
                        o_fp32=o_full[:, 0, :][None], o_bf16=pack(o_full[:, 0, :][None]),
                        prefill_seed=10, o_prefill_rows=o_pref[:, sample_rows(n), :],
                        prefill_rows=sample_rows(n), o_prefill_sha256=np.array(sha(o_pref)))
    manifest.append("decode_cfg1")
    (out / "MANIFEST.json").write_text(json.dumps({
        "generator": "tests/golden/make_golden.py",
        "reference_functions": [
            "sw/attn_driver.py:88-98 fp32_to_bf16_u16", "sw/attn_driver.py:101-103 bf16_u16_to_fp32",
            "sw/board_performance.py:158-192 cpu_attention_numpy",
            "sw/board_performance.py:222-227 _valid_pairs", "sw/benchmark.py:36-57 tile_pairs_per_head"],
        "numpy": np.__version__,
        "cases": manifest}, indent=1) + "\n")
    print(f"wrote {len(manifest)} attention fixtures + kat_bf16 + counts to {out}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
