"""On-disk KV-cache format ``lara-kv-v1`` (save / restore of a device cache).

The reference's cache lives in FPGA BRAM for one transaction
(hw/rtl/mem/kv_cache_ram.sv) and has no persistent form; a B200 serving
process keeps long caches resident in HBM and needs to checkpoint them.  A
``lara-kv-v1`` file is an uncompressed NumPy ``.npz`` archive with:

* ``format``  : the string ``"lara-kv-v1"``;
* ``lens``    : int32 ``[B]`` -- tokens held per sequence;
* ``k``, ``v``: uint16 (bf16 words) ``[B, Hkv, T, D]`` with ``T >= max(lens)``;
  rows past ``lens[b]`` carry no meaning;
* ``sha256``  : hex digest of ``lens``, ``k`` and ``v`` bytes (checked on load).

Both :class:`lara_b200.attn_driver.AttentionAccelerator` (``save_kv`` /
``restore_kv``) and :class:`lara_b200.paged.PagedKVCache` (``save`` / ``load``)
read and write it, so a cache can move between the contiguous and the paged
layout.
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np

FORMAT = "lara-kv-v1"


def _digest(lens: np.ndarray, k: np.ndarray, v: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in (lens, k, v):
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def save(path, k: np.ndarray, v: np.ndarray, lens: np.ndarray) -> Path:
    k = np.ascontiguousarray(k, dtype=np.uint16)
    v = np.ascontiguousarray(v, dtype=np.uint16)
    lens = np.ascontiguousarray(lens, dtype=np.int32)
    if k.ndim != 4 or v.shape != k.shape or lens.shape != (k.shape[0],):
        raise ValueError("expected k/v [B, Hkv, T, D] and lens [B]")
    if lens.size and (lens.min() < 0 or lens.max() > k.shape[2]):
        raise ValueError("lengths must lie in [0, T]")
    path = Path(path)
    with path.open("wb") as f:
        np.savez(f, format=np.array(FORMAT), lens=lens, k=k, v=v, sha256=np.array(_digest(lens, k, v)))
    return path


def load(path) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """-> (k, v, lens) after checking the format tag and the digest."""
    with np.load(Path(path), allow_pickle=False) as z:
        if str(z["format"]) != FORMAT:
            raise ValueError(f"{path}: not a {FORMAT} file")
        lens, k, v = z["lens"].astype(np.int32), z["k"].astype(np.uint16), z["v"].astype(np.uint16)
        if _digest(lens, k, v) != str(z["sha256"]):
            raise ValueError(f"{path}: checksum mismatch")
    return k, v, lens
