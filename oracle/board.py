"""TEST INFRASTRUCTURE ONLY -- Python front end of the board-arithmetic oracle.

Compiles ``board_arith.c`` (plain C, ``gcc -O2``) into
``oracle/_build/libboard_oracle.so`` on first use, or when the source is newer
than the library, and exposes:

* ``attention_board(q, k, v, causal, q_pos_base, kv_pos_base)`` -- one
  transaction in the reference layout (q/o ``[Hq, L, 128]``, k/v
  ``[Hkv, L, 128]`` bf16 words), returning the bf16 words LARA's synthesized
  datapath produces (see ``board_arith.c`` for the RTL lines each step
  restates);
* the element-wise primitives (``fp32_add``, ``fp32_mul``, ``bf16_mul``,
  ``exp_lookup``, ``recip_lut_bits``) for the primitive tests.

Parity of the full transaction with the FPGA is unpinned (the reference ships
no board case files); the tables are pinned (``oracle/board_luts.py``).
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

from . import board_luts

HERE = Path(__file__).resolve().parent
SRC = HERE / "board_arith.c"
LIB = HERE / "_build" / "libboard_oracle.so"

_lib = None
_tables = None


def build(force: bool = False) -> Path:
    if force or not LIB.exists() or LIB.stat().st_mtime < SRC.stat().st_mtime:
        LIB.parent.mkdir(exist_ok=True)
        tmp = LIB.with_suffix(".so.tmp")
        subprocess.run(["gcc", "-O2", "-std=c11", "-fopenmp", "-fno-semantic-interposition", "-shared", "-fPIC", "-o", str(tmp),
                        str(SRC)], check=True)
        tmp.replace(LIB)
    return LIB


def _load():
    global _lib, _tables
    if _lib is None:
        lib = ctypes.CDLL(str(build()))
        P = ctypes.c_void_p
        for name in ("ob_fp32_add_n", "ob_fp32_mul_n", "ob_bf16_mul_n"):
            getattr(lib, name).argtypes = [P, P, P, ctypes.c_size_t]
        for name in ("ob_exp_lookup_n", "ob_recip_lut_n"):
            getattr(lib, name).argtypes = [P, P, ctypes.c_size_t, P]
        lib.ob_attention_board.argtypes = [P, P, P, P] + [ctypes.c_int] * 6 + [P, P]
        _tables = board_luts.load()
        _lib = lib
    return _lib


def tables() -> tuple[np.ndarray, np.ndarray]:
    _load()
    return _tables


def _u32(a) -> np.ndarray:
    a = np.asarray(a)
    if a.dtype == np.float32:
        a = a.view(np.uint32)
    return np.ascontiguousarray(a, dtype=np.uint32)


def _binary(name: str, a, b, dtype=np.uint32) -> np.ndarray:
    lib = _load()
    a = np.ascontiguousarray(a, dtype=dtype)
    b = np.ascontiguousarray(b, dtype=dtype)
    out = np.empty(a.shape, np.uint32)
    getattr(lib, name)(a.ctypes.data, b.ctypes.data, out.ctypes.data, a.size)
    return out


def fp32_add(a, b) -> np.ndarray:
    return _binary("ob_fp32_add_n", _u32(a), _u32(b))


def fp32_mul(a, b) -> np.ndarray:
    return _binary("ob_fp32_mul_n", _u32(a), _u32(b))


def bf16_mul(a, b) -> np.ndarray:
    return _binary("ob_bf16_mul_n", a, b, dtype=np.uint16)


def exp_lookup(x) -> np.ndarray:
    lib = _load()
    x = _u32(x)
    out = np.empty(x.shape, np.uint32)
    lib.ob_exp_lookup_n(x.ctypes.data, out.ctypes.data, x.size, _tables[0].ctypes.data)
    return out


def recip_lut_bits(x) -> np.ndarray:
    lib = _load()
    x = _u32(x)
    out = np.empty(x.shape, np.uint32)
    lib.ob_recip_lut_n(x.ctypes.data, out.ctypes.data, x.size, _tables[1].ctypes.data)
    return out


def attention_board(q, k, v, *, causal: bool = True, q_pos_base: int = 0, kv_pos_base: int = 0) -> np.ndarray:
    """Board-arithmetic attention; q ``[Hq, L, 128]``, k/v ``[Hkv, L, 128]`` uint16 -> o ``[Hq, L, 128]``."""
    lib = _load()
    q = np.ascontiguousarray(q, dtype=np.uint16)
    k = np.ascontiguousarray(k, dtype=np.uint16)
    v = np.ascontiguousarray(v, dtype=np.uint16)
    hq, L, d = q.shape
    hkv = k.shape[0]
    if d != 128 or k.shape != (hkv, L, d) or v.shape != k.shape or hq % hkv:
        raise ValueError("board arithmetic covers head_dim 128 with q [Hq,L,128], k/v [Hkv,L,128]")
    o = np.empty_like(q)
    lib.ob_attention_board(q.ctypes.data, k.ctypes.data, v.ctypes.data, o.ctypes.data, hq, hkv, L, int(causal),
                           int(q_pos_base), int(kv_pos_base), _tables[0].ctypes.data, _tables[1].ctypes.data)
    return o
