"""ctypes binding of liblara_b200.so (the C ABI in include/lara_b200.h).

The library is loaded from this package directory; there is no fallback.  If
it is missing or cannot be loaded the import fails loudly, so no caller can
silently run a CPU path.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_size_t, c_uint16, c_uint64, c_void_p, c_double
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "liblara_b200.so"

# status codes (include/lara_b200.h; 0x00-0x12 mirror sw/attn_driver.py:80-85)
LARA_OK = 0x00
LARA_ERR_BAD_CFG = 0x01
LARA_ERR_BUSY_START = 0x02
LARA_ERR_STREAM_LEN = 0x10
LARA_ERR_STREAM_DEST = 0x11
LARA_ERR_RESULT_LEN = 0x12
LARA_ERR_CUDA = 0x20
LARA_ERR_TIMEOUT = 0x21
LARA_ERR_UNSUPPORTED = 0x22
LARA_ERR_DEVICE = 0x23

LARA_ARITH_IEEE = 0
LARA_ARITH_BOARD = 1
LARA_DECODE_KERNEL_CUDA_CORE = 0
LARA_DECODE_KERNEL_TENSOR = 1


class LaraError(RuntimeError):
    """A device-side or CUDA failure reported by liblara_b200.so."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{message} [status 0x{code:02x}]")
        self.code = code


class LaraConfigError(ValueError):
    """A shape, length or geometry rejected before launch (ERR_BAD_CFG / STREAM_*)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{message} [status 0x{code:02x}]")
        self.code = code


class LaraTimeout(TimeoutError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{message} [status 0x{code:02x}]")
        self.code = code


class LaraPerf(ctypes.Structure):
    _fields_ = [("cycles", c_uint64), ("mac_cycles", c_uint64), ("stall_cycles", c_uint64),
                ("clock_mhz", c_double)]


class LaraDeviceInfo(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 256), ("pci_bus_id", ctypes.c_char * 32), ("cc_major", c_int),
                ("cc_minor", c_int), ("sm_count", c_int), ("kernel_image_ok", c_int), ("driver_version", c_int),
                ("runtime_version", c_int), ("total_mem_bytes", ctypes.c_ulonglong)]


_I32P = POINTER(ctypes.c_int32)
_U16P = POINTER(c_uint16)

# name -> (restype, argtypes); every symbol include/lara_b200.h declares
SIGNATURES = {
    "lara_abi_version": (c_int, []),
    "lara_last_error_string": (c_char_p, []),
    "lara_status_name": (c_char_p, [c_int]),
    "lara_device_count": (c_int, [POINTER(c_int)]),
    "lara_selftest_wait_timeout": (c_int, [c_void_p, c_int, c_void_p]),
    "lara_device_query": (c_int, [c_int, POINTER(LaraDeviceInfo)]),
    "lara_decode_plan": (c_int, [c_int, c_int, c_int, c_int, c_int, c_void_p, POINTER(c_int), POINTER(c_int)]),
    "lara_decode_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "lara_decode_kernel": (c_int, [c_int, c_int, c_int]),
    "lara_workspace_init": (c_int, [c_void_p, c_size_t, c_void_p]),
    "lara_workspace_status": (c_int, [c_void_p, c_void_p, POINTER(c_int)]),
    "lara_gqa_decode": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                c_int, c_float, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "lara_gqa_decode_partial": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                        c_int, c_int, c_int, c_float, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "lara_gqa_decode_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                        c_int, c_int, c_float, c_int, c_int, c_void_p]),
    "lara_lse_combine": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "lara_lse_combine_strided": (c_int, [c_void_p, ctypes.c_longlong, c_void_p, ctypes.c_longlong, c_int, c_int,
                                         c_int, c_void_p, c_void_p]),
    "lara_kv_append": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                               c_void_p, c_void_p]),
    "lara_pack_bf16": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "lara_prefill_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "lara_gqa_prefill": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                 c_int, c_int, c_int, c_float, c_void_p, c_size_t, c_void_p]),
    "lara_dense_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int]),
    "lara_attention_dense": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                                     c_int, c_int, c_float, c_void_p, c_size_t, c_void_p]),
    "lara_attention_dense_board": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                           c_int, c_int, c_int, c_void_p]),
    "lara_gqa_decode_paged": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                      c_int, c_int, c_int, c_int, c_int, c_float, c_int, c_int, c_void_p, c_size_t,
                                      c_void_p]),
    "lara_kv_append_paged": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                     c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "lara_layer_prologue_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "lara_layer_prologue": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                    c_int, c_int, c_int, c_int, c_int, c_float, c_float, c_void_p, c_size_t,
                                    c_void_p]),
    "lara_create": (c_int, [c_int, POINTER(c_void_p)]),
    "lara_destroy": (c_int, [c_void_p]),
    "lara_configure_heads": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int]),
    "lara_configure": (c_int, [c_void_p, c_int, c_int, c_int, c_int]),
    "lara_kv_load": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int]),
    "lara_kv_append_ctx": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int]),
    "lara_run_prefill_chunk": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int]),
    "lara_get_seq_lens": (c_int, [c_void_p, c_void_p]),
    "lara_kv_truncate": (c_int, [c_void_p, c_void_p]),
    "lara_kv_read": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int]),
    "lara_run_query": (c_int, [c_void_p, c_void_p, c_void_p, c_int]),
    "lara_run_attention": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int]),
    "lara_read_perf": (c_int, [c_void_p, POINTER(LaraPerf)]),
    "lara_run_layer": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_float, c_float, c_int]),
    "lara_read_layer_perf": (c_int, [c_void_p, POINTER(c_uint64), POINTER(c_uint64)]),
    "lara_sync": (c_int, [c_void_p, c_int]),
    "lara_decode": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    "lara_prefill": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "lara_ctx_device": (c_int, [c_void_p]),
    "lara_ctx_selftest_timeout": (c_int, [c_void_p, c_int]),
    "lara_set_arithmetic": (c_int, [c_void_p, c_int]),
    "lara_get_arithmetic": (c_int, [c_void_p]),
}


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is not built; run `python -m lara_b200.build` (or __graft_entry__.build()). "
            "lara_b200 has no CPU fallback.")
    lib = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | ctypes.RTLD_LOCAL)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def last_error() -> str:
    msg = lib.lara_last_error_string()
    return msg.decode() if msg else ""


def check(rc: int, what: str = "") -> None:
    """Raise the Python exception matching a C-ABI status code.

    ValueError for configuration/shape errors (as the reference driver raises
    at sw/attn_driver.py:347-349,366-372,486-490), TimeoutError for timeouts
    (:453-454), RuntimeError for device errors (:446-448).
    """
    if rc == LARA_OK:
        return
    msg = f"{what}: {last_error()}" if what else last_error()
    if rc in (LARA_ERR_BAD_CFG, LARA_ERR_STREAM_LEN, LARA_ERR_STREAM_DEST, LARA_ERR_RESULT_LEN,
              LARA_ERR_UNSUPPORTED):
        raise LaraConfigError(rc, msg)
    if rc == LARA_ERR_TIMEOUT:
        raise LaraTimeout(rc, msg)
    raise LaraError(rc, msg)
