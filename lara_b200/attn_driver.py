"""B200 drop-in for LARA's host driver (``sw/attn_driver.py``).

The reference driver programs a KV260 overlay and services its load requests
over MMIO/DMA while one attention transaction runs.  This module keeps the
same call surface -- module constants, ``fp32_to_bf16_u16`` /
``bf16_u16_to_fp32``, ``TensorByteCounts``, ``RunProfile`` and
``AttentionAccelerator`` with ``configure``/``run_attention``/``read_perf``/
``last_profile``/``save_last_profile``/``close`` -- so ``board_test.py``,
``board_matrix.py``, ``board_performance.py`` and
``run_board_full_validation.py`` drive it unchanged.  Behind it is
``liblara_b200.so``: a C-ABI context that owns the HBM-resident KV cache and
runs hand-written sm_100a kernels.  There is no CPU fallback; constructing an
``AttentionAccelerator`` without a B200 raises.

Extensions (the north-star surface): ``configure_heads``, ``load_kv``,
``append_kv``, ``run_query`` (decode), ``run_prefill_chunk``, ``read_output``;
beyond it ``truncate_kv`` (rewind lengths), ``save_kv`` / ``restore_kv``.

Arithmetic of ``run_attention``: ``"ieee"`` (default; fp32 with a true exp,
within 2 bf16 ulp of the reference's CPU golden model) or ``"board"`` (the
FPGA datapath's output words bit for bit, the contract of the board case
files' ``expected_o``).  It is chosen by the ``arithmetic`` argument, else
the ``LARA_ARITHMETIC`` environment variable, else the ``"arithmetic"`` field
of the deployment descriptor named by ``bitstream_path`` (written by
``python -m lara_b200.deploy descriptors --arithmetic board``), so the
reference harnesses select it without code changes.

Timing: ``read_perf`` reports device time from CUDA events in nanoseconds,
and ``last_profile.clock_mhz`` is 1000.0, so the harnesses' cycles/(clock*1000)
conversion yields milliseconds (sw/board_performance.py:345-378).
"""

from __future__ import annotations

import ctypes
import hashlib
import json
import os
import subprocess
import time
from dataclasses import asdict, dataclass
from datetime import datetime, timezone
from pathlib import Path
from typing import Any

import numpy as np

from ._native import LARA_ARITH_BOARD, LARA_ARITH_IEEE, LaraPerf, check, lib

# CSR map and status bits of the reference (sw/attn_driver.py:33-61); kept so
# code that imports them keeps working.  The B200 status word uses the same
# START_READY / BUSY / DONE / ERROR bits.
CSR_CTRL = 0x000
CSR_STATUS = 0x004
CSR_SEQ_LEN = 0x008
CSR_Q_POS_BASE = 0x00C
CSR_KV_POS_BASE = 0x010
CSR_CFG = 0x014
CSR_ERROR_CODE = 0x018
CSR_LOAD_REQ = 0x01C
CSR_STREAM_LEN = 0x028
CSR_STREAM_DEST = 0x02C
CSR_RESULT_LEN = 0x058
CSR_PERF_CYCLES = 0x100
CSR_PERF_MAC_CYCLES = 0x108
CSR_PERF_STALLS = 0x10C

CTRL_START = 1 << 0
CTRL_CLEAR_STATUS = 1 << 1
STATUS_START_READY = 1 << 0
STATUS_BUSY = 1 << 1
STATUS_DONE = 1 << 2
STATUS_ERROR = 1 << 3
STATUS_STREAM_ERROR = 1 << 4
STATUS_KV_LOAD_REQ = 1 << 5
STATUS_Q_LOAD_REQ = 1 << 6

DEST_K_CACHE = 0
DEST_V_CACHE = 1
DEST_Q_BUF = 2

# Default geometry = the deployed RTL contract (hw/rtl/pkg/attn_pkg.sv:172-176).
HEAD_DIM = 128
TILE_Q = 32
N_Q_HEADS = 32
N_KV_HEADS = 8
GQA_GROUP_SIZE = N_Q_HEADS // N_KV_HEADS
MAX_SEQ_LEN = 512
ABSOLUTE_POSITION_LIMIT = 1 << 16
BF16_BYTES = 2
# The reference's signed-off PL clock, exported because harnesses import it.
PL_CLOCK_MHZ = 71.427856
# Device timestamps are nanoseconds: a 1000 MHz "clock".
DEVICE_CLOCK_MHZ = 1000.0
DMA_LENGTH_WIDTH = 26
DMA_MAX_TRANSFER_BYTES = (1 << DMA_LENGTH_WIDTH) - 1
MAX_KV_HEAD_BYTES = MAX_SEQ_LEN * HEAD_DIM * BF16_BYTES
Q_TILE_BYTES = TILE_Q * HEAD_DIM * BF16_BYTES
MAX_OUTPUT_BYTES = N_Q_HEADS * MAX_SEQ_LEN * HEAD_DIM * BF16_BYTES

ERR_NONE = 0x00
ERR_BAD_CFG = 0x01
ERR_BUSY_START = 0x02
ERR_STREAM_LEN = 0x10
ERR_STREAM_DEST = 0x11
ERR_RESULT_LEN = 0x12


def fp32_to_bf16_u16(values: np.ndarray) -> np.ndarray:
    """Pack float values into IEEE bf16 words, round to nearest even.

    Host-side input formatting with the reference's integer steps
    (sw/attn_driver.py:88-98); uint16 input passes through.  The device
    kernel ``lara_pack_bf16`` computes the same function on HBM tensors.
    """
    arr = np.asarray(values)
    if arr.dtype == np.uint16:
        return np.ascontiguousarray(arr)
    bits = np.asarray(arr, dtype=np.float32).view(np.uint32).copy()
    low = bits & np.uint32(0xFFFF)
    carry = ((low >> np.uint32(15)) & np.uint32(1)) & (
        ((bits >> np.uint32(16)) & np.uint32(1)) | (low & np.uint32(0x7FFF) != 0).astype(np.uint32))
    bits = (bits + carry.astype(np.uint32)) & np.uint32(0xFFFF0000)
    return np.ascontiguousarray((bits >> np.uint32(16)).astype(np.uint16))


def bf16_u16_to_fp32(values: np.ndarray) -> np.ndarray:
    """bf16 words -> fp32 (sw/attn_driver.py:101-103)."""
    words = np.asarray(values, dtype=np.uint16)
    return (words.astype(np.uint32) << np.uint32(16)).view(np.float32)


@dataclass(frozen=True)
class TensorByteCounts:
    q_bytes: int
    k_bytes: int
    v_bytes: int
    o_bytes: int


@dataclass
class RunProfile:
    """Per-transaction profile; same fields as sw/attn_driver.py:207-247.

    ``pl_*`` fields hold device time: cycles are nanoseconds (clock_mhz =
    1000); ``pl_mac_*`` is the attention kernels, ``pl_stall_*`` the
    host<->device copies.  The DMA fields count host<->device copies.
    """

    timestamp_utc: str
    git_commit: str
    bitstream_sha256: str | None
    clock_mhz: float
    seq_len: int
    causal: bool
    q_pos_base: int
    kv_pos_base: int
    host_rms_norm_ms: float = 0.0
    host_qkv_projection_ms: float = 0.0
    host_rope_ms: float = 0.0
    input_pack_ms: float = 0.0
    driver_setup_ms: float = 0.0
    request_service_ms: float = 0.0
    output_dma_setup_ms: float = 0.0
    output_dma_transfer_ms: float = 0.0
    attention_total_ms: float = 0.0
    layer_total_ms: float = 0.0
    kv_dma_setup_ms: float = 0.0
    kv_dma_transfer_ms: float = 0.0
    kv_dma_transfers: int = 0
    kv_dma_bytes: int = 0
    q_dma_setup_ms: float = 0.0
    q_dma_transfer_ms: float = 0.0
    q_dma_transfers: int = 0
    q_dma_bytes: int = 0
    output_dma_transfers: int = 0
    output_dma_bytes: int = 0
    pl_total_cycles: int = 0
    pl_mac_cycles: int = 0
    pl_stall_cycles: int = 0
    pl_core_active_cycles_excluding_stalls: int = 0
    pl_total_ms: float = 0.0
    pl_mac_ms: float = 0.0
    pl_stall_ms: float = 0.0
    pl_core_active_ms_excluding_stalls: float = 0.0

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _words(name: str, a, shape: tuple) -> np.ndarray:
    w = fp32_to_bf16_u16(a)
    if w.shape != shape:
        raise ValueError(f"expected {name}={shape}; got {w.shape}")
    return np.ascontiguousarray(w)


class AttentionAccelerator:
    """One B200 attention context (KV cache in HBM) with the reference's API."""

    def __init__(self, bitstream_path: str | None = None, overlay: Any | None = None, *,
                 device: int | None = None, arithmetic: str | None = None) -> None:
        # ``bitstream_path`` identifies the deployment artefact for provenance
        # (sha256 in RunProfile), as in the reference; no file is required.
        self.bitstream_path = str(Path(bitstream_path).resolve()) if bitstream_path else None
        self._git_hash = self._git_commit()
        self._bitstream_hash = self._bitstream_sha256()
        self._pl_clock_mhz = DEVICE_CLOCK_MHZ
        self.overlay = overlay
        self._closed = True
        self.last_profile: RunProfile | None = None
        if device is None:
            device = int(os.environ.get("LARA_DEVICE", os.environ.get("LOCAL_RANK", "0")))
        ctx = ctypes.c_void_p()
        check(lib.lara_create(int(device), ctypes.byref(ctx)), "lara_create")
        self._ctx = ctx
        self.device = int(device)
        self._closed = False
        self._hw_ready = True
        self.batch, self.n_q_heads, self.n_kv_heads, self.head_dim, self.max_seq_len = 1, N_Q_HEADS, N_KV_HEADS, \
            HEAD_DIM, MAX_SEQ_LEN
        self._status_word = STATUS_START_READY
        self.arithmetic = "ieee"
        self.set_arithmetic(arithmetic or os.environ.get("LARA_ARITHMETIC") or self._descriptor_arithmetic())
        self._last_output: np.ndarray | None = None
        self._perf = LaraPerf()
        self._max_len = 0  # longest cached sequence (profile field of run_query)

    # ------------------------------------------------------------------ basics
    @property
    def hw_ready(self) -> bool:
        return self._hw_ready and not self._closed

    @staticmethod
    def _git_commit() -> str:
        try:
            return subprocess.check_output(["git", "rev-parse", "--short", "HEAD"],
                                           cwd=Path(__file__).resolve().parents[1], stderr=subprocess.DEVNULL,
                                           text=True).strip()
        except (OSError, subprocess.SubprocessError):
            return "unknown"

    def _bitstream_sha256(self) -> str | None:
        if self.bitstream_path is None:
            return None
        path = Path(self.bitstream_path)
        if not path.is_file():
            return None
        digest = hashlib.sha256()
        with path.open("rb") as stream:
            for chunk in iter(lambda: stream.read(1024 * 1024), b""):
                digest.update(chunk)
        return digest.hexdigest()

    def _descriptor_arithmetic(self) -> str:
        if self.bitstream_path is None:
            return "ieee"
        try:
            doc = json.loads(Path(self.bitstream_path).read_text(encoding="utf-8"))
        except (OSError, UnicodeError, ValueError):
            return "ieee"  # not a lara_b200 descriptor: provenance only
        return str(doc.get("arithmetic", "ieee")) if isinstance(doc, dict) else "ieee"

    def set_arithmetic(self, mode: str) -> None:
        """Select ``"ieee"`` or ``"board"`` arithmetic for ``run_attention``."""
        self._require_open()
        codes = {"ieee": LARA_ARITH_IEEE, "board": LARA_ARITH_BOARD}
        if mode not in codes:
            raise ValueError(f"arithmetic must be 'ieee' or 'board', got {mode!r}")
        check(lib.lara_set_arithmetic(self._ctx, codes[mode]), "set_arithmetic")
        self.arithmetic = mode

    def _require_open(self) -> None:
        if self._closed:
            raise RuntimeError("attention accelerator buffers have been released")

    def close(self) -> None:
        if self._closed:
            return
        lib.lara_destroy(self._ctx)
        self._ctx = ctypes.c_void_p()
        self._closed = True

    def __del__(self) -> None:  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self) -> "AttentionAccelerator":
        self._require_open()
        return self

    def __exit__(self, exc_type: Any, exc: Any, traceback: Any) -> None:
        self.close()

    def save_last_profile(self, path: str | Path) -> None:
        if self.last_profile is None:
            raise RuntimeError("no completed attention run is available")
        Path(path).write_text(json.dumps(self.last_profile.to_dict(), indent=2) + "\n", encoding="utf-8")

    # ----------------------------------------------------- reference contract
    @staticmethod
    def _validate_seq_len(seq_len: int) -> None:
        if not 1 <= int(seq_len) <= MAX_SEQ_LEN:
            raise ValueError(f"seq_len must be in 1..{MAX_SEQ_LEN}, got {seq_len}")

    def _validate_len(self, seq_len: int) -> None:
        if not 1 <= int(seq_len) <= self.max_seq_len:
            raise ValueError(f"seq_len must be in 1..{self.max_seq_len}, got {seq_len}")

    @classmethod
    def byte_counts(cls, seq_len: int) -> TensorByteCounts:
        cls._validate_seq_len(seq_len)
        return TensorByteCounts(
            N_Q_HEADS * seq_len * HEAD_DIM * BF16_BYTES,
            N_KV_HEADS * seq_len * HEAD_DIM * BF16_BYTES,
            N_KV_HEADS * seq_len * HEAD_DIM * BF16_BYTES,
            N_Q_HEADS * seq_len * HEAD_DIM * BF16_BYTES,
        )

    def _counts(self, seq_len: int) -> TensorByteCounts:
        return TensorByteCounts(self.n_q_heads * seq_len * self.head_dim * BF16_BYTES,
                                self.n_kv_heads * seq_len * self.head_dim * BF16_BYTES,
                                self.n_kv_heads * seq_len * self.head_dim * BF16_BYTES,
                                self.n_q_heads * seq_len * self.head_dim * BF16_BYTES)

    def clear_status(self) -> None:
        self._require_open()
        self._status_word = STATUS_START_READY

    def status(self) -> int:
        return self._status_word

    def start(self) -> None:
        self._require_open()
        if not (self._status_word & STATUS_START_READY):
            raise RuntimeError("accelerator is not ready to accept start")

    def configure(self, seq_len: int, *, q_pos_base: int = 0, kv_pos_base: int = 0, causal: bool = True) -> None:
        self._require_open()
        self._validate_len(seq_len)
        if (q_pos_base < 0 or kv_pos_base < 0 or q_pos_base + seq_len > ABSOLUTE_POSITION_LIMIT
                or kv_pos_base + seq_len > ABSOLUTE_POSITION_LIMIT):
            raise ValueError("absolute position base + seq_len exceeds 16-bit range")
        check(lib.lara_configure(self._ctx, int(seq_len), int(q_pos_base), int(kv_pos_base), int(bool(causal))),
              "configure")

    def wait_done(self, q_heads=None, k_heads=None, v_heads=None, seq_len: int | None = None,
                  timeout_ms: int | None = None) -> None:
        """Wait for the context's device work (bounded by ``timeout_ms``)."""
        self._require_open()
        check(lib.lara_sync(self._ctx, -1 if timeout_ms is None else int(timeout_ms)), "wait_done")

    def readback_o(self, seq_len: int, out_buf: np.ndarray | None = None) -> np.ndarray:
        if self._last_output is None:
            raise RuntimeError("no completed attention run is available")
        return self._last_output

    def read_output(self) -> np.ndarray:
        return self.readback_o(0)

    def read_perf(self) -> dict[str, int]:
        self._require_open()
        check(lib.lara_read_perf(self._ctx, ctypes.byref(self._perf)), "read_perf")
        return {"cycles": int(self._perf.cycles), "mac_cycles": int(self._perf.mac_cycles),
                "stall_cycles": int(self._perf.stall_cycles)}

    def _new_profile(self, seq_len: int, causal: bool, q_pos_base: int, kv_pos_base: int) -> RunProfile:
        return RunProfile(timestamp_utc=datetime.now(timezone.utc).isoformat(), git_commit=self._git_hash,
                          bitstream_sha256=self._bitstream_hash, clock_mhz=self._pl_clock_mhz, seq_len=seq_len,
                          causal=causal, q_pos_base=q_pos_base, kv_pos_base=kv_pos_base)

    @property
    def last_profile(self) -> RunProfile | None:
        # run_query finishes its profile only when it is read (the device times
        # come from CUDA events; reading them is work a decode loop need not pay)
        query = self.__dict__.get("_pending_query")
        if query is not None:
            self._pending_query = None
            ts, t_start, t_call, t_end, q_bytes, o_bytes, seq_len = query
            prof = RunProfile(timestamp_utc=datetime.fromtimestamp(ts, timezone.utc).isoformat(),
                              git_commit=self._git_hash, bitstream_sha256=self._bitstream_hash,
                              clock_mhz=self._pl_clock_mhz, seq_len=seq_len, causal=False, q_pos_base=0,
                              kv_pos_base=0)
            prof.request_service_ms = (t_end - t_call) * 1000.0
            prof.q_dma_transfers, prof.q_dma_bytes = 1, q_bytes
            prof.output_dma_transfers, prof.output_dma_bytes = 1, o_bytes
            self._last_profile = prof
            self._pending_profile = (prof, t_start, t_end)
        pending = self.__dict__.get("_pending_profile")
        if pending is not None:
            self._pending_profile = None
            self._finish_profile(*pending)
        return self.__dict__.get("_last_profile")

    @last_profile.setter
    def last_profile(self, prof: RunProfile | None) -> None:
        self._pending_query = None
        self._pending_profile = None
        self._last_profile = prof

    def _finish_profile(self, prof: RunProfile, t_start: float, t_end: float | None = None) -> None:
        perf = self.read_perf()
        prof.pl_total_cycles = perf["cycles"]
        prof.pl_mac_cycles = perf["mac_cycles"]
        prof.pl_stall_cycles = perf["stall_cycles"]
        prof.pl_core_active_cycles_excluding_stalls = max(perf["cycles"] - perf["stall_cycles"], 0)
        per_ms = self._pl_clock_mhz * 1000.0
        prof.pl_total_ms = perf["cycles"] / per_ms
        prof.pl_mac_ms = perf["mac_cycles"] / per_ms
        prof.pl_stall_ms = perf["stall_cycles"] / per_ms
        prof.pl_core_active_ms_excluding_stalls = prof.pl_core_active_cycles_excluding_stalls / per_ms
        prof.attention_total_ms = ((time.perf_counter() if t_end is None else t_end) - t_start) * 1000.0

    def run_attention(self, q_heads: np.ndarray, k_heads: np.ndarray, v_heads: np.ndarray, *,
                      seq_len: int | None = None, q_pos_base: int = 0, kv_pos_base: int = 0, causal: bool = True,
                      timeout_ms: int | None = None) -> np.ndarray:
        """Run one full transaction; returns raw head-major bf16 words ``[Hq, L, D]``."""
        self._require_open()
        t_start = time.perf_counter()
        L = int(seq_len if seq_len is not None else q_heads.shape[1])
        self._validate_len(L)
        expected_q = (self.n_q_heads, L, self.head_dim)
        expected_kv = (self.n_kv_heads, L, self.head_dim)
        if (tuple(q_heads.shape) != expected_q or tuple(k_heads.shape) != expected_kv
                or tuple(v_heads.shape) != expected_kv):
            raise ValueError(f"expected Q={expected_q}, K/V={expected_kv}; got {q_heads.shape}, {k_heads.shape}, "
                             f"{v_heads.shape}")
        prof = self._new_profile(L, causal, q_pos_base, kv_pos_base)
        self.last_profile = prof

        t = time.perf_counter()
        q = np.ascontiguousarray(fp32_to_bf16_u16(q_heads))
        k = np.ascontiguousarray(fp32_to_bf16_u16(k_heads))
        v = np.ascontiguousarray(fp32_to_bf16_u16(v_heads))
        prof.input_pack_ms = (time.perf_counter() - t) * 1000.0

        t = time.perf_counter()
        self.configure(L, q_pos_base=q_pos_base, kv_pos_base=kv_pos_base, causal=causal)
        self.clear_status()
        counts = self._counts(L)
        out = np.empty(expected_q, dtype=np.uint16)
        prof.driver_setup_ms = (time.perf_counter() - t) * 1000.0

        self._status_word = STATUS_BUSY
        t = time.perf_counter()
        check(lib.lara_run_attention(self._ctx, _ptr(q), _ptr(k), _ptr(v), _ptr(out), 0), "run_attention")
        prof.request_service_ms = (time.perf_counter() - t) * 1000.0
        self._status_word = STATUS_DONE | STATUS_START_READY
        if timeout_ms is not None and prof.request_service_ms > timeout_ms:
            raise TimeoutError("attention accelerator timed out while servicing load requests")
        prof.kv_dma_transfers, prof.kv_dma_bytes = 2, counts.k_bytes + counts.v_bytes
        prof.q_dma_transfers, prof.q_dma_bytes = 1, counts.q_bytes
        prof.output_dma_transfers, prof.output_dma_bytes = 1, counts.o_bytes
        self._last_output = out
        self._finish_profile(prof, t_start)
        return out

    def run_layer(self, hidden_states: np.ndarray, wq: np.ndarray, wk: np.ndarray, wv: np.ndarray,
                  rms_weight: np.ndarray | None = None, *, q_pos_base: int = 0, kv_pos_base: int = 0,
                  causal: bool = True, timeout_ms: int | None = None) -> np.ndarray:
        """RMSNorm + QKV projection + RoPE, then attention; returns float32 ``[L, Hq * D]``.

        Same call and result layout as sw/attn_driver.py:552-586, but the
        prologue runs on the GPU (``lara_run_layer``): hidden_states
        ``[L, hidden]``, wq ``[hidden, Hq*D]``, wk/wv ``[hidden, Hkv*D]`` (the
        [IN][OUT] layout, Q = X @ Wq) and rms_weight ``[hidden]`` are packed to
        bf16; RMSNorm (eps 1e-5), the projection (fp32 accumulation) and RoPE
        (base 10000, dim pairs (2i, 2i+1), positions q/kv_pos_base + t) run in
        one fused launch sequence, and the attention uses this context's
        arithmetic.  RMSNorm and RoPE are fused into the projection kernels, so
        their device time is inside ``host_qkv_projection_ms`` and the
        ``host_rms_norm_ms`` / ``host_rope_ms`` fields stay 0.
        """
        self._require_open()
        t_start = time.perf_counter()
        x = np.asarray(hidden_states)
        if x.ndim != 2:
            raise ValueError(f"hidden_states must be [L, hidden], got {x.shape}")
        L, hidden = x.shape
        self._validate_len(L)
        nq, nkv = self.n_q_heads * self.head_dim, self.n_kv_heads * self.head_dim
        for name, w, cols in (("wq", wq, nq), ("wk", wk, nkv), ("wv", wv, nkv)):
            if tuple(np.shape(w)) != (hidden, cols):
                raise ValueError(f"expected {name}={(hidden, cols)}; got {np.shape(w)}")
        if rms_weight is not None and tuple(np.shape(rms_weight)) != (hidden,):
            raise ValueError(f"expected rms_weight=({hidden},); got {np.shape(rms_weight)}")
        if hidden % 64:
            raise ValueError("hidden size must be a multiple of 64")
        prof = self._new_profile(L, causal, q_pos_base, kv_pos_base)
        self.last_profile = prof
        t = time.perf_counter()
        xw = np.ascontiguousarray(fp32_to_bf16_u16(x))
        w_qkv = np.ascontiguousarray(np.concatenate([fp32_to_bf16_u16(np.asarray(w)) for w in (wq, wk, wv)], axis=1))
        gw = None if rms_weight is None else np.ascontiguousarray(fp32_to_bf16_u16(np.asarray(rms_weight)))
        prof.input_pack_ms = (time.perf_counter() - t) * 1000.0
        self.configure(L, q_pos_base=q_pos_base, kv_pos_base=kv_pos_base, causal=causal)
        self.clear_status()
        out = np.empty((self.n_q_heads, L, self.head_dim), dtype=np.uint16)
        self._status_word = STATUS_BUSY
        t = time.perf_counter()
        check(lib.lara_run_layer(self._ctx, _ptr(xw), _ptr(w_qkv), None if gw is None else _ptr(gw), int(hidden),
                                 _ptr(out), 1e-5, 10000.0, 0), "run_layer")
        prof.request_service_ms = (time.perf_counter() - t) * 1000.0
        self._status_word = STATUS_DONE | STATUS_START_READY
        if timeout_ms is not None and prof.request_service_ms > timeout_ms:
            raise TimeoutError("attention accelerator timed out while running the layer")
        self._last_output = out
        self._finish_profile(prof, t_start)
        pro, att = ctypes.c_uint64(0), ctypes.c_uint64(0)
        check(lib.lara_read_layer_perf(self._ctx, ctypes.byref(pro), ctypes.byref(att)), "read_layer_perf")
        prof.host_rms_norm_ms = 0.0
        prof.host_qkv_projection_ms = pro.value / 1e6
        prof.host_rope_ms = 0.0
        result = bf16_u16_to_fp32(out).transpose(1, 0, 2).reshape(L, nq)
        prof.layer_total_ms = (time.perf_counter() - t_start) * 1000.0
        return result

    # -------------------------------------------------------------- extensions
    def configure_heads(self, n_q_heads: int = N_Q_HEADS, n_kv_heads: int = N_KV_HEADS, head_dim: int = HEAD_DIM,
                        max_seq_len: int = MAX_SEQ_LEN, batch: int = 1) -> None:
        """Set the head geometry and KV-cache capacity (empties the cache)."""
        self._require_open()
        check(lib.lara_configure_heads(self._ctx, int(batch), int(n_q_heads), int(n_kv_heads), int(head_dim),
                                       int(max_seq_len)), "configure_heads")
        self._max_len = 0
        self.batch, self.n_q_heads, self.n_kv_heads, self.head_dim, self.max_seq_len = \
            int(batch), int(n_q_heads), int(n_kv_heads), int(head_dim), int(max_seq_len)

    @property
    def seq_lens(self) -> np.ndarray:
        self._require_open()
        out = np.zeros(self.batch, dtype=np.int32)
        check(lib.lara_get_seq_lens(self._ctx, _ptr(out)), "seq_lens")
        return out

    def load_kv(self, k: np.ndarray, v: np.ndarray, lens=None) -> None:
        """Load the cache from ``k/v[B, Hkv, L, D]``; ``lens[B]`` defaults to L."""
        self._require_open()
        L = int(np.asarray(k).shape[2])
        shape = (self.batch, self.n_kv_heads, L, self.head_dim)
        kw, vw = _words("K", k, shape), _words("V", v, shape)
        ln = np.full(self.batch, L, np.int32) if lens is None else np.ascontiguousarray(lens, dtype=np.int32)
        if ln.shape != (self.batch,):
            raise ValueError(f"lens must have shape ({self.batch},)")
        check(lib.lara_kv_load(self._ctx, _ptr(kw), _ptr(vw), _ptr(ln), L, 0), "load_kv")
        self._max_len = int(ln.max()) if ln.size else 0

    def save_kv(self, path) -> None:
        """Write the resident cache to ``path`` (the ``lara-kv-v1`` format of
        :mod:`lara_b200.kvfile`: lengths and the first max(len) tokens of every
        (sequence, kv head) row as bf16 words)."""
        from . import kvfile

        self._require_open()
        lens = self.seq_lens
        n = max(int(lens.max()) if lens.size else 0, 1)
        shape = (self.batch, self.n_kv_heads, n, self.head_dim)
        k = np.empty(shape, np.uint16)
        v = np.empty(shape, np.uint16)
        check(lib.lara_kv_read(self._ctx, _ptr(k), _ptr(v), _ptr(lens), n, 0), "kv_read")
        kvfile.save(path, k, v, lens)

    def restore_kv(self, path) -> None:
        """Load a cache written by :meth:`save_kv` (same batch, kv heads and
        head_dim as this context; lengths must fit max_seq_len)."""
        from . import kvfile

        self._require_open()
        k, v, lens = kvfile.load(path)
        if k.shape[0] != self.batch or k.shape[1] != self.n_kv_heads or k.shape[3] != self.head_dim:
            raise ValueError(f"{path}: cache geometry {k.shape} does not match batch={self.batch}, "
                             f"n_kv_heads={self.n_kv_heads}, head_dim={self.head_dim}")
        if k.shape[2] > self.max_seq_len:
            raise ValueError(f"{path}: {k.shape[2]} tokens exceed max_seq_len={self.max_seq_len}")
        self.load_kv(k, v, lens)

    def truncate_kv(self, lens) -> None:
        """Shorten the sequences to ``lens[B]`` (each at most its current length).

        The rows past the new lengths are dropped and later appends overwrite
        them: a prefill chunk or rejected speculative tokens are rewound
        without touching the rest of the cache.  Lengths cannot grow
        (``ValueError``)."""
        self._require_open()
        ln = np.ascontiguousarray(lens, dtype=np.int32)
        if ln.shape != (self.batch,):
            raise ValueError(f"lens must have shape ({self.batch},)")
        check(lib.lara_kv_truncate(self._ctx, _ptr(ln)), "truncate_kv")
        self._max_len = int(ln.max()) if ln.size else 0

    def append_kv(self, k_new: np.ndarray, v_new: np.ndarray) -> None:
        """Append ``k/v_new[B, Hkv, n, D]`` (or ``[B, Hkv, D]`` for one token)."""
        self._require_open()
        k_new = np.asarray(k_new)
        if k_new.ndim == 3:
            k_new, v_new = k_new[:, :, None, :], np.asarray(v_new)[:, :, None, :]
        n = int(k_new.shape[2])
        shape = (self.batch, self.n_kv_heads, n, self.head_dim)
        kw, vw = _words("K", k_new, shape), _words("V", v_new, shape)
        check(lib.lara_kv_append_ctx(self._ctx, _ptr(kw), _ptr(vw), n, 0), "append_kv")
        self._max_len += n

    def run_query(self, q: np.ndarray, *, out: np.ndarray | None = None) -> np.ndarray:
        """Decode one query token per sequence: ``q[B, Hq, D]`` -> ``o[B, Hq, D]`` (bf16 words)."""
        self._require_open()
        t_start = time.perf_counter()
        shape = (self.batch, self.n_q_heads, self.head_dim)
        if type(q) is np.ndarray and q.dtype == np.uint16 and q.shape == shape and q.flags.c_contiguous:
            qw = q  # the decode-loop case: already contiguous bf16 words
        else:
            qw = _words("Q", q, shape)
        if out is None:
            out = np.empty(shape, dtype=np.uint16)
        elif out.shape != shape or out.dtype != np.uint16 or not out.flags.c_contiguous:
            raise ValueError(f"out must be a contiguous uint16 array of shape {shape}")
        # data addresses of the last q / out arrays, held with the arrays themselves
        # (a decode loop passes the same buffers every step)
        cache = self.__dict__.get("_query_ptrs")
        if cache is None or cache[0] is not qw or cache[2] is not out:
            cache = self._query_ptrs = (qw, qw.ctypes.data, out, out.ctypes.data)
        self._status_word = STATUS_BUSY
        t = time.perf_counter()
        rc = lib.lara_run_query(self._ctx, cache[1], cache[3], 0)
        if rc:
            check(rc, "run_query")
        t_end = time.perf_counter()
        self._status_word = STATUS_DONE | STATUS_START_READY
        self._last_output = out
        # The RunProfile is built when last_profile is read: a decode loop pays
        # for two clock reads, not for the record.
        self._pending_profile = None
        self._pending_query = (time.time(), t_start, t, t_end, qw.nbytes, out.nbytes, self._max_len)
        return out

    def run_prefill_chunk(self, q: np.ndarray, k_new: np.ndarray, v_new: np.ndarray, *,
                          causal: bool = True, out: np.ndarray | None = None) -> np.ndarray:
        """Append ``n`` new tokens and attend them over cache + self.

        ``q[B, n, Hq, D]`` (token-major), ``k/v_new[B, Hkv, n, D]`` ->
        ``o[B, n, Hq, D]``.  Query i of sequence b sits at position
        ``len_b + i``; causal masking follows kv_pos <= q_pos.  ``out`` (a
        contiguous uint16 array of the output shape) receives the words; with
        page-locked inputs and output the copies overlap the kernels.
        """
        self._require_open()
        t_start = time.perf_counter()
        n = int(np.asarray(q).shape[1])
        qw = _words("Q", q, (self.batch, n, self.n_q_heads, self.head_dim))
        kv_shape = (self.batch, self.n_kv_heads, n, self.head_dim)
        kw, vw = _words("K", k_new, kv_shape), _words("V", v_new, kv_shape)
        if out is None:
            out = np.empty(qw.shape, dtype=np.uint16)
        elif out.shape != qw.shape or out.dtype != np.uint16 or not out.flags.c_contiguous:
            raise ValueError(f"out must be a contiguous uint16 array of shape {qw.shape}")
        prof = self._new_profile(n, causal, 0, 0)
        self.last_profile = prof
        t = time.perf_counter()
        check(lib.lara_run_prefill_chunk(self._ctx, _ptr(qw), _ptr(kw), _ptr(vw), _ptr(out), n, int(bool(causal)), 0),
              "run_prefill_chunk")
        self._max_len += n
        prof.request_service_ms = (time.perf_counter() - t) * 1000.0
        self._last_output = out
        self._finish_profile(prof, t_start)
        return out


def _self_test() -> None:
    """Zero input gives zero output (sw/board_test.py:78-79) on the B200 path."""
    with AttentionAccelerator() as accel:
        assert accel.hw_ready
        L = 16
        q = np.zeros((N_Q_HEADS, L, HEAD_DIM), dtype=np.uint16)
        k = np.zeros((N_KV_HEADS, L, HEAD_DIM), dtype=np.uint16)
        out = accel.run_attention(q, k, k, seq_len=L)
        assert out.shape == (N_Q_HEADS, L, HEAD_DIM) and not np.any(out)
    print("attn_driver B200 self-test PASSED")


if __name__ == "__main__":
    _self_test()
