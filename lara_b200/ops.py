"""Torch-tensor front end of the stateless C-ABI kernels.

PyTorch only provides device memory and the current stream here; every
computation runs in liblara_b200.so.  bf16 tensors may be ``torch.bfloat16``
or 16-bit integer views of the same words.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from ._native import check, lib

_WORD_DTYPES = (torch.bfloat16, torch.int16, torch.uint16)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _check_words(name: str, t: torch.Tensor, shape: tuple | None = None) -> None:
    if t.dtype not in _WORD_DTYPES:
        raise TypeError(f"{name} must hold bf16 words (bfloat16/int16/uint16), got {t.dtype}")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")


@dataclass
class DecodePlan:
    num_splits: int
    chunk_tokens: int
    workspace_bytes: int


def decode_plan(batch: int, n_q_heads: int, n_kv_heads: int, head_dim: int, max_seq_len: int,
                lens=None) -> DecodePlan:
    """Split plan for the current device (``lara_decode_plan``)."""
    ns, ch = ctypes.c_int(0), ctypes.c_int(0)
    arr = None
    if lens is not None:
        import numpy as np

        arr = np.ascontiguousarray(np.asarray(lens, dtype=np.int32))
    check(lib.lara_decode_plan(batch, n_q_heads, n_kv_heads, head_dim, max_seq_len,
                               None if arr is None else arr.ctypes.data, ctypes.byref(ns), ctypes.byref(ch)),
          "lara_decode_plan")
    ws = lib.lara_decode_workspace_bytes(batch, n_q_heads, n_kv_heads, head_dim, ns.value)
    return DecodePlan(ns.value, ch.value, int(ws))


def new_workspace(nbytes: int, device) -> torch.Tensor:
    """A zeroed device workspace (256-byte aligned by the caching allocator)."""
    ws = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
    check(lib.lara_workspace_init(ws.data_ptr(), ws.numel(), _stream(ws.device)), "lara_workspace_init")
    return ws


def workspace_status(ws: torch.Tensor) -> int:
    """Read and clear the device status word (synchronises the stream)."""
    bits = ctypes.c_int(0)
    check(lib.lara_workspace_status(ws.data_ptr(), _stream(ws.device), ctypes.byref(bits)), "lara_workspace_status")
    return bits.value


class Decoder:
    """Decode over a cache ``[B, Hkv, Lmax, D]`` with a fixed plan and workspace."""

    def __init__(self, batch: int, n_q_heads: int, n_kv_heads: int, head_dim: int, max_seq_len: int, device,
                 lens=None, num_splits: int = 0, chunk_tokens: int = 0, scale: float | None = None):
        self.batch, self.hq, self.hkv, self.d, self.lmax = batch, n_q_heads, n_kv_heads, head_dim, max_seq_len
        self.device = torch.device(device)
        plan = decode_plan(batch, n_q_heads, n_kv_heads, head_dim, max_seq_len, lens)
        if num_splits and chunk_tokens:
            plan = DecodePlan(num_splits, chunk_tokens,
                              int(lib.lara_decode_workspace_bytes(batch, n_q_heads, n_kv_heads, head_dim,
                                                                  num_splits)))
        self.plan = plan
        self.scale = 1.0 / math.sqrt(head_dim) if scale is None else float(scale)
        self.workspace = new_workspace(plan.workspace_bytes, self.device)

    def _shapes(self, q, k_cache, v_cache, seq_lens):
        _check_words("q", q, (self.batch, self.hq, self.d))
        _check_words("k_cache", k_cache, (self.batch, self.hkv, self.lmax, self.d))
        _check_words("v_cache", v_cache, (self.batch, self.hkv, self.lmax, self.d))
        if seq_lens.dtype != torch.int32 or not seq_lens.is_cuda or seq_lens.numel() != self.batch:
            raise ValueError("seq_lens must be a CUDA int32 tensor of length batch")

    def __call__(self, q, k_cache, v_cache, seq_lens, out=None):
        self._shapes(q, k_cache, v_cache, seq_lens)
        o = torch.empty_like(q) if out is None else out
        check(lib.lara_gqa_decode(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), seq_lens.data_ptr(),
                                  o.data_ptr(), self.batch, self.hq, self.hkv, self.d, self.lmax, self.scale,
                                  self.plan.num_splits, self.plan.chunk_tokens, self.workspace.data_ptr(),
                                  self.workspace.numel(), _stream(q.device)), "lara_gqa_decode")
        return o

    def partial(self, q, k_cache, v_cache, seq_lens, out_ml=None, out_acc=None):
        """Unnormalised (m, l) and acc per (b, h) row (split-KV across devices)."""
        self._shapes(q, k_cache, v_cache, seq_lens)
        rows = self.batch * self.hq
        ml = torch.empty((rows, 2), dtype=torch.float32, device=q.device) if out_ml is None else out_ml
        acc = torch.empty((rows, self.d), dtype=torch.float32, device=q.device) if out_acc is None else out_acc
        check(lib.lara_gqa_decode_partial(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), seq_lens.data_ptr(),
                                          ml.data_ptr(), acc.data_ptr(), self.batch, self.hq, self.hkv, self.d,
                                          self.lmax, self.scale, self.plan.num_splits, self.plan.chunk_tokens,
                                          self.workspace.data_ptr(), self.workspace.numel(), _stream(q.device)),
              "lara_gqa_decode_partial")
        return ml, acc


def decode_kernel(n_q_heads: int, n_kv_heads: int, head_dim: int) -> str:
    """``"tensor"`` (tcgen05 kernel) or ``"cuda_core"``: which decode kernel runs a geometry."""
    from ._native import LARA_DECODE_KERNEL_TENSOR

    k = int(lib.lara_decode_kernel(int(n_q_heads), int(n_kv_heads), int(head_dim)))
    return "tensor" if k == LARA_DECODE_KERNEL_TENSOR else "cuda_core"


def gqa_decode(q, k_cache, v_cache, seq_lens, *, scale=None, num_splits=0, chunk_tokens=0):
    """One-shot decode (plans and allocates a workspace per call)."""
    B, Hq, D = q.shape
    _, Hkv, Lmax, _ = k_cache.shape
    dec = Decoder(B, Hq, Hkv, D, Lmax, q.device, num_splits=num_splits, chunk_tokens=chunk_tokens, scale=scale)
    return dec(q, k_cache, v_cache, seq_lens)


def lse_combine(part_ml: torch.Tensor, part_acc: torch.Tensor) -> torch.Tensor:
    """Merge ``part_ml[P, rows, 2]``, ``part_acc[P, rows, D]`` into bf16 ``[rows, D]``."""
    P, rows, D = part_acc.shape
    if part_ml.shape != (P, rows, 2) or part_ml.dtype != torch.float32 or part_acc.dtype != torch.float32:
        raise ValueError("part_ml must be float32 [P, rows, 2] and part_acc float32 [P, rows, D]")
    o = torch.empty((rows, D), dtype=torch.bfloat16, device=part_acc.device)
    check(lib.lara_lse_combine(part_ml.contiguous().data_ptr(), part_acc.contiguous().data_ptr(), P, rows, D,
                               o.data_ptr(), _stream(o.device)), "lara_lse_combine")
    return o


def lse_combine_strided(buf: torch.Tensor, num_parts: int, rows: int, head_dim: int, *, ml_offset: int,
                        acc_offset: int, part_stride: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Merge partial states packed in one float32 buffer: part i's (m, l) pairs
    at ``buf[i*part_stride + ml_offset:]``, its acc rows at
    ``buf[i*part_stride + acc_offset:]``.  Returns bf16 ``[rows, head_dim]``
    (or writes ``out``)."""
    if buf.dtype != torch.float32 or not buf.is_contiguous():
        raise ValueError("buf must be a contiguous float32 tensor")
    need = (num_parts - 1) * part_stride + max(ml_offset + 2 * rows, acc_offset + rows * head_dim)
    if buf.numel() < need:
        raise ValueError(f"buf holds {buf.numel()} floats, {need} needed")
    o = torch.empty((rows, head_dim), dtype=torch.bfloat16, device=buf.device) if out is None else out
    base = buf.data_ptr()
    check(lib.lara_lse_combine_strided(base + 4 * ml_offset, part_stride, base + 4 * acc_offset, part_stride,
                                       num_parts, rows, head_dim, o.data_ptr(), _stream(buf.device)),
          "lara_lse_combine_strided")
    return o


def kv_append(k_cache, v_cache, seq_lens, k_new, v_new, workspace=None) -> None:
    """Write ``k_new/v_new[B, Hkv, n, D]`` at ``seq_lens[b]`` and advance ``seq_lens``."""
    B, Hkv, Lmax, D = k_cache.shape
    n = k_new.shape[2]
    _check_words("k_new", k_new, (B, Hkv, n, D))
    _check_words("v_new", v_new, (B, Hkv, n, D))
    check(lib.lara_kv_append(k_cache.data_ptr(), v_cache.data_ptr(), seq_lens.data_ptr(), k_new.data_ptr(),
                             v_new.data_ptr(), B, Hkv, D, Lmax, n, _ptr(workspace), _stream(k_cache.device)),
          "lara_kv_append")


def gqa_prefill(q, k_cache, v_cache, cached_lens, *, causal=True, scale=None, workspace=None, out=None):
    """Chunked prefill over the cache ("cache + self").

    ``q[B, n, Hq, D]`` (token-major) attends the cache ``k/v_cache[B, Hkv, Lmax, D]``
    whose rows ``cached_lens[b] .. cached_lens[b] + n - 1`` already hold the chunk's
    own K/V (``kv_append`` with the lengths before the append); query ``i`` of
    sequence ``b`` sits at position ``cached_lens[b] + i`` and, when ``causal``,
    sees keys ``0 .. cached_lens[b] + i``.  Returns ``o[B, n, Hq, D]`` (bf16).
    """
    B, n, Hq, D = q.shape
    _, Hkv, Lmax, _ = k_cache.shape
    _check_words("q", q)
    _check_words("k_cache", k_cache, (B, Hkv, Lmax, D))
    _check_words("v_cache", v_cache, (B, Hkv, Lmax, D))
    if cached_lens.dtype != torch.int32 or not cached_lens.is_cuda or cached_lens.numel() != B:
        raise ValueError("cached_lens must be a CUDA int32 tensor of length batch")
    nbytes = int(lib.lara_prefill_workspace_bytes(B, n, Hq, Hkv, D, Lmax))
    if nbytes == 0:
        raise ValueError(f"unsupported prefill geometry B={B} n={n} Hq={Hq} Hkv={Hkv} D={D} Lmax={Lmax}")
    if workspace is None or workspace.numel() < nbytes:
        workspace = new_workspace(nbytes, q.device)
    o = torch.empty_like(q) if out is None else out
    sc = 1.0 / math.sqrt(D) if scale is None else float(scale)
    check(lib.lara_gqa_prefill(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), cached_lens.data_ptr(),
                               o.data_ptr(), B, n, Hq, Hkv, D, Lmax, int(bool(causal)), sc, workspace.data_ptr(),
                               workspace.numel(), _stream(q.device)), "lara_gqa_prefill")
    return o


def pack_bf16(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> bf16 words (int16 view), bit-identical to the reference packer."""
    if x.dtype != torch.float32 or not x.is_cuda:
        raise ValueError("pack_bf16 takes a CUDA float32 tensor")
    x = x.contiguous()
    out = torch.empty(x.shape, dtype=torch.int16, device=x.device)
    check(lib.lara_pack_bf16(x.data_ptr(), out.data_ptr(), x.numel(), _stream(x.device)), "lara_pack_bf16")
    return out


def attention_dense(q, k, v, *, causal=True, q_pos_base=0, kv_pos_base=0, scale=None):
    """``run_attention`` semantics on device tensors: q[Hq,L,D], k/v[Hkv,L,D] -> o[Hq,L,D]."""
    Hq, L, D = q.shape
    Hkv = k.shape[0]
    _check_words("q", q)
    _check_words("k", k, (Hkv, L, D))
    _check_words("v", v, (Hkv, L, D))
    sc = 1.0 / math.sqrt(D) if scale is None else float(scale)
    nbytes = int(lib.lara_dense_workspace_bytes(Hq, Hkv, D, L))
    if nbytes == 0:
        raise ValueError(f"unsupported dense geometry Hq={Hq} Hkv={Hkv} D={D} L={L}")
    ws = new_workspace(nbytes, q.device)
    o = torch.empty_like(q)
    check(lib.lara_attention_dense(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), Hq, Hkv, D, L,
                                   q_pos_base, kv_pos_base, int(bool(causal)), sc, ws.data_ptr(), ws.numel(),
                                   _stream(q.device)), "lara_attention_dense")
    return o


def attention_dense_board(q, k, v, *, causal=True, q_pos_base=0, kv_pos_base=0):
    """``attention_dense`` in board arithmetic: the FPGA datapath's output words bit for bit
    (head_dim 128; see ``lara_attention_dense_board`` in include/lara_b200.h)."""
    Hq, L, D = q.shape
    Hkv = k.shape[0]
    _check_words("q", q)
    _check_words("k", k, (Hkv, L, D))
    _check_words("v", v, (Hkv, L, D))
    o = torch.empty_like(q)
    check(lib.lara_attention_dense_board(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), Hq, Hkv, D, L,
                                         int(bool(causal)), q_pos_base, kv_pos_base, _stream(q.device)),
          "lara_attention_dense_board")
    return o


def layer_prologue(x, w_qkv, rms_weight=None, *, n_q_heads=32, n_kv_heads=8, head_dim=128, q_pos_base=0,
                   kv_pos_base=0, rms_eps=1e-5, rope_base=10000.0, workspace=None, out=None):
    """RMSNorm -> QKV projection -> RoPE on device tensors (``lara_layer_prologue``).

    x: bf16 [L, hidden] or [B, L, hidden]; w_qkv: bf16 [hidden, (Hq + 2 Hkv) * D] (= [Wq | Wk | Wv]);
    rms_weight: bf16 [hidden] or None.  Returns bf16 q [(B,) Hq, L, D], k [(B,) Hkv, L, D], v likewise
    (into ``out = (q, k, v)`` when given).  ``workspace`` (from ``new_workspace``) is reused when large
    enough.
    """
    batched = x.dim() == 3
    B, L, hidden = x.shape if batched else (1, *x.shape)
    n_total = (n_q_heads + 2 * n_kv_heads) * head_dim
    _check_words("x", x, tuple(x.shape))
    _check_words("w_qkv", w_qkv, (hidden, n_total))
    if rms_weight is not None:
        _check_words("rms_weight", rms_weight, (hidden,))
    dev = x.device
    lead = (B,) if batched else ()
    if out is None:
        q = torch.empty((*lead, n_q_heads, L, head_dim), dtype=x.dtype, device=dev)
        k = torch.empty((*lead, n_kv_heads, L, head_dim), dtype=x.dtype, device=dev)
        v = torch.empty_like(k)
    else:
        q, k, v = out
        _check_words("q", q, (*lead, n_q_heads, L, head_dim))
        _check_words("k", k, (*lead, n_kv_heads, L, head_dim))
        _check_words("v", v, (*lead, n_kv_heads, L, head_dim))
    nbytes = int(lib.lara_layer_prologue_workspace_bytes(B, L, hidden))
    ws = workspace if workspace is not None and workspace.numel() >= nbytes else new_workspace(nbytes, dev)
    check(lib.lara_layer_prologue(x.data_ptr(), 0 if rms_weight is None else rms_weight.data_ptr(), w_qkv.data_ptr(),
                                  q.data_ptr(), k.data_ptr(), v.data_ptr(), B, L, hidden, n_q_heads, n_kv_heads,
                                  head_dim, q_pos_base, kv_pos_base, float(rms_eps), float(rope_base),
                                  ws.data_ptr(), ws.numel(), _stream(dev)), "lara_layer_prologue")
    return q, k, v
