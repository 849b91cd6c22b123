"""TEST INFRASTRUCTURE ONLY -- CPU oracle of the layer prologue.

``AttentionAccelerator.run_layer`` (sw/attn_driver.py:552-586) runs RMSNorm,
the QKV projection and RoPE on the host through ``host_attention.py``, a
module the reference does not ship.  Its contract is restated from the RTL
interface descriptions of the same steps and from ``run_layer``'s call
sequence:

* ``rms_norm``: ``y = x / sqrt(mean(x^2) + eps) * gamma``
  (hw/rtl/ext/rms_norm/rms_norm.sv:7), applied when ``rms_weight`` is given
  (sw/attn_driver.py:562); the B200 contract fixes its rounding: fp64 mean,
  ``inv`` rounded once to fp32, ``fp32(fp32(x * inv) * gamma)`` -> bf16;
* ``qkv_project``: ``Q = X @ Wq``, ``K = X @ Wk``, ``V = X @ Wv`` with weights
  stored ``[IN_DIM][OUT_DIM]`` (hw/rtl/ext/qkv_projection/qkv_projection.sv:
  8-10,32-35);
* ``reshape_to_heads``: ``[L, H*D] -> [H, L, D]`` (sw/attn_driver.py:571,580);
* ``apply_rope``: dims (2i, 2i+1) rotate by ``pos * theta_i``,
  ``theta_i = base^(-2i/D)``, ``pos = position_base + t``
  (hw/rtl/core/rope_engine.sv:1-11; sw/attn_driver.py:572-577), on q and k,
  not v.

The B200 path's operand precision (bf16 activations and weights, fp32
accumulation, bf16 outputs) is mirrored: x, rms_weight and W are bf16 words,
x_n is rounded to bf16 once before the projection, the projection sums in
float64 (the GPU's fp32 accumulation differs from it far below a bf16 ulp),
the RoPE rotation runs in float32 with cos/sin of the float32 angle, and the
returned q/k/v are float32 values (callers round them with
``fp32_to_bf16_u16`` for the parity check).
"""

from __future__ import annotations

import numpy as np

from .attention import bf16_u16_to_fp32, fp32_to_bf16_u16


def rope_theta(head_dim: int = 128, base: float = 10000.0) -> np.ndarray:
    """theta_i = base^(-2i/D) as float32 (hw/data/rope_theta.hex holds these for base 10000)."""
    i = np.arange(head_dim // 2, dtype=np.float64)
    return np.power(float(base), -2.0 * i / head_dim).astype(np.float32)


def rms_norm(x_words: np.ndarray, w_words: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """bf16 words [L, H] -> bf16 words of fp32(fp32(x * inv) * gamma), inv = fp32(1/sqrt(mean(x^2) + eps)).

    The mean is taken in float64 and ``inv`` rounded once to float32, so the
    statistic (and hence every x_n word) is reproducible across summation orders.
    """
    x = bf16_u16_to_fp32(x_words)
    g = bf16_u16_to_fp32(w_words)
    x64 = x.astype(np.float64)
    eps32 = float(np.float32(eps))
    inv = (1.0 / np.sqrt(np.mean(x64 * x64, axis=-1, keepdims=True) + eps32)).astype(np.float32)
    return fp32_to_bf16_u16((x * inv).astype(np.float32) * g)


def apply_rope(x: np.ndarray, position_base: int, base: float = 10000.0) -> np.ndarray:
    """x float32 [..., L, D]: rotate dim pairs (2i, 2i+1) of token t by (position_base + t) * theta_i."""
    L, D = x.shape[-2], x.shape[-1]
    theta = rope_theta(D, base)
    pos = (np.arange(L, dtype=np.int64) + int(position_base)).astype(np.float32)
    ang = (pos[:, None] * theta[None, :]).astype(np.float32)  # fp32 product, as on the device
    c = np.cos(ang.astype(np.float64)).astype(np.float32)
    s = np.sin(ang.astype(np.float64)).astype(np.float32)
    a, b = x[..., 0::2], x[..., 1::2]
    out = np.empty_like(x, dtype=np.float32)
    out[..., 0::2] = a * c - b * s
    out[..., 1::2] = a * s + b * c
    return out


def layer_prologue(x_words, w_qkv_words, rms_words=None, *, n_q_heads=32, n_kv_heads=8, head_dim=128,
                   q_pos_base=0, kv_pos_base=0, rms_eps=1e-5, rope_base=10000.0):
    """x [L, H], w_qkv [H, (Hq + 2 Hkv) D], rms [H] (bf16 words) -> float32 q [Hq,L,D], k, v [Hkv,L,D]."""
    xn = x_words if rms_words is None else rms_norm(x_words, rms_words, rms_eps)
    y = bf16_u16_to_fp32(xn).astype(np.float64) @ bf16_u16_to_fp32(w_qkv_words).astype(np.float64)
    y = y.astype(np.float32)
    L = y.shape[0]
    nq, nkv = n_q_heads * head_dim, n_kv_heads * head_dim
    q = y[:, :nq].reshape(L, n_q_heads, head_dim).transpose(1, 0, 2)
    k = y[:, nq:nq + nkv].reshape(L, n_kv_heads, head_dim).transpose(1, 0, 2)
    v = y[:, nq + nkv:].reshape(L, n_kv_heads, head_dim).transpose(1, 0, 2)
    return (apply_rope(np.ascontiguousarray(q), q_pos_base, rope_base),
            apply_rope(np.ascontiguousarray(k), kv_pos_base, rope_base), np.ascontiguousarray(v))
