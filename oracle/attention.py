"""NumPy restatement of LARA's CPU attention path -- TEST INFRASTRUCTURE ONLY.

This module is the checker for the CUDA kernels in ``lara_b200``; it is never
on the product path.  Every function names the reference code it restates
(paths relative to the LARA source tree).

* ``fp32_to_bf16_u16`` / ``bf16_u16_to_fp32`` restate ``sw/attn_driver.py:88-103``
  with the same integer operations, so the packing is bit-identical.
* ``cpu_attention_numpy`` restates ``sw/board_performance.py:158-192`` with the
  same NumPy operations in the same order (u16->fp32 by shift, fp32 matmul,
  multiply by ``float32(1/sqrt(D))``, ``-inf`` mask, max-subtract, ``np.exp``,
  divide by the row sum, matmul by V).  With the default geometry (32/8/128)
  it reproduces the reference's output bit-for-bit (pinned by
  ``tests/golden``).  The geometry is a parameter instead of module globals.
* ``decode_attention`` / ``prefill_attention`` apply the same per-group
  operations to the B200 KV-cache layout ``[B, Hkv, Lmax, D]``: a decode query
  sits at position ``len-1`` and sees every cached token (no mask, as in the
  reference's non-causal mode); a prefill chunk uses the reference's causal
  rule ``kv_pos <= q_pos`` (``sw/board_performance.py:174-177``).
* A row with no valid key produces zeros, the convention of the RTL output
  normaliser (``hw/rtl/mem/output_buffer.sv:271-286``: l == 0 -> 0); the
  reference's CPU function raises instead, and ``cpu_attention_numpy`` keeps
  that behaviour.
"""

from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------
# bf16 packing (sw/attn_driver.py:88-103)
# ---------------------------------------------------------------------------


def fp32_to_bf16_u16(values: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 words, round-to-nearest-even; uint16 input passes through.

    Restates ``sw/attn_driver.py:88-98``: round up when the dropped half-word
    is above one half, or exactly one half with an odd kept LSB; the carry is
    added to the full 32-bit word before truncation.
    """
    arr = np.asarray(values)
    if arr.dtype == np.uint16:
        return np.ascontiguousarray(arr)
    bits = np.asarray(arr, dtype=np.float32).view(np.uint32).copy()
    low = bits & np.uint32(0xFFFF)
    half_bit = (low >> np.uint32(15)) & np.uint32(1)
    sticky_or_odd = ((bits >> np.uint32(16)) & np.uint32(1)) | (low & np.uint32(0x7FFF) != 0).astype(np.uint32)
    carry = (half_bit & sticky_or_odd).astype(np.uint32)
    bits = (bits + carry) & np.uint32(0xFFFF0000)
    return np.ascontiguousarray((bits >> np.uint32(16)).astype(np.uint16))


def bf16_u16_to_fp32(values: np.ndarray) -> np.ndarray:
    """bf16 words -> fp32 by a 16-bit left shift (``sw/attn_driver.py:101-103``)."""
    words = np.asarray(values, dtype=np.uint16)
    return (words.astype(np.uint32) << np.uint32(16)).view(np.float32)


def bf16_ulp(words: np.ndarray) -> np.ndarray:
    """Size of one bf16 unit in the last place at each bf16 value (as fp32).

    bf16 keeps 7 stored mantissa bits, so a normal value with biased exponent
    ``e`` has ulp ``2**(e-127-7)``; zero and subnormals use ``2**-133``.
    """
    w = np.asarray(words, dtype=np.uint16).astype(np.int64)
    exp = (w >> 7) & 0xFF
    exp = np.maximum(exp, 1)
    return np.ldexp(np.float64(1.0), (exp - 127 - 7)).astype(np.float64)


def ulp_distance(actual_words: np.ndarray, expected_words: np.ndarray) -> np.ndarray:
    """|actual - expected| measured in bf16 ulps of ``expected`` (float64)."""
    a = bf16_u16_to_fp32(actual_words).astype(np.float64)
    e = bf16_u16_to_fp32(expected_words).astype(np.float64)
    return np.abs(a - e) / bf16_ulp(expected_words)


# Parity tolerance of the B200 kernels (<= 2 bf16 ulp of
# the golden model's result).  The ulp is taken at each golden element's
# magnitude, floored at 2**-8 of the largest magnitude in the same output
# vector (the last axis: one query head's D values), because near-zero
# elements produced by cancellation carry an fp32 rounding error that scales
# with the vector, and the golden model and the kernel both accumulate in
# fp32, in different orders.
PARITY_ULPS = 2.0
PARITY_FLOOR_FRAC = 2.0 ** -8
# The tensor-core kernels (tcgen05 decode for large groups, the prefill)
# feed P.V with each probability written as P_hi + P_lo, two bf16 words:
# |p - P_hi - P_lo| <= 2^-9 |P_lo| <= 2^-18 p.  Their P.V sum can therefore
# differ from an fp32 evaluation by up to 2^-18 * kappa (kappa = sum_j
# p_j |v_j| / l), on top of the fp32 accumulation both share.
TC_SPLIT_P_KAPPA = 2.0 ** -18


def _ulp_at(mag: np.ndarray) -> np.ndarray:
    m = np.maximum(np.asarray(mag, dtype=np.float64), 2.0 ** -126)
    return np.ldexp(1.0, (np.floor(np.log2(m)) - 7).astype(np.int64))


def bf16_parity_error(actual_words: np.ndarray, golden: np.ndarray, fp64: np.ndarray | None = None,
                      kappa_allowance: float = 0.0) -> dict:
    """Error of bf16 words against golden values (fp32 or fp64), in bf16 ulp.

    ``max_ulp`` uses the floored ulp above (the pass criterion is
    ``max_ulp <= PARITY_ULPS``); ``max_ulp_strict`` uses no floor and
    ``n_over_strict`` counts elements more than ``PARITY_ULPS`` strict ulp
    from the golden word.

    ``fp64`` is the same attention evaluated in float64 (the error reference
    of ``sw/board_performance.py:207-219``), as returned by the ``*_fp64``
    functions: ``[..., 2]`` holding each element's value ``t`` and the
    condition of its weighted sum ``kappa = sum_j p_j |v_j| / l`` (a plain
    array of values is taken with kappa = 0).  The fp64-anchored criterion is
    then evaluated for every element, with the ulp taken at the element's own
    fp64 magnitude (no floor):

        |actual - t| <= PARITY_ULPS * ulp(t) + max(|golden_bf16 - t|, eps_g * kappa)

    ``eps_g`` is the golden model's own largest fp32 error relative to kappa
    over the checked elements (``max |golden_fp32 - t| / kappa``): an fp32
    evaluation in another summation order has errors of the same size as the
    golden's, spread over different elements, and near an element produced by
    cancellation (|t| << kappa) that size is set by kappa, not by |t|.  So the
    kernel must be no more than 2 ulp worse than the golden model's own bf16
    result and its own error scale on the same inputs.  ``kappa_allowance``
    adds ``kappa_allowance * kappa`` to the bound for a kernel whose arithmetic
    differs from fp32 by a known amount (``TC_SPLIT_P_KAPPA`` for the
    tensor-core kernels' split P).  Reported:
    ``anchored_ratio`` (largest left/right quotient, pass <= 1),
    ``n_over_anchored``, ``eps_golden_u`` (eps_g in units of 2^-24),
    ``excess_kappa_u`` (the largest amount by which an element exceeds
    ``2 ulp(t) + |golden_bf16 - t|``, in units of 2^-24 kappa: the allowance a
    failing path would need), ``n_over_plain`` (elements above the bound
    without the eps_g term), and the kernel's and the golden model's largest
    strict-ulp distance from t.
    """
    golden32 = np.asarray(golden, dtype=np.float32)
    golden_words = fp32_to_bf16_u16(golden32)
    g = bf16_u16_to_fp32(golden_words).astype(np.float64)
    a = bf16_u16_to_fp32(np.asarray(actual_words, dtype=np.uint16)).astype(np.float64)
    err = np.abs(a - g)
    if err.size == 0:
        out = {"max_ulp": 0.0, "max_ulp_strict": 0.0, "n_over_strict": 0, "n": 0, "finite": True}
        if fp64 is not None:
            out.update({"anchored_ratio": 0.0, "n_over_anchored": 0, "n_over_plain": 0, "eps_golden_u": 0.0,
                        "excess_kappa_u": 0.0, "max_ulp_fp64_strict": 0.0, "golden_max_ulp_fp64_strict": 0.0})
        return out
    row_max = np.max(np.abs(g), axis=-1, keepdims=True)
    floored = _ulp_at(np.maximum(np.abs(g), PARITY_FLOOR_FRAC * row_max))
    strict = _ulp_at(np.abs(g))
    out = {
        "max_ulp": float(np.max(err / floored)),
        "max_ulp_strict": float(np.max(err / strict)),
        "n_over_strict": int(np.count_nonzero(err > PARITY_ULPS * strict)),
        "n": int(err.size),
        "finite": bool(np.all(np.isfinite(a))),
    }
    if fp64 is not None:
        f = np.asarray(fp64, dtype=np.float64)
        if f.shape == a.shape + (2,):
            t, kap = f[..., 0], f[..., 1]
        else:
            t, kap = f, np.zeros_like(f)
        u = 2.0 ** -24
        ulp_t = _ulp_at(np.abs(t))
        a_err = np.abs(a - t)
        g_err = np.abs(g - t)
        g32_err = np.abs(golden32.astype(np.float64) - t)
        pos = kap > 0
        eps_g = float(np.max(g32_err[pos] / kap[pos])) if np.any(pos) else 0.0
        plain = PARITY_ULPS * ulp_t + g_err
        bound = PARITY_ULPS * ulp_t + np.maximum(g_err, eps_g * kap) + kappa_allowance * kap
        ratio = np.where(np.isnan(a_err), np.inf, a_err / bound)
        excess = np.where(pos, np.maximum(a_err - plain, 0.0) / np.where(pos, kap, 1.0) / u, 0.0)
        out.update({
            "kappa_allowance_u": round(kappa_allowance / u, 3),
            "anchored_ratio": float(np.max(ratio)),
            "n_over_anchored": int(np.count_nonzero(ratio > 1.0)),
            "n_over_plain": int(np.count_nonzero(a_err > plain)),
            "eps_golden_u": round(eps_g / u, 3),
            "excess_kappa_u": round(float(np.max(excess)), 3),
            "max_ulp_fp64_strict": float(np.max(a_err / ulp_t)),
            "golden_max_ulp_fp64_strict": float(np.max(g_err / ulp_t)),
        })
    return out


# ---------------------------------------------------------------------------
# attention restatements
# ---------------------------------------------------------------------------


def cpu_attention_numpy(
    q: np.ndarray,
    k: np.ndarray,
    v: np.ndarray,
    *,
    causal: bool,
    q_pos_base: int,
    kv_pos_base: int,
    n_q_heads: int = 32,
    n_kv_heads: int = 8,
    head_dim: int = 128,
) -> np.ndarray:
    """Stable-softmax GQA attention, bf16 inputs, fp32 compute.

    Restates ``sw/board_performance.py:158-192`` operation for operation; the
    head geometry is an argument instead of the module constants.  Inputs are
    head-major bf16 words ``q[Hq, L, D]``, ``k/v[Hkv, L, D]``; returns fp32
    ``[Hq, L, D]``.
    """
    group = n_q_heads // n_kv_heads
    qf = bf16_u16_to_fp32(q)
    kf = bf16_u16_to_fp32(k)
    vf = bf16_u16_to_fp32(v)
    length = q.shape[1]
    output = np.empty((n_q_heads, length, head_dim), dtype=np.float32)
    valid = None
    if causal:
        q_positions = q_pos_base + np.arange(length)
        kv_positions = kv_pos_base + np.arange(length)
        valid = kv_positions[np.newaxis, :] <= q_positions[:, np.newaxis]
        if not np.all(np.any(valid, axis=1)):
            raise ValueError("causal workload contains a query with no valid K/V position")
    scale = np.float32(1.0 / np.sqrt(head_dim))
    for g in range(n_kv_heads):
        first = g * group
        q_group = qf[first:first + group]
        scores = np.matmul(q_group, kf[g].T) * scale
        if valid is not None:
            scores = np.where(valid[np.newaxis, :, :], scores, -np.inf)
        scores -= np.max(scores, axis=-1, keepdims=True)
        np.exp(scores, out=scores)
        scores /= np.sum(scores, axis=-1, keepdims=True)
        output[first:first + group] = np.matmul(scores, vf[g])
    return output


def dense_attention_fp64(q: np.ndarray, k: np.ndarray, v: np.ndarray, *, causal: bool, q_pos_base: int,
                         kv_pos_base: int, n_q_heads: int = 32, n_kv_heads: int = 8,
                         head_dim: int = 128, kappa: bool = True) -> np.ndarray:
    """``cpu_attention_numpy``'s transaction evaluated in float64 (the error reference).

    Same inputs, head map ``h // G``, scale and causal rule ``kv_pos <= q_pos``
    (``sw/board_performance.py:174-191``); rows without a visible key give
    zeros.  Returns float64 ``[Hq, L, D, 2]`` (value, condition; see
    ``decode_attention_fp64``), or ``[Hq, L, D]`` with ``kappa=False``."""
    group = n_q_heads // n_kv_heads
    length = q.shape[1]
    mask = None
    if causal:
        qp = q_pos_base + np.arange(length)
        kp = kv_pos_base + np.arange(length)
        mask = kp[np.newaxis, :] <= qp[:, np.newaxis]
    out = np.empty((n_q_heads, length, head_dim, 2) if kappa else (n_q_heads, length, head_dim), dtype=np.float64)
    sc = np.float64(1.0 / np.sqrt(head_dim))
    for g in range(n_kv_heads):
        qf = bf16_u16_to_fp32(q[g * group:(g + 1) * group]).astype(np.float64)
        kf = bf16_u16_to_fp32(k[g]).astype(np.float64)
        vf = bf16_u16_to_fp32(v[g]).astype(np.float64)
        out[g * group:(g + 1) * group] = _group_attention(qf, kf, vf, sc, mask, kappa=kappa)
    return out


def _group_attention(qf: np.ndarray, kf: np.ndarray, vf: np.ndarray, scale, mask=None, kappa: bool = False):
    """One GQA group, the operation order of ``board_performance.py:185-191``.

    ``qf[G, Lq, D]`` (or ``[G, D]``), ``kf/vf[L, D]``; ``mask[Lq, L]`` marks valid
    keys.  Rows without any valid key return zeros.  With ``kappa`` the result
    is stacked with the weighted sum's condition ``sum_j p_j |v_j| / l`` along
    a new last axis (``[..., D, 2]``).
    """
    scores = np.matmul(qf, kf.T) * scale
    if mask is not None:
        scores = np.where(mask, scores, -np.inf)
    row_max = np.max(scores, axis=-1, keepdims=True)
    dead = ~np.isfinite(row_max)
    row_max = np.where(dead, np.zeros_like(row_max), row_max)
    scores -= row_max
    np.exp(scores, out=scores)
    denom = np.sum(scores, axis=-1, keepdims=True)
    scores /= np.where(denom == 0, np.ones_like(denom), denom)
    out = np.matmul(scores, vf)
    if np.any(dead):
        out = np.where(dead, np.zeros_like(out), out)
    if kappa:
        cond = np.matmul(scores, np.abs(vf))
        if np.any(dead):
            cond = np.where(dead, np.zeros_like(cond), cond)
        out = np.stack([out, cond], axis=-1)
    return out


def decode_attention(
    q: np.ndarray,
    k_cache: np.ndarray,
    v_cache: np.ndarray,
    lens: np.ndarray,
    *,
    scale: float | None = None,
    dtype=np.float32,
    pairs=None,
    kappa: bool = False,
) -> np.ndarray:
    """One decode step over a KV cache.

    ``q[B, Hq, D]`` bf16 words, ``k_cache/v_cache[B, Hkv, Lmax, D]`` bf16
    words, ``lens[B]`` valid tokens per sequence.  The query of sequence ``b``
    attends to tokens ``0..lens[b]-1`` (it sits at position ``lens[b]-1``, so
    every cached token is visible).  Returns ``[B, Hq, D]`` in ``dtype``
    (float32 is the golden model, float64 the error reference).  ``pairs``
    optionally restricts the work to a list of ``(b, kv_head)``; other rows are
    left as NaN.
    """
    B, Hq, D = q.shape
    Hkv = k_cache.shape[1]
    G = Hq // Hkv
    sc = dtype(1.0 / np.sqrt(D)) if scale is None else dtype(scale)
    out = np.full((B, Hq, D, 2) if kappa else (B, Hq, D), np.nan, dtype=dtype)
    todo = pairs if pairs is not None else [(b, h) for b in range(B) for h in range(Hkv)]
    for b, h in todo:
        n = int(lens[b])
        if n <= 0:
            out[b, h * G:(h + 1) * G] = 0
            continue
        qf = bf16_u16_to_fp32(q[b, h * G:(h + 1) * G]).astype(dtype)
        kf = bf16_u16_to_fp32(k_cache[b, h, :n]).astype(dtype)
        vf = bf16_u16_to_fp32(v_cache[b, h, :n]).astype(dtype)
        out[b, h * G:(h + 1) * G] = _group_attention(qf, kf, vf, sc, kappa=kappa)
    return out


def decode_attention_fp64(q, k_cache, v_cache, lens, *, scale=None, pairs=None, kappa: bool = True) -> np.ndarray:
    """``decode_attention`` in float64: the error reference for parity reports.

    By default the result carries the condition of each output element along
    a last axis of 2 (``[..., 0]`` the value, ``[..., 1]`` ``sum_j p_j|v_j|/l``),
    the form ``bf16_parity_error`` takes as its ``fp64`` argument."""
    return decode_attention(q, k_cache, v_cache, lens, scale=scale, dtype=np.float64, pairs=pairs, kappa=kappa)


def prefill_attention(
    q: np.ndarray,
    k_cache: np.ndarray,
    v_cache: np.ndarray,
    kv_lens: np.ndarray,
    q_pos_base,
    *,
    causal: bool = True,
    scale: float | None = None,
    dtype=np.float32,
    kv_pos_base: int = 0,
    kappa: bool = False,
) -> np.ndarray:
    """A chunk of ``Lq`` queries per sequence over the cache (cache + self).

    ``q[B, Hq, Lq, D]``; query ``i`` of sequence ``b`` has absolute position
    ``q_pos_base[b] + i``; cached token ``j`` has position ``kv_pos_base + j``
    for ``j < kv_lens[b]``.  With ``causal`` a key is valid when
    ``kv_pos <= q_pos`` (``sw/board_performance.py:174-177``).
    """
    B, Hq, Lq, D = q.shape
    Hkv = k_cache.shape[1]
    G = Hq // Hkv
    qpb = np.broadcast_to(np.asarray(q_pos_base), (B,))
    sc = dtype(1.0 / np.sqrt(D)) if scale is None else dtype(scale)
    out = np.zeros((B, Hq, Lq, D, 2) if kappa else (B, Hq, Lq, D), dtype=dtype)
    for b in range(B):
        n = int(kv_lens[b])
        if n <= 0:
            continue
        mask = None
        if causal:
            qp = int(qpb[b]) + np.arange(Lq)
            kp = kv_pos_base + np.arange(n)
            mask = kp[np.newaxis, :] <= qp[:, np.newaxis]
        for h in range(Hkv):
            qf = bf16_u16_to_fp32(q[b, h * G:(h + 1) * G]).astype(dtype)
            kf = bf16_u16_to_fp32(k_cache[b, h, :n]).astype(dtype)
            vf = bf16_u16_to_fp32(v_cache[b, h, :n]).astype(dtype)
            out[b, h * G:(h + 1) * G] = _group_attention(qf, kf, vf, sc, mask, kappa=kappa)
    return out


def decode_partial(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, lens: np.ndarray, *,
                   scale: float | None = None):
    """Unnormalised partial state of a decode over a token slice.

    Same quantities as the kernel's partial-output mode: per (b, h) row,
    ``m = max_j s_j`` and ``l = sum_j 2^(s_j - m)``, ``acc = sum_j 2^(s_j - m) v_j``
    with ``s_j = scale * log2(e) * q.k_j`` (fp32); an empty slice gives
    ``m = -inf, l = 0, acc = 0``.  Returns ``ml[B*Hq, 2]``, ``acc[B*Hq, D]``.
    """
    B, Hq, D = q.shape
    Hkv = k_cache.shape[1]
    G = Hq // Hkv
    sc = np.float32((1.0 / np.sqrt(D) if scale is None else scale) * np.log2(np.e))
    ml = np.zeros((B * Hq, 2), np.float32)
    acc = np.zeros((B * Hq, D), np.float32)
    for b in range(B):
        n = int(lens[b])
        for h in range(Hkv):
            rows = slice(b * Hq + h * G, b * Hq + (h + 1) * G)
            if n <= 0:
                ml[rows, 0] = -np.inf
                continue
            qf = bf16_u16_to_fp32(q[b, h * G:(h + 1) * G])
            kf = bf16_u16_to_fp32(k_cache[b, h, :n])
            vf = bf16_u16_to_fp32(v_cache[b, h, :n])
            s = np.matmul(qf, kf.T) * sc
            m = np.max(s, axis=-1, keepdims=True)
            p = np.exp2(s - m)
            ml[rows, 0] = m[:, 0]
            ml[rows, 1] = np.sum(p, axis=-1)
            acc[rows] = np.matmul(p, vf)
    return ml, acc


def lse_combine(mls: np.ndarray, accs: np.ndarray) -> np.ndarray:
    """Merge partial states ``mls[P, rows, 2]``, ``accs[P, rows, D]`` -> fp32 ``[rows, D]``.

    M = max m_i, L = sum l_i 2^(m_i - M), O = sum acc_i 2^(m_i - M) / L; rows
    with L == 0 give zeros (``hw/rtl/mem/output_buffer.sv:271-286``)."""
    m = mls[..., 0]
    M = np.max(m, axis=0)
    Mu = np.where(np.isfinite(M), M, 0.0).astype(np.float32)
    w = np.exp2(m - Mu[None])
    L = np.sum(mls[..., 1] * w, axis=0)
    O = np.sum(accs * w[..., None], axis=0)
    return np.where(L[:, None] > 0, O / np.where(L > 0, L, 1)[:, None], 0).astype(np.float32)


# ---------------------------------------------------------------------------
# reports and counts
# ---------------------------------------------------------------------------


def numeric_error(actual: np.ndarray, reference: np.ndarray) -> dict:
    """Error metrics of ``sw/board_performance.py:207-219`` (same keys)."""
    a = np.asarray(actual, dtype=np.float64)
    r = np.asarray(reference, dtype=np.float64)
    delta = a - r
    denom = np.maximum(np.abs(r), 1.0e-6)
    ref_rms = float(np.sqrt(np.mean(r * r)))
    return {
        "max_abs": float(np.max(np.abs(delta))),
        "mean_abs": float(np.mean(np.abs(delta))),
        "rmse": float(np.sqrt(np.mean(delta * delta))),
        "normalized_rmse": float(np.sqrt(np.mean(delta * delta)) / max(ref_rms, 1.0e-12)),
        "max_relative_floor_1e-6": float(np.max(np.abs(delta) / denom)),
    }


def valid_pairs(seq_len: int, causal: bool, q_pos_base: int = 0, kv_pos_base: int = 0) -> int:
    """Valid (query, key) pairs per head (``sw/board_performance.py:222-227``)."""
    if not causal:
        return seq_len * seq_len
    qp = q_pos_base + np.arange(seq_len)
    kp = kv_pos_base + np.arange(seq_len)
    return int(np.count_nonzero(kp[np.newaxis, :] <= qp[:, np.newaxis]))


def tile_pairs_per_head(seq_len: int, causal: bool, q_pos_base: int = 0, kv_pos_base: int = 0,
                        tile_q: int = 32, tile_kv: int = 64) -> int:
    """Q-tile x KV-tile pairs visited per head with causal tile skipping.

    Restates ``sw/benchmark.py:36-57`` (the traversal of
    ``hw/rtl/core/attn_core.sv:138-153``).
    """
    n_q = -(-seq_len // tile_q)
    n_kv = -(-seq_len // tile_kv)
    if not causal:
        return n_q * n_kv
    pairs = 0
    for qt in range(n_q):
        rows = min(tile_q, seq_len - qt * tile_q)
        q_end = q_pos_base + qt * tile_q + rows - 1
        last = 0 if q_end < kv_pos_base else min((q_end - kv_pos_base) // tile_kv, n_kv - 1)
        pairs += last + 1
    return pairs
