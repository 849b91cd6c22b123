"""Parity helpers shared by the GPU tests.

The tolerance is the one BASELINE.json's north star states: the GPU output
may differ from the golden model's result (the CPU oracle's fp32 output,
rounded to bf16 with the reference packer) by at most 2 bf16 ulp.  The ulp is
taken at the magnitude of each golden element, floored at 2**-8 of the
largest magnitude in the same output vector (one query head's D values):
near-zero elements produced by cancellation carry an fp32 rounding error that
scales with the vector, not with the element, and both the golden model and
the kernel accumulate in fp32 in different orders.  The strict per-element
count (no floor) is returned too, for reporting.
"""

from __future__ import annotations

import numpy as np

import oracle

ULPS = 2.0
FLOOR_FRAC = 2.0 ** -8


def _ulp_at(mag: np.ndarray) -> np.ndarray:
    m = np.maximum(np.asarray(mag, dtype=np.float64), 2.0 ** -126)
    e = np.floor(np.log2(m))
    return np.ldexp(1.0, (e - 7).astype(np.int64))


def bf16_error(actual_words: np.ndarray, golden_fp: np.ndarray) -> dict:
    """Error of bf16 ``actual_words`` against golden values (fp32 or fp64)."""
    golden_words = oracle.fp32_to_bf16_u16(np.asarray(golden_fp, dtype=np.float32))
    g = oracle.bf16_u16_to_fp32(golden_words).astype(np.float64)
    a = oracle.bf16_u16_to_fp32(np.asarray(actual_words, dtype=np.uint16)).astype(np.float64)
    err = np.abs(a - g)
    row_max = np.max(np.abs(g), axis=-1, keepdims=True)
    floored = _ulp_at(np.maximum(np.abs(g), FLOOR_FRAC * row_max))
    strict = _ulp_at(np.abs(g))
    return {
        "max_ulp": float(np.max(err / floored)) if err.size else 0.0,
        "max_ulp_strict": float(np.max(err / strict)) if err.size else 0.0,
        "n_over_2ulp_strict": int(np.count_nonzero(err > ULPS * strict)),
        "n": int(err.size),
        "finite": bool(np.all(np.isfinite(a))),
    }


def assert_bf16_parity(actual_words, golden_fp32, fp64=None, what="") -> dict:
    """Assert <= 2 bf16 ulp vs the golden fp32 result (and vs fp64 if given)."""
    e = bf16_error(actual_words, golden_fp32)
    assert e["finite"], f"{what}: non-finite output"
    assert e["max_ulp"] <= ULPS, f"{what}: {e}"
    if fp64 is not None:
        e64 = bf16_error(actual_words, fp64)
        assert e64["max_ulp"] <= ULPS, f"{what} vs fp64: {e64}"
        e["fp64"] = e64
    return e


def words_of(t) -> np.ndarray:
    """bf16 torch tensor (any 16-bit dtype) -> numpy uint16 words on the host."""
    import torch

    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
