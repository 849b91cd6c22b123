"""Parity assertions shared by the GPU tests.

Tolerance (defined in ``oracle.attention``): the GPU output may differ from
the golden model's result -- the CPU oracle's fp32 output rounded to bf16 with
the reference packer -- by at most ``oracle.PARITY_ULPS`` = 2 bf16 ulp per
element, the ulp taken at the element's magnitude floored at
``oracle.PARITY_FLOOR_FRAC`` = 2**-8 of the largest magnitude of the same head
vector; the same bound is checked against the fp64 reference.
"""

from __future__ import annotations

import numpy as np

import oracle


def bf16_error(actual_words, golden) -> dict:
    return oracle.bf16_parity_error(actual_words, golden)


def assert_bf16_parity(actual_words, golden_fp32, fp64=None, what="") -> dict:
    """Assert <= 2 bf16 ulp vs the golden fp32 result (and vs fp64 if given)."""
    e = oracle.bf16_parity_error(actual_words, golden_fp32)
    assert e["finite"], f"{what}: non-finite output"
    assert e["max_ulp"] <= oracle.PARITY_ULPS, f"{what}: {e}"
    if fp64 is not None:
        e64 = oracle.bf16_parity_error(actual_words, fp64)
        assert e64["max_ulp"] <= oracle.PARITY_ULPS, f"{what} vs fp64: {e64}"
        e["fp64"] = e64
    return e


def words_of(t) -> np.ndarray:
    """bf16 torch tensor (any 16-bit dtype) -> numpy uint16 words on the host."""
    import torch

    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
