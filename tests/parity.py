"""Parity assertions shared by the GPU tests.

Two criteria, both defined in ``oracle.attention.bf16_parity_error``:

* golden: the GPU output may differ from the golden model's result -- the CPU
  oracle's fp32 output rounded to bf16 with the reference packer -- by at
  most ``oracle.PARITY_ULPS`` = 2 bf16 ulp per element, the ulp taken at the
  element's magnitude floored at ``oracle.PARITY_FLOOR_FRAC`` = 2**-8 of the
  largest magnitude of the same head vector.  The strict (unfloored) figures
  ``max_ulp_strict`` / ``n_over_strict`` are reported beside it.
* fp64-anchored (whenever the fp64 reference is given): for every element
  ``|gpu - fp64| <= 2 * ulp(fp64) + |golden_bf16 - fp64|`` with the ulp at the
  element's own magnitude, no floor -- never more than 2 ulp worse than the
  golden model's own bf16 result.  This is the bound that covers near-zero
  elements, where the floored ulp is loose.
"""

from __future__ import annotations

import numpy as np

import oracle


def bf16_error(actual_words, golden, fp64=None) -> dict:
    return oracle.bf16_parity_error(actual_words, golden, fp64)


def assert_bf16_parity(actual_words, golden_fp32, fp64=None, what="") -> dict:
    """Assert <= 2 bf16 ulp vs the golden fp32 result and, given ``fp64``, the
    fp64-anchored bound; the message carries every figure of the report."""
    e = oracle.bf16_parity_error(actual_words, golden_fp32, fp64)
    assert e["finite"], f"{what}: non-finite output {e}"
    assert e["max_ulp"] <= oracle.PARITY_ULPS, f"{what}: {e}"
    if fp64 is not None:
        assert e["n_over_anchored"] == 0, f"{what}: fp64-anchored bound exceeded: {e}"
    return e


def words_of(t) -> np.ndarray:
    """bf16 torch tensor (any 16-bit dtype) -> numpy uint16 words on the host."""
    import torch

    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
