"""Parity assertions shared by the GPU tests.

Two criteria, both defined in ``oracle.attention.bf16_parity_error``:

* golden: the GPU output may differ from the golden model's result -- the CPU
  oracle's fp32 output rounded to bf16 with the reference packer -- by at
  most ``oracle.PARITY_ULPS`` = 2 bf16 ulp per element, the ulp taken at the
  element's magnitude floored at ``oracle.PARITY_FLOOR_FRAC`` = 2**-8 of the
  largest magnitude of the same head vector.  The strict (unfloored) figures
  ``max_ulp_strict`` / ``n_over_strict`` are reported beside it.
* fp64-anchored (whenever the fp64 reference is given): for every element
  ``|gpu - t| <= 2 ulp(t) + max(|golden_bf16 - t|, eps_g * kappa)`` with t the
  fp64 value, the ulp at the element's own magnitude (no floor), kappa the
  condition ``sum_j p_j |v_j| / l`` of its weighted sum and eps_g the golden
  model's own largest fp32 error relative to kappa on the same inputs.  The
  tensor-core kernels add ``oracle.TC_SPLIT_P_KAPPA * kappa`` (2^-18 kappa,
  the representation error of their split P) to the bound; the CUDA-core
  kernels keep P in fp32 and get no allowance.
"""

from __future__ import annotations

import json
import os

import numpy as np

import oracle


def bf16_error(actual_words, golden, fp64=None) -> dict:
    return oracle.bf16_parity_error(actual_words, golden, fp64)


def _log(what: str, e: dict) -> None:
    """Append the report to the JSON-lines file named by LARA_PARITY_LOG (if set)."""
    path = os.environ.get("LARA_PARITY_LOG")
    if path:
        with open(path, "a") as fh:
            fh.write(json.dumps({"test": os.environ.get("PYTEST_CURRENT_TEST", ""), "what": what, **e}) + "\n")


def decode_on_tensor_cores(n_q_heads: int, n_kv_heads: int, head_dim: int) -> bool:
    """True when the decode of this geometry runs on the tcgen05 kernel (the
    library's own choice, LARA_DECODE_PATH included)."""
    from lara_b200 import ops

    return ops.decode_kernel(n_q_heads, n_kv_heads, head_dim) == "tensor"


def prefill_on_tensor_cores(n_q_heads: int, n_kv_heads: int, head_dim: int) -> bool:
    """True when prefill / dense attention of this geometry runs on a tcgen05
    kernel: the prefill kernel for head_dim 128 unless LARA_ATTN_PATH=stream,
    otherwise the decode kernels' choice."""
    if os.environ.get("LARA_ATTN_PATH") != "stream" and head_dim == 128:
        return True
    return decode_on_tensor_cores(n_q_heads, n_kv_heads, head_dim)


def assert_bf16_parity(actual_words, golden_fp32, fp64=None, what="", tensor_core=False) -> dict:
    """Assert <= 2 bf16 ulp vs the golden fp32 result and, given ``fp64``, the
    fp64-anchored bound (with the split-P allowance when ``tensor_core``); the
    message carries every figure of the report."""
    e = oracle.bf16_parity_error(actual_words, golden_fp32, fp64,
                                 oracle.TC_SPLIT_P_KAPPA if tensor_core else 0.0)
    _log(what, e)
    assert e["finite"], f"{what}: non-finite output {e}"
    assert e["max_ulp"] <= oracle.PARITY_ULPS, f"{what}: {e}"
    if fp64 is not None:
        assert e["n_over_anchored"] == 0, f"{what}: fp64-anchored bound exceeded: {e}"
    return e


def words_of(t) -> np.ndarray:
    """bf16 torch tensor (any 16-bit dtype) -> numpy uint16 words on the host."""
    import torch

    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
