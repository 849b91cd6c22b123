"""LARA B200: the grouped-query streaming-attention path on sm_100a.

* ``lara_b200.attn_driver`` -- drop-in for the reference host driver
  (``sw/attn_driver.py``), backed by the C-ABI context of liblara_b200.so.
* ``lara_b200.ops`` -- torch-tensor front end of the stateless kernels
  (decode, split-KV partials + LSE combine, KV append, bf16 pack, dense
  transaction, prefill).
* ``lara_b200.parallel`` -- one process per GPU: batch/KV-head sharding and
  split-KV across GPUs (NCCL all-gather of partials + LSE combine).

Importing the package loads liblara_b200.so and fails if it is not built.
"""

from ._native import LaraConfigError, LaraError, LaraTimeout, check, lib  # noqa: F401

__all__ = ["LaraConfigError", "LaraError", "LaraTimeout", "check", "lib"]
