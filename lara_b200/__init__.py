"""LARA B200: the grouped-query streaming-attention path on sm_100a.

* ``lara_b200.attn_driver`` -- drop-in for the reference host driver
  (``sw/attn_driver.py``), backed by the C-ABI context of liblara_b200.so.
* ``lara_b200.ops`` -- torch-tensor front end of the stateless kernels
  (decode, split-KV partials + LSE combine, KV append, bf16 pack, dense
  transaction, prefill).
* ``lara_b200.workloads`` -- seeded synthetic inputs of the benchmark configs.
* ``lara_b200.build`` -- compiles liblara_b200.so in-tree with nvcc.

The library is loaded by ``lara_b200._native`` (on first use of ``lib`` /
``check`` here, or on import of any module that computes); a missing or
stale library raises there -- there is no CPU fallback.
"""

_NATIVE = ("lib", "check", "LaraError", "LaraConfigError", "LaraTimeout")

__all__ = list(_NATIVE)


def __getattr__(name):
    if name in _NATIVE:
        from . import _native

        return getattr(_native, name)
    raise AttributeError(f"module 'lara_b200' has no attribute {name!r}")
