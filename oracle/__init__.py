"""CPU oracle for the GQA streaming-attention path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path (the ``lara_b200``
package, the C-ABI library) imports, links or executes anything in this
directory.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
``cpu_baseline`` / ``--impl reference`` legs use it, and only as the checker
or as the timed CPU baseline.

Parity pins: ``oracle.attention`` is checked bit-for-bit against fixtures that
were produced by importing the reference's own ``cpu_attention_numpy``
(``sw/board_performance.py:158-192``) and ``fp32_to_bf16_u16``
(``sw/attn_driver.py:88-98``); see ``tests/golden/make_golden.py``.
"""

from .attention import (  # noqa: F401
    PARITY_FLOOR_FRAC,
    PARITY_ULPS,
    TC_SPLIT_P_KAPPA,
    bf16_parity_error,
    bf16_u16_to_fp32,
    bf16_ulp,
    cpu_attention_numpy,
    decode_attention,
    decode_attention_fp64,
    decode_partial,
    dense_attention_fp64,
    lse_combine,
    fp32_to_bf16_u16,
    numeric_error,
    prefill_attention,
    tile_pairs_per_head,
    ulp_distance,
    valid_pairs,
)
