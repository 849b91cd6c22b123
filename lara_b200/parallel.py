"""One process per GPU: batch sharding and split-KV (sequence) sharding.

The reference is a single FPGA with no parallelism beyond its 16x16 array
(hw/rtl/core/attn_core.sv:327-350); this module is the B200 build's own
distribution layer (torch.distributed for the plumbing, NCCL over NVLink on
GPUs, gloo for CPU tests).

* ``batch_range`` / ``balanced_partition``: independent sequences are split
  across ranks with no collective on the data path (configs 2, 3, 5).  Ragged
  batches are balanced by token count (greedy longest-first).
* ``token_range``: a long sequence is split into contiguous, balanced token
  ranges, one per rank (config 4).
* ``SplitKVDecoder``: each rank decodes its token range into an unnormalised
  partial state (m, l, acc) per query row, packed as
  ``[rows*2 (m, l) | rows*D acc]``; one ``all_gather_into_tensor`` brings every
  rank's packed state into each GPU's own memory (no peer-memory loads, no
  multicast), and ``lara_lse_combine_strided`` merges them:
  M = max m_i, L = sum l_i 2^(m_i - M), O = sum acc_i 2^(m_i - M) / L.
"""

from __future__ import annotations

import heapq
from typing import Sequence


def token_range(length: int, world: int, rank: int) -> tuple[int, int]:
    """(start, count) of rank's contiguous share of ``length`` tokens (sizes differ by <= 1)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, rem = divmod(int(length), world)
    start = rank * base + min(rank, rem)
    return start, base + (1 if rank < rem else 0)


def batch_range(batch: int, world: int, rank: int) -> tuple[int, int]:
    """(start, count) of rank's contiguous share of ``batch`` sequences."""
    return token_range(batch, world, rank)


def balanced_partition(lens: Sequence[int], world: int) -> list[list[int]]:
    """Assign sequences to ranks so the token totals are balanced.

    Greedy longest-processing-time: sequences in decreasing length go to the
    currently lightest rank.  Returns sorted sequence indices per rank.
    """
    if world < 1:
        raise ValueError("world must be >= 1")
    heap = [(0, r) for r in range(world)]
    parts: list[list[int]] = [[] for _ in range(world)]
    for idx in sorted(range(len(lens)), key=lambda i: (-int(lens[i]), i)):
        load, r = heapq.heappop(heap)
        parts[r].append(idx)
        heapq.heappush(heap, (load + int(lens[idx]), r))
    return [sorted(p) for p in parts]


class SplitKVDecoder:
    """Decode of sequences whose KV cache is split along tokens across ranks.

    Every rank holds the same queries ``q[B, Hq, D]`` and its own cache slice
    ``k/v[B, Hkv, local_capacity, D]`` with ``lens_local[B]`` valid tokens (its
    ``token_range`` of each sequence).  ``__call__`` returns the full bf16
    output ``[B, Hq, D]`` on every rank.
    """

    def __init__(self, batch: int, n_q_heads: int, n_kv_heads: int, head_dim: int, local_capacity: int, device,
                 group=None, lens_local=None):
        import torch
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.batch, self.hq, self.hkv, self.d = batch, n_q_heads, n_kv_heads, head_dim
        self.rows = batch * n_q_heads
        self.device = torch.device(device)
        self.part_floats = self.rows * (2 + head_dim)
        self.packed = torch.empty(self.part_floats, dtype=torch.float32, device=self.device)
        self.gathered = torch.empty(self.world * self.part_floats, dtype=torch.float32, device=self.device)
        self._init_local(local_capacity, lens_local)

    # -- the two device steps (kept as methods so CPU tests can stand in) ----
    def _init_local(self, local_capacity, lens_local) -> None:
        from . import ops

        self.decoder = ops.Decoder(self.batch, self.hq, self.hkv, self.d, local_capacity, self.device,
                                   lens=lens_local)

    def _local_partial(self, q, k_local, v_local, lens_local, ml, acc) -> None:
        self.decoder.partial(q, k_local, v_local, lens_local, out_ml=ml, out_acc=acc)

    def _combine(self, gathered, out) -> None:
        from . import ops

        ops.lse_combine_strided(gathered, self.world, self.rows, self.d, ml_offset=0, acc_offset=2 * self.rows,
                                part_stride=self.part_floats, out=out)

    # -------------------------------------------------------------------------
    def __call__(self, q, k_local, v_local, lens_local, out=None):
        import torch
        import torch.distributed as dist

        ml = self.packed[:2 * self.rows].view(self.rows, 2)
        acc = self.packed[2 * self.rows:].view(self.rows, self.d)
        self._local_partial(q, k_local, v_local, lens_local, ml, acc)
        if self.world > 1:
            dist.all_gather_into_tensor(self.gathered, self.packed, group=self.group)
            gathered = self.gathered
        else:
            gathered = self.packed
        if out is None:
            out = torch.empty((self.batch, self.hq, self.d), dtype=torch.bfloat16, device=self.device)
        self._combine(gathered, out)
        return out
