"""CPU tests of the multi-GPU layer (``lara_b200.parallel``) with gloo ranks.

The sharding helpers are checked directly.  ``SplitKVDecoder``'s host
orchestration -- per-rank token ranges, the packed ``[m,l | acc]`` partial
buffer, the all-gather order and the strided combine layout -- runs on
world_size 2 with gloo; its two device steps are replaced by the oracle's
NumPy restatement of the same partial state and combine, reading the packed
layout exactly as ``lara_lse_combine_strided`` does.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from lara_b200 import parallel  # noqa: E402


def test_token_range_covers_exactly():
    for L in (1, 7, 8, 1_048_576, 1_000_003):
        for world in (1, 2, 3, 4, 8):
            parts = [parallel.token_range(L, world, r) for r in range(world)]
            assert parts[0][0] == 0
            assert all(parts[i][0] + parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            assert sum(c for _, c in parts) == L
            assert max(c for _, c in parts) - min(c for _, c in parts) <= 1
    with pytest.raises(ValueError):
        parallel.token_range(10, 2, 2)


def test_balanced_partition_ragged_config3():
    from lara_b200.workloads import ragged_lens

    lens = ragged_lens()
    for world in (2, 4, 8):
        parts = parallel.balanced_partition(lens, world)
        assert sorted(i for p in parts for i in p) == list(range(len(lens)))
        loads = [int(lens[p].sum()) for p in parts]
        assert max(loads) / (sum(loads) / world) < 1.01  # within 1% of perfect


class _CpuSplitKV(parallel.SplitKVDecoder):
    """SplitKVDecoder with the device steps replaced by the oracle (CPU tensors)."""

    def _init_local(self, local_capacity, lens_local):
        self.local_capacity = local_capacity

    def _local_partial(self, q, k_local, v_local, lens_local, ml, acc):
        m_l, a = oracle.decode_partial(q.numpy(), k_local.numpy(), v_local.numpy(), lens_local.numpy())
        ml.copy_(torch.from_numpy(m_l))
        acc.copy_(torch.from_numpy(a))

    def _combine(self, gathered, out):
        g = gathered.numpy()
        mls = np.stack([g[i * self.part_floats:i * self.part_floats + 2 * self.rows].reshape(self.rows, 2)
                        for i in range(self.world)])
        accs = np.stack([g[i * self.part_floats + 2 * self.rows:(i + 1) * self.part_floats].reshape(self.rows, self.d)
                         for i in range(self.world)])
        o = oracle.lse_combine(mls, accs).reshape(out.shape)
        out.copy_(torch.from_numpy(oracle.fp32_to_bf16_u16(o).view(np.int16)).view(torch.bfloat16))


def _worker(rank, world, port, result_q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)
        B, Hq, Hkv, D, L = 2, 8, 2, 64, 1001
        pk = oracle.fp32_to_bf16_u16
        q = pk(rng.standard_normal((B, Hq, D)).astype(np.float32))
        k = pk(rng.standard_normal((B, Hkv, L, D)).astype(np.float32))
        v = pk(rng.standard_normal((B, Hkv, L, D)).astype(np.float32))
        start, cnt = parallel.token_range(L, world, rank)
        kl = np.ascontiguousarray(k[:, :, start:start + cnt])
        vl = np.ascontiguousarray(v[:, :, start:start + cnt])
        dec = _CpuSplitKV(B, Hq, Hkv, D, cnt, "cpu")
        t = lambda a: torch.from_numpy(a.view(np.int16))  # noqa: E731
        out = dec(t(q), t(kl), t(vl), torch.full((B,), cnt, dtype=torch.int32))
        words = out.view(torch.int16).numpy().view(np.uint16)
        gold = oracle.decode_attention(q, k, v, np.full(B, L))
        err = oracle.bf16_parity_error(words.reshape(B, Hq, D), gold)
        result_q.put((rank, err["max_ulp"]))
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2])
def test_split_kv_orchestration_gloo(world):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=5) for _ in range(world))
    for rank, ulp in res:
        assert ulp <= oracle.PARITY_ULPS, (rank, ulp)
