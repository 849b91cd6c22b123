"""GPU tests of split-KV decode across ranks (``lara_b200.parallel``).

* world size 1: ``SplitKVDecoder`` runs partial decode + the strided LSE
  combine kernel on one GPU; compared with the oracle.
* world size 2 (needs two GPUs, NCCL): each rank holds half of every
  sequence's tokens; the gathered result must match the single-GPU decode of
  the whole sequence and the oracle (tolerance as in ``tests/parity.py``).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from parity import assert_bf16_parity, words_of  # noqa: E402

pytestmark = pytest.mark.gpu

B, HQ, HKV, D, L = 2, 32, 8, 128, 6000


def _global_inputs(dev):
    g = torch.Generator(device=dev)
    g.manual_seed(21)
    q = (torch.randn((B, HQ, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    k = (torch.randn((B, HKV, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    v = (torch.randn((B, HKV, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    return q, k, v


def test_split_kv_world1_matches_oracle():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    from lara_b200 import parallel

    dev = torch.device("cuda:0")
    q, k, v = _global_inputs(dev)
    lens = torch.full((B,), L, dtype=torch.int32, device=dev)
    dec = parallel.SplitKVDecoder(B, HQ, HKV, D, L, dev)
    o = dec(q, k, v, lens)
    args = (words_of(q), words_of(k), words_of(v), np.full(B, L))
    gold = oracle.decode_attention(*args)
    assert_bf16_parity(words_of(o), gold, oracle.decode_attention_fp64(*args), what="split-kv world 1")


def _rank_main(rank, world, port, q_out):
    import torch.distributed as dist

    from lara_b200 import ops, parallel

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        q, k, v = _global_inputs(dev)
        start, cnt = parallel.token_range(L, world, rank)
        kl = k[:, :, start:start + cnt].contiguous()
        vl = v[:, :, start:start + cnt].contiguous()
        lens = torch.full((B,), cnt, dtype=torch.int32, device=dev)
        dec = parallel.SplitKVDecoder(B, HQ, HKV, D, cnt, dev)
        o = dec(q, kl, vl, lens)
        full = ops.Decoder(B, HQ, HKV, D, L, dev)(q, k, v, torch.full((B,), L, dtype=torch.int32, device=dev))
        torch.cuda.synchronize(dev)
        if rank == 0:
            args = (words_of(q), words_of(k), words_of(v), np.full(B, L))
            gold = oracle.decode_attention(*args)
            e_gold = oracle.bf16_parity_error(words_of(o), gold, oracle.decode_attention_fp64(*args))
            e_full = oracle.bf16_parity_error(words_of(o), oracle.bf16_u16_to_fp32(words_of(full)))
            q_out.put((e_gold["max_ulp"], e_full["max_ulp"], e_gold["n_over_anchored"]))
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


def test_split_kv_two_gpus_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    ulp_gold, ulp_full, n_over = q_out.get(timeout=10)
    assert ulp_gold <= oracle.PARITY_ULPS and ulp_full <= oracle.PARITY_ULPS, (ulp_gold, ulp_full)
    assert n_over == 0, f"fp64-anchored bound exceeded on {n_over} elements"
