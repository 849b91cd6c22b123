"""Failure detection without a GPU fault.

The reference reports a stuck transaction through ERROR_CODE / STATUS_ERROR and
a host timeout (sw/attn_driver.py:446-454).  Here:

* GPU: every pipeline wait is bounded by %globaltimer; the self-test kernel
  waits on an mbarrier phase that nothing completes, gives up after a short
  limit and sets the timeout bit of the status word.  Through a context the
  call returns LARA_ERR_TIMEOUT (TimeoutError in Python), the status word is
  cleared, and the next decode on the same context is correct -- the context
  stays usable.  No fault, trap or hang is provoked.
* Host (gloo, CPU): a rank that fails before the split-KV all-gather does not
  leave its peer hanging -- the peer's collective ends with an error within the
  process group's timeout.
"""

from __future__ import annotations

import ctypes
import datetime
import os
import socket
import time

import numpy as np
import pytest
import torch

import oracle


@pytest.mark.gpu
def test_bounded_wait_times_out_and_reports():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    from lara_b200 import _native, ops

    ws = ops.new_workspace(256, torch.device("cuda:0"))
    t0 = time.perf_counter()
    _native.check(_native.lib.lara_selftest_wait_timeout(ws.data_ptr(), 50_000,
                                                          torch.cuda.current_stream().cuda_stream), "selftest")
    assert ops.workspace_status(ws) & 0x1  # kDevWaitTimeout
    assert time.perf_counter() - t0 >= 0.045
    assert ops.workspace_status(ws) == 0  # read-and-clear


@pytest.mark.gpu
def test_context_survives_a_timeout():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    from lara_b200 import _native
    from lara_b200.attn_driver import AttentionAccelerator
    from parity import assert_bf16_parity

    rng = np.random.default_rng(2)
    pk = oracle.fp32_to_bf16_u16
    B, Hq, Hkv, D, L = 2, 32, 8, 128, 300
    k = pk(rng.standard_normal((B, Hkv, L, D)).astype(np.float32) * 0.5)
    v = pk(rng.standard_normal((B, Hkv, L, D)).astype(np.float32) * 0.5)
    q = pk(rng.standard_normal((B, Hq, D)).astype(np.float32) * 0.5)
    with AttentionAccelerator() as acc:
        acc.configure_heads(Hq, Hkv, D, max_seq_len=L, batch=B)
        acc.load_kv(k, v)
        rc = _native.lib.lara_ctx_selftest_timeout(acc._ctx, 20_000)
        assert rc == _native.LARA_ERR_TIMEOUT
        with pytest.raises(TimeoutError):
            _native.check(_native.lib.lara_ctx_selftest_timeout(acc._ctx, 20_000), "selftest")
        o = acc.run_query(q)  # the context is still usable
    lens = np.full(B, L)
    assert_bf16_parity(o, oracle.decode_attention(q, k, v, lens), oracle.decode_attention_fp64(q, k, v, lens),
                       what="after timeout")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, result_q):
    import torch.distributed as dist

    from lara_b200 import parallel

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        if rank == 1:
            raise RuntimeError("rank 1 fails before the all-gather")

        class _Cpu(parallel.SplitKVDecoder):
            def _init_local(self, local_capacity, lens_local):
                pass

            def _local_partial(self, q, k_local, v_local, lens_local, ml, acc):
                ml.zero_()
                acc.zero_()

            def _combine(self, gathered, out):
                out.zero_()

        dec = _Cpu(1, 4, 1, 64, 16, "cpu")
        z = torch.zeros((1, 4, 64), dtype=torch.int16)
        t0 = time.perf_counter()
        try:
            dec(z, torch.zeros((1, 1, 16, 64), dtype=torch.int16), torch.zeros((1, 1, 16, 64), dtype=torch.int16),
                torch.full((1,), 16, dtype=torch.int32))
            result_q.put((rank, "completed", time.perf_counter() - t0))
        except Exception as exc:  # the peer's failure surfaces as an error, not a hang
            result_q.put((rank, type(exc).__name__, time.perf_counter() - t0))
    except RuntimeError:
        result_q.put((rank, "raised", 0.0))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_peer_failure_ends_the_collective_with_an_error():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    res = dict((r, (what, secs)) for r, what, secs in (q.get(timeout=5) for _ in range(2)))
    assert res[1][0] == "raised"
    assert res[0][0] != "completed" and res[0][1] < 60, res
