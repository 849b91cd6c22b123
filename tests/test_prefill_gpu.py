"""GPU parity of chunked prefill ("cache + self") and of the tensor-core path.

``lara_gqa_prefill`` runs the tcgen05/TMEM kernel for head_dim 128 and the
CUDA-core streaming kernel otherwise; ``LARA_ATTN_PATH=tc|stream`` selects one
explicitly, so both are checked against the CPU oracle (``prefill_attention``,
the causal rule of ``sw/board_performance.py:174-177`` over cache + self).
Tolerance as in ``tests/parity.py`` (<= 2 bf16 ulp, also vs fp64).  The
tensor-core path splits P into P_hi + P_lo (two bf16 terms, two P.V passes) by
default; ``LARA_TC_SPLIT_P=0`` rounds P to one bf16 (round to nearest even) and
is checked against its own, stated bound (``test_prefill_bf16_p_error_bound``).
"""

from __future__ import annotations

import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from parity import assert_bf16_parity, decode_on_tensor_cores, prefill_on_tensor_cores, words_of  # noqa: E402

pytestmark = pytest.mark.gpu


def _prefill(dev, q, k, v, cached, causal):
    from lara_b200 import _native, ops

    B, n, Hq, D = q.shape
    _, Hkv, Lmax, _ = k.shape
    lens = torch.tensor(cached, dtype=torch.int32, device=dev)
    nbytes = int(_native.lib.lara_prefill_workspace_bytes(B, n, Hq, Hkv, D, Lmax))
    ws = ops.new_workspace(nbytes, dev)
    o = torch.empty_like(q)
    _native.check(_native.lib.lara_gqa_prefill(q.data_ptr(), k.data_ptr(), v.data_ptr(), lens.data_ptr(),
                                               o.data_ptr(), B, n, Hq, Hkv, D, Lmax, int(causal),
                                               1.0 / math.sqrt(D), ws.data_ptr(), ws.numel(),
                                               torch.cuda.current_stream().cuda_stream), "prefill")
    torch.cuda.synchronize()
    assert ops.workspace_status(ws) == 0
    return o


CASES = [
    # (B, Hq, Hkv, D, cached, n, causal)
    (2, 32, 8, 128, [300, 250], 40, True),
    (1, 32, 8, 128, [0], 200, True),        # pure self-attention prefill, 2 query tiles
    (2, 16, 2, 128, [130, 5], 129, False),  # non-causal, G=8, query tile of 1 row
    (1, 8, 8, 128, [1000], 257, True),      # MHA, 3 query tiles
    (2, 64, 8, 128, [513, 1024], 130, True),
    (1, 8, 2, 64, [77], 33, True),          # head_dim 64: streaming kernel only
]


@pytest.mark.parametrize("path", ["tc", "stream"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: "B{}_Hq{}_Hkv{}_D{}_c{}_n{}_{}".format(
    c[0], c[1], c[2], c[3], max(c[4]), c[5], "causal" if c[6] else "full"))
def test_prefill_parity(monkeypatch, path, case):
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    B, Hq, Hkv, D, cached, n, causal = case
    if path == "tc" and D != 128:
        pytest.skip("tensor-core kernel is for head_dim 128")
    monkeypatch.setenv("LARA_ATTN_PATH", path)
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(B * 1000 + n)
    Lmax = max(cached) + n + 7
    q = (torch.randn((B, n, Hq, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    k = (torch.randn((B, Hkv, Lmax, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    v = (torch.randn((B, Hkv, Lmax, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    o = words_of(_prefill(dev, q, k, v, cached, causal))
    qw, kw, vw = words_of(q), words_of(k), words_of(v)
    for b in range(B):
        c = cached[b]
        # the new tokens' K/V sit at positions c .. c+n-1 of the cache
        gold = oracle.prefill_attention(qw[b:b + 1].transpose(0, 2, 1, 3), kw[b:b + 1], vw[b:b + 1],
                                        np.array([c + n]), c, causal=causal)[0]
        g64 = oracle.prefill_attention(qw[b:b + 1].transpose(0, 2, 1, 3), kw[b:b + 1], vw[b:b + 1],
                                       np.array([c + n]), c, causal=causal, dtype=np.float64, kappa=True)[0]
        assert_bf16_parity(o[b].transpose(1, 0, 2), gold, g64, what=f"{path} b={b}",
                           tensor_core=prefill_on_tensor_cores(Hq, Hkv, D))


@pytest.mark.parametrize("case", CASES[:5], ids=lambda c: "B{}_Hq{}_Hkv{}_c{}_n{}".format(
    c[0], c[1], c[2], max(c[4]), c[5]))
def test_prefill_bf16_p_error_bound(monkeypatch, case):
    """LARA_TC_SPLIT_P=0: P rounded to one bf16 before P.V (relative error up to
    2^-9 per probability).  Bound: |o - golden_fp64| <= 2^-5 * max|golden| of
    the same head vector (8 bf16 ulp of the vector's largest element; the worst
    case measured on these inputs is 2^-6.9).  The <= 2 ulp element-wise bound
    of the default split-P mode does not hold for this mode."""
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    B, Hq, Hkv, D, cached, n, causal = case
    monkeypatch.setenv("LARA_ATTN_PATH", "tc")
    monkeypatch.setenv("LARA_TC_SPLIT_P", "0")
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(B * 1000 + n + 1)
    Lmax = max(cached) + n + 7
    q = (torch.randn((B, n, Hq, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    k = (torch.randn((B, Hkv, Lmax, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    v = (torch.randn((B, Hkv, Lmax, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    o = oracle.bf16_u16_to_fp32(words_of(_prefill(dev, q, k, v, cached, causal)))
    qw, kw, vw = words_of(q), words_of(k), words_of(v)
    for b in range(B):
        c = cached[b]
        gold = oracle.prefill_attention(qw[b:b + 1].transpose(0, 2, 1, 3), kw[b:b + 1], vw[b:b + 1],
                                        np.array([c + n]), c, causal=causal, dtype=np.float64)[0]
        got = o[b].transpose(1, 0, 2)
        scale = np.max(np.abs(gold), axis=-1, keepdims=True)
        assert np.all(np.isfinite(got))
        assert np.all(np.abs(got - gold) <= 2.0 ** -5 * scale), f"b={b}: {np.max(np.abs(got - gold) / scale)}"


def test_dense_tc_matches_stream(monkeypatch):
    """The reference transaction (Lq = Lkv = 512, bases 31/7) on both kernels."""
    import make_golden as mg
    from lara_b200 import ops

    dev = torch.device("cuda:0")
    q, k, v = mg.board_inputs(77, 512, oracle.fp32_to_bf16_u16)
    t = lambda a: torch.from_numpy(a.astype(np.int16)).to(dev)  # noqa: E731
    outs = {}
    for path in ("tc", "stream"):
        monkeypatch.setenv("LARA_ATTN_PATH", path)
        outs[path] = words_of(ops.attention_dense(t(q), t(k), t(v), causal=True, q_pos_base=31, kv_pos_base=7))
    gold = oracle.cpu_attention_numpy(q, k, v, causal=True, q_pos_base=31, kv_pos_base=7)
    g64 = oracle.dense_attention_fp64(q, k, v, causal=True, q_pos_base=31, kv_pos_base=7)
    for path, o in outs.items():
        assert_bf16_parity(o, gold, g64, what=f"dense {path}",
                           tensor_core=path == "tc" or decode_on_tensor_cores(32, 8, 128))


@pytest.mark.slow
def test_config5_full_size_sampled(monkeypatch):
    """Config 5 (B=4, 2048 new tokens over 8192 cached, causal) through the
    context API on device buffers: ``lara_kv_load`` of the cached tokens, then
    ``lara_prefill`` appends the new K/V and attends on the tensor-core path.
    The appended cache rows are read back (``lara_kv_read``) and must equal the
    new K/V word for word; the output is checked against the oracle (golden
    and fp64-anchored bounds) on the rows either side of every 128-row query
    tile boundary (0, 127/128, ..., 1919/1920, 2047) of every sequence, which
    covers the first and last row of every causal diagonal tile."""
    import ctypes

    from lara_b200 import _native
    from lara_b200.attn_driver import AttentionAccelerator
    from lara_b200.workloads import PREFILL, make_prefill_inputs

    monkeypatch.setenv("LARA_ATTN_PATH", "tc")
    dev = torch.device("cuda:0")
    cfg = PREFILL
    q, k, v, kn, vn, lens = make_prefill_inputs(cfg, dev)
    B, C, n = cfg.batch, cfg.cached, cfg.new
    Hq, Hkv, D = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    lib = _native.lib
    o = torch.empty_like(q)
    lens_np = np.full(B, C, np.int32)
    with AttentionAccelerator() as acc:
        acc.configure_heads(Hq, Hkv, D, max_seq_len=C + n, batch=B)
        _native.check(lib.lara_kv_load(acc._ctx, k.data_ptr(), v.data_ptr(),
                                       lens_np.ctypes.data_as(ctypes.c_void_p), C + n, 1), "kv_load")
        torch.cuda.synchronize()
        _native.check(lib.lara_prefill(acc._ctx, q.data_ptr(), kn.data_ptr(), vn.data_ptr(), o.data_ptr(), n, 1,
                                       torch.cuda.current_stream().cuda_stream), "lara_prefill")
        _native.check(lib.lara_sync(acc._ctx, 60_000), "lara_sync")
        assert acc.seq_lens.tolist() == [C + n] * B
        k_back, v_back = torch.empty_like(k), torch.empty_like(v)
        lens_back = np.zeros(B, np.int32)
        _native.check(lib.lara_kv_read(acc._ctx, k_back.data_ptr(), v_back.data_ptr(),
                                       lens_back.ctypes.data_as(ctypes.c_void_p), C + n, 1), "kv_read")
    assert lens_back.tolist() == [C + n] * B
    assert torch.equal(k_back[:, :, C:].view(torch.int16), kn.view(torch.int16))
    assert torch.equal(v_back[:, :, C:].view(torch.int16), vn.view(torch.int16))
    assert torch.equal(k_back[:, :, :C].view(torch.int16), k[:, :, :C].view(torch.int16))
    ow, qw = words_of(o), words_of(q)
    starts = [0] + [t * 128 - 1 for t in range(1, n // 128)] + [n - 2]
    for b in range(B):
        kw, vw = words_of(k_back[b:b + 1]), words_of(v_back[b:b + 1])
        for i0 in starts:
            qs = qw[b:b + 1, i0:i0 + 2].transpose(0, 2, 1, 3)
            args = (qs, kw, vw, np.array([C + n]), C + i0)
            gold = oracle.prefill_attention(*args, causal=True)[0]
            g64 = oracle.prefill_attention(*args, causal=True, dtype=np.float64, kappa=True)[0]
            assert_bf16_parity(ow[b, i0:i0 + 2].transpose(1, 0, 2), gold, g64, what=f"cfg5 b={b} rows {i0}+2",
                               tensor_core=prefill_on_tensor_cores(Hq, Hkv, D))


def test_ops_gqa_prefill_matches_abi():
    """The torch front end ``ops.gqa_prefill`` returns the C ABI's words."""
    from lara_b200 import ops

    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    B, Hq, Hkv, D, cached, n = 2, 32, 8, 128, [300, 17], 150
    Lmax = max(cached) + n + 3
    q = (torch.randn((B, n, Hq, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    k = (torch.randn((B, Hkv, Lmax, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    v = (torch.randn((B, Hkv, Lmax, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    lens = torch.tensor(cached, dtype=torch.int32, device=dev)
    o_abi = words_of(_prefill(dev, q, k, v, cached, True))
    o_ops = words_of(ops.gqa_prefill(q, k, v, lens, causal=True))
    np.testing.assert_array_equal(o_ops, o_abi)
    with pytest.raises(ValueError):
        ops.gqa_prefill(q, k, v, lens.to(torch.int64))
