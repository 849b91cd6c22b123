"""GPU tests of the drop-in driver (``lara_b200.attn_driver``) and the dense path.

These replay what the reference harnesses do with ``AttentionAccelerator``:
``board_test.py`` (zero in -> zero out, NPZ comparison), ``board_matrix.py`` /
``board_performance.py`` (per-case ``run_attention``, ``save_last_profile``,
``read_perf`` validity, ``bf16_u16_to_fp32`` on outputs).  Expected outputs
are the reference's own ``cpu_attention_numpy`` results (fixture rows) and the
pinned oracle (full outputs); tolerance as in ``tests/parity.py``.
"""

from __future__ import annotations

import json

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import make_golden as mg  # noqa: E402
import oracle  # noqa: E402
from parity import assert_bf16_parity, decode_on_tensor_cores, prefill_on_tensor_cores, words_of  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def accel():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    from lara_b200.attn_driver import AttentionAccelerator

    a = AttentionAccelerator("lara_b200.bit")
    yield a
    a.close()


@pytest.mark.parametrize("case", mg.BOARD_CASES, ids=lambda c: f"L{c[0]}_{'c' if c[1] else 'nc'}_q{c[2]}kv{c[3]}")
def test_board_case_matrix(accel, golden_dir, case):
    L, causal, qb, kb = case
    name = f"board_L{L}_{'causal' if causal else 'noncausal'}_q{qb}_kv{kb}"
    fx = np.load(golden_dir / f"{name}.npz")
    q, k, v = mg.board_inputs(int(fx["seed"]), L, oracle.fp32_to_bf16_u16)
    out = accel.run_attention(q, k, v, seq_len=L, causal=causal, q_pos_base=qb, kv_pos_base=kb)
    assert out.dtype == np.uint16 and out.shape == (32, L, 128)
    rows = fx["rows"]
    g64 = oracle.dense_attention_fp64(q, k, v, causal=causal, q_pos_base=qb, kv_pos_base=kb)
    # against the reference's own output rows
    tc = prefill_on_tensor_cores(32, 8, 128)
    assert_bf16_parity(out[:, rows, :], fx["o_rows"], g64[:, rows, :], what=f"{name} vs reference rows", tensor_core=tc)
    # against the pinned oracle (full output) and fp64
    gold = oracle.cpu_attention_numpy(q, k, v, causal=causal, q_pos_base=qb, kv_pos_base=kb)
    assert_bf16_parity(out, gold, g64, what=f"{name} vs oracle", tensor_core=tc)
    # harness invariants (sw/board_performance.py:345-378)
    perf = accel.read_perf()
    prof = accel.last_profile
    assert prof is not None and prof.clock_mhz > 0 and perf["cycles"] > 0
    assert 0 <= perf["mac_cycles"] <= perf["cycles"] and 0 <= perf["stall_cycles"] <= perf["cycles"]


def test_zero_input_smoke(accel):
    """sw/board_test.py:45-79: a zero transaction returns all-zero words."""
    from lara_b200.attn_driver import HEAD_DIM, N_KV_HEADS, N_Q_HEADS

    q = np.zeros((N_Q_HEADS, 16, HEAD_DIM), np.uint16)
    k = np.zeros((N_KV_HEADS, 16, HEAD_DIM), np.uint16)
    out = accel.run_attention(q, k, k, seq_len=16)
    assert not np.any(out)


def test_profile_round_trip(accel, tmp_path):
    q, k, v = mg.board_inputs(5, 32, oracle.fp32_to_bf16_u16)
    accel.run_attention(q, k, v, seq_len=32)
    p = tmp_path / "profile.json"
    accel.save_last_profile(p)
    d = json.loads(p.read_text())
    assert d["seq_len"] == 32 and d["clock_mhz"] == 1000.0 and d["pl_total_cycles"] > 0


def test_fp32_inputs_are_packed(accel):
    rng = np.random.default_rng(1)
    qf = rng.standard_normal((32, 8, 128)).astype(np.float32)
    kf = rng.standard_normal((8, 8, 128)).astype(np.float32)
    vf = rng.standard_normal((8, 8, 128)).astype(np.float32)
    out_f = accel.run_attention(qf, kf, vf, seq_len=8)
    pk = oracle.fp32_to_bf16_u16
    out_w = accel.run_attention(pk(qf), pk(kf), pk(vf), seq_len=8)
    np.testing.assert_array_equal(out_f, out_w)


def test_validation_errors(accel):
    q = np.zeros((32, 4, 128), np.uint16)
    k = np.zeros((8, 4, 128), np.uint16)
    with pytest.raises(ValueError):
        accel.run_attention(q, k, k, seq_len=0)
    with pytest.raises(ValueError):
        accel.run_attention(np.zeros((32, 513, 128), np.uint16), np.zeros((8, 513, 128), np.uint16),
                            np.zeros((8, 513, 128), np.uint16))
    with pytest.raises(ValueError):
        accel.run_attention(q, k[:, :3], k, seq_len=4)
    with pytest.raises(ValueError):
        accel.configure(4, q_pos_base=65534)


def test_dead_causal_rows_are_zero(accel):
    """kv_pos_base beyond q positions: no visible key -> zeros (RTL l == 0 rule)."""
    q, k, v = mg.board_inputs(8, 16, oracle.fp32_to_bf16_u16)
    out = accel.run_attention(q, k, v, seq_len=16, causal=True, q_pos_base=0, kv_pos_base=8)
    assert not np.any(out[:, :8])
    args = (q[None], k[None], v[None], np.array([16]), 0)
    gold = oracle.prefill_attention(*args, causal=True, kv_pos_base=8)[0]
    g64 = oracle.prefill_attention(*args, causal=True, kv_pos_base=8, dtype=np.float64, kappa=True)[0]
    assert_bf16_parity(out[:, 8:], gold[:, 8:], g64[:, 8:], tensor_core=prefill_on_tensor_cores(32, 8, 128))


def test_closed_accelerator_raises():
    from lara_b200.attn_driver import AttentionAccelerator

    a = AttentionAccelerator()
    a.close()
    a.close()  # idempotent
    with pytest.raises(RuntimeError):
        a.run_attention(np.zeros((32, 1, 128), np.uint16), np.zeros((8, 1, 128), np.uint16),
                        np.zeros((8, 1, 128), np.uint16))
    with pytest.raises(RuntimeError):
        with a:
            pass


def test_decode_extension_cfg1(golden_dir):
    """configure_heads / load_kv / append_kv / run_query on the config-1 golden step."""
    from lara_b200.attn_driver import AttentionAccelerator

    fx = np.load(golden_dir / "decode_cfg1.npz")
    with AttentionAccelerator() as a:
        a.configure_heads(8, 2, 64, max_seq_len=600, batch=1)
        a.load_kv(fx["k_cache"], fx["v_cache"])
        a.append_kv(fx["k_new"], fx["v_new"])
        assert a.seq_lens.tolist() == [513]
        o = a.run_query(fx["q"])
        k_all = np.concatenate([fx["k_cache"], fx["k_new"][:, :, None, :]], axis=2)
        v_all = np.concatenate([fx["v_cache"], fx["v_new"][:, :, None, :]], axis=2)
        g64 = oracle.decode_attention_fp64(fx["q"], k_all, v_all, np.array([513]))
        assert_bf16_parity(o, fx["o_fp32"], g64, what="driver run_query cfg1", tensor_core=decode_on_tensor_cores(8, 2, 64))
        np.testing.assert_array_equal(a.read_output(), o)
        perf = a.read_perf()
        assert 0 <= perf["mac_cycles"] <= perf["cycles"]


def test_decode_extension_ragged_batch():
    from lara_b200.attn_driver import AttentionAccelerator

    rng = np.random.default_rng(4)
    B, Hq, Hkv, D, L = 5, 32, 8, 128, 1000
    pk = oracle.fp32_to_bf16_u16
    k = pk(rng.standard_normal((B, Hkv, L, D)).astype(np.float32) * 0.5)
    v = pk(rng.standard_normal((B, Hkv, L, D)).astype(np.float32) * 0.5)
    q = pk(rng.standard_normal((B, Hq, D)).astype(np.float32) * 0.5)
    lens = np.array([1000, 1, 513, 0, 64], np.int32)
    with AttentionAccelerator() as a:
        a.configure_heads(Hq, Hkv, D, max_seq_len=1024, batch=B)
        a.load_kv(k, v, lens)
        o = a.run_query(q)
    gold = oracle.decode_attention(q, k, v, lens)
    assert_bf16_parity(o, gold, oracle.decode_attention_fp64(q, k, v, lens), what="ragged run_query",
                       tensor_core=decode_on_tensor_cores(Hq, Hkv, D))


def test_prefill_chunk_extension():
    from lara_b200.attn_driver import AttentionAccelerator

    rng = np.random.default_rng(6)
    B, Hq, Hkv, D, C, n = 2, 32, 8, 128, 300, 40
    pk = oracle.fp32_to_bf16_u16
    k = pk(rng.standard_normal((B, Hkv, C, D)).astype(np.float32) * 0.5)
    v = pk(rng.standard_normal((B, Hkv, C, D)).astype(np.float32) * 0.5)
    kn = pk(rng.standard_normal((B, Hkv, n, D)).astype(np.float32) * 0.5)
    vn = pk(rng.standard_normal((B, Hkv, n, D)).astype(np.float32) * 0.5)
    q = pk(rng.standard_normal((B, n, Hq, D)).astype(np.float32) * 0.5)
    with AttentionAccelerator() as a:
        a.configure_heads(Hq, Hkv, D, max_seq_len=512, batch=B)
        a.load_kv(k, v, np.array([C, 250], np.int32))
        o = a.run_prefill_chunk(q, kn, vn, causal=True)
        assert a.seq_lens.tolist() == [C + n, 250 + n]
    for b, c in enumerate([C, 250]):
        k_all = np.concatenate([k[b:b + 1, :, :c], kn[b:b + 1]], axis=2)
        v_all = np.concatenate([v[b:b + 1, :, :c], vn[b:b + 1]], axis=2)
        args = (q[b:b + 1].transpose(0, 2, 1, 3), k_all, v_all, np.array([c + n]), c)
        gold = oracle.prefill_attention(*args, causal=True)
        g64 = oracle.prefill_attention(*args, causal=True, dtype=np.float64, kappa=True)
        assert_bf16_parity(o[b].transpose(1, 0, 2), gold[0], g64[0], what=f"prefill b={b}",
                           tensor_core=prefill_on_tensor_cores(Hq, Hkv, D))


def test_prefill_chunk_pinned_out_and_truncate_rewind():
    """Host-buffer prefill is pipelined by sequence: page-locked inputs with a
    page-locked ``out`` give the words of pageable buffers; ``truncate_kv``
    rewinds the chunk so the same call repeats bit for bit; lengths never grow."""
    from lara_b200.attn_driver import AttentionAccelerator
    from lara_b200._native import LaraConfigError

    rng = np.random.default_rng(17)
    B, Hq, Hkv, D, C, n = 4, 32, 8, 128, 700, 256
    pk = oracle.fp32_to_bf16_u16
    k = pk(rng.standard_normal((B, Hkv, C, D)).astype(np.float32) * 0.5)
    v = pk(rng.standard_normal((B, Hkv, C, D)).astype(np.float32) * 0.5)
    lens = np.array([700, 1, 0, 333], np.int32)

    def pinned(a):
        t = torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).pin_memory()
        return t, t.numpy().view(np.uint16)

    qt, q = pinned(pk(rng.standard_normal((B, n, Hq, D)).astype(np.float32) * 0.5))
    kt, kn = pinned(pk(rng.standard_normal((B, Hkv, n, D)).astype(np.float32) * 0.5))
    vt, vn = pinned(pk(rng.standard_normal((B, Hkv, n, D)).astype(np.float32) * 0.5))
    ot, out = pinned(np.zeros((B, n, Hq, D), np.uint16))
    with AttentionAccelerator() as a:
        a.configure_heads(Hq, Hkv, D, max_seq_len=1024, batch=B)
        a.load_kv(k, v, lens)
        o_page = a.run_prefill_chunk(q.copy(), kn.copy(), vn.copy(), causal=True).copy()
        assert a.seq_lens.tolist() == (lens + n).tolist()
        a.truncate_kv(lens)
        assert a.seq_lens.tolist() == lens.tolist()
        with pytest.raises(ValueError):
            a.run_prefill_chunk(q, kn, vn, causal=True, out=np.empty((B, n, Hq, D - 1), np.uint16))
        assert a.seq_lens.tolist() == lens.tolist()  # a rejected call appends nothing
        got = a.run_prefill_chunk(q, kn, vn, causal=True, out=out)
        assert got is out
        np.testing.assert_array_equal(out, o_page)
        with pytest.raises(LaraConfigError):
            a.truncate_kv(lens + n + 1)  # longer than the sequences
        a.truncate_kv(lens)
        a.append_kv(kn, vn)  # the rewound rows are overwritten by the same tokens
        assert a.seq_lens.tolist() == (lens + n).tolist()
    for b, c in enumerate(lens.tolist()):
        k_all = np.concatenate([k[b:b + 1, :, :c], kn[b:b + 1]], axis=2)
        v_all = np.concatenate([v[b:b + 1, :, :c], vn[b:b + 1]], axis=2)
        args = (q[b:b + 1].transpose(0, 2, 1, 3), k_all, v_all, np.array([c + n]), c)
        gold = oracle.prefill_attention(*args, causal=True)
        g64 = oracle.prefill_attention(*args, causal=True, dtype=np.float64, kappa=True)
        assert_bf16_parity(o_page[b].transpose(1, 0, 2), gold[0], g64[0], what=f"pipelined prefill b={b}",
                           tensor_core=prefill_on_tensor_cores(Hq, Hkv, D))


def test_dense_ops_matches_driver(accel):
    from lara_b200 import ops

    q, k, v = mg.board_inputs(12, 64, oracle.fp32_to_bf16_u16)
    out = accel.run_attention(q, k, v, seq_len=64, causal=True, q_pos_base=31, kv_pos_base=7)
    dev = torch.device("cuda:0")
    t = lambda a: torch.from_numpy(a.astype(np.int16)).to(dev)  # noqa: E731
    o2 = ops.attention_dense(t(q), t(k), t(v), causal=True, q_pos_base=31, kv_pos_base=7)
    np.testing.assert_array_equal(words_of(o2), out)


def test_run_query_pinned_host_buffers_match_pageable():
    """Page-locked host q/o are used in place by the kernel; pageable ones are
    staged.  Both give the same words."""
    from lara_b200.attn_driver import AttentionAccelerator

    rng = np.random.default_rng(9)
    B, Hq, Hkv, D, L = 3, 32, 8, 128, 700
    pk = oracle.fp32_to_bf16_u16
    k = pk(rng.standard_normal((B, Hkv, L, D)).astype(np.float32) * 0.5)
    v = pk(rng.standard_normal((B, Hkv, L, D)).astype(np.float32) * 0.5)
    q = pk(rng.standard_normal((B, Hq, D)).astype(np.float32) * 0.5)
    qp = torch.from_numpy(q.view(np.int16)).pin_memory()
    op = torch.empty_like(qp).pin_memory()
    with AttentionAccelerator() as a:
        a.configure_heads(Hq, Hkv, D, max_seq_len=L, batch=B)
        a.load_kv(k, v, np.array([700, 1, 350], np.int32))
        o_pageable = a.run_query(q).copy()
        o_pinned = a.run_query(qp.numpy().view(np.uint16), out=op.numpy().view(np.uint16))
        np.testing.assert_array_equal(o_pinned, o_pageable)
        perf = a.read_perf()
        assert 0 <= perf["mac_cycles"] <= perf["cycles"]
    lens = np.array([700, 1, 350])
    gold = oracle.decode_attention(q, k, v, lens)
    assert_bf16_parity(o_pinned, gold, oracle.decode_attention_fp64(q, k, v, lens), what="pinned run_query",
                       tensor_core=decode_on_tensor_cores(Hq, Hkv, D))


def test_run_layer_composes_prologue_and_attention():
    """run_layer (sw/attn_driver.py:552-586) = the GPU prologue followed by
    run_attention on its q/k/v: the words match that composition exactly, the
    result has the reference's [L, Hq*D] float32 layout, and the prologue
    meets the oracle's tolerance."""
    from lara_b200 import ops
    from lara_b200.attn_driver import AttentionAccelerator
    from oracle import prologue

    rng = np.random.default_rng(21)
    L, hidden = 96, 512
    x = rng.standard_normal((L, hidden)).astype(np.float32)
    wq = (rng.standard_normal((hidden, 32 * 128)) / np.sqrt(hidden)).astype(np.float32)
    wk = (rng.standard_normal((hidden, 8 * 128)) / np.sqrt(hidden)).astype(np.float32)
    wv = (rng.standard_normal((hidden, 8 * 128)) / np.sqrt(hidden)).astype(np.float32)
    g = (1.0 + 0.1 * rng.standard_normal(hidden)).astype(np.float32)
    pk = oracle.fp32_to_bf16_u16
    with AttentionAccelerator() as acc:
        out = acc.run_layer(x, wq, wk, wv, g, q_pos_base=31, kv_pos_base=7, causal=True)
        prof = acc.last_profile
        assert out.shape == (L, 32 * 128) and out.dtype == np.float32
        assert prof.host_qkv_projection_ms > 0 and prof.layer_total_ms >= prof.host_qkv_projection_ms
        dev = torch.device("cuda:0")
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev)  # noqa: E731
        w_qkv = np.concatenate([pk(wq), pk(wk), pk(wv)], axis=1)
        q, k, v = ops.layer_prologue(t(pk(x)), t(w_qkv), t(pk(g)), q_pos_base=31, kv_pos_base=7)
        qw, kw, vw = words_of(q), words_of(k), words_of(v)
        ref_words = acc.run_attention(qw, kw, vw, seq_len=L, q_pos_base=31, kv_pos_base=7, causal=True)
    np.testing.assert_array_equal(out, oracle.bf16_u16_to_fp32(ref_words).transpose(1, 0, 2).reshape(L, 32 * 128))
    gq, gk, gv = prologue.layer_prologue(pk(x), w_qkv, pk(g), q_pos_base=31, kv_pos_base=7)
    assert_bf16_parity(qw, gq, what="run_layer q")
    assert_bf16_parity(vw, gv, what="run_layer v")


def test_async_decode_and_prefill_match_synchronous_calls():
    """lara_decode / lara_prefill (stream-ordered, device buffers) + lara_sync give
    the words of lara_run_query / lara_run_prefill_chunk."""
    from lara_b200 import _native
    from lara_b200.attn_driver import AttentionAccelerator

    lib = _native.lib
    rng = np.random.default_rng(13)
    pk = oracle.fp32_to_bf16_u16
    B, Hq, Hkv, D, L, n = 3, 32, 8, 128, 600, 40
    k = pk(rng.standard_normal((B, Hkv, L, D)).astype(np.float32) * 0.5)
    v = pk(rng.standard_normal((B, Hkv, L, D)).astype(np.float32) * 0.5)
    q = pk(rng.standard_normal((B, Hq, D)).astype(np.float32) * 0.5)
    qp = pk(rng.standard_normal((B, n, Hq, D)).astype(np.float32) * 0.5)
    kn = pk(rng.standard_normal((B, Hkv, n, D)).astype(np.float32) * 0.5)
    vn = pk(rng.standard_normal((B, Hkv, n, D)).astype(np.float32) * 0.5)
    lens = np.array([500, 3, 250], np.int32)
    dev = torch.device("cuda:0")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev)  # noqa: E731
    stream = torch.cuda.Stream(device=dev)
    with AttentionAccelerator() as sync_acc, AttentionAccelerator() as async_acc:
        for acc in (sync_acc, async_acc):
            acc.configure_heads(Hq, Hkv, D, max_seq_len=1024, batch=B)
            acc.load_kv(k, v, lens)
        want = sync_acc.run_query(q).copy()
        qd = t(q)
        torch.cuda.current_stream().synchronize()  # qd is written on torch's stream, read on `stream`
        for splits in (0, 3):
            od = torch.empty_like(qd)
            _native.check(lib.lara_decode(async_acc._ctx, qd.data_ptr(), od.data_ptr(), splits, stream.cuda_stream),
                          "lara_decode")
            _native.check(lib.lara_sync(async_acc._ctx, 10_000), "lara_sync")
            got = words_of(od)
            if splits == 0:
                np.testing.assert_array_equal(got, want)
            else:
                assert_bf16_parity(got, oracle.decode_attention(q, k, v, lens),
                                   oracle.decode_attention_fp64(q, k, v, lens), what="lara_decode splits=3",
                                   tensor_core=decode_on_tensor_cores(Hq, Hkv, D))
        want_p = sync_acc.run_prefill_chunk(qp, kn, vn, causal=True)
        # keep the device inputs referenced until lara_sync: the call is asynchronous
        qpd, knd, vnd = t(qp), t(kn), t(vn)
        op = torch.empty_like(qpd)
        torch.cuda.current_stream().synchronize()  # the inputs are written on torch's stream
        _native.check(lib.lara_prefill(async_acc._ctx, qpd.data_ptr(), knd.data_ptr(), vnd.data_ptr(),
                                       op.data_ptr(), n, 1, stream.cuda_stream), "lara_prefill")
        _native.check(lib.lara_sync(async_acc._ctx, 10_000), "lara_sync")
        np.testing.assert_array_equal(words_of(op), want_p)
        assert async_acc.seq_lens.tolist() == (lens + n).tolist()


def test_run_query_profile_is_built_on_read():
    """run_query records two clock reads; last_profile builds the RunProfile (with
    the device times of the call) on its first read and describes the query,
    not the cache as it is when the profile is read."""
    from lara_b200.attn_driver import AttentionAccelerator

    rng = np.random.default_rng(4)
    B, Hq, Hkv, D, L = 2, 32, 8, 128, 300
    pk = oracle.fp32_to_bf16_u16
    k = pk(rng.standard_normal((B, Hkv, L, D)).astype(np.float32))
    v = pk(rng.standard_normal((B, Hkv, L, D)).astype(np.float32))
    q = pk(rng.standard_normal((B, Hq, D)).astype(np.float32))
    with AttentionAccelerator() as a:
        a.configure_heads(Hq, Hkv, D, max_seq_len=L + 8, batch=B)
        a.load_kv(k, v)
        a.run_query(q)
        prof = a.last_profile
        assert prof is not None and prof.pl_total_cycles > 0
        assert 0 <= prof.pl_mac_cycles <= prof.pl_total_cycles
        assert prof.q_dma_bytes == q.nbytes and prof.output_dma_bytes == q.nbytes
        assert prof.seq_len == L and prof.timestamp_utc and prof.attention_total_ms > 0
        assert a.last_profile is prof
        a.run_query(q)
        a.append_kv(np.zeros((B, Hkv, 1, D), np.uint16), np.zeros((B, Hkv, 1, D), np.uint16))
        assert a.last_profile.seq_len == L
