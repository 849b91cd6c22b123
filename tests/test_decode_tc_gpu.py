"""GPU parity of the tensor-core decode kernel (tcgen05 + TMEM) against the CPU oracle.

``LARA_DECODE_PATH=tc`` forces the tensor-core kernel for every group size it
is compiled for (1, 2, 4, 8 and 16 query heads per KV head, head_dim 128);
``=simt`` forces the CUDA-core kernel.  Both are checked against the same
oracle (``oracle.decode_attention``, the reference's ``cpu_attention_numpy``
restated for a KV cache) with the tolerance of ``tests/parity.py``: <= 2 bf16
ulp per element (ulp floored at 2**-8 of the head vector's largest
magnitude), also against the fp64 reference.
"""

from __future__ import annotations

import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from parity import assert_bf16_parity, decode_on_tensor_cores, words_of  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture
def dev():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    from lara_b200 import ops  # noqa: F401  (loads liblara_b200.so)

    return torch.device("cuda:0")


@pytest.fixture
def tc(dev, monkeypatch):
    monkeypatch.setenv("LARA_DECODE_PATH", "tc")
    return dev


def _words(g, shape, dev, std=1.0):
    return (torch.randn(shape, generator=g, device=dev) * std).to(torch.bfloat16)


def _case(dev, B, Hq, Hkv, lens, cap, *, seed, std=1.0, splits=(0, 0), boost=None, poison=False):
    from lara_b200 import ops

    D = 128
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    q = _words(g, (B, Hq, D), dev, std)
    k = _words(g, (B, Hkv, cap, D), dev, std)
    v = _words(g, (B, Hkv, cap, D), dev, std)
    if boost is not None:
        k[..., :4] = (k[..., :4].float() * boost).to(torch.bfloat16)
    if poison:
        # cache rows past each length hold NaN / Inf: they must not reach the output
        for b, n in enumerate(lens):
            k[b, :, n:] = float("nan")
            v[b, :, n:] = float("inf") if b % 2 else float("nan")
    lens_t = torch.tensor(lens, dtype=torch.int32, device=dev)
    dec = ops.Decoder(B, Hq, Hkv, D, cap, dev, lens=np.asarray(lens), num_splits=splits[0],
                      chunk_tokens=splits[1])
    o = dec(q, k, v, lens_t)
    torch.cuda.synchronize()
    assert ops.workspace_status(dec.workspace) == 0
    qw, kw, vw = words_of(q), words_of(k), words_of(v)
    gold = oracle.decode_attention(qw, kw, vw, np.asarray(lens))
    g64 = oracle.decode_attention_fp64(qw, kw, vw, np.asarray(lens))
    return words_of(o), gold, g64, dec


def test_kernel_selection(dev, monkeypatch):
    from lara_b200 import ops

    monkeypatch.delenv("LARA_DECODE_PATH", raising=False)
    assert ops.decode_kernel(64, 8, 128) == "tensor"      # G = 8
    assert ops.decode_kernel(32, 2, 128) == "tensor"      # G = 16
    assert ops.decode_kernel(32, 8, 128) == "cuda_core"   # G = 4
    assert ops.decode_kernel(64, 8, 64) == "cuda_core"    # head_dim 64
    monkeypatch.setenv("LARA_DECODE_PATH", "tc")
    assert ops.decode_kernel(32, 8, 128) == "tensor"
    assert ops.decode_kernel(8, 8, 128) == "tensor"
    assert ops.decode_kernel(64, 2, 128) == "cuda_core"   # G = 32: not compiled
    monkeypatch.setenv("LARA_DECODE_PATH", "simt")
    assert ops.decode_kernel(64, 8, 128) == "cuda_core"


GEOMS = [
    # (B, Hq, Hkv)
    (2, 8, 8),     # G = 1
    (2, 16, 8),    # G = 2
    (3, 32, 8),    # G = 4 (Llama-3-8B)
    (2, 64, 8),    # G = 8 (config 3)
    (2, 32, 2),    # G = 16
    (1, 16, 1),    # G = 16, the Q box covers every head
    (1, 8, 1),     # G = 8 with fewer than 16 query heads
    (2, 4, 1),     # G = 4 with fewer than 16 query heads
]


@pytest.mark.parametrize("geom", GEOMS, ids=lambda g: "B{}_Hq{}_Hkv{}".format(*g))
def test_tc_geometries_ragged(tc, geom):
    B, Hq, Hkv = geom
    cap = 700
    lens = [cap, 1, 333, 128, 129][:B]
    o, gold, g64, _ = _case(tc, B, Hq, Hkv, lens, cap, seed=B * 100 + Hq)
    assert_bf16_parity(o, gold, g64, what=f"tc {geom}", tensor_core=decode_on_tensor_cores(Hq, Hkv, 128))


@pytest.mark.parametrize("splits", [(1, 4096), (4, 1024), (64, 64), (7, 640), (3, 1376), (3, 1024), (5, 384),
                                    (1, 128)])
def test_tc_forced_splits(tc, splits):
    """Split partials and the last-arriver merge for several plans (G = 8),
    including plans whose splits do not cover the cache, so split 0 takes the
    rest (3 x 1024: 2048 tokens; 5 x 384: 2560; 1 x 128: all 4096)."""
    o, gold, g64, _ = _case(tc, 2, 64, 8, [4096, 2999], 4096, seed=7, std=0.5, splits=splits)
    assert_bf16_parity(o, gold, g64, what=f"tc splits={splits}", tensor_core=decode_on_tensor_cores(64, 8, 128))


def test_tc_many_items_per_cta(tc):
    """More work items than SMs: each CTA streams several items back to back."""
    rng = np.random.default_rng(12)
    lens = [int(x) for x in rng.integers(0, 3000, 40)]
    lens[3] = 0
    lens[7] = 3000
    o, gold, g64, _ = _case(tc, 40, 64, 8, lens, 3000, seed=12, std=0.5, splits=(12, 256))
    assert not np.any(o[3])
    keep = [b for b in range(40) if lens[b] > 0]
    assert_bf16_parity(o[keep], gold[keep], g64[keep], what="tc many items",
                       tensor_core=decode_on_tensor_cores(64, 8, 128))


@pytest.mark.parametrize("path", ["tc", "simt"])
def test_poisoned_cache_tail(dev, monkeypatch, path):
    """NaN / Inf past each sequence's length (the unwritten part of a cache) is never read into the output."""
    monkeypatch.setenv("LARA_DECODE_PATH", path)
    o, gold, g64, _ = _case(dev, 4, 64, 8, [700, 5, 129, 256], 700, seed=21, poison=True)
    assert_bf16_parity(o, gold, g64, what=f"{path} poisoned tail", tensor_core=decode_on_tensor_cores(64, 8, 128))


def test_tc_zero_length_gives_zero(tc):
    o, gold, g64, _ = _case(tc, 3, 64, 8, [0, 5, 0], 64, seed=11)
    assert not np.any(o[0]) and not np.any(o[2])
    assert_bf16_parity(o[1:2], gold[1:2], g64[1:2], tensor_core=decode_on_tensor_cores(64, 8, 128))


def test_tc_large_logits(tc):
    """Config-3 style: K channels 0..3 scaled by 20 (large logits)."""
    o, gold, g64, _ = _case(tc, 2, 64, 8, [4100, 777], 4100, seed=2, boost=20.0)
    assert_bf16_parity(o, gold, g64, what="tc large logits", tensor_core=decode_on_tensor_cores(64, 8, 128))


def test_tc_repeat_is_deterministic_and_queue_resets(tc):
    from lara_b200 import ops

    B, Hq, Hkv, D, cap = 3, 64, 8, 128, 2048
    g = torch.Generator(device=tc)
    g.manual_seed(3)
    q = _words(g, (B, Hq, D), tc)
    k = _words(g, (B, Hkv, cap, D), tc)
    v = _words(g, (B, Hkv, cap, D), tc)
    lens = torch.tensor([cap, 1500, 77], dtype=torch.int32, device=tc)
    dec = ops.Decoder(B, Hq, Hkv, D, cap, tc, num_splits=8, chunk_tokens=256)
    outs = [dec(q, k, v, lens).clone() for _ in range(3)]
    torch.cuda.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    ctr = dec.workspace[256:256 + 4 * B * Hkv].view(torch.int32)
    assert int(ctr.abs().sum()) == 0
    queue = dec.workspace[128:136].view(torch.int32)
    assert queue.tolist() == [0, 0]


def test_tc_partial_plus_lse_combine_equals_full(tc):
    """4 KV shards (as 4 GPUs would hold them), partial outputs, LSE combine (G = 8)."""
    from lara_b200 import ops

    B, Hq, Hkv, D, L, P = 2, 64, 8, 128, 4096, 4
    g = torch.Generator(device=tc)
    g.manual_seed(9)
    q = _words(g, (B, Hq, D), tc, 0.5)
    k = _words(g, (B, Hkv, L, D), tc, 0.5)
    v = _words(g, (B, Hkv, L, D), tc, 0.5)
    shard = L // P
    mls, accs = [], []
    for i in range(P):
        ks = k[:, :, i * shard:(i + 1) * shard].contiguous()
        vs = v[:, :, i * shard:(i + 1) * shard].contiguous()
        lens = torch.full((B,), shard, dtype=torch.int32, device=tc)
        dec = ops.Decoder(B, Hq, Hkv, D, shard, tc, num_splits=2, chunk_tokens=512)
        ml, acc = dec.partial(q, ks, vs, lens)
        mls.append(ml)
        accs.append(acc)
    # the partial state itself matches the oracle's restatement of it
    qw = words_of(q)
    ml0, acc0 = oracle.decode_partial(qw, words_of(k[:, :, :shard]), words_of(v[:, :, :shard]), np.full(B, shard))
    np.testing.assert_allclose(mls[0][:, 0].cpu().numpy(), ml0[:, 0], rtol=1e-5, atol=1e-5)
    o = ops.lse_combine(torch.stack(mls), torch.stack(accs)).view(B, Hq, D)
    kw, vw = words_of(k), words_of(v)
    gold = oracle.decode_attention(qw, kw, vw, np.full(B, L))
    assert_bf16_parity(words_of(o), gold, oracle.decode_attention_fp64(qw, kw, vw, np.full(B, L)), what="tc combine",
                       tensor_core=decode_on_tensor_cores(Hq, Hkv, D))


@pytest.mark.parametrize("path", ["tc", "simt"])
def test_prefill_rows_on_decode_kernels(dev, monkeypatch, path):
    """Chunked prefill through the decode kernels (one query row per new token,
    causal lengths per row) for G = 8 and 16."""
    from lara_b200 import _native, ops

    monkeypatch.setenv("LARA_ATTN_PATH", "stream")
    monkeypatch.setenv("LARA_DECODE_PATH", path)
    for (B, Hq, Hkv, cached, n) in ((2, 16, 2, [130, 5], 129), (1, 32, 2, [300], 40)):
        if path == "simt" and Hq // Hkv > 8:
            continue  # group 16 runs on the tensor-core kernel only
        D = 128
        g = torch.Generator(device=dev)
        g.manual_seed(B * 1000 + n + Hq)
        Lmax = max(cached) + n + 7
        q = (torch.randn((B, n, Hq, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
        k = (torch.randn((B, Hkv, Lmax, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
        v = (torch.randn((B, Hkv, Lmax, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
        lens = torch.tensor(cached, dtype=torch.int32, device=dev)
        nbytes = int(_native.lib.lara_prefill_workspace_bytes(B, n, Hq, Hkv, D, Lmax))
        ws = ops.new_workspace(nbytes, dev)
        o = torch.empty_like(q)
        _native.check(_native.lib.lara_gqa_prefill(q.data_ptr(), k.data_ptr(), v.data_ptr(), lens.data_ptr(),
                                                   o.data_ptr(), B, n, Hq, Hkv, D, Lmax, 1, 1.0 / math.sqrt(D),
                                                   ws.data_ptr(), ws.numel(),
                                                   torch.cuda.current_stream().cuda_stream), "prefill")
        torch.cuda.synchronize()
        assert ops.workspace_status(ws) == 0
        ow, qw, kw, vw = words_of(o), words_of(q), words_of(k), words_of(v)
        for b in range(B):
            c = cached[b]
            args = (qw[b:b + 1].transpose(0, 2, 1, 3), kw[b:b + 1], vw[b:b + 1], np.array([c + n]), c)
            gold = oracle.prefill_attention(*args, causal=True)[0]
            g64 = oracle.prefill_attention(*args, causal=True, dtype=np.float64, kappa=True)[0]
            assert_bf16_parity(ow[b].transpose(1, 0, 2), gold, g64, what=f"{path} prefill rows b={b}",
                               tensor_core=decode_on_tensor_cores(Hq, Hkv, D))


@pytest.mark.parametrize("path", ["tc", "simt"])
def test_dense_transaction_on_decode_kernels(dev, monkeypatch, path):
    """run_attention's dense transaction (one K/V shared by every query row) for G = 8."""
    from lara_b200 import ops

    monkeypatch.setenv("LARA_ATTN_PATH", "stream")
    monkeypatch.setenv("LARA_DECODE_PATH", path)
    rng = np.random.default_rng(5)
    L, Hq, Hkv, D = 300, 16, 2, 128
    q = oracle.fp32_to_bf16_u16(rng.standard_normal((Hq, L, D), dtype=np.float32))
    k = oracle.fp32_to_bf16_u16(rng.standard_normal((Hkv, L, D), dtype=np.float32))
    v = oracle.fp32_to_bf16_u16(rng.standard_normal((Hkv, L, D), dtype=np.float32))
    t = lambda a: torch.from_numpy(a.astype(np.int16)).to(dev)  # noqa: E731
    o = words_of(ops.attention_dense(t(q), t(k), t(v), causal=True, q_pos_base=31, kv_pos_base=7))
    geo = dict(causal=True, q_pos_base=31, kv_pos_base=7, n_q_heads=Hq, n_kv_heads=Hkv, head_dim=D)
    gold = oracle.cpu_attention_numpy(q, k, v, **geo)
    assert_bf16_parity(o, gold, oracle.dense_attention_fp64(q, k, v, **geo), what=f"dense {path}",
                       tensor_core=decode_on_tensor_cores(Hq, Hkv, D))


def _list_schedule_plan(lens, L, hkv, sms, overhead=1.0, max_items=1 << 18):
    """The planner's model restated: items in ticket order (split-major) go to the
    earliest-free CTA; an item costs its 128-token tiles plus `overhead` tiles.
    Candidates: equal splits of 2^k tiles; then, for the best of those chunks,
    a quarter and half of it and twice it, split counts whose split 0 (the
    rest of max_seq_len, rounded up to 128 tokens) is about 1.5^j chunks long."""
    import heapq

    max_tiles = -(-L // 128)
    best = [None]

    def consider(c, ns):
        c0 = c if ns * c >= L else -(-(L - (ns - 1) * c) // 128) * 128
        items = sum(1 if n <= c0 else 1 + -(-(n - c0) // c) for n in lens)
        if items * hkv > max_items:
            return
        heap = [0.0] * sms
        for sp in range(ns):
            for n in lens:
                begin = 0 if sp == 0 else c0 + (sp - 1) * c
                if n == 0 and sp == 0:
                    for _ in range(hkv):
                        heapq.heapreplace(heap, heap[0] + overhead)
                    continue
                if begin >= n:
                    continue
                cost = -(-min(c0 if sp == 0 else c, n - begin) // 128) + overhead
                for _ in range(hkv):
                    heapq.heapreplace(heap, heap[0] + cost)
        span = max(heap)
        if best[0] is None or span < best[0][0] * (1 - 1e-9):
            best[0] = (span, ns, c)

    chunks = []
    c = 128
    while True:
        c = min(c, max_tiles * 128)
        chunks.append(c)
        consider(c, -(-L // c))
        if c >= max_tiles * 128:
            break
        c *= 2
    best_equal = best[0][2]
    for c in chunks:
        if best_equal not in (c, 2 * c, 4 * c) and c != 2 * best_equal:
            continue
        last = -(-L // c)
        m = 1.5
        while m * c < L:
            ns = 1 + (L - int(m * c)) // c
            if 1 <= ns < last:
                consider(c, ns)
                last = ns
            m *= 1.5
    return best[0][1], best[0][2]


def test_tc_plan_matches_list_schedule_model(tc):
    import ctypes

    from lara_b200 import _native
    from lara_b200.workloads import CONFIGS

    sms = torch.cuda.get_device_properties(0).multi_processor_count
    cases = [(CONFIGS[3].lens(), 32768), (CONFIGS[3].lens(16), 32535), (np.full(64, 4096), 4096),
             (np.full(8, 4096), 4096), (np.full(16, 4096), 4096), (np.array([0, 5, 3000, 129]), 3000)]
    for lens, L in cases:
        lens = np.ascontiguousarray(lens, np.int32)
        ns, ch = ctypes.c_int(0), ctypes.c_int(0)
        _native.check(_native.lib.lara_decode_plan(len(lens), 64, 8, 128, L, lens.ctypes.data, ctypes.byref(ns),
                                                    ctypes.byref(ch)), "plan")
        assert (ns.value, ch.value) == _list_schedule_plan(lens.tolist(), L, 8, sms), (len(lens), L)


@pytest.mark.slow
def test_tc_long_sequence_many_splits(tc):
    """One 300,000-token sequence at G = 8 (the planner's split count, and a
    forced 300-way split whose merge spans more than 32 splits per pass)."""
    B, Hq, Hkv, L = 1, 64, 8, 300_000
    for splits in ((0, 0), (300, 1024)):
        o, gold, g64, dec = _case(tc, B, Hq, Hkv, [L], L, seed=31, std=0.5, splits=splits)
        assert_bf16_parity(o, gold, g64, what=f"tc long sequence splits={splits} plan={dec.plan}",
                           tensor_core=decode_on_tensor_cores(Hq, Hkv, 128))
