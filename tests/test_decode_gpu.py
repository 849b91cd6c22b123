"""GPU parity of the decode path (C ABI through ``lara_b200.ops``) vs the CPU oracle.

Tolerance: <= 2 bf16 ulp of the golden model's bf16 result per element, ulp
floored at 2**-8 of the head vector's largest magnitude (``tests/parity.py``),
and the same bound against the fp64 reference.
"""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from parity import assert_bf16_parity, decode_on_tensor_cores, words_of  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    from lara_b200 import ops  # noqa: F401  (loads liblara_b200.so)

    return torch.device("cuda:0")


def _rand_words(g, shape, dev, std=1.0):
    return (torch.randn(shape, generator=g, device=dev) * std).to(torch.bfloat16)


def _run_case(dev, B, Hq, Hkv, D, lens, cap, *, seed=0, std=1.0, splits=(0, 0), boost=None):
    from lara_b200 import ops

    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    q = _rand_words(g, (B, Hq, D), dev, std)
    k = _rand_words(g, (B, Hkv, cap, D), dev, std)
    v = _rand_words(g, (B, Hkv, cap, D), dev, std)
    if boost is not None:
        k[..., :4] = (k[..., :4].float() * boost).to(torch.bfloat16)
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


GEOMS = [
    # (B, Hq, Hkv, D)
    (2, 8, 2, 64),    # config-1 geometry (G=4, D=64)
    (3, 32, 8, 128),  # Llama-3-8B geometry (G=4)
    (2, 64, 8, 128),  # config-3 geometry (G=8)
    (2, 8, 8, 128),   # MHA (G=1)
    (2, 16, 8, 64),   # G=2, D=64
    (2, 16, 2, 64),   # G=8, D=64
    (1, 8, 4, 128),   # G=2
    (1, 8, 8, 64),    # G=1, D=64
]


@pytest.mark.parametrize("geom", GEOMS, ids=lambda g: "B{}_Hq{}_Hkv{}_D{}".format(*g))
def test_decode_geometries_ragged(dev, geom):
    B, Hq, Hkv, D = geom
    cap = 700
    lens = [cap, 1, 333, 64, 65][:B] if B <= 5 else [cap] * B
    o, gold, g64, _ = _run_case(dev, B, Hq, Hkv, D, lens, cap, seed=B * 100 + Hq)
    assert_bf16_parity(o, gold, g64, what=str(geom), tensor_core=decode_on_tensor_cores(Hq, Hkv, D))


@pytest.mark.parametrize("splits", [(1, 4096), (4, 1024), (64, 64), (7, 640), (3, 1024), (5, 384)])
def test_decode_forced_splits(dev, splits):
    """Split-KV merge inside the kernel (last-arriving CTA) for several plans,
    including plans whose splits do not cover the cache (3 x 1024, 5 x 384 over
    4096 tokens: split 0 takes the rest, 2048 and 2560 tokens)."""
    B, Hq, Hkv, D, cap = 2, 32, 8, 128, 4096
    lens = [4096, 2999]
    o, gold, g64, _ = _run_case(dev, B, Hq, Hkv, D, lens, cap, seed=7, std=0.5, splits=splits)
    assert_bf16_parity(o, gold, g64, what=f"splits={splits}", tensor_core=decode_on_tensor_cores(Hq, Hkv, D))


@pytest.mark.parametrize("splits", [(0, 0), (4, 1024), (7, 640), (64, 64), (3, 1024)])
def test_decode_cuda_core_group4(dev, monkeypatch, splits):
    """The CUDA-core kernel on the Llama-3-8B geometry, selected explicitly with
    LARA_DECODE_PATH=simt (the default for G = 4 as well)."""
    from lara_b200 import ops

    monkeypatch.setenv("LARA_DECODE_PATH", "simt")
    B, Hq, Hkv, D, cap = 3, 32, 8, 128, 4096
    assert ops.decode_kernel(Hq, Hkv, D) == "cuda_core"
    lens = [4096, 2999, 65]
    o, gold, g64, _ = _run_case(dev, B, Hq, Hkv, D, lens, cap, seed=17, std=0.5, splits=splits)
    assert_bf16_parity(o, gold, g64, what=f"cuda-core G=4 splits={splits}", tensor_core=False)


def test_decode_repeat_is_deterministic_and_counters_reset(dev):
    from lara_b200 import ops

    B, Hq, Hkv, D, cap = 2, 32, 8, 128, 2048
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    q = _rand_words(g, (B, Hq, D), dev)
    k = _rand_words(g, (B, Hkv, cap, D), dev)
    v = _rand_words(g, (B, Hkv, cap, D), dev)
    lens = torch.tensor([cap, 1500], dtype=torch.int32, device=dev)
    dec = ops.Decoder(B, Hq, Hkv, D, cap, dev, num_splits=8, chunk_tokens=256)
    outs = [dec(q, k, v, lens).clone() for _ in range(3)]
    torch.cuda.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    ctr = dec.workspace[256:256 + 4 * B * Hkv].view(torch.int32)
    assert int(ctr.abs().sum()) == 0


def test_decode_zero_length_gives_zero(dev):
    o, gold, g64, _ = _run_case(dev, 3, 8, 2, 64, [0, 5, 0], 64, seed=11)
    assert not np.any(o[0]) and not np.any(o[2])
    assert_bf16_parity(o[1:2], gold[1:2], g64[1:2], tensor_core=decode_on_tensor_cores(8, 2, 64))


def test_decode_large_logits_stress(dev):
    """Config-3 style: K channels 0..3 scaled by 20 (large logits)."""
    o, gold, g64, _ = _run_case(dev, 2, 64, 8, 128, [4100, 777], 4100, seed=2, boost=20.0)
    assert_bf16_parity(o, gold, g64, what="large logits", tensor_core=decode_on_tensor_cores(64, 8, 128))


def test_decode_zero_inputs(dev):
    from lara_b200 import ops

    B, Hq, Hkv, D, cap = 2, 32, 8, 128, 300
    z = torch.zeros((B, Hkv, cap, D), dtype=torch.bfloat16, device=dev)
    q = torch.zeros((B, Hq, D), dtype=torch.bfloat16, device=dev)
    o = ops.gqa_decode(q, z, z, torch.tensor([300, 17], dtype=torch.int32, device=dev))
    assert not torch.any(o.view(torch.int16) != 0)


def test_golden_cfg1_decode_with_append(dev, golden_dir):
    """Config 1: 512 cached tokens, append 1 through the kernel, decode."""
    from lara_b200 import ops

    fx = np.load(golden_dir / "decode_cfg1.npz")
    to_dev = lambda a: torch.from_numpy(a.astype(np.int16)).to(dev)  # noqa: E731
    cap = 520
    kc = torch.zeros((1, 2, cap, 64), dtype=torch.int16, device=dev)
    vc = torch.zeros((1, 2, cap, 64), dtype=torch.int16, device=dev)
    kc[:, :, :512] = to_dev(fx["k_cache"])
    vc[:, :, :512] = to_dev(fx["v_cache"])
    lens = torch.tensor([512], dtype=torch.int32, device=dev)
    ops.kv_append(kc, vc, lens, to_dev(fx["k_new"])[:, :, None, :].contiguous(),
                  to_dev(fx["v_new"])[:, :, None, :].contiguous())
    assert int(lens.item()) == 513
    q = to_dev(fx["q"])
    o = ops.gqa_decode(q, kc, vc, lens)
    ow = words_of(o)
    k_all = np.concatenate([fx["k_cache"], fx["k_new"][:, :, None, :]], axis=2)
    v_all = np.concatenate([fx["v_cache"], fx["v_new"][:, :, None, :]], axis=2)
    g64 = oracle.decode_attention_fp64(fx["q"], k_all, v_all, np.array([513]))
    e = assert_bf16_parity(ow, fx["o_fp32"], g64, what="config 1 vs reference golden")
    assert e["max_ulp_strict"] <= 2.0


def test_kv_append_round_trip(dev):
    """Appended rows land bit-exactly at seq_lens[b] and lengths advance."""
    from lara_b200 import ops

    B, Hkv, cap, D, n = 3, 4, 100, 128, 5
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    kc = _rand_words(g, (B, Hkv, cap, D), dev)
    vc = _rand_words(g, (B, Hkv, cap, D), dev)
    k0, v0 = kc.clone(), vc.clone()
    lens = torch.tensor([0, 17, 95], dtype=torch.int32, device=dev)
    kn = _rand_words(g, (B, Hkv, n, D), dev)
    vn = _rand_words(g, (B, Hkv, n, D), dev)
    ops.kv_append(kc, vc, lens, kn, vn)
    torch.cuda.synchronize()
    assert lens.tolist() == [5, 22, 100]
    for b, start in enumerate([0, 17, 95]):
        assert torch.equal(kc[b, :, start:start + n], kn[b])
        assert torch.equal(vc[b, :, start:start + n], vn[b])
        mask = torch.ones(cap, dtype=torch.bool, device=dev)
        mask[start:start + n] = False
        assert torch.equal(kc[b, :, mask], k0[b, :, mask])


def test_kv_append_overflow_is_flagged(dev):
    from lara_b200 import ops

    kc = torch.zeros((1, 1, 8, 64), dtype=torch.bfloat16, device=dev)
    lens = torch.tensor([6], dtype=torch.int32, device=dev)
    kn = torch.ones((1, 1, 4, 64), dtype=torch.bfloat16, device=dev)
    ws = ops.new_workspace(256, dev)
    ops.kv_append(kc, kc.clone(), lens, kn, kn, workspace=ws)
    assert ops.workspace_status(ws) != 0
    assert int(lens.item()) == 8  # clamped at capacity, rows past it dropped


def test_pack_bf16_matches_reference_kat(dev, golden_dir):
    from lara_b200 import ops

    kat = np.load(golden_dir / "kat_bf16.npz")
    x = torch.from_numpy(kat["fp32_bits"].view(np.float32).copy()).to(dev)
    got = ops.pack_bf16(x).cpu().numpy().view(np.uint16)
    np.testing.assert_array_equal(got, kat["bf16_words"])
    # ragged tail lengths
    for n in (1, 3, 5, 4099):
        got = ops.pack_bf16(x[:n].contiguous()).cpu().numpy().view(np.uint16)
        np.testing.assert_array_equal(got, kat["bf16_words"][:n])


def test_partial_plus_lse_combine_equals_full(dev):
    """Split a sequence into 4 KV shards (as 4 GPUs would), decode partials, combine."""
    from lara_b200 import ops

    B, Hq, Hkv, D, L, P = 2, 32, 8, 128, 4096, 4
    g = torch.Generator(device=dev)
    g.manual_seed(9)
    q = _rand_words(g, (B, Hq, D), dev, 0.5)
    k = _rand_words(g, (B, Hkv, L, D), dev, 0.5)
    v = _rand_words(g, (B, Hkv, L, D), dev, 0.5)
    shard = L // P
    mls, accs = [], []
    for i in range(P):
        ks = k[:, :, i * shard:(i + 1) * shard].contiguous()
        vs = v[:, :, i * shard:(i + 1) * shard].contiguous()
        lens = torch.full((B,), shard, dtype=torch.int32, device=dev)
        dec = ops.Decoder(B, Hq, Hkv, D, shard, dev)
        ml, acc = dec.partial(q, ks, vs, lens)
        mls.append(ml)
        accs.append(acc)
    o = ops.lse_combine(torch.stack(mls), torch.stack(accs)).view(B, Hq, D)
    qw, kw, vw = words_of(q), words_of(k), words_of(v)
    gold = oracle.decode_attention(qw, kw, vw, np.full(B, L))
    assert_bf16_parity(words_of(o), gold, oracle.decode_attention_fp64(qw, kw, vw, np.full(B, L)), what="combine",
                       tensor_core=decode_on_tensor_cores(Hq, Hkv, D))


def test_rejects_bad_geometry(dev):
    from lara_b200 import ops

    q = torch.zeros((1, 12, 128), dtype=torch.bfloat16, device=dev)
    k = torch.zeros((1, 5, 16, 128), dtype=torch.bfloat16, device=dev)
    with pytest.raises(ValueError):
        ops.gqa_decode(q, k, k, torch.tensor([16], dtype=torch.int32, device=dev))


@pytest.mark.slow
def test_config2_full_size_sampled(dev):
    """Config 2 at full size (B=64, L=4096); oracle on 24 sampled (b, kv-head) pairs."""
    from lara_b200 import ops
    from lara_b200.workloads import CONFIGS, make_decode_inputs

    cfg = CONFIGS[2]
    q, k, v, lens = make_decode_inputs(cfg, dev)
    dec = ops.Decoder(cfg.batch, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, cfg.seq_len, dev)
    o = words_of(dec(q, k, v, lens))
    rng = np.random.default_rng(0)
    pairs = sorted({(int(b), int(h)) for b, h in zip(rng.integers(0, 64, 24), rng.integers(0, 8, 24))})
    bs = sorted({b for b, _ in pairs})
    qw = words_of(q)
    G = cfg.group
    for b in bs:
        kw, vw = words_of(k[b:b + 1]), words_of(v[b:b + 1])
        hs = [h for bb, h in pairs if bb == b]
        gold = oracle.decode_attention(qw[b:b + 1], kw, vw, np.array([4096]), pairs=[(0, h) for h in hs])
        g64 = oracle.decode_attention_fp64(qw[b:b + 1], kw, vw, np.array([4096]), pairs=[(0, h) for h in hs])
        for h in hs:
            sl = slice(h * G, (h + 1) * G)
            assert_bf16_parity(o[b, sl], gold[0, sl], g64[0, sl], what=f"cfg2 b={b} kvh={h}",
                               tensor_core=decode_on_tensor_cores(cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim))


@pytest.mark.slow
def test_config3_ragged_sampled(dev):
    """Config 3 at full size: 256 ragged sequences (128..32768 tokens), K
    channels 0-3 scaled by 20, on the default kernel for its group of 8.  The
    oracle checks one kv head (rotating) of every 16th sequence, all 8 kv heads
    of the 3 longest sequences, and all 8 kv heads of the 3 sequences whose
    largest |logit| (found on the GPU) is the largest of the batch."""
    from lara_b200 import ops
    from lara_b200.workloads import CONFIGS, make_decode_inputs

    cfg = CONFIGS[3]
    B, G, Hkv, D = cfg.batch, cfg.group, cfg.n_kv_heads, cfg.head_dim
    q, k, v, lens = make_decode_inputs(cfg, dev)
    cap = k.shape[2]
    lens_np = lens.cpu().numpy()
    dec = ops.Decoder(B, cfg.n_q_heads, Hkv, D, cap, dev, lens=lens_np)
    o = words_of(dec(q, k, v, lens))
    torch.cuda.synchronize()
    assert ops.workspace_status(dec.workspace) == 0
    peak = np.zeros(B)
    for b in range(B):
        n = int(lens_np[b])
        s = torch.matmul(q[b].float().view(Hkv, G, D), k[b, :, :n].float().transpose(1, 2))
        peak[b] = float(s.abs().max()) / np.sqrt(D)
    longest = [int(b) for b in np.argsort(lens_np)[-3:]]
    hottest = [int(b) for b in np.argsort(peak)[-3:]]
    pairs = {(b, (b // 16) % Hkv) for b in range(0, B, 16)}
    pairs |= {(b, h) for b in longest + hottest for h in range(Hkv)}
    qw = words_of(q)
    for b in sorted({b for b, _ in pairs}):
        n = int(lens_np[b])
        hs = sorted(h for bb, h in pairs if bb == b)
        kw, vw = words_of(k[b:b + 1, :, :n]), words_of(v[b:b + 1, :, :n])
        sel = [(0, h) for h in hs]
        gold = oracle.decode_attention(qw[b:b + 1], kw, vw, np.array([n]), pairs=sel)
        g64 = oracle.decode_attention_fp64(qw[b:b + 1], kw, vw, np.array([n]), pairs=sel)
        for h in hs:
            sl = slice(h * G, (h + 1) * G)
            assert_bf16_parity(o[b, sl], gold[0, sl], g64[0, sl],
                               what=f"cfg3 b={b} len={n} kvh={h} max|logit|={peak[b]:.1f}",
                               tensor_core=decode_on_tensor_cores(cfg.n_q_heads, Hkv, D))


@pytest.mark.slow
def test_config4_long_context_sampled(dev):
    """Config 4 at full size (8 sequences of 1,048,576 cached tokens, N(0,1)*0.5,
    seed 3): the single-GPU decode (the planner's many-split plan) and the
    split-KV path -- four token ranges decoded as partials and merged by the LSE
    combine, as four GPUs would -- both checked against the oracle on 8
    (sequence, kv head) pairs, one per sequence."""
    import torch

    from lara_b200 import ops, parallel
    from lara_b200.workloads import CONFIGS, make_decode_inputs

    cfg = CONFIGS[4]
    B, L = cfg.batch, cfg.seq_len
    q, k, v, lens = make_decode_inputs(cfg, dev, batch=B)
    dec = ops.Decoder(B, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, L, dev)
    o_full = words_of(dec(q, k, v, lens))
    mls, accs = [], []
    for r in range(4):
        start, cnt = parallel.token_range(L, 4, r)
        part = ops.Decoder(B, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, cnt, dev)
        # the rank's token range as a strided view of the full cache (no copy)
        kr, vr = k[:, :, start:start + cnt], v[:, :, start:start + cnt]
        ml, acc = part.partial(q, kr.contiguous(), vr.contiguous(),
                               torch.full((B,), cnt, dtype=torch.int32, device=dev))
        mls.append(ml)
        accs.append(acc)
        del kr, vr
        torch.cuda.empty_cache()
    o_split = words_of(ops.lse_combine(torch.stack(mls), torch.stack(accs)).view(B, cfg.n_q_heads, cfg.head_dim))
    qw = words_of(q)
    G = cfg.group
    for b in range(B):
        h = (3 * b + 1) % cfg.n_kv_heads
        kw, vw = words_of(k[b:b + 1, h:h + 1]), words_of(v[b:b + 1, h:h + 1])
        qs = qw[b:b + 1, h * G:(h + 1) * G]
        gold = oracle.decode_attention(qs, kw, vw, np.array([L]))
        g64 = oracle.decode_attention_fp64(qs, kw, vw, np.array([L]))
        tc = decode_on_tensor_cores(cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim)
        assert_bf16_parity(o_full[b, h * G:(h + 1) * G], gold[0], g64[0], what=f"cfg4 full b={b} kvh={h}",
                           tensor_core=tc)
        assert_bf16_parity(o_split[b, h * G:(h + 1) * G], gold[0], g64[0], what=f"cfg4 split b={b} kvh={h}",
                           tensor_core=tc)
