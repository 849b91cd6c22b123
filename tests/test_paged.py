"""Paged KV cache (``lara_gqa_decode_paged`` / ``lara_kv_append_paged``,
``lara_b200.paged.PagedKVCache``) and cache persistence (``lara-kv-v1``).

Row (f)4 of the scope: a paged layout for many concurrent sequences and
save/restore of the device cache.  The paged decode must return the same words
as the contiguous decode over the same tokens (same kernel arithmetic, only the
tile addressing differs) and meet the oracle's tolerance; appends must land
every row where the block table says; a shared prefix is read through both
sequences' tables; a bad block-table entry is reported, never dereferenced;
files round-trip bit for bit between the contiguous and the paged layout.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle
from lara_b200 import kvfile


# ------------------------------------------------------------------ CPU tests
def test_kvfile_round_trip_and_tamper(tmp_path):
    rng = np.random.default_rng(0)
    k = rng.integers(0, 1 << 16, (3, 2, 10, 8)).astype(np.uint16)
    v = rng.integers(0, 1 << 16, (3, 2, 10, 8)).astype(np.uint16)
    lens = np.array([10, 0, 7], np.int32)
    p = kvfile.save(tmp_path / "c.npz", k, v, lens)
    k2, v2, l2 = kvfile.load(p)
    np.testing.assert_array_equal(k2, k)
    np.testing.assert_array_equal(v2, v)
    np.testing.assert_array_equal(l2, lens)
    with np.load(p) as z:
        d = {n: z[n] for n in z.files}
    d["k"] = d["k"].copy()
    d["k"][0, 0, 0, 0] ^= 1
    np.savez(tmp_path / "bad.npz", **d)
    with pytest.raises(ValueError, match="checksum"):
        kvfile.load(tmp_path / "bad.npz")
    with pytest.raises(ValueError):
        kvfile.save(tmp_path / "x.npz", k, v, np.array([11, 0, 0], np.int32))


def test_paged_geometry_validated_before_launch():
    from lara_b200 import _native

    lib = _native.lib
    dummy = ctypes.c_void_p(16)
    for ps in (8, 48, 1 << 17):
        rc = lib.lara_gqa_decode_paged(dummy, dummy, dummy, dummy, dummy, dummy, 1, 8, 2, 128, ps, 4, 4, 0.1, 0, 0,
                                       dummy, 1 << 20, None)
        assert rc == _native.LARA_ERR_BAD_CFG
        rc = lib.lara_kv_append_paged(dummy, dummy, dummy, dummy, dummy, dummy, 1, 2, 128, ps, 4, 4, 1, None, None)
        assert rc == _native.LARA_ERR_BAD_CFG
    rc = lib.lara_gqa_decode_paged(dummy, dummy, dummy, None, dummy, dummy, 1, 8, 2, 128, 64, 4, 4, 0.1, 0, 0, dummy,
                                   1 << 20, None)
    assert rc == _native.LARA_ERR_STREAM_DEST


# ------------------------------------------------------------------ GPU tests
def _torch():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    return torch


def _bf16(torch, a, dev):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev).view(torch.bfloat16)


def _fill(cache, torch, k, v, lens, dev, chunks=(None,)):
    """Create one sequence per row and append its tokens in the given chunk sizes."""
    slots = [cache.new_sequence() for _ in range(len(lens))]
    for i, n in enumerate(lens):
        pos = 0
        sizes = list(chunks) if chunks != (None,) else [n]
        while pos < n:
            step = min(sizes[0] or n, n - pos)
            sizes = sizes[1:] + sizes[:1]
            cache.append(_bf16(torch, k[i:i + 1, :, pos:pos + step], dev), _bf16(torch, v[i:i + 1, :, pos:pos + step], dev),
                         slots=[slots[i]])
            pos += step
    return slots


GEOMS = [(128, 4), (128, 8), (64, 4), (128, 1), (128, 16)]


@pytest.mark.gpu
@pytest.mark.parametrize("path", ["auto", "tc", "simt"])
@pytest.mark.parametrize("page_size", [16, 64, 256])
@pytest.mark.parametrize("geom", GEOMS, ids=lambda g: f"D{g[0]}_G{g[1]}")
def test_paged_decode_equals_contiguous(monkeypatch, page_size, geom, path):
    """Both decode kernels (LARA_DECODE_PATH=tc|simt, and the default choice)."""
    torch = _torch()
    from lara_b200 import ops
    from lara_b200.paged import PagedKVCache
    from parity import assert_bf16_parity, decode_on_tensor_cores, words_of

    D, G = geom
    if (path == "tc" and D != 128) or (path == "simt" and G > 8):
        pytest.skip("geometry not compiled for this kernel")
    if path != "auto":
        monkeypatch.setenv("LARA_DECODE_PATH", path)
    hkv = 2
    hq = hkv * G
    lens = [700, 1, 0, 513, 64]
    L = max(lens)
    rng = np.random.default_rng(page_size + D + G)
    pk = oracle.fp32_to_bf16_u16
    k = pk(rng.standard_normal((len(lens), hkv, L, D)).astype(np.float32) * 0.5)
    v = pk(rng.standard_normal((len(lens), hkv, L, D)).astype(np.float32) * 0.5)
    q = pk(rng.standard_normal((len(lens), hq, D)).astype(np.float32) * 0.5)
    dev = torch.device("cuda:0")
    cache = PagedKVCache(num_pages=64 * 1024 // page_size, page_size=page_size, n_kv_heads=hkv, head_dim=D,
                         max_seqs=8, max_seq_len=1024, device=dev)
    # scramble the free list so consecutive tokens land in non-adjacent pages
    order = rng.permutation(cache.num_pages)
    cache._free = [int(p) for p in order]
    slots = _fill(cache, torch, k, v, lens, dev, chunks=(37, 1, 128))
    o_paged = words_of(cache.decode(_bf16(torch, q, dev), slots=slots))
    assert cache.status() == 0
    kc = _bf16(torch, k, dev)
    vc = _bf16(torch, v, dev)
    lt = torch.tensor(lens, dtype=torch.int32, device=dev)
    o_contig = words_of(ops.gqa_decode(_bf16(torch, q, dev), kc, vc, lt))
    np.testing.assert_array_equal(o_paged, o_contig)
    gold = oracle.decode_attention(q, k, v, np.array(lens))
    g64 = oracle.decode_attention_fp64(q, k, v, np.array(lens))
    assert_bf16_parity(o_paged, gold, g64, what=f"paged ps={page_size} D={D} G={G}",
                       tensor_core=decode_on_tensor_cores(hq, hkv, D))
    for i, s in enumerate(slots):  # every row landed where the table says
        ks, vs = cache.gather(s)
        np.testing.assert_array_equal(words_of(ks), k[i, :, :lens[i]])
        np.testing.assert_array_equal(words_of(vs), v[i, :, :lens[i]])


@pytest.mark.gpu
def test_shared_prefix_and_free():
    torch = _torch()
    from lara_b200 import ops
    from lara_b200.paged import PagedKVCache
    from parity import words_of

    dev = torch.device("cuda:0")
    rng = np.random.default_rng(3)
    pk = oracle.fp32_to_bf16_u16
    hkv, D, G = 8, 128, 4
    a_k = pk(rng.standard_normal((1, hkv, 300, D)).astype(np.float32))
    a_v = pk(rng.standard_normal((1, hkv, 300, D)).astype(np.float32))
    b_k = pk(rng.standard_normal((1, hkv, 50, D)).astype(np.float32))
    b_v = pk(rng.standard_normal((1, hkv, 50, D)).astype(np.float32))
    cache = PagedKVCache(num_pages=32, page_size=64, n_kv_heads=hkv, head_dim=D, max_seqs=4, max_seq_len=1024,
                         device=dev)
    a = _fill(cache, torch, a_k, a_v, [300], dev)[0]
    b = cache.new_sequence()
    assert cache.share_prefix(a, b, 280) == 256  # whole pages only
    used = cache.num_pages - cache.free_pages
    cache.append(_bf16(torch, b_k, dev), _bf16(torch, b_v, dev), slots=[b])
    assert cache.num_pages - cache.free_pages == used + 1  # 50 new tokens: one fresh page
    q = pk(rng.standard_normal((1, hkv * G, D)).astype(np.float32))
    o_b = words_of(cache.decode(_bf16(torch, q, dev), slots=[b]))
    kc = np.concatenate([a_k[:, :, :256], b_k], axis=2)
    vc = np.concatenate([a_v[:, :, :256], b_v], axis=2)
    o_ref = words_of(ops.gqa_decode(_bf16(torch, q, dev), _bf16(torch, kc, dev), _bf16(torch, vc, dev),
                                    torch.tensor([306], dtype=torch.int32, device=dev)))
    np.testing.assert_array_equal(o_b, o_ref)
    cache.free_sequence(a)  # the shared pages stay with b
    np.testing.assert_array_equal(words_of(cache.decode(_bf16(torch, q, dev), slots=[b])), o_ref)
    cache.free_sequence(b)
    assert cache.free_pages == cache.num_pages


@pytest.mark.gpu
def test_bad_page_is_reported_not_dereferenced():
    torch = _torch()
    from lara_b200.paged import PagedKVCache

    dev = torch.device("cuda:0")
    cache = PagedKVCache(num_pages=8, page_size=64, n_kv_heads=2, head_dim=128, max_seqs=2, max_seq_len=512,
                         device=dev)
    s = cache.new_sequence()
    kn = torch.zeros((1, 2, 100, 128), dtype=torch.bfloat16, device=dev)
    cache.append(kn, kn, slots=[s])
    cache.block_table[s, 1] = 1000  # corrupt: outside the pool
    cache.decode(torch.zeros((1, 8, 128), dtype=torch.bfloat16, device=dev), slots=[s])
    torch.cuda.synchronize()
    assert cache.status() & 0x8  # kDevBadPage


@pytest.mark.gpu
@pytest.mark.parametrize("path", ["tc", "simt"])
def test_paged_chunk_past_the_page_cache(monkeypatch, path):
    """One split over 9000 tokens in 16-token pages: 563 pages per chunk, past the
    kernels' shared-memory caches of block-table entries (256 on CUDA cores, 512 on
    the tensor-core kernel), so the later tiles read the table through the
    out-of-cache path.  Same words as the contiguous decode with the same split,
    within the oracle's tolerance; then a bad entry past the cache is reported."""
    torch = _torch()
    from lara_b200 import _native
    from lara_b200.ops import _stream, new_workspace, workspace_status
    from parity import assert_bf16_parity, decode_on_tensor_cores, words_of

    monkeypatch.setenv("LARA_DECODE_PATH", path)
    lib = _native.lib
    dev = torch.device("cuda:0")
    hkv, G, D, ps = 2, 8, 128, 16
    hq = hkv * G
    lens = [9000, 8200]
    cap = 9216  # 72 tiles of 128 tokens: one split covers every sequence
    pps = cap // ps
    rng = np.random.default_rng(21)
    pk = oracle.fp32_to_bf16_u16
    B = len(lens)
    k = pk(rng.standard_normal((B, hkv, cap, D)).astype(np.float32) * 0.5)
    v = pk(rng.standard_normal((B, hkv, cap, D)).astype(np.float32) * 0.5)
    q = pk(rng.standard_normal((B, hq, D)).astype(np.float32) * 0.5)
    npg = [(n + ps - 1) // ps for n in lens]
    total = sum(npg)
    perm = rng.permutation(total)
    table = np.full((B, pps), -1, np.int32)
    kp = np.zeros((total, hkv, ps, D), np.uint16)
    vp = np.zeros_like(kp)
    base = 0
    for b, n in enumerate(npg):
        pages = perm[base:base + n]
        table[b, :n] = pages
        kp[pages] = k[b, :, :n * ps].reshape(hkv, n, ps, D).transpose(1, 0, 2, 3)
        vp[pages] = v[b, :, :n * ps].reshape(hkv, n, ps, D).transpose(1, 0, 2, 3)
        base += n
    qt, kt, vt = _bf16(torch, q, dev), _bf16(torch, kp, dev), _bf16(torch, vp, dev)
    tt = torch.from_numpy(table).to(dev)
    lt = torch.tensor(lens, dtype=torch.int32, device=dev)
    nbytes = int(lib.lara_decode_workspace_bytes(B, hq, hkv, D, 1))
    ws = new_workspace(nbytes, dev)
    st = _stream(dev)

    def paged():
        o = torch.empty_like(qt)
        rc = lib.lara_gqa_decode_paged(qt.data_ptr(), kt.data_ptr(), vt.data_ptr(), tt.data_ptr(), lt.data_ptr(),
                                       o.data_ptr(), B, hq, hkv, D, ps, pps, total, 1.0 / np.sqrt(D), 1, cap,
                                       ws.data_ptr(), ws.numel(), st)
        assert rc == 0, _native.last_error()
        return o

    o_paged = words_of(paged())
    assert workspace_status(ws) == 0
    kc, vc = _bf16(torch, k, dev), _bf16(torch, v, dev)
    oc = torch.empty_like(qt)
    rc = lib.lara_gqa_decode(qt.data_ptr(), kc.data_ptr(), vc.data_ptr(), lt.data_ptr(), oc.data_ptr(), B, hq, hkv, D,
                             cap, 1.0 / np.sqrt(D), 1, cap, ws.data_ptr(), ws.numel(), st)
    assert rc == 0, _native.last_error()
    np.testing.assert_array_equal(o_paged, words_of(oc))
    gold = oracle.decode_attention(q, k, v, np.array(lens))
    g64 = oracle.decode_attention_fp64(q, k, v, np.array(lens))
    assert_bf16_parity(o_paged, gold, g64, what=f"paged ps=16, 563 pages in one chunk ({path})",
                       tensor_core=decode_on_tensor_cores(hq, hkv, D))
    tt[0, 540] = total + 5  # past both caches, inside the sequence
    paged()
    assert workspace_status(ws) & 0x8  # kDevBadPage


@pytest.mark.gpu
def test_persistence_round_trips(tmp_path):
    """driver cache -> file -> paged cache (other page size) -> file -> driver cache."""
    torch = _torch()
    from lara_b200.attn_driver import AttentionAccelerator
    from lara_b200.paged import PagedKVCache
    from parity import words_of

    rng = np.random.default_rng(9)
    pk = oracle.fp32_to_bf16_u16
    B, hq, hkv, D, L = 3, 32, 8, 128, 400
    k = pk(rng.standard_normal((B, hkv, L, D)).astype(np.float32) * 0.5)
    v = pk(rng.standard_normal((B, hkv, L, D)).astype(np.float32) * 0.5)
    q = pk(rng.standard_normal((B, hq, D)).astype(np.float32) * 0.5)
    lens = np.array([400, 17, 256], np.int32)
    with AttentionAccelerator() as acc:
        acc.configure_heads(hq, hkv, D, max_seq_len=512, batch=B)
        acc.load_kv(k, v, lens)
        o1 = acc.run_query(q).copy()
        acc.save_kv(tmp_path / "a.npz")
    dev = torch.device("cuda:0")
    cache = PagedKVCache(num_pages=64, page_size=32, n_kv_heads=hkv, head_dim=D, max_seqs=4, max_seq_len=512,
                         device=dev)
    slots = cache.load(tmp_path / "a.npz")
    o2 = words_of(cache.decode(torch.from_numpy(q.view(np.int16)).to(dev).view(torch.bfloat16), slots=slots))
    np.testing.assert_array_equal(o2, o1)
    cache.save(tmp_path / "b.npz", slots=slots)
    with AttentionAccelerator() as acc:
        acc.configure_heads(hq, hkv, D, max_seq_len=512, batch=B)
        acc.restore_kv(tmp_path / "b.npz")
        assert acc.seq_lens.tolist() == lens.tolist()
        np.testing.assert_array_equal(acc.run_query(q), o1)
