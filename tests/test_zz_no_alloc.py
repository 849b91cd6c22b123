"""GPU test of ``lara_gqa_decode_noalloc``, the decode entry point that allocates nothing.

It exists for callers that cannot allocate device memory where they run
attention (a plugin inside a framework that owns every device allocation, a
serving loop that may not pay cudaMalloc's implicit synchronisation, a
binding that can pass only the operation's tensors): its scratch is a fixed
array in the library's own device memory.  The test calls it through the C
ABI twice in a row and checks each output against the existing entry point
``lara_gqa_decode`` (caller workspace) within the parity tolerance used by the
other GPU tests (``oracle.PARITY_ULPS`` bf16 ulp, ``tests/parity.py``).  It
allocates its inputs with torch; the entry point under test allocates
nothing.  This file is collected last so a failure here does not stop the
rest of the suite.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

import oracle  # noqa: E402
from parity import assert_bf16_parity, decode_on_tensor_cores, words_of  # noqa: E402

pytestmark = pytest.mark.gpu


def _noalloc(lib, q, k, v, lens, o, B, Hq, Hkv, D, L, splits=0, chunk=0):
    return lib.lara_gqa_decode_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), lens.data_ptr(), o.data_ptr(), B,
                                       Hq, Hkv, D, L, 1.0 / math.sqrt(D), splits, chunk,
                                       torch.cuda.current_stream().cuda_stream)


def _inputs(dev, B, Hq, Hkv, D, L, seed):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    q = (torch.randn((B, Hq, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    k = (torch.randn((B, Hkv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    v = (torch.randn((B, Hkv, L, D), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    return q, k, v


@pytest.mark.parametrize("geom", [(4, 32, 8, 128, 4096, [4096, 3000, 1, 2222]), (3, 8, 2, 64, 700, [513, 0, 700])],
                         ids=["llama3_8b", "cfg1_geometry"])
def test_noalloc_matches_workspace_entry_point_twice(geom):
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    from lara_b200 import _native, ops

    dev = torch.device("cuda:0")
    B, Hq, Hkv, D, L, lens_list = geom
    q, k, v = _inputs(dev, B, Hq, Hkv, D, L, seed=B * 31 + D)
    lens = torch.tensor(lens_list, dtype=torch.int32, device=dev)
    expected = ops.Decoder(B, Hq, Hkv, D, L, dev)(q, k, v, lens)  # existing entry point, caller workspace
    torch.cuda.synchronize()
    golden = oracle.bf16_u16_to_fp32(words_of(expected))
    for call in range(2):
        o = torch.full_like(q, float("nan"))
        rc = _noalloc(_native.lib, q, k, v, lens, o, B, Hq, Hkv, D, L)
        assert rc == 0, _native.last_error()
        torch.cuda.synchronize()
        assert_bf16_parity(words_of(o), golden, what=f"no-alloc call {call + 1}")
    # and against the CPU oracle, as for every decode path
    args = (words_of(q), words_of(k), words_of(v), np.asarray(lens_list))
    gold = oracle.decode_attention(*args)
    assert_bf16_parity(words_of(o), gold, oracle.decode_attention_fp64(*args), what="no-alloc vs oracle",
                       tensor_core=decode_on_tensor_cores(Hq, Hkv, D))


def test_noalloc_forced_splits_then_other_shape():
    """Explicit split plan (the in-kernel merge uses the shared counters), then a
    different workload: the second call must not see the first call's state."""
    from lara_b200 import _native, ops

    dev = torch.device("cuda:0")
    q, k, v = _inputs(dev, 2, 32, 8, 128, 4096, seed=5)
    lens = torch.tensor([4096, 2500], dtype=torch.int32, device=dev)
    exp = ops.Decoder(2, 32, 8, 128, 4096, dev, num_splits=8, chunk_tokens=512)(q, k, v, lens)
    o = torch.empty_like(q)
    assert _noalloc(_native.lib, q, k, v, lens, o, 2, 32, 8, 128, 4096, 8, 512) == 0, _native.last_error()
    torch.cuda.synchronize()
    # the same plan runs the same kernel on the same inputs: the same words
    np.testing.assert_array_equal(words_of(o), words_of(exp))
    q2, k2, v2 = _inputs(dev, 5, 64, 8, 128, 1000, seed=6)
    lens2 = torch.tensor([1000, 7, 999, 64, 500], dtype=torch.int32, device=dev)
    exp2 = ops.Decoder(5, 64, 8, 128, 1000, dev)(q2, k2, v2, lens2)
    o2 = torch.empty_like(q2)
    assert _noalloc(_native.lib, q2, k2, v2, lens2, o2, 5, 64, 8, 128, 1000) == 0, _native.last_error()
    torch.cuda.synchronize()
    assert_bf16_parity(words_of(o2), oracle.bf16_u16_to_fp32(words_of(exp2)), what="second workload")


def test_noalloc_rejects_sizes_beyond_the_scratch():
    from lara_b200 import _native

    dev = torch.device("cuda:0")
    q, k, v = _inputs(dev, 64, 32, 8, 128, 256, seed=7)
    lens = torch.full((64,), 256, dtype=torch.int32, device=dev)
    o = torch.empty_like(q)
    # 64 sequences x 32 heads x 64 splits x (128 + 2) floats is ~68 MB > 8 MiB
    rc = _noalloc(_native.lib, q, k, v, lens, o, 64, 32, 8, 128, 256, 64, 64)
    assert rc == _native.LARA_ERR_RESULT_LEN
    assert "no-alloc scratch" in _native.last_error()


def _stage_tokens(head_dim, group):
    """The split-chunk granule: tokens per pipeline stage of the CUDA-core
    decode kernel (``Traits<D, G>::kTile`` in lara_b200/csrc/decode.cu), or the
    tensor-core kernel's 128-token tile for groups only it serves (> 8)."""
    if group > 8:
        return 128
    vec = 4 if group >= 8 else 8
    lanes = head_dim // vec
    rows = 32 // lanes
    passes = max(1, min(4, lanes // group))
    return 8 * passes * rows


def test_noalloc_reduces_a_plan_that_does_not_fit():
    """The one path of its own: with splits = chunk = 0, a workload whose
    planned split partials exceed LARA_NOALLOC_SCRATCH_BYTES is re-planned with
    fewer splits until they fit.  The result must equal, word for word, the
    workspace entry point run with that reduced plan, and meet the oracle."""
    from lara_b200 import _native, ops

    lib = _native.lib
    cap = 8 * 1024 * 1024
    dev = torch.device("cuda:0")
    # groups of 16 query heads: the most partial state per split, so the
    # planner's split count overflows the scratch at moderate batch sizes
    Hq, Hkv, D = 128, 8, 128
    chosen = None
    for B, L in ((8, 32768), (16, 16384), (32, 8192), (16, 32768)):
        s_, c_ = ctypes.c_int(0), ctypes.c_int(0)
        assert lib.lara_decode_plan(B, Hq, Hkv, D, L, None, ctypes.byref(s_), ctypes.byref(c_)) == 0
        if lib.lara_decode_workspace_bytes(B, Hq, Hkv, D, s_.value) > cap:
            chosen = (B, L, s_.value, c_.value)
            break
    assert chosen is not None, "no candidate workload plans more split partials than the scratch holds"
    B, L, splits, chunk = chosen
    planned = splits
    tile = _stage_tokens(D, Hq // Hkv)
    while splits > 1 and lib.lara_decode_workspace_bytes(B, Hq, Hkv, D, splits) > cap:
        splits -= 1
        chunk = -(-L // (tile * splits)) * tile
        splits = -(-L // chunk)
    assert splits < planned and lib.lara_decode_workspace_bytes(B, Hq, Hkv, D, splits) <= cap
    q, k, v = _inputs(dev, B, Hq, Hkv, D, L, seed=9)
    lens = torch.full((B,), L, dtype=torch.int32, device=dev)
    exp = ops.Decoder(B, Hq, Hkv, D, L, dev, num_splits=splits, chunk_tokens=chunk)(q, k, v, lens)
    o = torch.empty_like(q)
    assert _noalloc(lib, q, k, v, lens, o, B, Hq, Hkv, D, L) == 0, _native.last_error()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(words_of(o), words_of(exp))
    qw, ow = words_of(q), words_of(o)
    G = Hq // Hkv
    for b, h in ((0, 0), (B // 2, 3), (B - 1, Hkv - 1)):
        kw, vw = words_of(k[b:b + 1, h:h + 1]), words_of(v[b:b + 1, h:h + 1])
        qs = qw[b:b + 1, h * G:(h + 1) * G]
        gold = oracle.decode_attention(qs, kw, vw, np.array([L]))
        g64 = oracle.decode_attention_fp64(qs, kw, vw, np.array([L]))
        assert_bf16_parity(ow[b, h * G:(h + 1) * G], gold[0], g64[0], tensor_core=decode_on_tensor_cores(Hq, Hkv, D),
                           what=f"no-alloc reduced plan {planned} -> {splits} splits b={b} kvh={h}")
