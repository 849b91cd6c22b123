"""Seeded synthetic workloads for the five BASELINE configurations.

No public dataset is involved: every input is drawn on the device from
``torch.Generator(device).manual_seed(seed)`` as fp32 N(0,1) (times the stated
scale) and rounded to bf16 (round to nearest even, the reference packer's
rounding for finite values).  Draw order per config is fixed: Q first, then
for each sequence K then V (whole [Hkv, L, D] blocks), then new K/V rows.

1. golden decode step: B=1, 8/2 heads, D=64, 512 cached + 1 appended, seed 0
   (the exact inputs of this case come from numpy, ``tests/golden``);
2. Llama-3-8B decode: B=64, 32/8 heads, D=128, L=4096, N(0,1)*0.5, seed 1;
3. ragged stress: B=256, 64/8 heads, D=128, lengths
   ``numpy.random.default_rng(2).integers(128, 32768, 256, endpoint=True)``,
   N(0,1) with K channels 0..3 scaled by 20;
4. long-context split-KV: B=8, 32/8 heads, D=128, L=1,048,576, N(0,1)*0.5, seed 3;
5. chunked prefill: B=4, 2048 new tokens over 8192 cached (causal), 32/8
   heads, D=128, N(0,1)*0.5, seed 4.

``make_decode_inputs`` / ``make_prefill_inputs`` draw a whole workload from
one generator (the tests' inputs).  The sharded forms ``decode_shard`` /
``prefill_shard`` (the benchmark's inputs) draw every piece from its own
generator keyed by (seed, tensor, sequence, token block), so a sequence's --
or a token range's -- words are the same whichever rank holds it and however
many ranks there are, and any rank can redraw any piece to check it.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass(frozen=True)
class DecodeConfig:
    name: str
    batch: int
    n_q_heads: int
    n_kv_heads: int
    head_dim: int
    seq_len: int          # tokens per sequence (max for ragged)
    std: float
    seed: int
    ragged: bool = False
    k_boost_channels: tuple = field(default_factory=tuple)
    k_boost: float = 1.0

    @property
    def group(self) -> int:
        return self.n_q_heads // self.n_kv_heads

    def lens(self, batch: int | None = None) -> np.ndarray:
        b = self.batch if batch is None else batch
        if self.ragged:
            return ragged_lens()[:b].astype(np.int32)
        return np.full(b, self.seq_len, np.int32)

    def kv_bytes(self, lens: np.ndarray) -> int:
        """Algorithmic KV-stream bytes of one decode step: sum(len) * Hkv * D * 2 (K,V) * 2 B."""
        return int(np.sum(lens, dtype=np.int64)) * self.n_kv_heads * self.head_dim * 2 * 2


def ragged_lens() -> np.ndarray:
    """Config 3 lengths, pinned: sum = 4,291,565 tokens."""
    return np.random.default_rng(2).integers(128, 32768, 256, endpoint=True)


CONFIGS = {
    2: DecodeConfig("llama3_8b_decode", 64, 32, 8, 128, 4096, 0.5, 1),
    3: DecodeConfig("ragged_decode_stress", 256, 64, 8, 128, 32768, 1.0, 2, ragged=True,
                    k_boost_channels=(0, 1, 2, 3), k_boost=20.0),
    4: DecodeConfig("long_context_splitkv", 8, 32, 8, 128, 1_048_576, 0.5, 3),
}


@dataclass(frozen=True)
class PrefillConfig:
    name: str = "chunked_prefill"
    batch: int = 4
    n_q_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128
    cached: int = 8192
    new: int = 2048
    std: float = 0.5
    seed: int = 4

    def flops(self) -> int:
        """Valid (query, key) pairs x 4 D FLOP (QK^T and PV, 2 FLOP per MAC)."""
        pairs = self.batch * self.n_q_heads * (self.new * self.cached + self.new * (self.new + 1) // 2)
        return pairs * self.head_dim * 4


PREFILL = PrefillConfig()


def make_decode_inputs(cfg: DecodeConfig, device, *, batch: int | None = None, seq_len: int | None = None,
                       seed: int | None = None, capacity: int | None = None, lens=None):
    """Device tensors (q, k_cache, v_cache, lens) for a decode config.

    ``batch``/``seq_len`` shrink the workload (tests); ``lens`` gives explicit
    per-sequence lengths (a rank's share of a ragged batch); ``capacity`` is
    the cache's token capacity (default: the longest sequence).
    """
    import torch

    if lens is not None:
        lens = np.asarray(lens, dtype=np.int32)
        B = len(lens)
    else:
        B = cfg.batch if batch is None else batch
        lens = cfg.lens(B) if seq_len is None else np.full(B, seq_len, np.int32)
        if seq_len is not None and cfg.ragged:
            lens = np.minimum(cfg.lens(B), seq_len).astype(np.int32)
    cap = int(lens.max()) if capacity is None else int(capacity)
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(cfg.seed if seed is None else seed)
    H, Hkv, D = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    q = (torch.randn((B, H, D), generator=g, device=dev) * cfg.std).to(torch.bfloat16)
    k = torch.empty((B, Hkv, cap, D), dtype=torch.bfloat16, device=dev)
    v = torch.empty((B, Hkv, cap, D), dtype=torch.bfloat16, device=dev)
    scale = torch.ones(D, device=dev)
    for ch in cfg.k_boost_channels:
        scale[ch] = cfg.k_boost
    for b in range(B):
        n = int(lens[b])
        kb = torch.randn((Hkv, n, D), generator=g, device=dev) * cfg.std
        if cfg.k_boost_channels:
            kb *= scale
        k[b, :, :n] = kb.to(torch.bfloat16)
        v[b, :, :n] = (torch.randn((Hkv, n, D), generator=g, device=dev) * cfg.std).to(torch.bfloat16)
        if n < cap:
            k[b, :, n:] = 0
            v[b, :, n:] = 0
    return q, k, v, torch.from_numpy(lens).to(dev)


def make_prefill_inputs(cfg: PrefillConfig, device, *, batch: int | None = None, cached: int | None = None,
                        new: int | None = None):
    """Device tensors for chunked prefill: cache (capacity cached+new, first
    ``cached`` tokens filled), new K/V ``[B, Hkv, n, D]``, q ``[B, n, Hq, D]``,
    cached lengths."""
    import torch

    B = cfg.batch if batch is None else batch
    C = cfg.cached if cached is None else cached
    n = cfg.new if new is None else new
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(cfg.seed)
    H, Hkv, D = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    q = (torch.randn((B, n, H, D), generator=g, device=dev) * cfg.std).to(torch.bfloat16)
    k = torch.zeros((B, Hkv, C + n, D), dtype=torch.bfloat16, device=dev)
    v = torch.zeros((B, Hkv, C + n, D), dtype=torch.bfloat16, device=dev)
    for b in range(B):
        k[b, :, :C] = (torch.randn((Hkv, C, D), generator=g, device=dev) * cfg.std).to(torch.bfloat16)
        v[b, :, :C] = (torch.randn((Hkv, C, D), generator=g, device=dev) * cfg.std).to(torch.bfloat16)
    k_new = (torch.randn((B, Hkv, n, D), generator=g, device=dev) * cfg.std).to(torch.bfloat16)
    v_new = (torch.randn((B, Hkv, n, D), generator=g, device=dev) * cfg.std).to(torch.bfloat16)
    lens = torch.full((B,), C, dtype=torch.int32, device=dev)
    return q, k, v, k_new, v_new, lens


# ---------------------------------------------------------------------------
# sharded, rank-independent draws (benchmark inputs)
# ---------------------------------------------------------------------------

TOKEN_BLOCK = 65536  # tokens per generator stream of a (sequence, K or V) row
_Q, _K, _V, _KNEW, _VNEW = 1, 2, 3, 4, 5


def _generator(device, *key):
    """A device generator seeded from a tuple of small ints."""
    import torch

    seed = 0
    for x in key:
        seed = (seed * 1_000_003 + int(x)) % (2 ** 61 - 1)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _draw_rows(cfg, device, kind: int, b: int, start: int, count: int, total: int, std: float,
               heads: int, boost=None):
    """fp32 rows [heads, count, D] of token range [start, start+count) of one
    sequence whose row holds ``total`` tokens: token block j of the row comes
    from generator (seed, kind, b, j) as N(0,1)*std [, K channels boosted]."""
    import torch

    D = cfg.head_dim
    out = torch.empty((heads, count, D), dtype=torch.float32, device=device)
    j = start // TOKEN_BLOCK
    while count > 0 and j * TOKEN_BLOCK < start + count:
        b0 = j * TOKEN_BLOCK
        n = min(TOKEN_BLOCK, total - b0)
        blk = torch.randn((heads, n, D), generator=_generator(device, cfg.seed, kind, b, j), device=device) * std
        if boost is not None:
            blk *= boost
        lo, hi = max(start, b0), min(start + count, b0 + n)
        out[:, lo - start:hi - start] = blk[:, lo - b0:hi - b0]
        j += 1
    return out


def decode_shard(cfg: DecodeConfig, device, seqs, lens_all, *, token_start: int = 0, token_count=None,
                 capacity=None):
    """Decode inputs of the global sequences ``seqs`` (indices into the
    workload's batch, lengths ``lens_all[b]``), restricted to the token range
    [token_start, token_start + token_count) of every sequence (a split-KV
    rank's slice; default: every token).

    Returns q [len(seqs), Hq, D], k/v [len(seqs), Hkv, capacity, D] (rows past
    a sequence's slice zeroed) and the int32 slice lengths, all on ``device``."""
    import torch

    dev = torch.device(device)
    Hq, Hkv, D = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    lens_all = np.asarray(lens_all)
    local = []
    for b in seqs:
        total = int(lens_all[b])
        cnt = total - token_start if token_count is None else min(int(token_count), total - token_start)
        local.append(max(0, cnt))
    cap = max(1, max(local) if capacity is None else int(capacity))
    boost = None
    if cfg.k_boost_channels:
        boost = torch.ones(D, device=dev)
        for ch in cfg.k_boost_channels:
            boost[ch] = cfg.k_boost
    q = torch.empty((len(seqs), Hq, D), dtype=torch.bfloat16, device=dev)
    k = torch.zeros((len(seqs), Hkv, cap, D), dtype=torch.bfloat16, device=dev)
    v = torch.zeros_like(k)
    for i, b in enumerate(seqs):
        q[i] = (torch.randn((Hq, D), generator=_generator(dev, cfg.seed, _Q, b), device=dev) * cfg.std).to(
            torch.bfloat16)
        n, total = local[i], int(lens_all[b])
        if n > 0:
            k[i, :, :n] = _draw_rows(cfg, dev, _K, b, token_start, n, total, cfg.std, Hkv, boost).to(torch.bfloat16)
            v[i, :, :n] = _draw_rows(cfg, dev, _V, b, token_start, n, total, cfg.std, Hkv).to(torch.bfloat16)
    return q, k, v, torch.tensor(local, dtype=torch.int32, device=dev)


def prefill_units(cfg: PrefillConfig, world: int, rank: int):
    """Rank's share of the prefill's (sequence, kv head) units: a contiguous
    range of the B * Hkv units, returned as [(sequence, first kv head, kv
    heads)] pieces (one per sequence the range touches)."""
    units = cfg.batch * cfg.n_kv_heads
    base, rem = divmod(units, world)
    u0 = rank * base + min(rank, rem)
    u1 = u0 + base + (1 if rank < rem else 0)
    pieces = []
    u = u0
    while u < u1:
        b, h = divmod(u, cfg.n_kv_heads)
        n = min(u1 - u, cfg.n_kv_heads - h)
        pieces.append((b, h, n))
        u += n
    return pieces


def prefill_launch_groups(cfg: PrefillConfig, pieces):
    """Pieces grouped for launching: consecutive whole sequences (all kv heads)
    form one batched group [(first sequence, sequences, 0, Hkv)]; a partial
    sequence is a group of its own [(sequence, 1, first kv head, kv heads)]."""
    groups = []
    for b, h0, nh in pieces:
        whole = h0 == 0 and nh == cfg.n_kv_heads
        if whole and groups and groups[-1][2] == 0 and groups[-1][3] == cfg.n_kv_heads \
                and groups[-1][0] + groups[-1][1] == b:
            groups[-1] = (groups[-1][0], groups[-1][1] + 1, 0, nh)
        else:
            groups.append((b, 1, h0, nh))
    return groups


def prefill_shard(cfg: PrefillConfig, device, b: int, h0: int, nh: int, nb: int = 1):
    """Chunked-prefill inputs of kv heads [h0, h0+nh) of sequences [b, b+nb)
    (and their query heads): q [nb, n, nh*G, D], cache k/v [nb, nh, C+n, D]
    with the first C tokens drawn, new k/v [nb, nh, n, D], cached lengths [C]*nb.
    Each (sequence, tensor) is one generator stream over all heads, sliced to
    the requested heads."""
    import torch

    dev = torch.device(device)
    G, D, C, n = cfg.n_q_heads // cfg.n_kv_heads, cfg.head_dim, cfg.cached, cfg.new
    Hq, Hkv = cfg.n_q_heads, cfg.n_kv_heads
    q = torch.empty((nb, n, nh * G, D), dtype=torch.bfloat16, device=dev)
    k = torch.zeros((nb, nh, C + n, D), dtype=torch.bfloat16, device=dev)
    v = torch.zeros_like(k)
    kn = torch.empty((nb, nh, n, D), dtype=torch.bfloat16, device=dev)
    vn = torch.empty_like(kn)
    for i in range(nb):
        def draw(kind, shape):
            return torch.randn(shape, generator=_generator(dev, cfg.seed, kind, b + i), device=dev) * cfg.std

        q[i] = draw(_Q, (n, Hq, D))[:, h0 * G:(h0 + nh) * G].to(torch.bfloat16)
        k[i, :, :C] = draw(_K, (Hkv, C, D))[h0:h0 + nh].to(torch.bfloat16)
        v[i, :, :C] = draw(_V, (Hkv, C, D))[h0:h0 + nh].to(torch.bfloat16)
        kn[i] = draw(_KNEW, (Hkv, n, D))[h0:h0 + nh].to(torch.bfloat16)
        vn[i] = draw(_VNEW, (Hkv, n, D))[h0:h0 + nh].to(torch.bfloat16)
    return q, k, v, kn, vn, torch.full((nb,), C, dtype=torch.int32, device=dev)
