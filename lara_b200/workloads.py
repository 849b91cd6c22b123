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
