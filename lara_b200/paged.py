"""Paged KV cache for many concurrent sequences (device pool + host page allocator).

The reference attends one sequence per transaction out of BRAM
(hw/rtl/mem/kv_cache_ram.sv); a B200 serving process holds thousands of
sequences of different lengths and cannot give each a max-length slab.  Here
K/V live in page pools ``[num_pages, Hkv, page_size, D]`` (bf16; the rows of
one (page, kv head) are contiguous, so the decode kernel still moves each
64-token tile with one or a few bulk copies) and a device block table
``int32[max_seqs, pages_per_seq]`` maps token ``t`` of sequence ``s`` to page
``block_table[s, t // page_size]``.  Pages are allocated on the host from a
free list with reference counts, so a common prefix can be shared between
sequences (``share_prefix``); an append never writes into a shared page.

The kernels are ``lara_gqa_decode_paged`` / ``lara_kv_append_paged``
(include/lara_b200.h); a decode over a paged cache returns the same words as
over a contiguous cache holding the same tokens.  ``save`` / ``load`` use the
``lara-kv-v1`` file format of :mod:`lara_b200.kvfile`.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from . import kvfile
from ._native import check, lib
from .ops import _check_words, _stream, new_workspace


class PagedKVCache:
    def __init__(self, num_pages: int, page_size: int, n_kv_heads: int, head_dim: int, max_seqs: int,
                 max_seq_len: int, device="cuda:0"):
        if page_size < 16 or page_size & (page_size - 1):
            raise ValueError("page_size must be a power of two >= 16")
        self.device = torch.device(device)
        self.page_size, self.n_kv_heads, self.head_dim = int(page_size), int(n_kv_heads), int(head_dim)
        self.num_pages, self.max_seqs = int(num_pages), int(max_seqs)
        self.pages_per_seq = int(math.ceil(max_seq_len / page_size))
        shape = (self.num_pages, self.n_kv_heads, self.page_size, self.head_dim)
        self.k_pages = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        self.v_pages = torch.zeros(shape, dtype=torch.bfloat16, device=self.device)
        self._table = np.full((self.max_seqs, self.pages_per_seq), -1, np.int32)
        self.block_table = torch.from_numpy(self._table).to(self.device)
        self._lens = np.zeros(self.max_seqs, np.int32)
        self.lens = torch.zeros(self.max_seqs, dtype=torch.int32, device=self.device)
        self._refs = np.zeros(self.num_pages, np.int32)
        self._free = list(range(self.num_pages - 1, -1, -1))
        self._active = np.zeros(self.max_seqs, bool)
        self._ws = None
        self._status = new_workspace(256, self.device)

    # ------------------------------------------------------------ allocation
    @property
    def capacity(self) -> int:
        return self.pages_per_seq * self.page_size

    @property
    def free_pages(self) -> int:
        return len(self._free)

    def seq_len(self, slot: int) -> int:
        return int(self._lens[slot])

    def new_sequence(self) -> int:
        idle = np.flatnonzero(~self._active)
        if idle.size == 0:
            raise RuntimeError("no free sequence slot")
        slot = int(idle[0])
        self._active[slot] = True
        self._lens[slot] = 0
        self._sync_rows([slot])
        return slot

    def free_sequence(self, slot: int) -> None:
        for j in range(self.pages_per_seq):
            page = int(self._table[slot, j])
            if page >= 0:
                self._release(page)
                self._table[slot, j] = -1
        self._lens[slot] = 0
        self._active[slot] = False
        self._sync_rows([slot])

    def share_prefix(self, src: int, dst: int, n_tokens: int) -> int:
        """Give ``dst`` the first full pages of ``src`` covering up to ``n_tokens``
        tokens (reference-counted, read-only); returns the tokens shared."""
        if self._lens[dst] != 0 or not self._active[src] or not self._active[dst]:
            raise ValueError("share_prefix needs an active source and an empty active destination")
        n_pages = min(int(n_tokens), int(self._lens[src])) // self.page_size
        for j in range(n_pages):
            page = int(self._table[src, j])
            self._refs[page] += 1
            self._table[dst, j] = page
        self._lens[dst] = n_pages * self.page_size
        self._sync_rows([dst])
        return n_pages * self.page_size

    def reserve(self, slots, n_new: int) -> None:
        """Make sure each slot has pages for n_new more tokens."""
        changed = []
        for slot in slots:
            need_end = int(self._lens[slot]) + int(n_new)
            if need_end > self.capacity:
                raise ValueError(f"sequence {slot} would hold {need_end} tokens > capacity {self.capacity}")
            first = int(self._lens[slot]) // self.page_size
            last = (need_end - 1) // self.page_size if need_end > 0 else -1
            for j in range(first, last + 1):
                page = int(self._table[slot, j])
                if page >= 0 and self._refs[page] > 1:
                    raise ValueError(f"sequence {slot} would append into shared page {page}")
                if page < 0:
                    if not self._free:
                        raise MemoryError("page pool exhausted")
                    page = self._free.pop()
                    self._refs[page] = 1
                    self._table[slot, j] = page
                    changed.append(slot)
        if changed:
            self._sync_rows(sorted(set(changed)))

    def _release(self, page: int) -> None:
        self._refs[page] -= 1
        if self._refs[page] == 0:
            self._free.append(page)

    def _sync_rows(self, slots) -> None:
        idx = torch.as_tensor(np.asarray(slots, np.int64), device=self.device)
        self.block_table.index_copy_(0, idx, torch.from_numpy(self._table[slots]).to(self.device))
        self.lens.index_copy_(0, idx, torch.from_numpy(self._lens[slots]).to(self.device))

    def _slots(self, slots):
        if slots is None:
            slots = np.flatnonzero(self._active)
        slots = np.asarray(slots, np.int64)
        if slots.size == 0 or not np.all(self._active[slots]):
            raise ValueError("slots must name active sequences")
        return slots

    # --------------------------------------------------------------- kernels
    def append(self, k_new, v_new, slots=None) -> None:
        """k/v_new ``[n_seq, Hkv, n, D]`` (bf16) for the given slots (default: all active, ascending)."""
        slots = self._slots(slots)
        n = int(k_new.shape[2])
        _check_words("k_new", k_new, (len(slots), self.n_kv_heads, n, self.head_dim))
        _check_words("v_new", v_new, (len(slots), self.n_kv_heads, n, self.head_dim))
        self.reserve(slots, n)
        idx = torch.as_tensor(slots, device=self.device)
        table = self.block_table.index_select(0, idx)
        lens = self.lens.index_select(0, idx)
        check(lib.lara_kv_append_paged(self.k_pages.data_ptr(), self.v_pages.data_ptr(), table.data_ptr(),
                                       lens.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), len(slots),
                                       self.n_kv_heads, self.head_dim, self.page_size, self.pages_per_seq,
                                       self.num_pages, n, self._status.data_ptr(), _stream(self.device)),
              "lara_kv_append_paged")
        self.lens.index_copy_(0, idx, lens)
        self._lens[slots] += n

    def decode(self, q, slots=None, scale=None):
        """q ``[n_seq, Hq, D]`` (bf16) -> o ``[n_seq, Hq, D]`` over each slot's cached tokens."""
        import ctypes

        slots = self._slots(slots)
        B, hq, d = q.shape
        _check_words("q", q, (len(slots), hq, self.head_dim))
        idx = torch.as_tensor(slots, device=self.device)
        table = self.block_table.index_select(0, idx)
        lens = self.lens.index_select(0, idx)
        lens_host = np.ascontiguousarray(self._lens[slots])
        ns, ch = ctypes.c_int(0), ctypes.c_int(0)
        check(lib.lara_decode_plan(B, hq, self.n_kv_heads, d, self.capacity, lens_host.ctypes.data,
                                   ctypes.byref(ns), ctypes.byref(ch)), "lara_decode_plan")
        nbytes = int(lib.lara_decode_workspace_bytes(B, hq, self.n_kv_heads, d, ns.value))
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = new_workspace(nbytes, self.device)
        o = torch.empty_like(q)
        sc = 1.0 / math.sqrt(d) if scale is None else float(scale)
        check(lib.lara_gqa_decode_paged(q.data_ptr(), self.k_pages.data_ptr(), self.v_pages.data_ptr(),
                                        table.data_ptr(), lens.data_ptr(), o.data_ptr(), B, hq, self.n_kv_heads, d,
                                        self.page_size, self.pages_per_seq, self.num_pages, sc, ns.value, ch.value,
                                        self._ws.data_ptr(), self._ws.numel(), _stream(self.device)),
              "lara_gqa_decode_paged")
        return o

    def status(self) -> int:
        """Device status bits of the last appends and decodes (read and cleared)."""
        from .ops import workspace_status

        bits = workspace_status(self._status)
        if self._ws is not None:
            bits |= workspace_status(self._ws)
        return bits

    # ------------------------------------------------------------ contents
    def gather(self, slot: int):
        """(k, v) ``[Hkv, len, D]`` of one sequence, read through its block table."""
        n = int(self._lens[slot])
        pages = self._table[slot, : (n + self.page_size - 1) // self.page_size]
        idx = torch.as_tensor(pages.astype(np.int64), device=self.device)
        k = self.k_pages.index_select(0, idx).permute(1, 0, 2, 3).reshape(self.n_kv_heads, -1, self.head_dim)
        v = self.v_pages.index_select(0, idx).permute(1, 0, 2, 3).reshape(self.n_kv_heads, -1, self.head_dim)
        return k[:, :n].contiguous(), v[:, :n].contiguous()

    def save(self, path, slots=None) -> None:
        slots = self._slots(slots)
        T = max(int(self._lens[slots].max()), 1)
        k = np.zeros((len(slots), self.n_kv_heads, T, self.head_dim), np.uint16)
        v = np.zeros_like(k)
        for i, s in enumerate(slots):
            ks, vs = self.gather(int(s))
            n = ks.shape[1]
            k[i, :, :n] = ks.view(torch.int16).cpu().numpy().view(np.uint16)
            v[i, :, :n] = vs.view(torch.int16).cpu().numpy().view(np.uint16)
        kvfile.save(path, k, v, self._lens[slots])

    def load(self, path) -> list[int]:
        """Create one new sequence per stored sequence; returns their slots."""
        k, v, lens = kvfile.load(path)
        if k.shape[1] != self.n_kv_heads or k.shape[3] != self.head_dim:
            raise ValueError(f"{path}: geometry {k.shape} does not match this cache")
        slots = []
        for i in range(k.shape[0]):
            s = self.new_sequence()
            slots.append(s)
            n = int(lens[i])
            if n:
                t = lambda a: torch.from_numpy(np.ascontiguousarray(a[None, :, :n]).view(np.int16)).to(  # noqa: E731
                    self.device).view(torch.bfloat16)
                self.append(t(k[i]), t(v[i]), slots=[s])
        return slots
