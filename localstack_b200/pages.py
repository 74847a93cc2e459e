"""Device-side KV-cache bookkeeping (lstk_kv_pages, include/lstk_cuda_attn.h).

The reference's KvCache (src/kv_cache.cpp:59-132) hands out cells on the host, so every decode
step uploads cells, positions and block tables. DevicePages keeps the same state (LIFO stack of
free 32-cell blocks, per-slot block tables and lengths, high-water mark) in device memory and
applies KvCache's rules in kernels: `alloc` is KvCache::alloc(slot, count) per listed slot, in
list order (prompt chunks and decode tokens of one continuous-batching step in one launch);
`release` is truncate_seq / remove_seq (prefix reuse truncates, a finished request removes). The tables and lengths are the arrays
attn_decode reads, so allocate -> kv_append -> attn_decode runs without a host round trip.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from ._lib import KvPages, check, lib
from .attn import _p, _stream

BLOCK = 32


class DevicePages:
    """Bookkeeping for `size` cells and `n_slots` sequence slots of up to `max_blocks` blocks each.

    The free stack starts as KvCache::init builds it (block 0 on top) unless `free_blocks` gives
    another order (bottom first, as KvCache::set_free_blocks)."""

    def __init__(self, size, n_slots, max_blocks, device="cuda", free_blocks=None):
        if size <= 0 or size % BLOCK:
            raise ValueError("size must be a positive multiple of 32")
        n_blocks = size // BLOCK
        if free_blocks is None:
            free_blocks = np.arange(n_blocks - 1, -1, -1, dtype=np.uint32)
        fb = np.ascontiguousarray(free_blocks, np.uint32)
        if fb.size > n_blocks or (fb.size and int(fb.max()) >= n_blocks) or np.unique(fb).size != fb.size:
            raise ValueError("free_blocks must be distinct block ids below size / 32")
        self.size, self.n_slots, self.max_blocks = size, n_slots, max_blocks
        self.free_blocks = torch.zeros(n_blocks, dtype=torch.int32, device=device)
        self.device = self.free_blocks.device
        self.free_blocks[: fb.size] = torch.from_numpy(fb.view(np.int32)).to(device)
        self.free_top = torch.tensor([fb.size], dtype=torch.int32, device=device)
        self.block_tables = torch.zeros(n_slots, max_blocks, dtype=torch.int32, device=device)
        self.seq_lens = torch.zeros(n_slots, dtype=torch.int32, device=device)
        self.used_hwm = torch.zeros(1, dtype=torch.int32, device=device)
        self.state = KvPages(self.free_blocks.data_ptr(), self.free_top.data_ptr(), self.block_tables.data_ptr(),
                             self.seq_lens.data_ptr(), self.used_hwm.data_ptr(), n_slots, max_blocks, BLOCK)

    def alloc(self, slots, counts=None, max_tokens=None, cells=None, positions=None, ok=None, stream=None):
        """KvCache::alloc(slots[i], counts[i]) for each (distinct) slot in order, on the device.

        counts: None (one token each) or an int32 device tensor; max_tokens bounds their sum (the
        outputs' length; defaults to len(cells) when given, else one token per slot). Returns
        (cells int64 [tokens], positions int32 [tokens], ok int32 [n]); slot i's tokens follow
        those of slots 0..i-1."""
        n = slots.numel()
        if slots.dtype != torch.int32 or slots.device != self.device or not slots.is_contiguous():
            raise ValueError("slots must be a contiguous int32 tensor on the cache's device")
        if counts is not None and (counts.dtype != torch.int32 or counts.device != self.device
                                   or counts.numel() != n or not counts.is_contiguous()):
            raise ValueError("counts must be a contiguous int32 tensor on the cache's device, one per slot")
        if max_tokens is None:
            if counts is not None and cells is None:
                raise ValueError("give max_tokens (or cells) with counts")
            max_tokens = cells.numel() if cells is not None else n
        cells = torch.empty(max_tokens, dtype=torch.int64, device=self.device) if cells is None else cells
        positions = torch.empty(max_tokens, dtype=torch.int32, device=self.device) if positions is None else positions
        ok = torch.empty(n, dtype=torch.int32, device=self.device) if ok is None else ok
        if cells.numel() < max_tokens or positions.numel() < max_tokens or ok.numel() < n:
            raise ValueError("output tensors are shorter than max_tokens / the slot count")
        check(lib().lstk_cuda_kv_alloc(ctypes.byref(self.state), _p(slots), _p(counts), n, int(max_tokens), _p(cells),
                                       _p(positions), _p(ok), _stream(stream, self.device)))
        return cells, positions, ok

    def alloc_step(self, slots, cells=None, positions=None, ok=None, stream=None):
        """One decode token for each (distinct) slot."""
        return self.alloc(slots, None, slots.numel(), cells, positions, ok, stream)

    def release(self, slot, keep=0, stream=None):
        """KvCache::truncate_seq(slot, keep) for keep > 0, remove_seq(slot) otherwise."""
        check(lib().lstk_cuda_kv_release(ctypes.byref(self.state), int(slot), int(keep),
                                         _stream(stream, self.device)))

    def free_list(self):
        """The free stack bottom first (KvCache::free_blocks order)."""
        top = int(self.free_top.item())
        return self.free_blocks[:top].cpu().numpy().view(np.uint32).copy()
