"""Python view of the host-side KV-cache bookkeeping (include/lstk_kv_cache.h).

Same rules as the reference's KvCache (src/kv_cache.h:24-62): 32-cell blocks from a LIFO free
list, per-sequence block tables, per-cell (seq, pos) ownership. `block_tables()` produces the
int32 tables the decode / prefill kernels read instead of the reference's dense masked scan.
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import LSTK_OK, LstkError, lib

_P = ctypes.c_void_p
_U32 = ctypes.c_uint32
_I32 = ctypes.c_int32

_bound = False


def _bind():
    global _bound
    if _bound:
        return lib()
    L = lib()
    L.lstk_kv_cache_create.argtypes = [_U32, _U32]
    L.lstk_kv_cache_create.restype = _P
    L.lstk_kv_cache_destroy.argtypes = [_P]
    L.lstk_kv_cache_set_free_blocks.argtypes = [_P, _P, _I32]
    L.lstk_kv_cache_alloc.argtypes = [_P, _I32, _I32, _P, _P]
    L.lstk_kv_cache_remove_seq.argtypes = [_P, _I32]
    L.lstk_kv_cache_truncate_seq.argtypes = [_P, _I32, _I32]
    L.lstk_kv_cache_length.argtypes = [_P, _I32]
    L.lstk_kv_cache_length.restype = _I32
    L.lstk_kv_cache_used_hwm.argtypes = [_P]
    L.lstk_kv_cache_used_hwm.restype = _U32
    L.lstk_kv_cache_n_free_cells.argtypes = [_P]
    L.lstk_kv_cache_n_free_cells.restype = _U32
    L.lstk_kv_cache_free_blocks.argtypes = [_P, _P, _I32]
    L.lstk_kv_cache_free_blocks.restype = _I32
    L.lstk_kv_cache_seq_blocks.argtypes = [_P, _I32, _P, _I32]
    L.lstk_kv_cache_seq_blocks.restype = _I32
    L.lstk_kv_cache_cells.argtypes = [_P, _P, _P]
    L.lstk_kv_cache_block_tables.argtypes = [_P, _P, _I32, _I32, _P, _P]
    L.lstk_kv_cache_fill_mask.argtypes = [_P, _I32, _P, _I32, _I32, _P]
    L.lstk_n_kv_for.argtypes = [_U32, _I32]
    L.lstk_n_kv_for.restype = _I32
    _bound = True
    return L


def _ptr(a):
    return a.ctypes.data_as(_P)


class KvCache:
    """Bookkeeping for `size` cells in 32-cell blocks (KvCache::init, src/kv_cache.cpp:11-42)."""

    def __init__(self, size, block_size=32):
        L = _bind()
        self.size = int(size)
        self.block_size = int(block_size)
        self.h = L.lstk_kv_cache_create(self.size, self.block_size)
        if not self.h:
            raise ValueError("size must be a positive multiple of block_size")

    def __del__(self):
        if getattr(self, "h", None):
            _bind().lstk_kv_cache_destroy(self.h)
            self.h = None

    def set_free_blocks(self, blocks):
        b = np.ascontiguousarray(blocks, np.uint32)
        rc = _bind().lstk_kv_cache_set_free_blocks(self.h, _ptr(b), b.size)
        if rc != LSTK_OK:
            raise LstkError(rc, "invalid free-block list")

    def alloc(self, seq, n_tokens):
        """(cells int64, positions int32), or None when the cache is full (nothing allocated)."""
        cells = np.empty(n_tokens, np.int64)
        pos = np.empty(n_tokens, np.int32)
        rc = _bind().lstk_kv_cache_alloc(self.h, seq, n_tokens, _ptr(cells), _ptr(pos))
        return (cells, pos) if rc == LSTK_OK else None

    def remove_seq(self, seq):
        _bind().lstk_kv_cache_remove_seq(self.h, seq)

    def truncate_seq(self, seq, keep):
        _bind().lstk_kv_cache_truncate_seq(self.h, seq, keep)

    def length(self, seq):
        return _bind().lstk_kv_cache_length(self.h, seq)

    @property
    def used_hwm(self):
        return _bind().lstk_kv_cache_used_hwm(self.h)

    def n_free_cells(self):
        return _bind().lstk_kv_cache_n_free_cells(self.h)

    def free_blocks(self):
        out = np.empty(self.size // self.block_size + 1, np.uint32)
        n = _bind().lstk_kv_cache_free_blocks(self.h, _ptr(out), out.size)
        return out[:n].copy()

    def seq_blocks(self, seq):
        out = np.empty(self.size // self.block_size + 1, np.uint32)
        n = _bind().lstk_kv_cache_seq_blocks(self.h, seq, _ptr(out), out.size)
        return out[:n].copy()

    def cells(self):
        cs = np.empty(self.size, np.int32)
        cp = np.empty(self.size, np.int32)
        _bind().lstk_kv_cache_cells(self.h, _ptr(cs), _ptr(cp))
        return cs, cp

    def block_tables(self, seqs, max_blocks=None):
        """(block_tables int32 [n][max_blocks], seq_lens int32 [n]) for the kernels."""
        seqs = np.ascontiguousarray(seqs, np.int32)
        if max_blocks is None:
            max_blocks = max([1] + [(self.length(int(s)) + self.block_size - 1) // self.block_size for s in seqs])
        bt = np.empty((seqs.size, max_blocks), np.int32)
        lens = np.empty(seqs.size, np.int32)
        rc = _bind().lstk_kv_cache_block_tables(self.h, _ptr(seqs), seqs.size, max_blocks, _ptr(bt), _ptr(lens))
        if rc != LSTK_OK:
            raise LstkError(rc, "a sequence needs more than max_blocks blocks")
        return bt, lens

    def fill_mask(self, seq, pos, n_kv):
        pos = np.ascontiguousarray(pos, np.int32)
        mask = np.empty((pos.size, n_kv), np.uint16)
        _bind().lstk_kv_cache_fill_mask(self.h, seq, _ptr(pos), pos.size, n_kv, _ptr(mask))
        return mask


def n_kv_for(cache_size, n_total):
    """Engine::n_kv_for (src/engine.cpp:193-196)."""
    return _bind().lstk_n_kv_for(cache_size, n_total)
