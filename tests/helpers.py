"""Seeded synthetic inputs shared by the tests (harness code, not product code)."""
from __future__ import annotations

import numpy as np

from oracle import oracle as O

PAGE = 32
D = 128


def pages_for(n):
    return (int(n) + PAGE - 1) // PAGE


def scattered_block_tables(rng, seq_lens, extra_pages=3):
    """Block tables for sequences of the given lengths, pages drawn from a seeded permutation of
    all pages (the way a permuted free list scatters them through KvCache::alloc). Returns
    (block_tables int32 [B][max_blocks], n_pages)."""
    need = [pages_for(n) for n in seq_lens]
    n_pages = sum(need) + extra_pages
    order = rng.permutation(n_pages).astype(np.int32)
    max_blocks = max(1, max(need) if need else 1)
    bt = np.full((len(seq_lens), max_blocks), -1, np.int32)
    at = 0
    for b, k in enumerate(need):
        bt[b, :k] = order[at:at + k]
        at += k
    # unused entries point at a valid page so a stray read stays in bounds
    bt[bt < 0] = order[-1]
    return bt, n_pages


def random_cache(rng, n_pages, n_head_kv, norm_k=True):
    """f16 bit arrays [n_pages*32][Hkv][128]: K rows RMS-normalised N(0,1), V rows N(0,1)."""
    n_cells = n_pages * PAGE
    k = rng.standard_normal((n_cells, n_head_kv, D), dtype=np.float32)
    if norm_k:
        k = k / np.sqrt(np.mean(k * k, axis=-1, keepdims=True) + 1e-6)
    v = rng.standard_normal((n_cells, n_head_kv, D), dtype=np.float32)
    return O.f32_to_f16_bits(k), O.f32_to_f16_bits(v)


def random_q(rng, n, n_head, normed=True):
    q = rng.standard_normal((n, n_head, D), dtype=np.float32)
    if normed:
        q = q / np.sqrt(np.mean(q * q, axis=-1, keepdims=True) + 1e-6)
    return q.astype(np.float32)


def within(a, b, atol=2e-3, rtol=1e-2):
    """The parity tolerance: |a - b| <= atol + rtol * |b| elementwise (f32 outputs)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return bool(np.all(np.abs(a - b) <= atol + rtol * np.abs(b)))


def max_err(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)))) if np.size(a) else 0.0
