"""The product's host KV bookkeeping (include/lstk_kv_cache.h) against the reference's own
KvCache (src/kv_cache.cpp): the committed golden fixture (generated from the reference by
tests/golden/gen_kv_cache_golden.py) and, where the reference sources exist, live fuzzing of
oracle/_ref/libref_kv_cache.so."""
import json
import os
import zlib

import numpy as np
import pytest

from localstack_b200.kv_cache import KvCache, n_kv_for
from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "kv_cache_ops.json")


def _state(kv, seqs):
    cs, cp = kv.cells()
    return {
        "used_hwm": int(kv.used_hwm),
        "n_free_cells": int(kv.n_free_cells()),
        "free_blocks": kv.free_blocks().tolist(),
        "seq_blocks": {str(s): kv.seq_blocks(s).tolist() for s in seqs},
        "lengths": {str(s): int(kv.length(s)) for s in seqs},
        "cell_seq_crc": zlib.crc32(np.ascontiguousarray(cs, np.int32).tobytes()),
        "cell_pos_crc": zlib.crc32(np.ascontiguousarray(cp, np.int32).tobytes()),
    }


def test_replays_reference_golden_ops():
    with open(GOLDEN) as f:
        data = json.load(f)
    assert data["cases"]
    for case in data["cases"]:
        kv = KvCache(case["size"])
        seqs = list(range(4))
        for op in case["ops"]:
            if op["op"] == "set_free_blocks":
                kv.set_free_blocks(op["blocks"])
                continue
            if op["op"] == "alloc":
                res = kv.alloc(op["seq"], op["n"])
                assert (res is not None) == op["ok"]
                if res is not None:
                    assert res[0].tolist() == op["cells"] and res[1].tolist() == op["positions"]
            elif op["op"] == "truncate_seq":
                kv.truncate_seq(op["seq"], op["keep"])
            else:
                kv.remove_seq(op["seq"])
            assert _state(kv, seqs) == op["state"], op["op"]
            if "mask" in op:
                m = op["mask"]
                mask = kv.fill_mask(m["seq"], m["pos"], m["n_kv"])
                assert [np.nonzero(r == 0)[0].tolist() for r in mask] == m["visible"]
                assert np.all((mask == 0) | (mask == 0xFC00))
        cs, cp = kv.cells()
        assert cs.tolist() == case["final_cell_seq"] and cp.tolist() == case["final_cell_pos"]


@pytest.mark.skipif(not O.ref_available(), reason="reference sources not present (oracle/_ref not built)")
@pytest.mark.parametrize("seed", range(6))
def test_fuzz_against_compiled_reference(seed):
    rng = np.random.default_rng(100 + seed)
    size = int(rng.choice([64, 256, 2048]))
    a, b = KvCache(size), O.RefKvCache(size)
    if seed % 2:
        perm = rng.permutation(size // 32).astype(np.uint32)
        a.set_free_blocks(perm)
        b.set_free_blocks(perm)
    for _ in range(150):
        s = int(rng.integers(0, 5))
        r = rng.random()
        if r < 0.6:
            n = int(rng.integers(0, 90))
            ra, rb = a.alloc(s, n), b.alloc(s, n)
            assert (ra is None) == (rb is None)
            if ra is not None:
                assert np.array_equal(ra[0], rb[0]) and np.array_equal(ra[1], rb[1])
        elif r < 0.8:
            keep = int(rng.integers(-2, a.length(s) + 3))
            a.truncate_seq(s, keep)
            b.truncate_seq(s, keep)
        else:
            a.remove_seq(s)
            b.remove_seq(s)
        assert a.used_hwm == b.used_hwm and a.n_free_cells() == b.n_free_cells()
        assert np.array_equal(a.free_blocks(), b.free_blocks())
        for q in range(5):
            assert a.length(q) == b.length(q) and np.array_equal(a.seq_blocks(q), b.seq_blocks(q))
        ca, cb = a.cells(), b.cells()
        assert np.array_equal(ca[0], cb[0]) and np.array_equal(ca[1], cb[1])
        L = a.length(s)
        if L:
            pos = np.array([0, L - 1], np.int32)
            n_kv = n_kv_for(size, a.used_hwm)
            assert np.array_equal(a.fill_mask(s, pos, n_kv), b.fill_mask(s, pos, n_kv))


def test_block_tables_give_exactly_the_mask_visible_cells():
    rng = np.random.default_rng(9)
    kv = KvCache(512)
    kv.set_free_blocks(rng.permutation(16).astype(np.uint32))
    for seq, n in [(0, 50), (1, 100), (0, 20), (2, 1), (1, 64)]:
        kv.alloc(seq, n)
    kv.truncate_seq(1, 120)
    bt, lens = kv.block_tables([0, 1, 2, 7])
    assert lens.tolist() == [70, 120, 1, 0]
    for i, seq in enumerate([0, 1, 2]):
        for p in [0, lens[i] // 2, lens[i] - 1]:
            mask = kv.fill_mask(seq, [p], 512)[0]
            visible = set(np.nonzero(mask == 0)[0].tolist())
            via_table = {int(bt[i, j // 32]) * 32 + j % 32 for j in range(p + 1)}
            assert visible == via_table


def test_n_kv_for_matches_engine_rule():
    for size in [256, 4096]:
        for n in [1, 255, 256, 257, 3000, 5000]:
            assert n_kv_for(size, n) == min(size, max(256, (n + 255) // 256 * 256))


def test_capacity_and_bad_free_list():
    kv = KvCache(64)
    assert kv.alloc(0, 65) is None and kv.length(0) == 0
    assert kv.alloc(0, 64) is not None and kv.alloc(1, 1) is None
    with pytest.raises(Exception):
        kv.set_free_blocks([0, 2])  # block 2 does not exist in a 64-cell cache
    with pytest.raises(ValueError):
        KvCache(33)
