"""Generates tests/golden/kv_cache_ops.json from the reference's own KvCache.

Run in a container where the reference sources exist (oracle/Makefile compiles
src/kv_cache.cpp unchanged into oracle/_ref/libref_kv_cache.so against oracle/ref_shim). The
script applies seeded random sequences of alloc / remove_seq / truncate_seq (the operations the
reference's Engine and server issue, src/engine.cpp:200-243, src/server.cpp:212-219) and
records, after every operation, what the reference returned and its full bookkeeping state. The
fixture lets tests check the product's host bookkeeping (include/lstk_kv_cache.h) on machines
without the reference.

    python tests/golden/gen_kv_cache_golden.py
"""
import json
import os
import sys
import zlib

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as O  # noqa: E402

OUT = os.path.join(HERE, "kv_cache_ops.json")


def snapshot(kv, seqs):
    cs, cp = kv.cells()
    return {
        "used_hwm": int(kv.used_hwm),
        "n_free_cells": int(kv.n_free_cells()),
        "free_blocks": kv.free_blocks().tolist(),
        "seq_blocks": {str(s): kv.seq_blocks(s).tolist() for s in seqs},
        "lengths": {str(s): int(kv.length(s)) for s in seqs},
        # per-cell ownership as CRC32 of the int32 arrays (full arrays only in each case's last op)
        "cell_seq_crc": zlib.crc32(np.ascontiguousarray(cs, np.int32).tobytes()),
        "cell_pos_crc": zlib.crc32(np.ascontiguousarray(cp, np.int32).tobytes()),
    }


def run_case(seed, size, n_ops, permute):
    rng = np.random.default_rng(seed)
    kv = O.RefKvCache(size)
    ops = []
    if permute:
        perm = rng.permutation(size // 32).astype(np.uint32)
        kv.set_free_blocks(perm)
        ops.append({"op": "set_free_blocks", "blocks": perm.tolist()})
    seqs = list(range(4))
    for _ in range(n_ops):
        r = rng.random()
        s = int(rng.integers(0, 4))
        if r < 0.6:
            n = int(rng.choice([1, 1, 3, 31, 32, 33, 70]))
            res = kv.alloc(s, n)
            rec = {"op": "alloc", "seq": s, "n": n, "ok": res is not None}
            if res is not None:
                rec["cells"] = res[0].tolist()
                rec["positions"] = res[1].tolist()
        elif r < 0.8:
            keep = int(rng.integers(-1, kv.length(s) + 2))
            kv.truncate_seq(s, keep)
            rec = {"op": "truncate_seq", "seq": s, "keep": keep}
        else:
            kv.remove_seq(s)
            rec = {"op": "remove_seq", "seq": s}
        rec["state"] = snapshot(kv, seqs)
        # mask rows for the sequence's last two positions over the reference's dense scan length
        L = kv.length(s)
        if L > 0:
            pos = np.array([max(0, L - 2), L - 1], np.int32)
            n_kv = min(size, max(256, (kv.used_hwm + 255) // 256 * 256))
            mask = kv.fill_mask(s, pos, n_kv)
            rec["mask"] = {"seq": s, "pos": pos.tolist(), "n_kv": n_kv,
                           "visible": [np.nonzero(row == 0)[0].tolist() for row in mask],
                           "neg_inf_bits_ok": bool(np.all((mask == 0) | (mask == 0xFC00)))}
        ops.append(rec)
    cs, cp = kv.cells()
    return {"seed": seed, "size": size, "ops": ops, "final_cell_seq": cs.tolist(), "final_cell_pos": cp.tolist()}


def main():
    if not O.ref_available():
        O.build()
    if not O.ref_available():
        raise SystemExit("reference sources absent: cannot regenerate the fixture")
    cases = [run_case(seed, size, n_ops, permute)
             for seed, size, n_ops, permute in [(1, 256, 60, False), (2, 512, 80, True), (3, 1024, 120, True)]]
    with open(OUT, "w") as f:
        json.dump({"source": "reference src/kv_cache.cpp via oracle/_ref/libref_kv_cache.so", "cases": cases}, f,
                  separators=(",", ":"))
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes)")


if __name__ == "__main__":
    main()
