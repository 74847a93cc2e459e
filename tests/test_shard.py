"""Host logic of the multi-GPU paths (LPT sequence partition, contiguous page chunks, the
[O | lse] record exchange) on CPU, including a world_size-2 gloo run."""
import json
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from localstack_b200.shard import chunk_keys, lpt_partition, page_chunks


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_lpt_partition_covers_every_sequence_once():
    rng = np.random.default_rng(3)
    lens = rng.integers(1024, 32769, 64)
    for world in (1, 2, 3, 8):
        parts, loads = lpt_partition(lens, world)
        allidx = np.sort(np.concatenate(parts))
        assert np.array_equal(allidx, np.arange(64))
        assert [int(lens[p].sum()) for p in parts] == loads.tolist()
        # LPT guarantee: the heaviest rank exceeds the mean by less than the longest sequence
        assert loads.max() <= lens.sum() / world + lens.max()


def test_lpt_partition_small_cases():
    parts, loads = lpt_partition([5, 1, 4, 3], 2)
    assert [p.tolist() for p in parts] == [[0, 1], [2, 3]] and loads.tolist() == [6, 7]
    parts, loads = lpt_partition([7], 3)  # more ranks than sequences: the others get nothing
    assert [p.tolist() for p in parts] == [[0], [], []] and loads.tolist() == [7, 0, 0]
    parts, _ = lpt_partition([], 2)
    assert all(len(p) == 0 for p in parts)
    with pytest.raises(ValueError):
        lpt_partition([1], 0)


def test_page_chunks_and_keys():
    assert page_chunks(4096, 8) == [(512 * r, 512 * (r + 1)) for r in range(8)]
    ch = page_chunks(10, 4)
    assert ch[0][0] == 0 and ch[-1][1] == 10 and all(a[1] == b[0] for a, b in zip(ch, ch[1:]))
    assert max(e - s for s, e in ch) - min(e - s for s, e in ch) <= 1
    assert page_chunks(1, 4) == [(0, 0), (0, 0), (0, 0), (0, 1)]
    ctx = 1000  # 32 pages, the last holding 8 keys
    assert sum(chunk_keys(ctx, s, e) for s, e in page_chunks(32, 3)) == ctx
    assert chunk_keys(ctx, 31, 32) == 8 and chunk_keys(ctx, 0, 0) == 0


def test_kv_split_and_sequence_sharding_gloo(tmp_path):
    from shard_workers import kv_split_cpu

    world = 2
    mp.spawn(kv_split_cpu, args=(world, free_port(), str(tmp_path)), nprocs=world, join=True)
    res = [json.load(open(os.path.join(tmp_path, f"rank{r}.json"))) for r in range(world)]
    for r in range(world):
        for ctx in (1000, 70, 33, 20):
            ok, err = res[r][f"split_{ctx}"]
            assert ok, (r, ctx, err)
    assert res[0]["seq_shard"][0], res[0]["seq_shard"]
    assert sorted(res[0]["mine"] + res[1]["mine"]) == list(range(9))
