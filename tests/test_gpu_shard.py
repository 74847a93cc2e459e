"""Multi-GPU decode paths on the device: the KV-split record exchange and its strided LSE merge
(one GPU, ranks emulated by page chunks), and the NCCL run over two ranks when two GPUs exist."""
import json
import math
import os
import socket

import numpy as np
import pytest
import torch

import localstack_b200 as L
from helpers import D, max_err, random_cache, random_q, scattered_block_tables, within
from localstack_b200.shard import chunk_keys, page_chunks, record_views
from oracle import oracle as O

SCALE = 1.0 / math.sqrt(D)


@pytest.mark.gpu
@pytest.mark.parametrize("R", [1, 3, 8])
def test_records_and_strided_merge(R):
    rng = np.random.default_rng(100 + R)
    hq, hkv, ctx = 32, 4, 9000 + 5
    bt, n_pages = scattered_block_tables(rng, [ctx])
    kc, vc = random_cache(rng, n_pages, hkv)
    q = random_q(rng, 1, hq)
    dev = "cuda"
    f16 = lambda a: torch.from_numpy(a.view(np.int16)).to(dev).view(torch.float16)
    kc_t, vc_t, q_t = f16(kc), f16(vc), torch.from_numpy(q).to(dev)
    rows = hq
    buf = torch.full((R * (rows * D + rows),), float("nan"), device=dev)
    o_parts, lse_parts = record_views(buf, rows)
    for r, (s, e) in enumerate(page_chunks((ctx + 31) // 32, R)):
        sub = torch.from_numpy(np.ascontiguousarray(bt[:, s:e])).to(dev)
        L.attn_decode(kc_t, vc_t, q_t, sub, torch.tensor([chunk_keys(ctx, s, e)], dtype=torch.int32, device=dev),
                      SCALE, out=o_parts[r].view(1, hq, D), lse_out=lse_parts[r].view(1, hq))
    out, lse = L.attn_merge(o_parts, lse_parts)
    L.check_status()
    ex, ex_lse = O.paged_attn(q, [0], [ctx - 1], kc, vc, bt, [ctx], SCALE, mode=O.MODE_EXACT, want_lse=True)
    assert within(out.cpu().numpy(), ex.reshape(hq, D)), max_err(out.cpu().numpy(), ex.reshape(hq, D))
    assert np.allclose(lse.cpu().numpy(), ex_lse.reshape(hq), atol=1e-3)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_kv_split_nccl_two_ranks(tmp_path):
    import torch.multiprocessing as mp
    from shard_workers import kv_split_nccl

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = {"NCCL_NVLS_ENABLE": "0"}
    old = {k: os.environ.get(k) for k in env}
    os.environ.update(env)
    try:
        mp.spawn(kv_split_nccl, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    finally:
        for k, v in old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    for r in range(2):
        ok, err = json.load(open(os.path.join(tmp_path, f"rank{r}.json")))["split"]
        assert ok, (r, err)
