"""Rank bodies for the multi-process sharding tests (spawned children import this module).

Each worker joins a process group on 127.0.0.1, runs its shard and writes a small JSON verdict
to `result_dir/rank<r>.json`; the parent test asserts on those files. Harness code only.
"""
import json
import math
import os
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

from helpers import D, random_cache, random_q, scattered_block_tables, within, max_err
from oracle import oracle as O

SCALE = 1.0 / math.sqrt(D)


def _join(rank, world, port, backend):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    kw = {}
    if backend == "nccl":
        torch.cuda.set_device(rank)
        kw["device_id"] = torch.device("cuda", rank)
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=timedelta(seconds=60), **kw)


def _chunk_table(bt, s, e):
    sub = np.ascontiguousarray(bt[:, s:e]) if e > s else np.zeros((bt.shape[0], 1), np.int32)
    return sub


def kv_split_cpu(rank, world, port, result_dir):
    """Config-4 shape on the host: one long context split over the ranks in contiguous page
    chunks; each rank's partial (oracle, exact) goes through the product's record layout and
    gather, then the oracle's LSE merge; compared with the whole-context oracle decode. Also the
    LPT sequence partition: every rank decodes its own sequences, rank 0 gathers them and
    compares with the unsharded batch."""
    from localstack_b200.shard import all_gather_records, chunk_keys, lpt_partition, page_chunks, record_views

    _join(rank, world, port, "gloo")
    res = {}
    try:
        rng = np.random.default_rng(41)
        hq, hkv = 32, 4
        # 32 pages; 3 pages (uneven chunks); 2 pages; 1 page (rank 0's chunk is empty: lse -inf)
        for ctx in (1000, 70, 33, 20):
            bt, n_pages = scattered_block_tables(rng, [ctx])
            kc, vc = random_cache(rng, n_pages, hkv)
            q = random_q(rng, 1, hq)
            s, e = page_chunks((ctx + 31) // 32, world)[rank]
            n = chunk_keys(ctx, s, e)
            o, lse = O.paged_attn(q, [0], [ctx - 1], kc, vc, _chunk_table(bt, s, e), [n], SCALE,
                                  mode=O.MODE_EXACT, want_lse=True)
            local = torch.from_numpy(np.concatenate([o.reshape(-1), lse.reshape(-1)]).astype(np.float32))
            gathered = torch.empty(world * local.numel(), dtype=torch.float32)
            all_gather_records(gathered, local)
            o_parts, lse_parts = record_views(gathered, hq)
            merged, _ = O.lse_merge(o_parts.numpy(), lse_parts.numpy())
            whole = O.paged_attn(q, [0], [ctx - 1], kc, vc, bt, [ctx], SCALE, mode=O.MODE_EXACT)
            res[f"split_{ctx}"] = [within(merged, whole.reshape(hq, D), atol=1e-5, rtol=1e-5),
                                   max_err(merged, whole.reshape(hq, D))]
        # sequence sharding: same seeded batch on every rank, LPT partition, no data-path collective
        lens = rng.integers(1, 400, 9).astype(np.int64)
        bt, n_pages = scattered_block_tables(rng, lens.tolist())
        kc, vc = random_cache(rng, n_pages, hkv)
        q = random_q(rng, len(lens), hq)
        parts, loads = lpt_partition(lens, world)
        mine = parts[rank]
        out = np.zeros((len(lens), hq, D), np.float32)
        if len(mine):
            o = O.paged_attn(q[mine], np.arange(len(mine)), lens[mine] - 1, kc, vc, bt[mine], lens[mine], SCALE,
                             mode=O.MODE_EXACT)
            out[mine] = o
        # gathered to rank 0 for verification only (sum of disjoint rows)
        t = torch.from_numpy(out)
        dist.reduce(t, dst=0)
        if rank == 0:
            whole = O.paged_attn(q, np.arange(len(lens)), lens - 1, kc, vc, bt, lens, SCALE, mode=O.MODE_EXACT)
            res["seq_shard"] = [within(t.numpy(), whole, atol=1e-6, rtol=1e-6), max_err(t.numpy(), whole)]
        res["loads"] = loads.tolist()
        res["mine"] = mine.tolist()
    finally:
        dist.destroy_process_group()
    with open(os.path.join(result_dir, f"rank{rank}.json"), "w") as f:
        json.dump(res, f)


def kv_split_nccl(rank, world, port, result_dir):
    """The product's KvSplitDecode over NCCL: rank r's block table lists only its chunk's pages."""
    import localstack_b200 as L
    from localstack_b200.shard import KvSplitDecode, PeerBarrier, chunk_keys, page_chunks

    _join(rank, world, port, "nccl")
    res = {}
    try:
        dev = torch.device("cuda", rank)
        rng = np.random.default_rng(43)
        hq, hkv, ctx = 32, 4, 20000 + 13
        bt, n_pages = scattered_block_tables(rng, [ctx])
        kc, vc = random_cache(rng, n_pages, hkv)
        q = random_q(rng, 1, hq)
        s, e = page_chunks((ctx + 31) // 32, world)[rank]
        n = chunk_keys(ctx, s, e)
        f16 = lambda a: torch.from_numpy(a.view(np.int16)).to(dev).view(torch.float16)
        args = (f16(kc), f16(vc), torch.from_numpy(q).to(dev), torch.from_numpy(_chunk_table(bt, s, e)).to(dev),
                torch.tensor([n], dtype=torch.int32, device=dev), SCALE)
        ex = O.paged_attn(q, [0], [ctx - 1], kc, vc, bt, [ctx], SCALE, mode=O.MODE_EXACT)
        for exchange in ("fused", "p2p", "collective"):
            dec = KvSplitDecode(1, hq, hkv, dev, exchange=exchange)
            for _ in range(3):  # repeated calls: epochs / banks alternate
                out = dec(*args)
            torch.cuda.synchronize()
            L.check_status()
            res[f"split_{exchange}"] = [within(out.cpu().numpy(), ex), max_err(out.cpu().numpy(), ex)]
            if exchange in ("fused", "p2p"):
                # one step captured in a CUDA graph and replayed
                side = torch.cuda.Stream()
                side.wait_stream(torch.cuda.current_stream())
                with torch.cuda.stream(side):
                    dec(*args)
                torch.cuda.current_stream().wait_stream(side)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    dec(*args)
                dec.out.zero_()
                for _ in range(3):
                    g.replay()
                torch.cuda.synchronize()
                L.check_status()
                res[f"split_{exchange}_graph"] = [within(dec.out.cpu().numpy(), ex), max_err(dec.out.cpu().numpy(), ex)]
                del g
            dec.close()
        # The device-side barrier of the ranks' streams that starts each timed split step.
        pbar = PeerBarrier(dev)
        for _ in range(5):
            pbar()
        torch.cuda.synchronize()
        L.check_status()
        pbar.close()
        res["peer_barrier"] = [True, 0.0]
    finally:
        dist.destroy_process_group()
    with open(os.path.join(result_dir, f"rank{rank}.json"), "w") as f:
        json.dump(res, f)
