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


def _mailbox(n_ranks, rows):
    import ctypes
    lib = L.lib()
    own, h = ctypes.c_void_p(), (ctypes.c_char * 64)()
    assert lib.lstk_cuda_mailbox_alloc(lib.lstk_cuda_mailbox_bytes(n_ranks, rows, 128), ctypes.byref(own), h) == 0
    return own


@pytest.mark.gpu
def test_exchange_merge_single_rank_epochs_and_graph():
    """R = 1: the merged rows are the local rows exactly, over several calls (epochs advance in
    the mailbox) and from a CUDA graph replayed with new inputs."""
    import ctypes
    lib = L.lib()
    rows = 32
    own = _mailbox(1, rows)
    try:
        boxes = torch.tensor([own.value], dtype=torch.int64, device="cuda")
        o = torch.empty(rows, 128, device="cuda")
        lse = torch.empty(rows, device="cuda")
        out = torch.empty_like(o)
        lse_out = torch.empty_like(lse)
        P = lambda t: ctypes.c_void_p(t.data_ptr())
        call = lambda: lib.lstk_cuda_attn_exchange_merge(P(boxes), 0, 1, P(o), P(lse), rows, 128, 0, P(out),
                                                         P(lse_out), ctypes.c_void_p(
                                                             torch.cuda.current_stream().cuda_stream))
        for i in range(3):
            o.normal_()
            lse.normal_()
            assert call() == 0
            torch.cuda.synchronize()
            assert torch.equal(out, o) and torch.equal(lse_out, lse)
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            call()
        torch.cuda.current_stream().wait_stream(side)
        with torch.cuda.graph(g):
            call()
        for i in range(3):
            o.normal_()
            lse.normal_()
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, o) and torch.equal(lse_out, lse)
        del g
        L.check_status()
    finally:
        torch.cuda.synchronize()
        lib.lstk_cuda_mailbox_free(own)


def _fused_case(seed, ctx):
    rng = np.random.default_rng(seed)
    bt, n_pages = scattered_block_tables(rng, [ctx])
    kc, vc = random_cache(rng, n_pages, 4)
    q = random_q(rng, 1, 32)
    f16 = lambda a: torch.from_numpy(a.view(np.int16)).cuda().view(torch.float16)
    return (f16(kc), f16(vc), torch.from_numpy(q).cuda(), torch.from_numpy(bt).cuda(),
            torch.tensor([ctx], dtype=torch.int32, device="cuda"))


def _decode_exchange(args, ws, boxes, rank, n_ranks, out, lse, wait_ns=0):
    import ctypes
    from localstack_b200.attn import _DT, layout_of
    kc, vc, q, bt, lens = args
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    return L.lib().lstk_cuda_attn_decode_exchange(
        ctypes.byref(layout_of(kc)), P(kc), P(vc), P(q), _DT[q.dtype], 1, 32, P(bt), bt.shape[1], P(lens), 0, SCALE,
        P(out), P(lse), P(ws.buf), ws.buf.numel(), 0, P(boxes), rank, n_ranks, wait_ns,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.gpu
@pytest.mark.parametrize("ctx", [20000, 33, 0])
def test_decode_exchange_single_rank_equals_decode(ctx):
    """R = 1: the decode with the exchange fused into its combine gives the plain decode's rows
    and lse exactly (a merge of one record), for a context split over every CTA, one finished
    inside one CTA, and an empty one; over repeated calls (epochs advance) and graph replays."""
    args = _fused_case(5, max(ctx, 1))
    if ctx == 0:
        args = args[:4] + (torch.zeros(1, dtype=torch.int32, device="cuda"),)
    ref, ref_lse = L.attn_decode(*args, SCALE, want_lse=True)
    rows = 32
    own = _mailbox(1, rows)
    try:
        boxes = torch.tensor([own.value], dtype=torch.int64, device="cuda")
        ws = L.DecodeWorkspace(1, 32, 4)
        out = torch.empty((1, 32, 128), device="cuda")
        lse = torch.empty((1, 32), device="cuda")
        for _ in range(3):
            out.fill_(7.0)
            assert _decode_exchange(args, ws, boxes, 0, 1, out, lse) == 0
            torch.cuda.synchronize()
            L.check_status()
            assert torch.equal(out, ref) and torch.equal(lse, ref_lse)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            _decode_exchange(args, ws, boxes, 0, 1, out, lse)
        torch.cuda.current_stream().wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            _decode_exchange(args, ws, boxes, 0, 1, out, lse)
        for _ in range(3):
            out.fill_(7.0)
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, ref) and torch.equal(lse, ref_lse)
        del g
        L.check_status()
    finally:
        torch.cuda.synchronize()
        L.lib().lstk_cuda_mailbox_free(own)


@pytest.mark.gpu
def test_decode_exchange_times_out_when_a_peer_never_writes():
    """Failure detection of the fused path: rank 0 of 2 waits for rank 1's flags, which nothing
    sets; each combine CTA's bounded wait (20 ms) runs out, LSTK_ERR_TIMEOUT is recorded, the rows
    are zeros and the context still decodes correctly afterwards."""
    args = _fused_case(6, 5000)
    before = L.attn_decode(*args, SCALE)
    own, other = _mailbox(2, 32), _mailbox(2, 32)
    try:
        boxes = torch.tensor([own.value, other.value], dtype=torch.int64, device="cuda")
        ws = L.DecodeWorkspace(1, 32, 4)
        out = torch.full((1, 32, 128), 7.0, device="cuda")
        lse = torch.empty((1, 32), device="cuda")
        assert _decode_exchange(args, ws, boxes, 0, 2, out, lse, wait_ns=20_000_000) == 0
        with pytest.raises(L.LstkError) as e:
            L.check_status()
        assert e.value.code == -3
        assert torch.count_nonzero(out).item() == 0
        after = L.attn_decode(*args, SCALE)
        L.check_status()
        assert torch.equal(after, before)
    finally:
        torch.cuda.synchronize()
        L.lib().lstk_cuda_mailbox_free(own)
        L.lib().lstk_cuda_mailbox_free(other)


@pytest.mark.gpu
def test_exchange_merge_times_out_when_a_peer_never_writes():
    """Failure detection: rank 0 of 2 waits for source 1's flags, which nothing sets; the bounded
    wait (20 ms here) runs out, the kernel records LSTK_ERR_TIMEOUT and returns zeros, and the
    device stays usable."""
    import ctypes
    lib = L.lib()
    rows = 8
    own, other = _mailbox(2, rows), _mailbox(2, rows)
    try:
        boxes = torch.tensor([own.value, other.value], dtype=torch.int64, device="cuda")
        o = torch.randn(rows, 128, device="cuda")
        lse = torch.randn(rows, device="cuda")
        out = torch.full_like(o, 7.0)
        P = lambda t: ctypes.c_void_p(t.data_ptr())
        assert lib.lstk_cuda_attn_exchange_merge(P(boxes), 0, 2, P(o), P(lse), rows, 128, 20_000_000, P(out),
                                                 None, ctypes.c_void_p(
                                                     torch.cuda.current_stream().cuda_stream)) == 0
        with pytest.raises(L.LstkError) as e:
            L.check_status()
        assert e.value.code == -3
        assert torch.count_nonzero(out).item() == 0
        L.check_status()  # cleared by the read; the context still works
        assert torch.equal(torch.ones(4, device="cuda") * 2, torch.full((4,), 2.0, device="cuda"))
    finally:
        torch.cuda.synchronize()
        lib.lstk_cuda_mailbox_free(own)
        lib.lstk_cuda_mailbox_free(other)


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
        res = json.load(open(os.path.join(tmp_path, f"rank{r}.json")))
        for key in ("split_fused", "split_fused_graph", "split_p2p", "split_collective", "split_p2p_graph",
                    "peer_barrier"):
            ok, err = res[key]
            assert ok, (r, key, err)
