"""Multi-GPU sharding of the attention node's decode, one process per GPU (torch.distributed).

The reference runs every layer in one process on one ggml backend (src/engine.cpp:282-298). Its
attention node shards in two ways, both built here on the single-GPU C ABI:

* Independent sequences (batched decode): sequences go to ranks by LPT - longest context first,
  each to the least-loaded rank. A rank holds its own sequences' pages, block tables and queries
  and runs the ordinary decode; nothing crosses GPUs on the data path.
* One long sequence: its page list is cut into R contiguous chunks, chunk r's pages resident on
  rank r. Each rank decodes its chunk with lse_out, then the partials are exchanged and merged
  by log-sum-exp, so the merged output is replicated on every rank. Three exchanges:
  - "fused": lstk_cuda_attn_decode_exchange - the decode's own combine kernel stores each row it
    finishes straight into every peer's mailbox over NVLink (CUDA IPC mappings set up once
    through the process group) as value+epoch words, waits until the peers' words of the row
    carry the call's epoch and merges: no launch after the decode;
  - "p2p": the same protocol in a kernel of its own (lstk_cuda_attn_exchange_merge) after the
    decode;
  - "collective": one record [O (rows x D) | lse (rows)] per rank, all-gathered through the
    process group (NCCL on GPUs, gloo on CPUs) and merged with lstk_cuda_attn_merge straight
    out of the gathered buffer through the merge's part strides.
"""
import ctypes
import heapq
import math

import numpy as np
import torch
import torch.distributed as dist

from ._lib import check, lib
from .attn import _DT, HEAD_DIM, DecodeWorkspace, _p, _stream, attn_decode, attn_merge, layout_of


def lpt_partition(lengths, world):
    """Sequences per rank by LPT greedy: longest first (ties: lower index), each to the rank with
    the least total length so far (ties: lower rank). Returns (list of index arrays, ascending
    within a rank; int64 array of per-rank total lengths)."""
    if world <= 0:
        raise ValueError("world must be positive")
    lengths = np.asarray(lengths, np.int64)
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    heap = [(0, r) for r in range(world)]
    parts = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        parts[r].append(i)
        heapq.heappush(heap, (load + int(lengths[i]), r))
    loads = np.zeros(world, np.int64)
    for load, r in heap:
        loads[r] = load
    return [np.array(sorted(p), np.int64) for p in parts], loads


def page_chunks(n_pages, world):
    """Contiguous [start, end) ranges of a page list, one per rank, sizes differing by at most one."""
    if world <= 0 or n_pages < 0:
        raise ValueError("bad page chunking")
    return [(r * n_pages // world, (r + 1) * n_pages // world) for r in range(world)]


def chunk_keys(seq_len, start, end, block_size=32):
    """Number of the sequence's keys that live in pages [start, end) of its block table."""
    return max(0, min(seq_len, end * block_size) - start * block_size)


def record_views(buf, rows, head_dim=HEAD_DIM):
    """(O [R][rows][D], lse [R][rows]) views of a buffer of R records [O | lse]."""
    rec = rows * head_dim + rows
    g = buf.view(-1, rec)
    return g[:, :rows * head_dim].view(g.shape[0], rows, head_dim), g[:, rows * head_dim:]


def all_gather_records(gathered, local, group=None):
    """Gather every rank's record into `gathered` ([world * rec], rank order)."""
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(gathered, local, group=group)
    else:
        dist.all_gather(list(gathered.view(dist.get_world_size(group), -1).unbind(0)), local, group=group)
    return gathered


class PeerMailboxes:
    """This rank's exchange mailbox for `rows` rows (allocated by the library in this GPU's memory)
    and the peers' mailboxes mapped through CUDA IPC handles shared once over the process group;
    `ptrs` is the int64 device tensor of the R mailbox addresses the exchange kernels take. Every
    rank of `group` builds it collectively and calls close() collectively."""

    def __init__(self, rows, device, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        L = lib()
        nbytes = L.lstk_cuda_mailbox_bytes(self.world, rows, HEAD_DIM)
        own, handle = ctypes.c_void_p(), (ctypes.c_char * 64)()
        with torch.cuda.device(device):
            check(L.lstk_cuda_mailbox_alloc(nbytes, ctypes.byref(own), handle))
        self._own = own
        self._peers = []
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(own.value)
                continue
            peer = ctypes.c_void_p()
            check(L.lstk_cuda_mailbox_open(ctypes.create_string_buffer(h, 64), ctypes.byref(peer)))
            self._peers.append(peer)
            ptrs.append(peer.value)
        self.ptrs = torch.tensor(ptrs, dtype=torch.int64, device=device)
        dist.barrier(group=group)

    def close(self):
        """Releases the peer mappings and the own mailbox once every rank is done with them."""
        if self._own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # no rank still writes into another's mailbox
        L = lib()
        for peer in self._peers:
            check(L.lstk_cuda_mailbox_close(peer))
        self._peers = []
        dist.barrier(group=self.group)  # no rank still maps this rank's mailbox
        check(L.lstk_cuda_mailbox_free(self._own))
        self._own = None


class PeerBarrier:
    """A barrier of the ranks' CUDA streams, on the device: one exchange-merge of a single dummy
    row over peer memory (lstk_cuda_attn_exchange_merge), so each rank's kernel returns once every
    rank's stream has reached the same call (bounded by wait_ns; a timeout sets
    LSTK_ERR_TIMEOUT). Its exit skew across ranks is about one NVLink store latency, far below
    the exit skew of a small NCCL collective; used to start the ranks of a timed step together."""

    def __init__(self, device, group=None, wait_ns=0):
        self.mb = PeerMailboxes(1, device, group)
        self.wait_ns = int(wait_ns)
        self.o = torch.zeros(HEAD_DIM, dtype=torch.float32, device=device)
        self.lse = torch.zeros(1, dtype=torch.float32, device=device)
        self.out = torch.empty_like(self.o)
        self.lse_out = torch.empty_like(self.lse)

    def __call__(self):
        check(lib().lstk_cuda_attn_exchange_merge(_p(self.mb.ptrs), self.mb.rank, self.mb.world, _p(self.o),
                                                  _p(self.lse), 1, HEAD_DIM, self.wait_ns, _p(self.out),
                                                  _p(self.lse_out), _stream(None, self.o.device)))

    def close(self):
        self.mb.close()


class KvSplitDecode:
    """Decode of sequences whose pages are split over the ranks of `group` in contiguous chunks.

    Every rank calls it with the same n_seqs / n_head, the same number of times; rank r passes
    its own chunk's block tables and per-sequence key counts (chunk_keys). Returns the merged
    output [n_seqs][n_head][D] f32, identical on every rank, and keeps the merged natural-log
    lse in `self.lse`. Call close() on every rank before the process group goes away."""

    def __init__(self, n_seqs, n_head, n_head_kv, device, group=None, exchange="p2p", wait_ns=0):
        if exchange not in ("fused", "p2p", "collective"):
            raise ValueError("exchange must be 'fused', 'p2p' or 'collective'")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.exchange = exchange
        self.wait_ns = int(wait_ns)
        self.n_seqs, self.n_head = n_seqs, n_head
        self.rows = n_seqs * n_head
        rec = self.rows * HEAD_DIM + self.rows
        self.local = torch.empty(rec, dtype=torch.float32, device=device)
        self.ws = DecodeWorkspace(n_seqs, n_head, n_head_kv, device)
        self.out = torch.empty((n_seqs, n_head, HEAD_DIM), dtype=torch.float32, device=device)
        self.lse = torch.empty((n_seqs, n_head), dtype=torch.float32, device=device)
        self._mb = None
        if exchange == "collective":
            self.gathered = torch.empty(self.world * rec, dtype=torch.float32, device=device)
        else:
            self._mb = PeerMailboxes(self.rows, device, group)
            self.mailboxes = self._mb.ptrs

    def close(self):
        """Releases the peer mappings and the own mailbox once every rank is done with them."""
        if self._mb is not None:
            self._mb.close()
            self._mb = None

    def __call__(self, k_cache, v_cache, q, block_tables, chunk_lens, scale=None, max_seq_len=0):
        if self.exchange == "fused":
            L = layout_of(k_cache)
            if scale is None:
                scale = 1.0 / math.sqrt(HEAD_DIM)
            check(lib().lstk_cuda_attn_decode_exchange(
                ctypes.byref(L), _p(k_cache), _p(v_cache), _p(q), _DT[q.dtype], self.n_seqs, self.n_head,
                _p(block_tables), block_tables.shape[1], _p(chunk_lens), int(max_seq_len), float(scale), _p(self.out),
                _p(self.lse), _p(self.ws.buf), self.ws.buf.numel(), 0, _p(self.mailboxes), self.rank, self.world,
                self.wait_ns, _stream(None, q.device)))
            return self.out
        o_loc, lse_loc = record_views(self.local, self.rows)
        attn_decode(k_cache, v_cache, q, block_tables, chunk_lens, scale, max_seq_len,
                    out=o_loc[0].view(self.n_seqs, self.n_head, HEAD_DIM),
                    lse_out=lse_loc[0].view(self.n_seqs, self.n_head), workspace=self.ws)
        if self.exchange == "p2p":
            check(lib().lstk_cuda_attn_exchange_merge(_p(self.mailboxes), self.rank, self.world, _p(o_loc[0]),
                                                      _p(lse_loc[0]), self.rows, HEAD_DIM, self.wait_ns,
                                                      _p(self.out), _p(self.lse), _stream(None, q.device)))
            return self.out
        all_gather_records(self.gathered, self.local, self.group)
        o_parts, lse_parts = record_views(self.gathered, self.rows)
        attn_merge(o_parts, lse_parts, out=self.out.view(self.rows, HEAD_DIM), lse_out=self.lse.view(self.rows))
        return self.out
