"""q8_0 KV cache: the reference's planned alternative to its f16 cache (docs/plan.md:389-395).

Values are ggml's block_q8_0 (per 32 consecutive values of a row: d = amax / 127 as f16, q =
round-to-nearest-even(x / d) as int8), kept in two planes so every 128-byte row is 16-byte
aligned for TMA: `qs` int8 [n_cells][n_head_kv][128] and `d` f16 [n_cells][n_head_kv][4]. About
0.53 of the f16 cache's bytes, so a decode step reads half as much.
"""
import ctypes
import math

import torch

from ._lib import KvLayout, check, lib
from .attn import _DT, BLOCK_SIZE, HEAD_DIM, DecodeWorkspace, _p, _stream


class Q8Cache:
    """One K or V cache as q8_0 planes (zeroed: masked cells hold finite values)."""

    def __init__(self, n_cells, n_head_kv, device="cuda"):
        if n_cells % BLOCK_SIZE:
            raise ValueError("n_cells must be a multiple of 32")
        self.qs = torch.zeros((n_cells, n_head_kv, HEAD_DIM), dtype=torch.int8, device=device)
        self.d = torch.zeros((n_cells, n_head_kv, HEAD_DIM // 32), dtype=torch.float16, device=device)

    @property
    def layout(self):
        n_cells, hkv, hd = self.qs.shape
        return KvLayout(n_cells, hkv, hd, BLOCK_SIZE)

    @property
    def device(self):
        return self.qs.device

    def to_ggml_blocks(self, stream=None):
        """The cache as ggml's block_q8_0 rows: uint8 [n_cells][n_head_kv][4 * 34]."""
        n_cells, hkv, _ = self.qs.shape
        out = torch.empty((n_cells, hkv, 4 * 34), dtype=torch.uint8, device=self.device)
        check(lib().lstk_cuda_q8_to_ggml_blocks(_p(self.qs), _p(self.d), n_cells * hkv, _p(out),
                                                _stream(stream, self.device)))
        return out

    @staticmethod
    def from_ggml_blocks(blocks, stream=None):
        """A cache from ggml's block_q8_0 rows (uint8 [n_cells][n_head_kv][4 * 34])."""
        n_cells, hkv, nb = blocks.shape
        if blocks.dtype != torch.uint8 or nb != 4 * 34 or not blocks.is_contiguous():
            raise ValueError("blocks must be a contiguous uint8 [n_cells][n_head_kv][136] tensor")
        c = Q8Cache(n_cells, hkv, blocks.device)
        check(lib().lstk_cuda_q8_from_ggml_blocks(_p(blocks), n_cells * hkv, _p(c.qs), _p(c.d),
                                                  _stream(stream, blocks.device)))
        return c

    def dequantize(self):
        """f32 values d * q [n_cells][n_head_kv][128]."""
        return self.qs.float() * self.d.float().repeat_interleave(32, dim=-1)


def alloc_cache_q8(n_cells, n_head_kv, device="cuda"):
    return Q8Cache(n_cells, n_head_kv, device)


def kv_append_q8(kq: Q8Cache, vq: Q8Cache, q, k, v, positions, cells, rope, q_gamma=None, k_gamma=None, eps=1e-6,
                 q_out_dtype=torch.float32, q_out=None, stream=None):
    """kv_append into q8_0 planes: QK-RMSNorm + NEOX RoPE as the f16 path, then the K and V rows
    quantised to q8_0. Returns q_out [T][Hq][D] (f32 or f16)."""
    L = kq.layout
    T = q.shape[0]
    Hq = q.shape[1] if q.dim() == 3 else q.shape[1] // HEAD_DIM
    if q.dtype not in (torch.float32, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q/k/v must share dtype f32 or bf16")
    if positions.dtype != torch.int32 or cells.dtype != torch.int64:
        raise ValueError("positions must be int32 and cells int64")
    if q_out is None:
        q_out = torch.empty((T, Hq, HEAD_DIM), dtype=q_out_dtype, device=q.device)
    check(lib().lstk_cuda_kv_append_q8(ctypes.byref(L), _p(kq.qs), _p(kq.d), _p(vq.qs), _p(vq.d), _p(q), _p(k), _p(v),
                                       _DT[q.dtype], q.stride(0), k.stride(0), v.stride(0), T, Hq, _p(positions),
                                       _p(cells), _p(q_gamma), _p(k_gamma), eps, _p(rope), rope.shape[0], _p(q_out),
                                       _DT[q_out.dtype], _stream(stream, kq.device)))
    return q_out


def attn_decode_q8(kq: Q8Cache, vq: Q8Cache, q, block_tables, seq_lens, scale=None, max_seq_len=0, out=None,
                   lse_out=None, want_lse=False, workspace=None, n_ctas=0, stream=None):
    """Paged decode over q8_0 planes with ggml's CPU semantics for a q8_0 cache (query quantised to
    q8_0, integer block dots, f32 accumulation of the dequantised V). Arguments as attn_decode."""
    L = kq.layout
    B, Hq, _ = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(HEAD_DIM)
    if block_tables.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise ValueError("block_tables and seq_lens must be int32")
    if not (q.is_contiguous() and block_tables.is_contiguous() and seq_lens.is_contiguous()):
        raise ValueError("q, block_tables and seq_lens must be contiguous")
    if out is None:
        out = torch.empty((B, Hq, HEAD_DIM), dtype=torch.float32, device=q.device)
    if want_lse and lse_out is None:
        lse_out = torch.empty((B, Hq), dtype=torch.float32, device=q.device)
    if workspace is None or workspace.n_seqs < B:
        workspace = DecodeWorkspace(B, Hq, L.n_head_kv, q.device)
    check(lib().lstk_cuda_attn_decode_q8(ctypes.byref(L), _p(kq.qs), _p(kq.d), _p(vq.qs), _p(vq.d), _p(q),
                                         _DT[q.dtype], B, Hq, _p(block_tables), block_tables.shape[1], _p(seq_lens),
                                         int(max_seq_len), float(scale), _p(out), _p(lse_out), _p(workspace.buf),
                                         workspace.buf.numel(), int(n_ctas), _stream(stream, kq.device)))
    return (out, lse_out) if want_lse else out


def attn_prefill_q8(kq: Q8Cache, vq: Q8Cache, q, q_seq_start, q_pos0, kv_lens, block_tables, max_q_len, scale=None,
                    out=None, workspace=None, scratch=None, stream=None):
    """Causal prefill over q8_0 planes: the pages the call reads are dequantised into a compact f16
    scratch cache (`scratch`: uint8 of lstk_cuda_q8_prefill_scratch_size bytes, allocated when
    None) and the tensor-core prefill runs on it. Arguments and result as attn_prefill."""
    L = kq.layout
    total, Hq, _ = q.shape
    B = q_pos0.shape[0]
    if scale is None:
        scale = 1.0 / math.sqrt(HEAD_DIM)
    if q.dtype not in (torch.float16, torch.float32) or not q.is_contiguous():
        raise ValueError("q must be a contiguous f16 or f32 tensor [total_tokens][Hq][128]")
    for name, t in (("q_seq_start", q_seq_start), ("q_pos0", q_pos0), ("kv_lens", kv_lens),
                    ("block_tables", block_tables)):
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous int32 tensor")
    max_blocks = block_tables.shape[1]
    if out is None:
        out = torch.empty((total, Hq, HEAD_DIM), dtype=torch.float32, device=q.device)
    ws_need = lib().lstk_cuda_attn_prefill_workspace_size(B, Hq, L.n_head_kv, HEAD_DIM, int(max_q_len), max_blocks,
                                                          total, _DT[q.dtype])
    if ws_need and (workspace is None or workspace.numel() < ws_need):
        workspace = torch.empty(ws_need, dtype=torch.uint8, device=q.device)
    sc_need = lib().lstk_cuda_q8_prefill_scratch_size(B, max_blocks, L.n_head_kv)
    if scratch is None or scratch.numel() < sc_need:
        scratch = torch.empty(sc_need, dtype=torch.uint8, device=q.device)
    check(lib().lstk_cuda_attn_prefill_q8(ctypes.byref(L), _p(kq.qs), _p(kq.d), _p(vq.qs), _p(vq.d), _p(q),
                                          _DT[q.dtype], B, Hq, _p(q_seq_start), int(max_q_len), total, _p(q_pos0),
                                          _p(kv_lens), _p(block_tables), max_blocks, float(scale), _p(out),
                                          _p(workspace), workspace.numel() if workspace is not None else 0,
                                          _p(scratch), scratch.numel(), _stream(stream, kq.device)))
    return out
