"""Python bindings of the attention-node C ABI over torch device tensors.

Each function mirrors one group of the ggml nodes that the reference's attn_block
(src/qwen3.cpp:128-171) records, and forwards to the sm_100a kernels in liblstk_attn.so through
the C ABI of include/lstk_cuda_attn.h. Tensors only carry device memory and the current CUDA
stream; all compute happens in the library. Errors raise LstkError with the library's message,
as the reference returns `false` with `err` set.
"""
from __future__ import annotations

import ctypes
import math

import torch

from . import _lib
from ._lib import DTYPE_BF16, DTYPE_F16, DTYPE_F32, KvLayout, check, lib

HEAD_DIM = 128
BLOCK_SIZE = 32

_DT = {torch.float32: DTYPE_F32, torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16}


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(stream=None, device=None):
    """Stream handle to launch on: `stream`, else the current stream of `device` (the tensors'
    device; the current device when None). The raw handle avoids building a torch Stream object,
    which costs several microseconds per call."""
    if stream is not None:
        return ctypes.c_void_p(stream.cuda_stream)
    idx = device.index if isinstance(device, torch.device) else device
    if idx is None:
        idx = torch.cuda.current_device()
    if _raw_stream is not None:
        return ctypes.c_void_p(_raw_stream(idx))
    return ctypes.c_void_p(torch.cuda.current_stream(idx).cuda_stream)


def layout_of(k_cache: torch.Tensor) -> KvLayout:
    """Layout of a [n_cells][n_head_kv][head_dim] f16 cache tensor (KvCache::k[l], src/kv_cache.h:32)."""
    if k_cache.dtype != torch.float16 or k_cache.dim() != 3 or not k_cache.is_contiguous():
        raise ValueError("cache must be a contiguous f16 [n_cells, n_head_kv, head_dim] tensor")
    n_cells, hkv, hd = k_cache.shape
    return KvLayout(n_cells, hkv, hd, BLOCK_SIZE)


def alloc_cache(n_cells, n_head_kv, device="cuda", head_dim=HEAD_DIM):
    """A zeroed f16 cache tensor; KvCache::init also clears its buffer (src/kv_cache.cpp:31-32) so
    that masked cells never hold non-finite values."""
    if n_cells % BLOCK_SIZE:
        raise ValueError("n_cells must be a multiple of 32")
    return torch.zeros((n_cells, n_head_kv, head_dim), dtype=torch.float16, device=device)


def rope_table_host(n_pos, head_dim=HEAD_DIM, freq_base=1e6, freq_scale=1.0):
    """[n_pos][head_dim/2][2] f32 (cos, sin) table, filled on the host by the library."""
    t = torch.empty((n_pos, head_dim // 2, 2), dtype=torch.float32)
    check(lib().lstk_rope_table_fill(ctypes.c_void_p(t.data_ptr()), n_pos, head_dim, freq_base, freq_scale))
    return t


def rope_table(n_pos, device="cuda", head_dim=HEAD_DIM, freq_base=1e6, freq_scale=1.0):
    return rope_table_host(n_pos, head_dim, freq_base, freq_scale).to(device)


def kv_append(k_cache, v_cache, q, k, v, positions, cells, rope, q_gamma=None, k_gamma=None, eps=1e-6,
              q_out_dtype=torch.float32, q_out=None, stream=None):
    """QK-RMSNorm + NEOX RoPE + f16 scatter of K/V into the cache (src/qwen3.cpp:139-153).

    q [T][Hq][D] (or a [T][>= Hq*D] view), k/v [T][Hkv][D]; f32 or bf16. positions int32 [T],
    cells int64 [T]. Returns q_out [T][Hq][D] in q_out_dtype (f32 or f16)."""
    L = layout_of(k_cache)
    T = q.shape[0]
    Hq = q.shape[1] if q.dim() == 3 else q.shape[1] // HEAD_DIM
    if q.dtype not in (torch.float32, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q/k/v must share dtype f32 or bf16")
    if positions.dtype != torch.int32 or cells.dtype != torch.int64:
        raise ValueError("positions must be int32 and cells int64")
    if q_out is None:
        q_out = torch.empty((T, Hq, HEAD_DIM), dtype=q_out_dtype, device=q.device)
    check(lib().lstk_cuda_kv_append(ctypes.byref(L), _p(k_cache), _p(v_cache), _p(q), _p(k), _p(v), _DT[q.dtype],
                                    q.stride(0), k.stride(0), v.stride(0), T, Hq, _p(positions), _p(cells),
                                    _p(q_gamma), _p(k_gamma), eps, _p(rope), rope.shape[0], _p(q_out),
                                    _DT[q_out.dtype], _stream(stream, k_cache.device)))
    return q_out


class DecodeWorkspace:
    """Caller-owned scratch for attn_decode (sized by lstk_cuda_attn_decode_workspace_size)."""

    def __init__(self, n_seqs, n_head, n_head_kv, device="cuda"):
        nbytes = lib().lstk_cuda_attn_decode_workspace_size(n_seqs, n_head, n_head_kv, HEAD_DIM)
        self.buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        self.n_seqs = n_seqs


def attn_decode(k_cache, v_cache, q, block_tables, seq_lens, scale=None, max_seq_len=0, out=None, lse_out=None,
                want_lse=False, workspace=None, n_ctas=0, stream=None, kv_range=None):
    """Paged decode attention, one query token per sequence (src/qwen3.cpp:155-167).

    q [B][Hq][D] f32/f16; block_tables int32 [B][max_blocks]; seq_lens int32 [B]. Returns out
    [B][Hq][D] f32 (and lse [B][Hq] natural log when want_lse). kv_range=(begin, end) restricts
    every sequence to its keys [begin, min(end, len)) (begin a multiple of 32; the partial
    entry point), for results to be combined with attn_merge."""
    L = layout_of(k_cache)
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
    if kv_range is None:
        check(lib().lstk_cuda_attn_decode(ctypes.byref(L), _p(k_cache), _p(v_cache), _p(q), _DT[q.dtype], B, Hq,
                                          _p(block_tables), block_tables.shape[1], _p(seq_lens), int(max_seq_len),
                                          float(scale), _p(out), _p(lse_out), _p(workspace.buf),
                                          workspace.buf.numel(), int(n_ctas), _stream(stream, k_cache.device)))
    else:
        check(lib().lstk_cuda_attn_decode_partial(ctypes.byref(L), _p(k_cache), _p(v_cache), _p(q), _DT[q.dtype], B,
                                                  Hq, _p(block_tables), block_tables.shape[1], _p(seq_lens),
                                                  int(max_seq_len), int(kv_range[0]), int(kv_range[1]),
                                                  float(scale), _p(out), _p(lse_out), _p(workspace.buf),
                                                  workspace.buf.numel(), int(n_ctas),
                                                  _stream(stream, k_cache.device)))
    return (out, lse_out) if want_lse else out


def attn_merge(o_parts, lse_parts, out=None, lse_out=None, stream=None):
    """Log-sum-exp merge of partial results over disjoint key ranges.

    o_parts [R][rows][D] f32, lse_parts [R][rows] f32 (natural log); each part's rows are dense,
    parts may be strided (e.g. views into one gathered buffer of [O | lse] records).
    Returns (out, lse)."""
    R, rows, D = o_parts.shape
    if o_parts.stride(2) != 1 or o_parts.stride(1) != D or lse_parts.shape != (R, rows) or lse_parts.stride(1) != 1:
        raise ValueError("attn_merge: each part must be a dense [rows][D] / [rows] block")
    if out is None:
        out = torch.empty((rows, D), dtype=torch.float32, device=o_parts.device)
    if lse_out is None:
        lse_out = torch.empty((rows,), dtype=torch.float32, device=o_parts.device)
    check(lib().lstk_cuda_attn_merge(_p(o_parts), _p(lse_parts), R, rows, D, o_parts.stride(0), lse_parts.stride(0),
                                     _p(out), _p(lse_out), _stream(stream, o_parts.device)))
    return out, lse_out


def attn_prefill(k_cache, v_cache, q, q_seq_start, q_pos0, kv_lens, block_tables, max_q_len, scale=None, out=None,
                 workspace=None, stream=None):
    """Paged causal prefill attention on the tensor cores (src/qwen3.cpp:155-167, n_tokens > 1).

    q [total_tokens][Hq][D] f16 (or f32, converted in the workspace); q_seq_start int32 [B+1];
    q_pos0, kv_lens int32 [B]; block_tables int32 [B][max_blocks]. Returns out f32 like q."""
    L = layout_of(k_cache)
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
    if q_seq_start.numel() != B + 1 or kv_lens.numel() != B or block_tables.shape[0] != B:
        raise ValueError("q_seq_start [B+1], q_pos0 / kv_lens [B] and block_tables [B][max_blocks] must agree")
    if out is None:
        out = torch.empty((total, Hq, HEAD_DIM), dtype=torch.float32, device=q.device)
    elif out.dtype != torch.float32 or not out.is_contiguous() or out.numel() < total * Hq * HEAD_DIM:
        raise ValueError("out must be a contiguous f32 tensor with total_tokens * Hq * 128 elements")
    if q.dtype == torch.float32:  # the f16 copy of q lives in the workspace; f16 queries need none
        need = lib().lstk_cuda_attn_prefill_workspace_size(B, Hq, L.n_head_kv, HEAD_DIM, int(max_q_len),
                                                           block_tables.shape[1], total, _DT[q.dtype])
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=q.device)
    check(lib().lstk_cuda_attn_prefill(ctypes.byref(L), _p(k_cache), _p(v_cache), _p(q), _DT[q.dtype], B, Hq,
                                       _p(q_seq_start), int(max_q_len), total, _p(q_pos0), _p(kv_lens),
                                       _p(block_tables), block_tables.shape[1], float(scale), _p(out),
                                       _p(workspace), workspace.numel() if workspace is not None else 0,
                                       _stream(stream, k_cache.device)))
    return out


def check_status(stream=None):
    """Synchronise and raise if a kernel recorded a timeout or an out-of-range index."""
    check(lib().lstk_cuda_status(_stream(stream)))
