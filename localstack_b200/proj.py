"""Python bindings of the projection entry points (lstk_cuda_proj, lstk_cuda_rms_norm,
lstk_cuda_to_bf16) over torch device tensors.

They replace the dense nodes around the reference's attention: rms(x, attn_norm), the Wq / Wk /
Wv projections and the Wo projection with its residual add (src/qwen3.cpp:112-120, 134-138,
169-170). Weights are in ggml's mul_mat layout, [out_features][in_features] (in contiguous).
"""
from __future__ import annotations

import torch

from ._lib import check, lib
from .attn import _DT, _p, _stream


def _rows(t, name):
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a 2-D tensor with contiguous rows")
    return t.shape[0], t.shape[1], t.stride(0)


_workspaces = {}  # device -> uint8 tensor for the K split of small-m projections (grown on demand)


def _split_workspace(m, n, k, device):
    need = lib().lstk_cuda_proj_workspace_size(m, n, k)
    if need == 0:
        return None
    ws = _workspaces.get(device)
    if ws is None or ws.numel() < need:
        ws = torch.empty(need, dtype=torch.uint8, device=device)
        _workspaces[device] = ws
    return ws


def proj(x, w, residual=None, out=None, out_dtype=torch.bfloat16, stream=None, split_k=True):
    """out = x @ w.T (+ residual) on the tensor cores. x [m][k] bf16, w [n][k] bf16, residual
    [m][n] bf16 (may be `out` itself); out [m][n] bf16 or f32. With split_k, small-m shapes split K
    over the idle SMs through a workspace kept per device (allocated on first use of a shape: make
    that call before any stream capture)."""
    m, k, ldx = _rows(x, "x")
    n, kw, ldw = _rows(w, "w")
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or kw != k:
        raise ValueError("x [m][k] and w [n][k] must be bf16 with the same k")
    if residual is not None:
        mr, nr, ldr = _rows(residual, "residual")
        if residual.dtype != torch.bfloat16 or (mr, nr) != (m, n):
            raise ValueError("residual must be bf16 [m][n]")
    else:
        ldr = 0
    if out is None:
        out = torch.empty((m, n), dtype=out_dtype, device=x.device)
    mo, no, ldo = _rows(out, "out")
    if (mo, no) != (m, n) or out.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("out must be [m][n] bf16 or f32")
    ws = _split_workspace(m, n, k, x.device) if split_k else None
    if ws is not None:
        check(lib().lstk_cuda_proj_ws(_p(x), ldx, _p(w), ldw, m, n, k, _p(residual), ldr, _p(out), _DT[out.dtype], ldo,
                                      _p(ws), ws.numel(), _stream(stream, x.device)))
    else:
        check(lib().lstk_cuda_proj(_p(x), ldx, _p(w), ldw, m, n, k, _p(residual), ldr, _p(out), _DT[out.dtype], ldo,
                                   _stream(stream, x.device)))
    return out


def rms_norm(x, gamma=None, eps=1e-6, out=None, stream=None):
    """Row RMSNorm times gamma (f32 [cols] or None), bf16 out. x [rows][cols] bf16 or f32."""
    rows, cols, ldx = _rows(x, "x")
    if out is None:
        out = torch.empty((rows, cols), dtype=torch.bfloat16, device=x.device)
    _, _, ldy = _rows(out, "out")
    if out.dtype != torch.bfloat16 or tuple(out.shape) != (rows, cols):
        raise ValueError("out must be bf16 [rows][cols]")
    if gamma is not None and (gamma.dtype != torch.float32 or gamma.numel() != cols or not gamma.is_contiguous()):
        raise ValueError("gamma must be a contiguous f32 [cols] tensor")
    check(lib().lstk_cuda_rms_norm(_p(x), _DT[x.dtype], ldx, _p(gamma), float(eps), _p(out), ldy, rows, cols,
                                   _stream(stream, x.device)))
    return out


def to_bf16(x, out=None, stream=None):
    """bf16 copy of an f32 [rows][cols] tensor (or a view with contiguous rows)."""
    if x.dim() != 2:
        x = x.reshape(x.shape[0], -1)
    rows, cols, ldx = _rows(x, "x")
    if out is None:
        out = torch.empty((rows, cols), dtype=torch.bfloat16, device=x.device)
    _, _, ldy = _rows(out, "out")
    check(lib().lstk_cuda_to_bf16(_p(x), ldx, _p(out), ldy, rows, cols, _stream(stream, x.device)))
    return out
