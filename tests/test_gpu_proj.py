"""Projection GEMM (tcgen05), RMSNorm and the f32 -> bf16 cast on the GPU against an fp32 (fp64
accumulated) torch reference of the same op.

Tolerance. Operands are bf16 (exact in f32), products exact in f32; the tensor core accumulates in
f32 in its own order, so an f32 output is within a few units of 2^-24 of sum_k |x w| per term:
|gpu - ref| <= 1e-5 * (|x| @ |w|.T) + 1e-6. A bf16 output adds its one rounding:
+ 2^-8 * |ref|.
"""
import numpy as np
import pytest
import torch

import localstack_b200 as L

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ref(x, w, res=None):
    r = x.double() @ w.double().T
    if res is not None:
        r = r + res.double()
    mag = x.double().abs() @ w.double().abs().T
    return r, mag


def _check(out, ref, mag, bf16_out):
    err = (out.double() - ref).abs()
    bound = 1e-5 * mag + 1e-6 + (1.01 * 2.0 ** -8 * ref.abs() if bf16_out else 0)
    bad = err > bound
    assert not bool(bad.any()), f"{int(bad.sum())} of {bad.numel()} outside; max err {float(err.max()):.3e}"


def _operands(m, n, k, seed, scale_w=0.02):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn((m, k), generator=g, device=DEV).bfloat16()
    w = (torch.randn((n, k), generator=g, device=DEV) * scale_w).bfloat16()
    return x, w, g


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_config5_wqkv_shape(out_dtype):
    # Qwen3-30B-A3B fused Wq|Wk|Wv: 4352 tokens x 2048 -> 4096 + 2 x 512
    x, w, _ = _operands(4352, 5120, 2048, 1)
    out = L.proj(x, w, out_dtype=out_dtype)
    L.check_status()
    ref, mag = _ref(x, w)
    _check(out, ref, mag, out_dtype == torch.bfloat16)


def test_config5_wo_with_residual_in_place():
    # Wo: 4352 x 4096 -> 2048, plus the residual stream, written over the residual itself
    x, w, g = _operands(4352, 2048, 4096, 2)
    res = torch.randn((4352, 2048), generator=g, device=DEV).bfloat16()
    ref, mag = _ref(x, w, res)
    out = L.proj(x, w, residual=res, out=res)
    L.check_status()
    _check(out, ref, mag + res.double().abs(), True)


@pytest.mark.parametrize("m,n,k", [(1, 256, 64), (77, 264, 40), (300, 24, 72), (129, 520, 2048), (4500, 64, 136)])
def test_ragged_shapes(m, n, k):
    # tails in every dimension: partial row tiles, partial column chunks, K not a multiple of 64
    x, w, g = _operands(m, n, k, m + n + k)
    res = torch.randn((m, n), generator=g, device=DEV).bfloat16()
    out = L.proj(x, w, residual=res, out_dtype=torch.float32)
    L.check_status()
    ref, mag = _ref(x, w, res)
    _check(out, ref, mag + res.double().abs(), False)


def test_strided_views_and_neighbours_untouched():
    # x and w as column slices of wider buffers; out a column slice: its neighbours keep their bytes
    g = torch.Generator(device=DEV).manual_seed(9)
    xb = torch.randn((200, 256 + 64), generator=g, device=DEV).bfloat16()
    wb = (torch.randn((300, 256 + 32), generator=g, device=DEV) * 0.05).bfloat16()
    ob = torch.full((200, 300 + 40), 7.0, device=DEV)
    x, w = xb[:, 64:], wb[:, :256]
    out = L.proj(x, w, out=ob[:, 8:308])
    L.check_status()
    ref, mag = _ref(x, w)
    _check(out, ref, mag, False)
    assert bool((ob[:, :8] == 7).all()) and bool((ob[:, 308:] == 7).all())


def test_repeated_calls_are_bit_identical():
    x, w, _ = _operands(1000, 1024, 512, 4)
    a = L.proj(x, w)
    b = L.proj(x, w)
    L.check_status()
    assert torch.equal(a, b)


def test_rms_norm_bf16_and_f32_inputs():
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn((4352, 2048), generator=g, device=DEV) * 3
    gamma = 1 + 0.1 * torch.randn(2048, generator=g, device=DEV)
    for xin in (x, x.bfloat16()):
        y = L.rms_norm(xin, gamma, 1e-6)
        L.check_status()
        xd = xin.double()
        ref = xd * torch.rsqrt(xd.square().mean(-1, keepdim=True) + 1e-6) * gamma.double()
        err = (y.double() - ref).abs()
        assert bool((err <= 1.01 * 2.0 ** -8 * ref.abs() + 1e-6).all()), float(err.max())


def test_to_bf16_is_round_to_nearest_even():
    g = torch.Generator(device=DEV).manual_seed(6)
    x = torch.randn((333, 4096), generator=g, device=DEV) * 10
    y = L.to_bf16(x)
    L.check_status()
    assert torch.equal(y, x.bfloat16())
    # a strided source (rows of a wider buffer)
    xb = torch.randn((50, 200), generator=g, device=DEV)
    assert torch.equal(L.to_bf16(xb[:, 8:136]), xb[:, 8:136].bfloat16())


@pytest.mark.parametrize("m,n,k,res,split", [(544, 2048, 4096, True, True), (1088, 5120, 2048, False, False),
                                             (544, 5120, 2048, False, False), (77, 264, 2048, True, True),
                                             (300, 1024, 8192, False, True)])
def test_small_m_split_k(m, n, k, res, split):
    # per-GPU shapes of a sharded config 5 (few tiles): K split over the idle SMs into f32 slices of
    # a workspace, summed with the residual by the reduce kernel; the residual written in place
    need = L.lib().lstk_cuda_proj_workspace_size(m, n, k)
    x, w, g = _operands(m, n, k, m + k)
    r = torch.randn((m, n), generator=g, device=DEV).bfloat16() if res else None
    ref, mag = _ref(x, w, r)
    out = L.proj(x, w, residual=r, out=r, out_dtype=torch.bfloat16) if res else L.proj(x, w, out_dtype=torch.float32)
    L.check_status()
    _check(out, ref, mag + (r.double().abs() if res else 0), res)
    assert (need > 0) == split  # on 148 SMs: split when the tiles fill at most half of them
