"""The BASELINE configurations at their full sizes, end to end, against the CPU oracle.

* Config 2 as one chain: bf16 N(0,1) Q/K/V -> lstk_cuda_kv_append (QK-RMSNorm, NEOX RoPE 1e6, f16
  pages at seeded random page ids; pages and Q bit-exact against the oracle's append) ->
  lstk_cuda_attn_prefill over the pages the append wrote (causal, 2048 tokens, Hq 16 / Hkv 8).
* Config 3 with all 64 sequences (ctx U[1024, 32768], Hq 32 / Hkv 4, one global page permutation).
* Config 4: one 131072-token context (4096 pages at random places).

Gate (the tolerance of the north star, on f32 outputs): |gpu - exact| <= 2e-3 + 1e-2 |exact|,
where exact is the oracle with f32 accumulation - the precision the reference's call site asks
for (GGML_PREC_F32, src/qwen3.cpp:165-167). Against the oracle's model of ggml's CPU kernel (Q
rounded to f16 for the dot, an f16 V accumulator) the GPU must be no further than the exact answer
itself is, plus the same tolerance: that model already sits up to ~2.6e-3 from the exact result
at these sizes, so a plain 2e-3 band around it cannot be met by any f32-accumulating kernel.
Large inputs are drawn on the device (seeded) and copied to the host for the oracle.
"""
import math

import numpy as np
import pytest
import torch

import localstack_b200 as L
from oracle import oracle as O
from tests.helpers import max_err, within

pytestmark = pytest.mark.gpu
SCALE = 1.0 / math.sqrt(128)
DEV = "cuda"
D = 128


def _bits(t):
    """f16 / bf16 tensor -> host uint16 bit pattern array."""
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def _check_both_modes(out, ex, gg):
    assert within(out, ex), f"max |gpu - exact| = {max_err(out, ex)}"
    gap = np.abs(ex.astype(np.float64) - gg)
    assert np.all(np.abs(out.astype(np.float64) - gg) <= gap + 2e-3 + 1e-2 * np.abs(gg)), max_err(out, gg)


def _device_cache(n_cells, hkv, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    k = torch.randn((n_cells, hkv, D), generator=g, device=DEV)
    k = (k * torch.rsqrt(k.square().mean(-1, keepdim=True) + 1e-6)).half()
    v = torch.randn((n_cells, hkv, D), generator=g, device=DEV).half()
    return k, v


def test_config2_chain_bf16_append_then_prefill():
    T, hq, hkv = 2048, 16, 8
    rng = np.random.default_rng(2)
    n_pages = 64 + 8
    perm = rng.permutation(n_pages)[:64].astype(np.int32)  # 64 pages at seeded random ids
    pos = np.arange(T, dtype=np.int32)
    cells = (perm[pos // 32].astype(np.int64) * 32 + pos % 32)
    g = torch.Generator(device=DEV).manual_seed(2)
    q_in = torch.randn((T, hq, D), generator=g, device=DEV).bfloat16()
    k_in = torch.randn((T, hkv, D), generator=g, device=DEV).bfloat16()
    v_in = torch.randn((T, hkv, D), generator=g, device=DEV).bfloat16()
    gamma = torch.ones(D, device=DEV)
    kc, vc = L.alloc_cache(n_pages * 32, hkv, DEV), L.alloc_cache(n_pages * 32, hkv, DEV)
    rope = L.rope_table(T, DEV)
    q16 = L.kv_append(kc, vc, q_in, k_in, v_in, torch.from_numpy(pos).to(DEV), torch.from_numpy(cells).to(DEV), rope,
                      gamma, gamma, 1e-6, q_out_dtype=torch.float16)
    bt = perm[None, :]
    i32 = lambda *v: torch.tensor(v, dtype=torch.int32, device=DEV)
    out = L.attn_prefill(kc, vc, q16, i32(0, T), i32(0), i32(T), torch.from_numpy(bt).to(DEV), T, SCALE)
    L.check_status()
    # the append, bit for bit
    kc_ref = np.zeros((n_pages * 32, hkv, D), np.uint16)
    vc_ref = np.zeros_like(kc_ref)
    q_ref = O.kv_append(_bits(q_in), _bits(k_in), _bits(v_in), pos, cells, kc_ref, vc_ref, np.ones(D, np.float32),
                        np.ones(D, np.float32), 1e-6, 1e6, 1.0, in_dtype="bf16")
    assert np.array_equal(_bits(kc), kc_ref), "K pages differ"
    assert np.array_equal(_bits(vc), vc_ref), "V pages differ"
    assert np.array_equal(_bits(q16), O.f32_to_f16_bits(q_ref)), "f16 Q differs"
    # the prefill over those pages
    qr = q16.float().cpu().numpy()
    q_seq = np.zeros(T, np.int32)
    ex = O.paged_attn(qr, q_seq, pos, kc_ref, vc_ref, bt, [T], SCALE, causal=True, mode=O.MODE_EXACT)
    gg = O.paged_attn(qr, q_seq, pos, kc_ref, vc_ref, bt, [T], SCALE, causal=True, mode=O.MODE_GGML)
    _check_both_modes(out.cpu().numpy(), ex, gg)


def test_config3_full_batch_64_sequences():
    hq, hkv, B = 32, 4, 64
    rng = np.random.default_rng(3)
    ctx = rng.integers(1024, 32768 + 1, B)
    lens = (ctx + 1).astype(np.int32)  # the step's own token is appended before attention
    need = (lens + 31) // 32
    n_pages = int(need.sum())
    perm = rng.permutation(n_pages).astype(np.int32)  # one global permutation of every page
    bt = np.zeros((B, int(need.max())), np.int32)
    at = 0
    for b in range(B):
        bt[b, :need[b]] = perm[at:at + need[b]]
        at += need[b]
    kc, vc = _device_cache(n_pages * 32, hkv, 3)
    q = torch.randn((B, hq, D), generator=torch.Generator(device=DEV).manual_seed(33), device=DEV)
    out = L.attn_decode(kc, vc, q, torch.from_numpy(bt).to(DEV), torch.from_numpy(lens).to(DEV), SCALE,
                        max_seq_len=int(lens.max()))
    L.check_status()
    kh, vh, qh = _bits(kc), _bits(vc), q.cpu().numpy()
    del kc, vc
    torch.cuda.empty_cache()
    ex = O.paged_attn(qh, np.arange(B), lens - 1, kh, vh, bt, lens, SCALE, mode=O.MODE_EXACT)
    gg = O.paged_attn(qh, np.arange(B), lens - 1, kh, vh, bt, lens, SCALE, mode=O.MODE_GGML)
    _check_both_modes(out.cpu().numpy(), ex, gg)


def test_config4_131072_keys():
    hq, hkv, ctx = 32, 4, 131072
    n_pages = ctx // 32
    bt = np.random.default_rng(4).permutation(n_pages).astype(np.int32)[None]
    kc, vc = _device_cache(ctx, hkv, 4)
    q = torch.randn((1, hq, D), generator=torch.Generator(device=DEV).manual_seed(44), device=DEV)
    lens = np.array([ctx], np.int32)
    out, lse = L.attn_decode(kc, vc, q, torch.from_numpy(bt).to(DEV), torch.from_numpy(lens).to(DEV), SCALE,
                             max_seq_len=ctx, want_lse=True)
    L.check_status()
    kh, vh, qh = _bits(kc), _bits(vc), q.cpu().numpy()
    ex, lse_ex = O.paged_attn(qh, [0], [ctx - 1], kh, vh, bt, lens, SCALE, mode=O.MODE_EXACT, want_lse=True)
    gg = O.paged_attn(qh, [0], [ctx - 1], kh, vh, bt, lens, SCALE, mode=O.MODE_GGML)
    _check_both_modes(out.cpu().numpy(), ex, gg)
    assert np.allclose(lse.cpu().numpy(), lse_ex, atol=1e-3, rtol=1e-4)
