"""The BASELINE configurations at their full sizes, run on the GPU through the C ABI and on the CPU
oracle in both precision modes (harness code, not product code; used by tests/test_gpu_configs.py
and __graft_entry__.smoke()).

Each case returns (gpu, exact, ggml): the GPU output and the oracle's f32-accumulating ("exact")
and ggml-CPU-kernel ("ggml": Q rounded to f16 for the dot, f16 V accumulator) results on the same
inputs. Large inputs are drawn on the device (seeded) and copied to the host for the oracle.
"""
from __future__ import annotations

import math

import numpy as np
import torch

import localstack_b200 as L
from oracle import oracle as O

SCALE = 1.0 / math.sqrt(128)
D = 128


def bits(t):
    """f16 / bf16 tensor -> host uint16 bit pattern array."""
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def device_cache(n_cells, hkv, seed, dev="cuda"):
    g = torch.Generator(device=dev).manual_seed(seed)
    k = torch.randn((n_cells, hkv, D), generator=g, device=dev)
    k = (k * torch.rsqrt(k.square().mean(-1, keepdim=True) + 1e-6)).half()
    v = torch.randn((n_cells, hkv, D), generator=g, device=dev).half()
    return k, v


def both_modes(q, q_seq, q_pos, kc, vc, bt, kv_lens, causal=True):
    ex = O.paged_attn(q, q_seq, q_pos, kc, vc, bt, kv_lens, SCALE, causal=causal, mode=O.MODE_EXACT)
    gg = O.paged_attn(q, q_seq, q_pos, kc, vc, bt, kv_lens, SCALE, causal=causal, mode=O.MODE_GGML)
    return ex, gg


def config1(dev="cuda"):
    """Config 1: B=1, Hq 16 / Hkv 8, 512 cached tokens + the appended query token = 513 keys in 17
    pages of a seeded permutation of 20."""
    hq, hkv, keys = 16, 8, 513
    bt = np.random.default_rng(1).permutation(20)[:17].astype(np.int32)[None]
    kc, vc = device_cache(20 * 32, hkv, 1, dev)
    q = torch.randn((1, hq, D), generator=torch.Generator(device=dev).manual_seed(11), device=dev)
    out = L.attn_decode(kc, vc, q, torch.from_numpy(bt).to(dev), torch.tensor([keys], dtype=torch.int32, device=dev),
                        SCALE, max_seq_len=keys)
    L.check_status()
    ex, gg = both_modes(q.cpu().numpy(), [0], [keys - 1], bits(kc), bits(vc), bt, [keys])
    return out.cpu().numpy(), ex, gg


def config2_chain(dev="cuda", check_append=True):
    """Config 2 as one chain: bf16 N(0,1) Q/K/V -> kv_append (QK-RMSNorm unit gamma, NEOX RoPE 1e6,
    f16 K/V into 64 pages at seeded random ids) -> causal prefill of the 2048 tokens, Hq 16 / Hkv 8.
    With check_append, the pages and f16 Q are compared bit for bit with the oracle's append."""
    T, hq, hkv = 2048, 16, 8
    rng = np.random.default_rng(2)
    n_pages = 64 + 8
    perm = rng.permutation(n_pages)[:64].astype(np.int32)
    pos = np.arange(T, dtype=np.int32)
    cells = perm[pos // 32].astype(np.int64) * 32 + pos % 32
    g = torch.Generator(device=dev).manual_seed(2)
    q_in = torch.randn((T, hq, D), generator=g, device=dev).bfloat16()
    k_in = torch.randn((T, hkv, D), generator=g, device=dev).bfloat16()
    v_in = torch.randn((T, hkv, D), generator=g, device=dev).bfloat16()
    gamma = torch.ones(D, device=dev)
    kc, vc = L.alloc_cache(n_pages * 32, hkv, dev), L.alloc_cache(n_pages * 32, hkv, dev)
    q16 = L.kv_append(kc, vc, q_in, k_in, v_in, torch.from_numpy(pos).to(dev), torch.from_numpy(cells).to(dev),
                      L.rope_table(T, dev), gamma, gamma, 1e-6, q_out_dtype=torch.float16)
    bt = perm[None, :]
    i32 = lambda *v: torch.tensor(v, dtype=torch.int32, device=dev)
    out = L.attn_prefill(kc, vc, q16, i32(0, T), i32(0), i32(T), torch.from_numpy(bt).to(dev), T, SCALE)
    L.check_status()
    kc_ref = np.zeros((n_pages * 32, hkv, D), np.uint16)
    vc_ref = np.zeros_like(kc_ref)
    q_ref = O.kv_append(bits(q_in), bits(k_in), bits(v_in), pos, cells, kc_ref, vc_ref, np.ones(D, np.float32),
                        np.ones(D, np.float32), 1e-6, 1e6, 1.0, in_dtype="bf16")
    if check_append:
        assert np.array_equal(bits(kc), kc_ref), "K pages differ"
        assert np.array_equal(bits(vc), vc_ref), "V pages differ"
        assert np.array_equal(bits(q16), O.f32_to_f16_bits(q_ref)), "f16 Q differs"
    ex, gg = both_modes(q16.float().cpu().numpy(), np.zeros(T, np.int32), pos, kc_ref, vc_ref, bt, [T])
    return out.cpu().numpy(), ex, gg


def config3(dev="cuda"):
    """Config 3 with all 64 sequences: ctx U[1024, 32768] (+ the appended token), Hq 32 / Hkv 4, one
    global permutation of every page."""
    hq, hkv, B = 32, 4, 64
    rng = np.random.default_rng(3)
    lens = (rng.integers(1024, 32768 + 1, B) + 1).astype(np.int32)
    need = (lens + 31) // 32
    n_pages = int(need.sum())
    perm = rng.permutation(n_pages).astype(np.int32)
    bt = np.zeros((B, int(need.max())), np.int32)
    at = 0
    for b in range(B):
        bt[b, :need[b]] = perm[at:at + need[b]]
        at += need[b]
    kc, vc = device_cache(n_pages * 32, hkv, 3, dev)
    q = torch.randn((B, hq, D), generator=torch.Generator(device=dev).manual_seed(33), device=dev)
    out = L.attn_decode(kc, vc, q, torch.from_numpy(bt).to(dev), torch.from_numpy(lens).to(dev), SCALE,
                        max_seq_len=int(lens.max()))
    L.check_status()
    kh, vh = bits(kc), bits(vc)
    del kc, vc
    torch.cuda.empty_cache()
    ex, gg = both_modes(q.cpu().numpy(), np.arange(B), lens - 1, kh, vh, bt, lens)
    return out.cpu().numpy(), ex, gg


def config4(dev="cuda", want_lse=False):
    """Config 4: one 131072-token context (4096 pages at random places), Hq 32 / Hkv 4."""
    hq, hkv, ctx = 32, 4, 131072
    bt = np.random.default_rng(4).permutation(ctx // 32).astype(np.int32)[None]
    kc, vc = device_cache(ctx, hkv, 4, dev)
    q = torch.randn((1, hq, D), generator=torch.Generator(device=dev).manual_seed(44), device=dev)
    lens = np.array([ctx], np.int32)
    out, lse = L.attn_decode(kc, vc, q, torch.from_numpy(bt).to(dev), torch.from_numpy(lens).to(dev), SCALE,
                             max_seq_len=ctx, want_lse=True)
    L.check_status()
    kh, vh, qh = bits(kc), bits(vc), q.cpu().numpy()
    ex, lse_ex = O.paged_attn(qh, [0], [ctx - 1], kh, vh, bt, lens, SCALE, mode=O.MODE_EXACT, want_lse=True)
    gg = O.paged_attn(qh, [0], [ctx - 1], kh, vh, bt, lens, SCALE, mode=O.MODE_GGML)
    if want_lse:
        return out.cpu().numpy(), ex, gg, lse.cpu().numpy(), lse_ex
    return out.cpu().numpy(), ex, gg


def distances(gpu, ex, gg):
    """Max |gpu - exact|, max |gpu - ggml|, max |exact - ggml|, and whether the gate holds."""
    g = gpu.astype(np.float64)
    within = bool(np.all(np.abs(g - ex) <= 2e-3 + 1e-2 * np.abs(ex)))
    return {"vs_exact": float(np.max(np.abs(g - ex))), "vs_ggml": float(np.max(np.abs(g - gg))),
            "exact_vs_ggml": float(np.max(np.abs(ex.astype(np.float64) - gg))), "within_tol_exact": within}
