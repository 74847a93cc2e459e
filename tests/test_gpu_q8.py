"""q8_0 KV cache on the GPU against the CPU oracle.

* Append: the q8_0 planes (int8 values and f16 scales) bit-identical to the oracle's (ggml's
  quantize_row_q8_0, ties to even) of the normed and roped rows, f32 and bf16 inputs, and Q
  bit-identical to the f16 path's.
* Decode: within the north-star tolerance (|gpu - oracle| <= 2e-3 + 1e-2 |oracle|) of the oracle in
  ggml's semantics for a q8_0 cache (query quantised to q8_0, integer block dots, f32 V
  accumulation), which the kernel follows; the distance to the exact mode (f32 query against the
  dequantised cache) is bounded by the same tolerance plus the query's own rounding.
"""
import math

import numpy as np
import pytest
import torch

import localstack_b200 as L
from oracle import oracle as O
from tests.helpers import max_err, random_q, scattered_block_tables, within

pytestmark = pytest.mark.gpu
SCALE = 1.0 / math.sqrt(128)
DEV = "cuda"


def _planes(q8):
    return (q8.qs.cpu().numpy(), q8.d.cpu().view(torch.int16).numpy().view(np.uint16))


@pytest.mark.parametrize("dtype,T,Hq,Hkv", [("f32", 64, 32, 4), ("bf16", 2048, 16, 8), ("bf16", 4352, 32, 4),
                                            ("f32", 1, 16, 8), ("bf16", 3000, 2, 2)])
def test_append_q8_bit_exact(dtype, T, Hq, Hkv):
    rng = np.random.default_rng(T + Hq)
    D = 128
    q_in = rng.standard_normal((T, Hq, D)).astype(np.float32) * 3
    k_in = rng.standard_normal((T, Hkv, D)).astype(np.float32) * 3
    v_in = rng.standard_normal((T, Hkv, D)).astype(np.float32) * 3
    v_in[::7, :, :32] = 0  # whole zero blocks
    n_cells = ((T + 31) // 32 + 4) * 32
    pos = rng.integers(0, 20000, T).astype(np.int32)
    cells = rng.permutation(n_cells)[:T].astype(np.int64)
    g = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    if dtype == "bf16":
        bits = lambda a: torch.from_numpy(a).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        q_h, k_h, v_h = bits(q_in), bits(k_in), bits(v_in)
    else:
        q_h, k_h, v_h = q_in, k_in, v_in
    kqs, vqs = np.zeros((n_cells, Hkv, D), np.int8), np.zeros((n_cells, Hkv, D), np.int8)
    kd, vd = np.zeros((n_cells, Hkv, 4), np.uint16), np.zeros((n_cells, Hkv, 4), np.uint16)
    q_ref = O.kv_append_q8(q_h, k_h, v_h, pos, cells, kqs, kd, vqs, vd, g, g, 1e-6, 1e6, 1.0, in_dtype=dtype)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    kq, vq = L.alloc_cache_q8(n_cells, Hkv, DEV), L.alloc_cache_q8(n_cells, Hkv, DEV)
    q = L.kv_append_q8(kq, vq, t(q_in).to(tdt), t(k_in).to(tdt), t(v_in).to(tdt), t(pos), t(cells),
                       L.rope_table(int(pos.max()) + 1, DEV), t(g), t(g), 1e-6)
    L.check_status()
    gk, gkd = _planes(kq)
    gv, gvd = _planes(vq)
    assert np.array_equal(gk, kqs) and np.array_equal(gkd, kd)
    assert np.array_equal(gv, vqs) and np.array_equal(gvd, vd)
    assert np.array_equal(q.cpu().numpy().view(np.uint32), q_ref.view(np.uint32))


def _decode_case(rng, lens, Hq, Hkv):
    bt, n_pages = scattered_block_tables(rng, lens)
    n_cells = n_pages * 32
    k = rng.standard_normal((n_cells, Hkv, 128)).astype(np.float32)
    k = k / np.sqrt(np.mean(k * k, axis=-1, keepdims=True) + 1e-6)
    v = rng.standard_normal((n_cells, Hkv, 128)).astype(np.float32)
    kqs, kd = O.quantize_q8_0(k)
    vqs, vd = O.quantize_q8_0(v)
    q = random_q(rng, len(lens), Hq)
    kq, vq = L.Q8Cache(n_cells, Hkv, DEV), L.Q8Cache(n_cells, Hkv, DEV)
    for cache, qs, d in ((kq, kqs, kd), (vq, vqs, vd)):
        cache.qs.copy_(torch.from_numpy(qs))
        cache.d.copy_(torch.from_numpy(d.view(np.int16)).view(torch.float16))
    return (kq, vq, torch.from_numpy(q).to(DEV), torch.from_numpy(bt).to(DEV),
            torch.tensor(lens, dtype=torch.int32, device=DEV)), (q, kqs, kd, vqs, vd, bt)


@pytest.mark.parametrize("lens,Hq,Hkv", [([1, 33, 4000, 700], 32, 4), ([513], 16, 8), ([17000, 5, 31, 32, 64], 32, 4),
                                         ([2048] * 3, 16, 2)])
def test_decode_q8_vs_oracle(lens, Hq, Hkv):
    rng = np.random.default_rng(sum(lens) + Hq)
    args, (q, kqs, kd, vqs, vd, bt) = _decode_case(rng, lens, Hq, Hkv)
    out, lse = L.attn_decode_q8(*args, SCALE, want_lse=True)
    L.check_status()
    seq, pos = np.arange(len(lens)), np.asarray(lens) - 1
    gg, lse_gg = O.paged_attn_q8(q, seq, pos, kqs, kd, vqs, vd, bt, lens, SCALE, mode=O.MODE_GGML, want_lse=True)
    ex = O.paged_attn_q8(q, seq, pos, kqs, kd, vqs, vd, bt, lens, SCALE, mode=O.MODE_EXACT)
    o = out.cpu().numpy()
    assert within(o, gg), max_err(o, gg)
    assert np.allclose(lse.cpu().numpy(), lse_gg, atol=1e-3, rtol=1e-4)
    gap = np.abs(gg.astype(np.float64) - ex)
    assert np.all(np.abs(o.astype(np.float64) - ex) <= gap + 2e-3 + 1e-2 * np.abs(ex)), max_err(o, ex)


def test_decode_q8_f16_query_and_ctas():
    """An f16 query (converted to f32 before its quantisation) and explicit CTA counts."""
    rng = np.random.default_rng(77)
    lens = [3000, 1]
    args, (q, kqs, kd, vqs, vd, bt) = _decode_case(rng, lens, 32, 4)
    q16 = args[2].half()
    ref = O.paged_attn_q8(q16.float().cpu().numpy(), np.arange(2), np.asarray(lens) - 1, kqs, kd, vqs, vd, bt, lens,
                          SCALE, mode=O.MODE_GGML)
    for n_ctas in (0, 7, 160):
        out = L.attn_decode_q8(args[0], args[1], q16, args[3], args[4], SCALE, n_ctas=n_ctas)
        L.check_status()
        assert within(out.cpu().numpy(), ref), (n_ctas, max_err(out.cpu().numpy(), ref))


def test_append_then_decode_q8_chain():
    """Config-3 shape: a decode step's append into q8_0 planes, then the decode over them."""
    rng = np.random.default_rng(5)
    lens = [900, 1500, 40, 2100]
    Hq, Hkv = 32, 4
    args, (q_unused, kqs, kd, vqs, vd, bt) = _decode_case(rng, [n - 1 for n in lens], Hq, Hkv)
    kq, vq, _, bt_t, _ = args
    # the new token of each sequence goes into its next cell
    bt2, _ = bt, None
    cells = np.array([bt[b, (n - 1) // 32] * 32 + (n - 1) % 32 for b, n in enumerate(lens)], np.int64)
    if (cells >= kqs.shape[0]).any() or any((n - 1) // 32 >= bt.shape[1] for n in lens):
        pytest.skip("case layout")
    q_in = rng.standard_normal((len(lens), Hq, 128)).astype(np.float32)
    k_in = rng.standard_normal((len(lens), Hkv, 128)).astype(np.float32)
    v_in = rng.standard_normal((len(lens), Hkv, 128)).astype(np.float32)
    pos = np.asarray(lens, np.int32) - 1
    g = np.ones(128, np.float32)
    q_ref = O.kv_append_q8(q_in, k_in, v_in, pos, cells, kqs, kd, vqs, vd, g, g, 1e-6, 1e6, 1.0)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    q_out = L.kv_append_q8(kq, vq, t(q_in), t(k_in), t(v_in), t(pos), t(cells), L.rope_table(4096, DEV), t(g), t(g),
                           1e-6)
    out = L.attn_decode_q8(kq, vq, q_out, bt_t, torch.tensor(lens, dtype=torch.int32, device=DEV), SCALE)
    L.check_status()
    ref = O.paged_attn_q8(q_ref, np.arange(len(lens)), pos, kqs, kd, vqs, vd, bt2, lens, SCALE, mode=O.MODE_GGML)
    assert within(out.cpu().numpy(), ref), max_err(out.cpu().numpy(), ref)


def test_ggml_block_layout_round_trip():
    """The planes hold exactly ggml's block_q8_0 bytes: packing a cache into 34-byte blocks (f16 d,
    then 32 int8) matches a numpy packing of the same planes, and unpacking restores them."""
    rng = np.random.default_rng(9)
    n_cells, hkv = 96, 4
    x = rng.standard_normal((n_cells, hkv, 128)).astype(np.float32)
    qs, d = O.quantize_q8_0(x)
    c = L.Q8Cache(n_cells, hkv, DEV)
    c.qs.copy_(torch.from_numpy(qs))
    c.d.copy_(torch.from_numpy(d.view(np.int16)).view(torch.float16))
    blocks = c.to_ggml_blocks()
    L.check_status()
    ref = np.empty((n_cells, hkv, 4, 34), np.uint8)
    ref[..., :2] = d.reshape(n_cells, hkv, 4, 1).view(np.uint8).reshape(n_cells, hkv, 4, 2)
    ref[..., 2:] = qs.reshape(n_cells, hkv, 4, 32).view(np.uint8)
    assert np.array_equal(blocks.cpu().numpy(), ref.reshape(n_cells, hkv, 136))
    back = L.Q8Cache.from_ggml_blocks(blocks)
    L.check_status()
    assert torch.equal(back.qs, c.qs) and torch.equal(back.d.view(torch.int16), c.d.view(torch.int16))


def test_decode_q8_config4_131072_keys():
    """Config 4 over a q8_0 cache: one 131072-key context (4096 pages at random places)."""
    rng = np.random.default_rng(131)
    args, (q, kqs, kd, vqs, vd, bt) = _decode_case(rng, [131072], 32, 4)
    out = L.attn_decode_q8(*args, SCALE, max_seq_len=131072)
    L.check_status()
    gg = O.paged_attn_q8(q, [0], [131071], kqs, kd, vqs, vd, bt, [131072], SCALE, mode=O.MODE_GGML)
    assert within(out.cpu().numpy(), gg), max_err(out.cpu().numpy(), gg)


@pytest.mark.parametrize("q_lens,ctx_before,Hq,Hkv", [([2048], [0], 16, 8), ([512, 512, 200, 512], [0, 512, 1000, 33], 32, 4),
                                                      ([1, 77, 300], [0, 5, 0], 16, 2)])
def test_prefill_q8_vs_oracle(q_lens, ctx_before, Hq, Hkv):
    """Prefill over q8_0 planes (pages dequantised into an f16 scratch, then the tensor-core
    prefill) against the oracle's exact mode over the same q8_0 cache (f32 query, the dequantised
    K / V, double): the north-star tolerance."""
    rng = np.random.default_rng(sum(q_lens) + Hq)
    kv_lens = [c + t for c, t in zip(ctx_before, q_lens)]
    bt, n_pages = scattered_block_tables(rng, kv_lens)
    n_cells = n_pages * 32
    k = rng.standard_normal((n_cells, Hkv, 128)).astype(np.float32)
    k = k / np.sqrt(np.mean(k * k, axis=-1, keepdims=True) + 1e-6)
    v = rng.standard_normal((n_cells, Hkv, 128)).astype(np.float32)
    kqs, kd = O.quantize_q8_0(k)
    vqs, vd = O.quantize_q8_0(v)
    kq, vq = L.Q8Cache(n_cells, Hkv, DEV), L.Q8Cache(n_cells, Hkv, DEV)
    for cache, qs, d in ((kq, kqs, kd), (vq, vqs, vd)):
        cache.qs.copy_(torch.from_numpy(qs))
        cache.d.copy_(torch.from_numpy(d.view(np.int16)).view(torch.float16))
    total = int(sum(q_lens))
    q = random_q(rng, total, Hq).astype(np.float16)
    starts = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    t32 = lambda a: torch.tensor(a, dtype=torch.int32, device=DEV)
    out = L.attn_prefill_q8(kq, vq, torch.from_numpy(q).to(DEV), torch.from_numpy(starts).to(DEV), t32(ctx_before),
                            t32(kv_lens), torch.from_numpy(bt).to(DEV), max(q_lens), SCALE)
    L.check_status()
    q_seq = np.concatenate([np.full(n, b, np.int32) for b, n in enumerate(q_lens)])
    q_pos = np.concatenate([np.arange(c, c + n, dtype=np.int32) for c, n in zip(ctx_before, q_lens)])
    ex = O.paged_attn_q8(q.astype(np.float32), q_seq, q_pos, kqs, kd, vqs, vd, bt, kv_lens, SCALE, causal=True,
                         mode=O.MODE_EXACT)
    o = out.cpu().numpy()
    assert within(o, ex), max_err(o, ex)
