"""Paged split-K decode attention on the GPU vs the CPU oracle.

Tolerance (north star): |gpu - oracle_exact| <= 2e-3 + 1e-2 * |oracle_exact| on the f32 outputs.
Against the ggml-precision oracle (f16 V accumulator) the GPU must be no further than the exact
result itself is, plus the same tolerance.
"""
import math

import numpy as np
import pytest
import torch

import localstack_b200 as L
from oracle import oracle as O
from tests.helpers import max_err, random_cache, random_q, scattered_block_tables, within

pytestmark = pytest.mark.gpu
SCALE = 1.0 / math.sqrt(128)


def _decode(seq_lens, Hq, Hkv, seed=0, n_ctas=0, q_dtype=torch.float32, want_lse=False):
    rng = np.random.default_rng(seed)
    bt, n_pages = scattered_block_tables(rng, seq_lens)
    kc, vc = random_cache(rng, n_pages, Hkv)
    q = random_q(rng, len(seq_lens), Hq)
    dev = "cuda"
    kc_t = torch.from_numpy(kc.view(np.int16)).to(dev).view(torch.float16)
    vc_t = torch.from_numpy(vc.view(np.int16)).to(dev).view(torch.float16)
    q_t = torch.from_numpy(q).to(dev).to(q_dtype)
    res = L.attn_decode(kc_t, vc_t, q_t, torch.from_numpy(bt).to(dev),
                        torch.from_numpy(np.asarray(seq_lens, np.int32)).to(dev), SCALE, n_ctas=n_ctas,
                        want_lse=want_lse)
    L.check_status()
    lens = np.asarray(seq_lens, np.int32)
    q_ref = q_t.float().cpu().numpy()
    B = len(seq_lens)
    ex, lse = O.paged_attn(q_ref, np.arange(B), lens - 1, kc, vc, bt, lens, SCALE, mode=O.MODE_EXACT, want_lse=True)
    gg = O.paged_attn(q_ref, np.arange(B), lens - 1, kc, vc, bt, lens, SCALE, mode=O.MODE_GGML)
    if want_lse:
        out, lse_gpu = res
        return out.cpu().numpy(), lse_gpu.cpu().numpy(), ex, gg, lse
    return res.cpu().numpy(), ex, gg


def _assert_parity(out, ex, gg):
    assert within(out, ex), f"max |gpu - exact| = {max_err(out, ex)}"
    # ggml-precision model: no further from it than the exact answer, plus tolerance
    gap = np.abs(ex.astype(np.float64) - gg)
    assert np.all(np.abs(out.astype(np.float64) - gg) <= gap + 2e-3 + 1e-2 * np.abs(gg)), max_err(out, gg)


def test_config1_decode_1p7b():
    # Config 1: B=1, Hq16/Hkv8, 512 context tokens + the appended query token = 513 keys.
    out, ex, gg = _decode([513], 16, 8, seed=0)
    _assert_parity(out, ex, gg)


@pytest.mark.parametrize("Hq,Hkv", [(32, 4), (16, 8), (8, 8), (16, 4), (4, 4), (16, 2), (8, 1)])
def test_group_sizes(Hq, Hkv):
    out, ex, gg = _decode([1, 31, 32, 33, 100, 257], Hq, Hkv, seed=Hq * 10 + Hkv)
    _assert_parity(out, ex, gg)


def test_ragged_batch_30b_shape_with_empty_sequence():
    lens = [0, 1, 5, 32, 64, 65, 1000, 4097, 0, 2500]
    out, ex, gg = _decode(lens, 32, 4, seed=7)
    _assert_parity(out, ex, gg)
    assert np.all(out[0] == 0) and np.all(out[8] == 0)  # a sequence with no keys reads as zeros


@pytest.mark.parametrize("n_ctas", [1, 3, 7, 148, 512])
def test_split_count_invariance(n_ctas):
    lens = [3000, 17, 700, 4096, 1]
    out, ex, gg = _decode(lens, 32, 4, seed=11, n_ctas=n_ctas)
    _assert_parity(out, ex, gg)


@pytest.mark.parametrize("Hq,Hkv,ctx,n_ctas,pad_pages", [
    (32, 4, 16384 + 5, 0, 0),    # one head group over the whole grid (148 pieces per row)
    (16, 8, 513, 0, 0),          # config 1: two head groups, grid 34 = 2 x 17
    (16, 8, 4000, 7, 0),         # a grid the head groups do not divide
    (48, 12, 3000, 30, 0),       # three head groups, grid 30 = 3 x 10
    (48, 12, 3000, 0, 0),        # three head groups, grid 148
    (32, 4, 300, 0, 40),         # table wider than the sequence: more CTAs than page-groups
    (16, 8, 200, 0, 20),         # the same with two head groups
])
def test_single_sequence_combine(Hq, Hkv, ctx, n_ctas, pad_pages):
    # One sequence split over many CTAs: the combine loads the row's pieces together with the
    # prefix when the head groups divide the grid and every CTA holds a page-group; the other
    # cases (uneven grid, empty CTA ranges from a table wider than the sequence) take the
    # general path. Every case against the oracle.
    rng = np.random.default_rng(ctx + Hkv)
    bt, n_pages = scattered_block_tables(rng, [ctx])
    if pad_pages:
        bt = np.concatenate([bt, np.full((1, pad_pages), bt[0, 0], np.int32)], axis=1)
    kc, vc = random_cache(rng, n_pages, Hkv)
    q = random_q(rng, 1, Hq)
    dev = "cuda"
    f = lambda a: torch.from_numpy(a.view(np.int16)).to(dev).view(torch.float16)
    out, lse = L.attn_decode(f(kc), f(vc), torch.from_numpy(q).to(dev), torch.from_numpy(bt).to(dev),
                             torch.tensor([ctx], dtype=torch.int32, device=dev), SCALE, n_ctas=n_ctas, want_lse=True)
    L.check_status()
    ex, lse_ex = O.paged_attn(q, [0], [ctx - 1], kc, vc, bt, [ctx], SCALE, mode=O.MODE_EXACT, want_lse=True)
    assert within(out.cpu().numpy(), ex), max_err(out.cpu().numpy(), ex)
    assert np.allclose(lse.cpu().numpy(), lse_ex, atol=1e-3, rtol=1e-4)


@pytest.mark.parametrize("Hq,Hkv,n_ctas", [(32, 4, 0), (16, 8, 0), (8, 1, 0), (32, 4, 300), (48, 12, 0)])
def test_many_sequences_combine_by_rows(Hq, Hkv, n_ctas):
    # A batch with more sequences than a few per CTA grid: the combine merges one row per warp
    # (pieces of rows split across CTA boundaries, rows a single CTA finished, empty sequences).
    rng = np.random.default_rng(Hq + Hkv + n_ctas)
    lens = rng.integers(1, 3000, 40).tolist()
    lens[3] = 0
    lens[17] = 0
    lens[20] = 20000
    out, lse_gpu, ex, gg, lse = _decode(lens, Hq, Hkv, seed=Hq + Hkv + n_ctas, n_ctas=n_ctas, want_lse=True)
    _assert_parity(out, ex, gg)
    assert np.all(out[3] == 0) and np.all(out[17] == 0)
    live = np.asarray(lens) > 0
    assert np.all(np.isneginf(lse_gpu[~live]))
    assert np.allclose(lse_gpu[live], lse[live], atol=1e-3, rtol=1e-4)


def test_page_permutation_is_bit_invariant():
    # Same K/V content placed in differently permuted pages -> identical output bits.
    rng = np.random.default_rng(5)
    lens = [700, 1500, 33]
    Hq, Hkv = 32, 4
    bt, n_pages = scattered_block_tables(rng, lens)
    kc, vc = random_cache(rng, n_pages, Hkv)
    q = random_q(rng, len(lens), Hq)
    perm = rng.permutation(n_pages)
    kc2 = np.empty_like(kc)
    vc2 = np.empty_like(vc)
    for p in range(n_pages):
        kc2[perm[p] * 32:(perm[p] + 1) * 32] = kc[p * 32:(p + 1) * 32]
        vc2[perm[p] * 32:(perm[p] + 1) * 32] = vc[p * 32:(p + 1) * 32]
    bt2 = perm[bt].astype(np.int32)
    dev = "cuda"
    f = lambda a: torch.from_numpy(a.view(np.int16)).to(dev).view(torch.float16)
    lens_t = torch.tensor(lens, dtype=torch.int32, device=dev)
    q_t = torch.from_numpy(q).to(dev)
    o1 = L.attn_decode(f(kc), f(vc), q_t, torch.from_numpy(bt).to(dev), lens_t, SCALE).cpu().numpy()
    o2 = L.attn_decode(f(kc2), f(vc2), q_t, torch.from_numpy(bt2).to(dev), lens_t, SCALE).cpu().numpy()
    assert np.array_equal(o1.view(np.uint32), o2.view(np.uint32))


def test_f16_query_and_lse():
    out, lse_gpu, ex, gg, lse = _decode([300, 1, 2048], 32, 4, seed=9, q_dtype=torch.float16, want_lse=True)
    _assert_parity(out, ex, gg)
    assert np.allclose(lse_gpu, lse, atol=1e-3, rtol=1e-4)


def test_config3_shape_sampled():
    # Config-3 shape (30B-A3B GQA 32/4) with 16 sequences of ctx U[1024, 32768]; all checked.
    rng = np.random.default_rng(3)
    lens = rng.integers(1024, 32769, 16).tolist()
    out, ex, gg = _decode(lens, 32, 4, seed=3)
    _assert_parity(out, ex, gg)


def test_long_context_split_and_merge():
    # Config-4 style: one sequence's pages split into R contiguous chunks (as R GPUs would hold
    # them); each chunk decoded with lse, then merged by log-sum-exp == whole-context decode.
    rng = np.random.default_rng(21)
    ctx, Hq, Hkv, R = 16384 + 7, 32, 4, 4
    bt, n_pages = scattered_block_tables(rng, [ctx])
    kc, vc = random_cache(rng, n_pages, Hkv)
    q = random_q(rng, 1, Hq)
    dev = "cuda"
    f = lambda a: torch.from_numpy(a.view(np.int16)).to(dev).view(torch.float16)
    kc_t, vc_t, q_t = f(kc), f(vc), torch.from_numpy(q).to(dev)
    n_blk = (ctx + 31) // 32
    cut = [round(r * n_blk / R) for r in range(R + 1)]
    o_parts, l_parts = [], []
    for r in range(R):
        sub_bt = torch.from_numpy(np.ascontiguousarray(bt[:, cut[r]:cut[r + 1]])).to(dev)
        sub_len = min(ctx, cut[r + 1] * 32) - cut[r] * 32
        o, lse = L.attn_decode(kc_t, vc_t, q_t, sub_bt, torch.tensor([sub_len], dtype=torch.int32, device=dev),
                               SCALE, want_lse=True)
        o_parts.append(o.reshape(Hq, 128))
        l_parts.append(lse.reshape(Hq))
    merged, _ = L.attn_merge(torch.stack(o_parts), torch.stack(l_parts))
    whole = L.attn_decode(kc_t, vc_t, q_t, torch.from_numpy(bt).to(dev),
                          torch.tensor([ctx], dtype=torch.int32, device=dev), SCALE)
    L.check_status()
    ex = O.paged_attn(q, [0], [ctx - 1], kc, vc, bt, [ctx], SCALE, mode=O.MODE_EXACT)
    assert within(merged.cpu().numpy(), ex.reshape(Hq, 128))
    assert within(whole.cpu().numpy(), ex)


def test_bad_page_reports_device_index():
    dev = "cuda"
    kc = L.alloc_cache(64, 4, dev)
    vc = L.alloc_cache(64, 4, dev)
    q = torch.randn(1, 32, 128, device=dev)
    bt = torch.tensor([[0, 5]], dtype=torch.int32, device=dev)  # page 5 >= 2 pages
    L.attn_decode(kc, vc, q, bt, torch.tensor([40], dtype=torch.int32, device=dev), SCALE)
    with pytest.raises(L.LstkError) as e:
        L.check_status()
    assert e.value.code == -6


def test_append_and_decode_replay_in_cuda_graph():
    """A decode step (append + split-K decode + combine) captured once in a CUDA graph and
    replayed gives the eager results bit for bit (no host work inside the entry points)."""
    rng = np.random.default_rng(17)
    lens = [700, 33, 1500]
    Hq, Hkv = 32, 4
    bt, n_pages = scattered_block_tables(rng, [n + 1 for n in lens])
    kc, vc = random_cache(rng, n_pages, Hkv)
    dev = "cuda"
    f16 = lambda a: torch.from_numpy(a.view(np.int16)).to(dev).view(torch.float16)
    kc_e, vc_e = f16(kc), f16(vc)
    kc_g, vc_g = kc_e.clone(), vc_e.clone()
    B = len(lens)
    q_in = torch.from_numpy(random_q(rng, B, Hq, normed=False)).to(dev)
    k_in = torch.from_numpy(random_q(rng, B, Hkv, normed=False)).to(dev)
    v_in = torch.from_numpy(random_q(rng, B, Hkv, normed=False)).to(dev)
    pos = torch.tensor(lens, dtype=torch.int32, device=dev)
    cells = torch.tensor([int(bt[b, lens[b] // 32]) * 32 + lens[b] % 32 for b in range(B)], dtype=torch.int64,
                         device=dev)
    rope = L.rope_table(2048, dev)
    gamma = torch.linspace(0.5, 1.5, 128, device=dev)
    bt_t = torch.from_numpy(bt).to(dev)
    kl = torch.tensor([n + 1 for n in lens], dtype=torch.int32, device=dev)
    ws = L.DecodeWorkspace(B, Hq, Hkv, dev)

    def step(kc_t, vc_t, q_out, out):
        L.kv_append(kc_t, vc_t, q_in, k_in, v_in, pos, cells, rope, gamma, gamma, 1e-6, q_out=q_out)
        L.attn_decode(kc_t, vc_t, q_out, bt_t, kl, SCALE, max_seq_len=max(lens) + 1, out=out, workspace=ws)

    q_e, o_e = torch.empty(B, Hq, 128, device=dev), torch.empty(B, Hq, 128, device=dev)
    step(kc_e, vc_e, q_e, o_e)
    q_g, o_g = torch.zeros_like(q_e), torch.zeros_like(o_e)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step(kc_g, vc_g, q_g, o_g)  # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(side)
    o_g.zero_()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step(kc_g, vc_g, q_g, o_g)
    g.replay()
    torch.cuda.synchronize()
    L.check_status()
    assert torch.equal(o_g, o_e) and torch.equal(q_g, q_e)
    assert torch.equal(kc_g.view(torch.int16), kc_e.view(torch.int16))
    del g


def test_decode_partial_key_ranges_merge_to_whole():
    """lstk_cuda_attn_decode_partial over page-aligned key ranges, each against the oracle on
    the same keys, and the LSE merge of the ranges against the whole decode (ragged batch: the
    ranges cut some sequences and miss others entirely)."""
    rng = np.random.default_rng(31)
    lens = [5000, 33, 700, 4096]
    Hq, Hkv = 32, 4
    bt, n_pages = scattered_block_tables(rng, lens)
    kc, vc = random_cache(rng, n_pages, Hkv)
    q = random_q(rng, len(lens), Hq)
    dev = "cuda"
    f16 = lambda a: torch.from_numpy(a.view(np.int16)).to(dev).view(torch.float16)
    kc_t, vc_t, q_t, bt_t = f16(kc), f16(vc), torch.from_numpy(q).to(dev), torch.from_numpy(bt).to(dev)
    lens_t = torch.tensor(lens, dtype=torch.int32, device=dev)
    ranges = [(0, 64), (64, 1024), (1024, 4096), (4096, 1 << 30)]
    parts, lses = [], []
    B = len(lens)
    for a, b in ranges:
        o, lse = L.attn_decode(kc_t, vc_t, q_t, bt_t, lens_t, SCALE, want_lse=True, kv_range=(a, b))
        parts.append(o.reshape(B * Hq, 128))
        lses.append(lse.reshape(B * Hq))
        # oracle on the same keys: the sub-range of every sequence's pages
        sub_lens = np.array([max(0, min(n, b) - a) for n in lens], np.int32)
        sub_bt = np.ascontiguousarray(bt[:, a // 32:]) if a // 32 < bt.shape[1] else np.zeros((B, 1), np.int32)
        if sub_bt.shape[1] == 0:
            sub_bt = np.zeros((B, 1), np.int32)
        ex = O.paged_attn(q, np.arange(B), np.maximum(sub_lens - 1, 0), kc, vc, sub_bt, sub_lens, SCALE,
                          mode=O.MODE_EXACT)
        got = o.cpu().numpy()
        for i in range(B):
            if sub_lens[i] == 0:
                assert np.all(got[i] == 0) and np.all(np.isneginf(lse.cpu().numpy()[i]))
            else:
                assert within(got[i], ex[i]), (a, b, i, max_err(got[i], ex[i]))
    merged, _ = L.attn_merge(torch.stack(parts), torch.stack(lses))
    L.check_status()
    lens_np = np.asarray(lens, np.int32)
    ex_whole = O.paged_attn(q, np.arange(B), lens_np - 1, kc, vc, bt, lens_np, SCALE, mode=O.MODE_EXACT)
    # the merged ranges meet the same tolerance against the exact whole-context result
    assert within(merged.cpu().numpy(), ex_whole.reshape(B * Hq, 128)), max_err(merged.cpu().numpy(),
                                                                                 ex_whole.reshape(B * Hq, 128))
