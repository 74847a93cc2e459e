"""Paged causal prefill (tcgen05 tensor cores) on the GPU vs the CPU oracle.

Tolerance (north star): |gpu - oracle_exact| <= 2e-3 + 1e-2 * |oracle_exact| on f32 outputs.
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
DEV = "cuda"


def _f16(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(DEV).view(torch.float16)


def _prefill_case(q_lens, ctx_before, Hq, Hkv, seed, q_dtype=torch.float16, ggml_check=False):
    """Sequence b has ctx_before[b] cached tokens and q_lens[b] new query tokens (already in the
    cache, as kv_append runs before attention). Returns (gpu, oracle_exact[, oracle_ggml])."""
    rng = np.random.default_rng(seed)
    kv_lens = [c + t for c, t in zip(ctx_before, q_lens)]
    bt, n_pages = scattered_block_tables(rng, kv_lens)
    kc, vc = random_cache(rng, n_pages, Hkv)
    total = int(sum(q_lens))
    q = random_q(rng, total, Hq)
    q16 = q.astype(np.float16)
    starts = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    q_t = torch.from_numpy(q16).to(DEV) if q_dtype == torch.float16 else torch.from_numpy(q).to(DEV)
    out = L.attn_prefill(_f16(kc), _f16(vc), q_t, torch.from_numpy(starts).to(DEV),
                         torch.tensor(ctx_before, dtype=torch.int32, device=DEV),
                         torch.tensor(kv_lens, dtype=torch.int32, device=DEV), torch.from_numpy(bt).to(DEV),
                         max(q_lens), SCALE)
    L.check_status()
    q_seq = np.concatenate([np.full(n, b, np.int32) for b, n in enumerate(q_lens)])
    q_pos = np.concatenate([np.arange(c, c + n, dtype=np.int32) for c, n in zip(ctx_before, q_lens)])
    qr = q16.astype(np.float32)
    ex = O.paged_attn(qr, q_seq, q_pos, kc, vc, bt, kv_lens, SCALE, causal=True, mode=O.MODE_EXACT)
    res = [out.cpu().numpy(), ex]
    if ggml_check:
        res.append(O.paged_attn(qr, q_seq, q_pos, kc, vc, bt, kv_lens, SCALE, causal=True, mode=O.MODE_GGML))
    return res


def test_config2_prefill_2048():
    # Config 2: one 2048-token prompt, Hq 16 / Hkv 8, pages scattered, causal.
    out, ex = _prefill_case([2048], [0], 16, 8, seed=2)
    assert within(out, ex), max_err(out, ex)


@pytest.mark.parametrize("Hq,Hkv", [(32, 4), (16, 8), (8, 8), (32, 8), (16, 2)])
def test_group_sizes_and_ragged_tiles(Hq, Hkv):
    out, ex = _prefill_case([1, 77, 300], [0, 0, 0], Hq, Hkv, seed=Hq + Hkv)
    assert within(out, ex), max_err(out, ex)


def test_chunked_prefill_with_prior_context_30b_shape():
    # Config-5 style: prefill chunks of 512 tokens behind existing context, batched.
    out, ex, gg = _prefill_case([512, 512, 200, 512], [0, 512, 1000, 33], 32, 4, seed=5, ggml_check=True)
    assert within(out, ex), max_err(out, ex)
    gap = np.abs(ex.astype(np.float64) - gg)
    assert np.all(np.abs(out.astype(np.float64) - gg) <= gap + 2e-3 + 1e-2 * np.abs(gg))


def test_long_ragged_batch():
    # Sequences of very different lengths (one with no new tokens) and prior context in one call.
    out, ex = _prefill_case([1100, 0, 40, 700, 1300], [0, 64, 2000, 100, 0], 32, 4, seed=21)
    assert within(out, ex), max_err(out, ex)


def test_long_prompt_many_key_tiles():
    """An 8192-token prompt (64 key tiles per query tile, 2048 CTAs), repeated: the pipeline's
    barriers must hold over long runs (a parity wait that skips a phase stalls until its bound and
    reports a timeout). Checked against a plain fp32 torch restatement of causal attention over
    the gathered pages (the oracle is too slow at this size)."""
    rng = np.random.default_rng(44)
    T, Hq, Hkv = 8192, 32, 4
    bt, n_pages = scattered_block_tables(rng, [T])
    kc, vc = random_cache(rng, n_pages, Hkv)
    q16 = random_q(rng, T, Hq).astype(np.float16)
    k_t, v_t, bt_t, q_t = _f16(kc), _f16(vc), torch.from_numpy(bt).to(DEV), torch.from_numpy(q16).to(DEV)
    i32 = lambda *v: torch.tensor(v, dtype=torch.int32, device=DEV)
    for _ in range(3):
        out = L.attn_prefill(k_t, v_t, q_t, i32(0, T), i32(0), i32(T), bt_t, T, SCALE)
        L.check_status()
    cells = (bt_t[0].long()[:, None] * 32 + torch.arange(32, device=DEV)).reshape(-1)[:T]
    K, V, Q = k_t[cells].float(), v_t[cells].float(), q_t.float()
    mask = torch.ones(T, T, dtype=torch.bool, device=DEV).tril()
    G = Hq // Hkv
    ref = torch.empty(T, Hq, 128, device=DEV)
    for h in range(Hq):
        s = (Q[:, h] @ K[:, h // G].T) * SCALE
        ref[:, h] = torch.softmax(s.masked_fill(~mask, float("-inf")), dim=-1) @ V[:, h // G]
    got, want = out.cpu().numpy(), ref.cpu().numpy()
    assert within(got, want), max_err(got, want)


def test_mostly_empty_items():
    """A 200-token and a 1-token prompt: 64 items on 64 CTAs, 24 of which get only items past the
    short prompt's end (no keys, no MMA). Those CTAs must skip the tensor-core drain rather than
    wait on it, and every live row must still match: three calls well inside half a second (a
    wait that ran to its bound would take a second)."""
    import time
    out, ex = _prefill_case([200, 1], [0, 0], 16, 8, seed=31)
    assert within(out, ex), max_err(out, ex)
    rng = np.random.default_rng(31)
    bt, n_pages = scattered_block_tables(rng, [200, 1])
    kc, vc = random_cache(rng, n_pages, 8)
    q = torch.from_numpy(random_q(rng, 201, 16).astype(np.float16)).to(DEV)
    i32 = lambda *v: torch.tensor(v, dtype=torch.int32, device=DEV)
    args = (_f16(kc), _f16(vc), q, i32(0, 200, 201), i32(0, 0), i32(200, 1), torch.from_numpy(bt).to(DEV), 200, SCALE)
    L.attn_prefill(*args)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(3):
        L.attn_prefill(*args)
    torch.cuda.synchronize()
    L.check_status()
    assert time.perf_counter() - t0 < 0.5


def test_f32_query_input():
    out, ex = _prefill_case([129, 64], [5, 0], 16, 8, seed=8, q_dtype=torch.float32)
    assert within(out, ex), max_err(out, ex)


def test_chunked_equals_single_prefill():
    # The reference splits long prompts into n_batch chunks (src/engine.cpp:254-264); attention of
    # the chunks over the growing cache must equal one pass over the whole prompt.
    rng = np.random.default_rng(13)
    T, Hq, Hkv = 1100, 16, 8
    bt, n_pages = scattered_block_tables(rng, [T])
    kc, vc = random_cache(rng, n_pages, Hkv)
    q16 = random_q(rng, T, Hq).astype(np.float16)
    k_t, v_t, bt_t = _f16(kc), _f16(vc), torch.from_numpy(bt).to(DEV)
    q_t = torch.from_numpy(q16).to(DEV)
    i32 = lambda *v: torch.tensor(v, dtype=torch.int32, device=DEV)
    whole = L.attn_prefill(k_t, v_t, q_t, i32(0, T), i32(0), i32(T), bt_t, T, SCALE)
    parts = []
    for a, b in [(0, 512), (512, 1024), (1024, T)]:
        parts.append(L.attn_prefill(k_t, v_t, q_t[a:b].contiguous(), i32(0, b - a), i32(a), i32(b), bt_t, b - a,
                                    SCALE))
    chunked = torch.cat(parts)
    L.check_status()
    assert within(chunked.cpu().numpy(), whole.cpu().numpy(), atol=1e-5, rtol=1e-5)


def test_bad_query_rows_report_device_index():
    """Sequence 1's rows run past total_tokens: it is skipped (its neighbour's rows are still
    right and nothing past the valid rows is written) and the status reports the sequence."""
    rng = np.random.default_rng(17)
    bt, n_pages = scattered_block_tables(rng, [70, 70])
    kc, vc = random_cache(rng, n_pages, 8)
    q16 = random_q(rng, 140, 16).astype(np.float16)
    i32 = lambda *v: torch.tensor(v, dtype=torch.int32, device=DEV)
    out = torch.full((140, 16, 128), 7.0, device=DEV)
    L.attn_prefill(_f16(kc), _f16(vc), torch.from_numpy(q16).to(DEV), i32(0, 70, 150), i32(0, 0), i32(70, 70),
                   torch.from_numpy(bt).to(DEV), 80, SCALE, out=out)
    with pytest.raises(L.LstkError) as e:
        L.check_status()
    assert e.value.code == -6 and "site 23" in str(e.value) and "detail 1" in str(e.value)
    got = out.cpu().numpy()
    assert np.all(got[70:] == 7.0)  # the skipped sequence's rows are untouched
    q_seq = np.zeros(70, np.int32)
    q_pos = np.arange(70, dtype=np.int32)
    ex = O.paged_attn(q16[:70].astype(np.float32), q_seq, q_pos, kc, vc, bt[:1], [70], SCALE, causal=True,
                      mode=O.MODE_EXACT)
    assert within(got[:70], ex), max_err(got[:70], ex)


def test_bad_page_reports_device_index():
    kc = L.alloc_cache(128, 8, DEV)
    vc = L.alloc_cache(128, 8, DEV)
    q = torch.randn(40, 16, 128, device=DEV).half()
    i32 = lambda *v: torch.tensor(v, dtype=torch.int32, device=DEV)
    bt = torch.tensor([[1, 9]], dtype=torch.int32, device=DEV)  # page 9 >= 4 pages
    L.attn_prefill(kc, vc, q, i32(0, 40), i32(0), i32(40), bt, 40, SCALE)
    with pytest.raises(L.LstkError) as e:
        L.check_status()
    assert e.value.code == -6
