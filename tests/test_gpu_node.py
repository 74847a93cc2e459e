"""The whole attention node, step by step, against the reference's own formulation.

The reference runs attn_block (src/qwen3.cpp:128-171) as: QK-RMSNorm, NEOX RoPE, set_rows of K/V
into the cells KvCache::alloc returned, then flash_attn_ext of Q over the first n_kv cells of the
cache (Engine::n_kv_for, src/engine.cpp:193-196) with the f16 mask KvCache::fill_mask builds
(src/kv_cache.cpp:140-150). Here the same steps run through the backend (kv_append, then
attn_prefill for a prompt chunk and attn_decode for the next token, over block tables) and through
the oracle's dense masked restatement, with the bookkeeping of the reference's KvCache rules.
Pages must be bit-identical; outputs within the parity tolerance of the exact mode.
"""
import math

import numpy as np
import pytest
import torch

import localstack_b200 as L
from localstack_b200.kv_cache import KvCache, n_kv_for
from oracle import oracle as O
from tests.helpers import max_err, within

pytestmark = pytest.mark.gpu
D = 128


@pytest.mark.parametrize("Hq,Hkv,prompt", [(16, 8, 512), (32, 4, 300)])
def test_prompt_then_decode_matches_dense_masked_reference(Hq, Hkv, prompt):
    rng = np.random.default_rng(Hq + prompt)
    size = 2048
    kv = KvCache(size)
    kv.set_free_blocks(rng.permutation(size // 32).astype(np.uint32))  # scattered pages
    kv.alloc(5, 70)  # another sequence holds cells too: the mask must hide them
    scale = 1.0 / math.sqrt(D)
    qg = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    kg = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    dev = "cuda"
    kc = L.alloc_cache(size, Hkv, dev)
    vc = L.alloc_cache(size, Hkv, dev)
    kc_ref = np.zeros((size, Hkv, D), np.uint16)
    vc_ref = np.zeros((size, Hkv, D), np.uint16)
    rope = L.rope_table(4096, dev)
    qg_t, kg_t = torch.from_numpy(qg).to(dev), torch.from_numpy(kg).to(dev)
    seq = 0
    for step, T in enumerate([prompt, 1]):  # prompt chunk, then one decode token
        cells, pos = kv.alloc(seq, T)
        q_in = rng.standard_normal((T, Hq, D), dtype=np.float32) * 2
        k_in = rng.standard_normal((T, Hkv, D), dtype=np.float32) * 2
        v_in = rng.standard_normal((T, Hkv, D), dtype=np.float32)
        # reference path (oracle): ops in attn_block order, dense masked attention over n_kv cells
        q_ref = O.kv_append(q_in, k_in, v_in, pos, cells, kc_ref, vc_ref, qg, kg, 1e-6, 1e6, 1.0)
        n_kv = n_kv_for(size, kv.used_hwm)
        mask = kv.fill_mask(seq, pos, n_kv)
        ex = O.flash_attn_ext(q_ref, kc_ref, vc_ref, n_kv, mask, scale, mode=O.MODE_EXACT)
        # backend path
        t = lambda a, dt=torch.float32: torch.from_numpy(np.ascontiguousarray(a)).to(dev).to(dt)
        q16 = L.kv_append(kc, vc, t(q_in), t(k_in), t(v_in), t(pos, torch.int32), t(cells, torch.int64), rope, qg_t,
                          kg_t, 1e-6, q_out_dtype=torch.float16 if T > 1 else torch.float32)
        bt, lens = kv.block_tables(np.array([seq]))
        bt_t, lens_t = t(bt, torch.int32), t(lens, torch.int32)
        if T > 1:
            out = L.attn_prefill(kc, vc, q16, t([0, T], torch.int32), t([int(pos[0])], torch.int32), lens_t, bt_t, T,
                                 scale)
            # the prefill consumes f16 queries: the exact reference with the same rounding
            ex = O.flash_attn_ext(q16.float().cpu().numpy(), kc_ref, vc_ref, n_kv, mask, scale, mode=O.MODE_EXACT)
        else:
            out = L.attn_decode(kc, vc, q16, bt_t, lens_t, scale)
        L.check_status()
        got = out.cpu().numpy().reshape(T, Hq, D)
        assert np.array_equal(kc.cpu().view(torch.int16).numpy().view(np.uint16), kc_ref), step
        assert np.array_equal(vc.cpu().view(torch.int16).numpy().view(np.uint16), vc_ref), step
        assert within(got, ex), (step, max_err(got, ex))
