"""Bounded waits of the decode and prefill kernels, made to run out on the GPU.

The kernels' loaders are gated on a start flag that nothing sets (lstk_cuda_set_wait_policy), with
a 2 ms pipeline limit: the loader's wait runs out, the kernel records LSTK_ERR_TIMEOUT, the other
warps see the abort in their own bounded waits, in-flight work drains, tensor memory is freed and
the kernel returns. The host reads the status; the same context then runs a normal call that must
still meet the parity tolerance against the oracle. No fault, trap or endless loop is involved:
every wait here ends by its limit.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

import localstack_b200 as L
from localstack_b200 import _lib
from oracle import oracle as O
from tests.helpers import random_cache, random_q, scattered_block_tables, within

pytestmark = pytest.mark.gpu
SCALE = 1.0 / math.sqrt(128)


def _policy(wait_ns, flag):
    _lib.check(L.lib().lstk_cuda_set_wait_policy(int(wait_ns), ctypes.c_void_p(flag.data_ptr()) if flag is not None
                                                 else None))


@pytest.fixture
def reset_policy():
    yield
    _policy(0, None)


def _decode_case(seed=3):
    rng = np.random.default_rng(seed)
    lens = [4000, 33, 1, 700]
    bt, n_pages = scattered_block_tables(rng, lens)
    kc, vc = random_cache(rng, n_pages, 4)
    q = random_q(rng, len(lens), 32)
    f16 = lambda a: torch.from_numpy(a.view(np.int16)).cuda().view(torch.float16)
    lens_np = np.asarray(lens, np.int32)
    ex = O.paged_attn(q, np.arange(len(lens)), lens_np - 1, kc, vc, bt, lens_np, SCALE, mode=O.MODE_EXACT)
    return (f16(kc), f16(vc), torch.from_numpy(q).cuda(), torch.from_numpy(bt).cuda(),
            torch.from_numpy(lens_np).cuda()), ex


def _prefill_case(seed=4):
    rng = np.random.default_rng(seed)
    T, Hq, Hkv = 700, 16, 8
    bt, n_pages = scattered_block_tables(rng, [T])
    kc, vc = random_cache(rng, n_pages, Hkv)
    q16 = random_q(rng, T, Hq).astype(np.float16)
    f16 = lambda a: torch.from_numpy(a.view(np.int16)).cuda().view(torch.float16)
    i32 = lambda *v: torch.tensor(v, dtype=torch.int32, device="cuda")
    ex = O.paged_attn(q16.astype(np.float32), np.zeros(T, np.int32), np.arange(T, dtype=np.int32), kc, vc, bt, [T],
                      SCALE, causal=True, mode=O.MODE_EXACT)
    args = (f16(kc), f16(vc), torch.from_numpy(q16).cuda(), i32(0, T), i32(0), i32(T), torch.from_numpy(bt).cuda(), T)
    return args, ex


def test_decode_wait_runs_out_then_context_still_works(reset_policy):
    args, ex = _decode_case()
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")  # nothing ever sets it
    _policy(2_000_000, flag)
    L.attn_decode(*args, SCALE)
    with pytest.raises(L.LstkError) as e:
        L.check_status()
    assert e.value.code == _lib.LSTK_ERR_TIMEOUT
    assert "timed out" in str(e.value)
    _policy(0, None)
    out = L.attn_decode(*args, SCALE)
    L.check_status()
    assert within(out.cpu().numpy(), ex)


def test_prefill_wait_runs_out_then_context_still_works(reset_policy):
    args, ex = _prefill_case()
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    _policy(2_000_000, flag)
    L.attn_prefill(*args, SCALE)
    with pytest.raises(L.LstkError) as e:
        L.check_status()
    assert e.value.code == _lib.LSTK_ERR_TIMEOUT
    _policy(0, None)
    out = L.attn_prefill(*args, SCALE)
    L.check_status()
    assert within(out.cpu().numpy(), ex)


def test_set_flag_and_explicit_limit_give_normal_results(reset_policy):
    """A start flag that is already set, and a non-default pipeline limit, change nothing."""
    dargs, dex = _decode_case(5)
    pargs, pex = _prefill_case(6)
    flag = torch.ones(1, dtype=torch.int32, device="cuda")
    _policy(500_000_000, flag)
    out = L.attn_decode(*dargs, SCALE)
    pre = L.attn_prefill(*pargs, SCALE)
    L.check_status()
    assert within(out.cpu().numpy(), dex)
    assert within(pre.cpu().numpy(), pex)
