"""lstk_cuda_attn_decode_static: decode for callers that cannot allocate device memory when they
decode (their memory is pooled up front, allocation is not allowed where they run, or they are a
C/FFI host that owns only the tensors it passes). It uses scratch built into the library instead
of a workspace argument. This file is collected last on purpose: it calls the C ABI directly and
must agree with the workspace entry point, call after call, whether it runs alone or after the
rest of the suite."""
import ctypes
import math

import numpy as np
import pytest
import torch

import localstack_b200 as L
from localstack_b200 import _lib
from oracle import oracle as O
from tests.helpers import max_err, random_cache, random_q, scattered_block_tables, within

pytestmark = pytest.mark.gpu
SCALE = 1.0 / math.sqrt(128)


def _static_fn():
    fn = L.lib().lstk_cuda_attn_decode_static
    P, I32, F = ctypes.c_void_p, ctypes.c_int32, ctypes.c_float
    fn.argtypes = [ctypes.POINTER(_lib.KvLayout), P, P, P, I32, I32, I32, P, I32, P, I32, F, P, P, I32, P]
    fn.restype = ctypes.c_int
    return fn


def _case(seed, lens, Hq, Hkv):
    rng = np.random.default_rng(seed)
    bt, n_pages = scattered_block_tables(rng, lens)
    kc, vc = random_cache(rng, n_pages, Hkv)
    q = random_q(rng, len(lens), Hq)
    dev = "cuda"
    f16 = lambda a: torch.from_numpy(a.view(np.int16)).to(dev).view(torch.float16)
    return (f16(kc), f16(vc), torch.from_numpy(q).to(dev), torch.from_numpy(bt).to(dev),
            torch.tensor(lens, dtype=torch.int32, device=dev))


def _call_static(fn, kc, vc, q, bt, lens, out, lse, n_ctas=0):
    lay = L.layout_of(kc)
    p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return fn(ctypes.byref(lay), p(kc), p(vc), p(q), _lib.DTYPE_F32, q.shape[0], q.shape[1], p(bt), bt.shape[1],
              p(lens), 0, SCALE, p(out), p(lse), n_ctas, stream)


def test_static_scratch_decode_matches_workspace_decode_twice():
    fn = _static_fn()
    # Two different batches back to back: the second call reuses scratch the first one filled.
    for seed, lens, Hq, Hkv in [(31, [513, 1, 4000, 77, 0, 2048], 32, 4), (32, [300, 9000, 33], 16, 8)]:
        kc, vc, q, bt, lens_t = _case(seed, lens, Hq, Hkv)
        ref, ref_lse = L.attn_decode(kc, vc, q, bt, lens_t, SCALE, want_lse=True)
        out = torch.empty_like(ref)
        lse = torch.empty_like(ref_lse)
        assert _call_static(fn, kc, vc, q, bt, lens_t, out, lse) == _lib.LSTK_OK, _lib.last_error()
        L.check_status()
        assert within(out.cpu().numpy(), ref.cpu().numpy())
        a, b = lse.cpu().numpy(), ref_lse.cpu().numpy()
        fin = np.isfinite(b)
        assert np.array_equal(np.isfinite(a), fin) and np.all(a[~fin] == b[~fin])  # empty sequence: -inf
        assert within(a[fin], b[fin], atol=1e-4, rtol=1e-5)


def test_static_scratch_at_its_limits_against_the_oracle():
    """The fixed array's two limits at once - 1024 sequences (mixed short lengths, some empty) on a
    160-CTA split - twice in a row with different data: against the CPU oracle directly, and bit
    for bit against the workspace entry point on the same grid."""
    fn = _static_fn()
    for seed, (Hq, Hkv) in ((41, (32, 4)), (42, (16, 8))):
        rng = np.random.default_rng(seed)
        lens = rng.integers(0, 400, 1024)
        lens[rng.choice(1024, 40, replace=False)] = 0
        lens = lens.tolist()
        kc, vc, q, bt, lens_t = _case(seed, lens, Hq, Hkv)
        out = torch.empty((1024, Hq, 128), device="cuda")
        lse = torch.empty((1024, Hq), device="cuda")
        assert _call_static(fn, kc, vc, q, bt, lens_t, out, lse, n_ctas=160) == _lib.LSTK_OK, _lib.last_error()
        ref, ref_lse = L.attn_decode(kc, vc, q, bt, lens_t, SCALE, want_lse=True, n_ctas=160)
        L.check_status()
        assert torch.equal(out, ref) and torch.equal(lse, ref_lse)
        lens_np = np.asarray(lens, np.int32)
        kh = kc.cpu().view(torch.int16).numpy().view(np.uint16)
        vh = vc.cpu().view(torch.int16).numpy().view(np.uint16)
        ex = O.paged_attn(q.cpu().numpy(), np.arange(1024), np.maximum(lens_np - 1, 0), kh, vh, bt.cpu().numpy(),
                          lens_np, SCALE, mode=O.MODE_EXACT)
        got = out.cpu().numpy()
        empty = lens_np == 0
        assert np.all(got[empty] == 0)
        assert within(got[~empty], ex[~empty]), max_err(got[~empty], ex[~empty])


def test_static_scratch_rejects_oversized_requests():
    fn = _static_fn()
    kc, vc, q, bt, lens_t = _case(33, [64], 32, 4)
    out = torch.empty((1, 32, 128), device="cuda")
    lse = torch.empty((1, 32), device="cuda")
    assert _call_static(fn, kc, vc, q, bt, lens_t, out, lse, n_ctas=161) == _lib.LSTK_ERR_CAPACITY
    assert "160" in _lib.last_error()
    big_q = torch.zeros((1025, 32, 128), device="cuda")
    big_bt = torch.zeros((1025, 1), dtype=torch.int32, device="cuda")
    big_lens = torch.zeros(1025, dtype=torch.int32, device="cuda")
    big_out = torch.empty((1025, 32, 128), device="cuda")
    rc = _call_static(fn, kc, vc, big_q, big_bt, big_lens, big_out, None)
    assert rc == _lib.LSTK_ERR_CAPACITY and "1024" in _lib.last_error()
