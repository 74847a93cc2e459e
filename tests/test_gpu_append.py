"""K/V append (QK-RMSNorm + NEOX RoPE + f16 set_rows) on the GPU vs the CPU oracle: bit-exact."""
import numpy as np
import pytest
import torch

import localstack_b200 as L
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _run(T, Hq, Hkv, n_cells, positions, cells, dtype="f32", gamma=True, seed=0, q_out_dtype=torch.float32,
         fused_rows=False):
    rng = np.random.default_rng(seed)
    D = 128
    if fused_rows:
        # One [T][(Hq + 2 Hkv) * D] projection output, passed as three strided views.
        qkv = rng.standard_normal((T, (Hq + 2 * Hkv) * D), dtype=np.float32) * 3
        q_in, k_in, v_in = (qkv[:, :Hq * D].reshape(T, Hq, D), qkv[:, Hq * D:(Hq + Hkv) * D].reshape(T, Hkv, D),
                            qkv[:, (Hq + Hkv) * D:].reshape(T, Hkv, D))
    else:
        q_in = rng.standard_normal((T, Hq, D), dtype=np.float32) * 3
        k_in = rng.standard_normal((T, Hkv, D), dtype=np.float32) * 3
        v_in = rng.standard_normal((T, Hkv, D), dtype=np.float32) * 3
    qg = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32) if gamma else None
    kg = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32) if gamma else None
    if dtype == "bf16":
        to_bits = lambda a: (torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).view(torch.int16).numpy()
                             .view(np.uint16))
        q_h, k_h, v_h = to_bits(q_in), to_bits(k_in), to_bits(v_in)
    else:
        q_h, k_h, v_h = q_in, k_in, v_in
    kc_ref = np.zeros((n_cells, Hkv, D), np.uint16)
    vc_ref = np.zeros((n_cells, Hkv, D), np.uint16)
    q_ref = O.kv_append(q_h, k_h, v_h, positions, cells, kc_ref, vc_ref, qg, kg, 1e-6, 1e6, 1.0, in_dtype=dtype)

    dev = "cuda"
    if fused_rows:
        qkv_t = torch.from_numpy(qkv).to(dev)
        if dtype == "bf16":
            qkv_t = qkv_t.to(torch.bfloat16)
        q_t, k_t, v_t = qkv_t[:, :Hq * D], qkv_t[:, Hq * D:(Hq + Hkv) * D], qkv_t[:, (Hq + Hkv) * D:]
    else:
        tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
        q_t, k_t, v_t = (torch.from_numpy(a).to(dev).to(tdt) for a in (q_in, k_in, v_in))
    kc = L.alloc_cache(n_cells, Hkv, dev)
    vc = L.alloc_cache(n_cells, Hkv, dev)
    rope = L.rope_table(int(max(positions)) + 1, dev)
    pos_t = torch.from_numpy(np.asarray(positions, np.int32)).to(dev)
    cells_t = torch.from_numpy(np.asarray(cells, np.int64)).to(dev)
    qg_t = torch.from_numpy(qg).to(dev) if gamma else None
    kg_t = torch.from_numpy(kg).to(dev) if gamma else None
    q_out = L.kv_append(kc, vc, q_t, k_t, v_t, pos_t, cells_t, rope, qg_t, kg_t, 1e-6, q_out_dtype=q_out_dtype)
    L.check_status()
    kc_gpu = kc.cpu().view(torch.int16).numpy().view(np.uint16)
    vc_gpu = vc.cpu().view(torch.int16).numpy().view(np.uint16)
    return q_out.float().cpu().numpy(), kc_gpu, vc_gpu, q_ref, kc_ref, vc_ref


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_append_prefill_chunk_bit_exact(dtype):
    # Config-2 shape: 2048 tokens, Hq 16 / Hkv 8, scattered into 64 seeded pages.
    rng = np.random.default_rng(1)
    T, n_pages = 2048, 64 + 3
    perm = rng.permutation(n_pages)[:64]
    pos = np.arange(T, dtype=np.int32)
    cells = (perm[pos // 32] * 32 + pos % 32).astype(np.int64)
    q, kc, vc, q_ref, kc_ref, vc_ref = _run(T, 16, 8, n_pages * 32, pos, cells, dtype=dtype)
    assert np.array_equal(kc, kc_ref), "K pages differ"
    assert np.array_equal(vc, vc_ref), "V pages differ"
    assert np.array_equal(q.view(np.uint32), q_ref.view(np.uint32)), "Q out differs"


def test_append_long_positions_and_fused_rows():
    # Positions up to 131071 (config 4), 30B-A3B heads, QKV as strided views of one projection.
    rng = np.random.default_rng(2)
    T = 97
    pos = np.sort(rng.choice(131072, T, replace=False)).astype(np.int32)
    cells = rng.permutation(4096 * 32)[:T].astype(np.int64)
    q, kc, vc, q_ref, kc_ref, vc_ref = _run(T, 32, 4, 4096 * 32, pos, cells, fused_rows=True, seed=3)
    assert np.array_equal(kc, kc_ref) and np.array_equal(vc, vc_ref)
    assert np.array_equal(q.view(np.uint32), q_ref.view(np.uint32))


def test_append_no_gamma_and_f16_q_out():
    rng = np.random.default_rng(4)
    T = 33
    pos = np.arange(500, 500 + T, dtype=np.int32)
    cells = rng.permutation(64)[:T].astype(np.int64)
    q, kc, vc, q_ref, kc_ref, vc_ref = _run(T, 16, 8, 64, pos, cells, gamma=False, q_out_dtype=torch.float16)
    assert np.array_equal(kc, kc_ref) and np.array_equal(vc, vc_ref)
    assert np.array_equal(q.astype(np.float16), q_ref.astype(np.float16))


def test_append_single_token_decode_step():
    q, kc, vc, q_ref, kc_ref, vc_ref = _run(1, 32, 4, 1024, np.array([512], np.int32), np.array([777], np.int64))
    assert np.array_equal(kc, kc_ref) and np.array_equal(vc, vc_ref)
    assert np.array_equal(q.view(np.uint32), q_ref.view(np.uint32))


def test_append_bad_cell_reports_device_index():
    dev = "cuda"
    kc = L.alloc_cache(64, 8, dev)
    vc = L.alloc_cache(64, 8, dev)
    q = torch.randn(2, 16, 128, device=dev)
    k = torch.randn(2, 8, 128, device=dev)
    v = torch.randn(2, 8, 128, device=dev)
    rope = L.rope_table(16, dev)
    pos = torch.tensor([0, 1], dtype=torch.int32, device=dev)
    cells = torch.tensor([3, 64], dtype=torch.int64, device=dev)  # 64 is out of range
    L.kv_append(kc, vc, q, k, v, pos, cells, rope)
    with pytest.raises(L.LstkError) as e:
        L.check_status()
    assert e.value.code == -6
    L.check_status()  # status is cleared once read
    assert torch.count_nonzero(kc[3]) > 0  # the valid token was still written


@pytest.mark.parametrize("dtype,q_out_dtype", [("bf16", torch.float16), ("bf16", torch.float32),
                                               ("f32", torch.float16)])
def test_append_large_batch_wide_groups(dtype, q_out_dtype):
    # Config-5 shape: 4352 tokens x (32 + 4 + 4) heads = 174,080 rows, QKV as strided views of one
    # projection output; enough rows for 32-row groups (bf16 in, f16 Q out) or 16-row groups.
    rng = np.random.default_rng(6)
    T, n_cells = 4352, 8192
    pos = rng.integers(0, 16384, T).astype(np.int32)
    cells = rng.permutation(n_cells)[:T].astype(np.int64)
    q, kc, vc, q_ref, kc_ref, vc_ref = _run(T, 32, 4, n_cells, pos, cells, dtype=dtype, q_out_dtype=q_out_dtype,
                                            fused_rows=True, seed=7)
    assert np.array_equal(kc, kc_ref) and np.array_equal(vc, vc_ref)
    if q_out_dtype == torch.float16:
        assert np.array_equal(q.astype(np.float16), q_ref.astype(np.float16))
    else:
        assert np.array_equal(q.view(np.uint32), q_ref.view(np.uint32))


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_append_groups_spanning_many_tokens(dtype):
    # Hq 1 / Hkv 1: 3 rows per token, and enough rows for 32-row (bf16) / 16-row (f32) groups, so
    # one group spans up to 12 tokens and the RoPE rows past its first four load in the write loop.
    rng = np.random.default_rng(8)
    T = 40000
    pos = rng.integers(0, 16384, T).astype(np.int32)
    cells = rng.permutation(T).astype(np.int64)
    q, kc, vc, q_ref, kc_ref, vc_ref = _run(T, 1, 1, T, pos, cells, dtype=dtype, seed=9)
    assert np.array_equal(kc, kc_ref) and np.array_equal(vc, vc_ref)
    assert np.array_equal(q.view(np.uint32), q_ref.view(np.uint32))


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_append_rms_sum_hard_rows(dtype):
    """Rows that stress the double sum of squares: values spanning many orders of magnitude (where
    summation order changes the rounding, so the kernel must sum in index order), denormal squares
    next to normal ones, a single nonzero, zeros, squares that overflow f32 (an infinite sum),
    squares just below that, and a moderate spread near the bound under which any order of
    summation is exact, in f32 and bf16. Pages and Q must equal the oracle's."""
    rng = np.random.default_rng(11)
    T, Hq, Hkv, D = 64, 16, 8, 128
    R = Hq + 2 * Hkv

    def rows(n):
        out = rng.standard_normal((n, D)).astype(np.float32) * 2
        kinds = rng.integers(0, 8, n)
        for r in range(n):
            if kinds[r] == 1:  # magnitudes from 1e-20 to 1e3: the exact bound fails
                out[r] *= (10.0 ** rng.uniform(-20, 3, D)).astype(np.float32)
            elif kinds[r] == 2:  # tiny values with denormal squares next to normal ones
                out[r, ::3] = 1e-21
            elif kinds[r] == 3:  # one nonzero element
                out[r] = 0
                out[r, rng.integers(D)] = 7.5
            elif kinds[r] == 4:  # all zeros
                out[r] = 0
            elif kinds[r] == 5:  # squares overflow f32: ggml's sum is inf, the scale 0
                out[r, rng.integers(D)] = 3e20
            elif kinds[r] == 6:  # squares up to ~1e36, their sum finite
                out[r] *= 3e17
            elif kinds[r] == 7:  # magnitudes over 2^-12..2^0: near the exact-summation bound
                out[r] *= (2.0 ** rng.uniform(-12, 0, D)).astype(np.float32)
        return out

    q_in = rows(T * Hq).reshape(T, Hq, D)
    k_in = rows(T * Hkv).reshape(T, Hkv, D)
    v_in = rng.standard_normal((T, Hkv, D)).astype(np.float32)
    if dtype == "bf16":
        bits = lambda a: (torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).view(torch.int16).numpy()
                          .view(np.uint16))
        q_h, k_h, v_h = bits(q_in), bits(k_in), bits(v_in)
    else:
        q_h, k_h, v_h = q_in, k_in, v_in
    pos = np.arange(T, dtype=np.int32) * 7
    cells = rng.permutation(256)[:T].astype(np.int64)
    g = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    kc_ref = np.zeros((256, Hkv, D), np.uint16)
    vc_ref = np.zeros_like(kc_ref)
    q_ref = O.kv_append(q_h, k_h, v_h, pos, cells, kc_ref, vc_ref, g, g, 1e-6, 1e6, 1.0, in_dtype=dtype)
    dev = "cuda"
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    kc, vc = L.alloc_cache(256, Hkv, dev), L.alloc_cache(256, Hkv, dev)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    q = L.kv_append(kc, vc, t(q_in).to(tdt), t(k_in).to(tdt), t(v_in).to(tdt), t(pos), t(cells),
                    L.rope_table(int(pos.max()) + 1, dev), t(g), t(g), 1e-6)
    L.check_status()
    assert np.array_equal(kc.cpu().view(torch.int16).numpy().view(np.uint16), kc_ref)
    assert np.array_equal(vc.cpu().view(torch.int16).numpy().view(np.uint16), vc_ref)
    assert np.array_equal(q.cpu().numpy().view(np.uint32), q_ref.view(np.uint32))
    assert R == 32
