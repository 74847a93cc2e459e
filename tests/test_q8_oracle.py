"""The q8_0 restatement in the oracle (CPU): ggml's block_q8_0 quantisation with known answers,
the q8_0 append equal to quantising the f16 path's f32 rows, and the two attention modes over a
q8_0 cache against each other and against attention over the dequantised cache."""
import numpy as np

from oracle import oracle as O
from tests.helpers import scattered_block_tables


def test_quantize_known_answers():
    x = np.zeros((2, 32), np.float32)
    x[0, :6] = [127, 2.5, -3.5, 0.5, -127, 1.5]  # amax 127: d = 1, q = x rounded, ties to even
    q, d = O.quantize_q8_0(x)
    assert list(q[0, :6]) == [127, 2, -4, 0, -127, 2]
    assert O.f16_bits_to_f32(d)[0, 0] == 1.0
    assert not q[1].any() and d[1, 0] == 0  # an all-zero block: d = 0, q = 0
    x = np.full((1, 32), -0.25, np.float32)  # d = 0.25 / 127; every value maps to -127
    q, d = O.quantize_q8_0(x)
    assert (q == -127).all()
    assert d[0, 0] == O.f32_to_f16_bits(np.float32(0.25) / np.float32(127))


def test_quantize_error_bound():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((200, 128)) * 10 ** rng.uniform(-3, 3, (200, 1))).astype(np.float32)
    q, d = O.quantize_q8_0(x)
    # q is x rounded in units of the unrounded d = amax / 127; the stored scale is the f16 of d
    # (subnormal for tiny blocks): |x - d16 q| <= d / 2 + |q| |d - d16| (+ f32 rounding)
    d_true = np.repeat(np.abs(x).reshape(200, 4, 32).max(-1) / np.float32(127), 32, axis=-1)
    d16 = np.repeat(O.f16_bits_to_f32(d), 32, axis=-1)
    bound = 0.5 * d_true + np.abs(q) * np.abs(d_true - d16) + 1e-6 * np.abs(x)
    assert np.all(np.abs(O.dequantize_q8_0(q, d) - x) <= bound)
    assert np.all(np.abs(q.astype(np.int32)) <= 127)


def test_append_q8_is_quantised_f32_rows():
    rng = np.random.default_rng(2)
    T, Hq, Hkv, D = 40, 8, 2, 128
    q_in = rng.standard_normal((T, Hq, D)).astype(np.float32) * 3
    k_in = rng.standard_normal((T, Hkv, D)).astype(np.float32) * 3
    v_in = rng.standard_normal((T, Hkv, D)).astype(np.float32) * 3
    pos = rng.integers(0, 5000, T).astype(np.int32)
    cells = rng.permutation(64)[:T].astype(np.int64)
    g = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    kqs, vqs = np.zeros((64, Hkv, D), np.int8), np.zeros((64, Hkv, D), np.int8)
    kd, vd = np.zeros((64, Hkv, 4), np.uint16), np.zeros((64, Hkv, 4), np.uint16)
    q8_q = O.kv_append_q8(q_in, k_in, v_in, pos, cells, kqs, kd, vqs, vd, g, g, 1e-6, 1e6, 1.0)
    kc, vc = np.zeros((64, Hkv, D), np.uint16), np.zeros((64, Hkv, D), np.uint16)
    f16_q = O.kv_append(q_in, k_in, v_in, pos, cells, kc, vc, g, g, 1e-6, 1e6, 1.0)
    assert np.array_equal(q8_q.view(np.uint32), f16_q.view(np.uint32))
    k_rows = O.rope_neox(O.rms_norm_mul(k_in, g, 1e-6), pos, 1e6)
    eq, ed = O.quantize_q8_0(k_rows)
    assert np.array_equal(kqs[cells], eq) and np.array_equal(kd[cells], ed)
    eq, ed = O.quantize_q8_0(v_in)
    assert np.array_equal(vqs[cells], eq) and np.array_equal(vd[cells], ed)


def test_attention_modes_over_q8_cache():
    rng = np.random.default_rng(3)
    lens = [1, 33, 700]
    bt, n_pages = scattered_block_tables(rng, lens)
    Hq, Hkv, D = 16, 4, 128
    k = rng.standard_normal((n_pages * 32, Hkv, D)).astype(np.float32)
    v = rng.standard_normal((n_pages * 32, Hkv, D)).astype(np.float32)
    kqs, kd = O.quantize_q8_0(k)
    vqs, vd = O.quantize_q8_0(v)
    q = rng.standard_normal((len(lens), Hq, D)).astype(np.float32)
    q = q / np.sqrt(np.mean(q * q, axis=-1, keepdims=True))
    seq = np.arange(len(lens))
    pos = np.asarray(lens) - 1
    scale = 1 / np.sqrt(D)
    gg = O.paged_attn_q8(q, seq, pos, kqs, kd, vqs, vd, bt, lens, scale, mode=O.MODE_GGML)
    ex = O.paged_attn_q8(q, seq, pos, kqs, kd, vqs, vd, bt, lens, scale, mode=O.MODE_EXACT)
    # the modes differ by the query's own q8_0 rounding (ggml) and the f32 / double arithmetic
    assert np.abs(gg - ex).max() < 1e-2
    # one key: the output is that key's dequantised V row exactly (softmax weight 1)
    row = bt[0, 0] * 32
    assert np.allclose(gg[0], np.repeat(O.dequantize_q8_0(vqs[row], vd[row]), Hq // Hkv, axis=0), atol=0, rtol=0)
