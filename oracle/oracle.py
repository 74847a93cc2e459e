"""ctypes wrapper over oracle/liblstk_oracle.so and oracle/_ref/libref_kv_cache.so.

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use
this module as the checker. The product (localstack_b200/) never imports it.

The oracle restates the ggml CPU semantics that the reference's attn_block
(src/qwen3.cpp:128-171) requests; see lstk_oracle.cpp's header for what is restated and why
parity with ggml itself is unpinned. `RefKvCache` drives the reference's own KvCache
(src/kv_cache.cpp) compiled unchanged against oracle/ref_shim.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblstk_oracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libref_kv_cache.so")

MODE_GGML = 0
MODE_EXACT = 1

_lib = None
_ref = None

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float


def build():
    """Compile the oracle libraries (and oracle/_ref when the reference sources are present)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.orc_f32_to_f16.argtypes = [_P, _P, _I64]
        L.orc_f16_to_f32.argtypes = [_P, _P, _I64]
        L.orc_rms_norm_mul.argtypes = [_P, _P, _I64, _I64, _P, _F]
        L.orc_rope_cache.argtypes = [_I64, _I, _F, _F, _P]
        L.orc_rope_neox.argtypes = [_P, _I64, _I64, _I64, _P, _I, _F, _F]
        L.orc_set_rows_f16.argtypes = [_P, _I64, _I64, _P, _I64, _I64, _P]
        L.orc_set_rows_f16.restype = _I
        L.orc_kv_append.argtypes = [_P, _P, _P, _I, _I64, _I64, _I64, _I, _I, _I, _I, _P, _P, _P, _P, _F, _F, _F,
                                    _P, _P, _I64, _P]
        L.orc_kv_append.restype = _I
        L.orc_flash_attn_ext.argtypes = [_P, _I, _I, _P, _P, _I, _I, _I64, _P, _F, _I, _P, _I]
        L.orc_paged_attn.argtypes = [_P, _I, _P, _P, _I, _P, _P, _I, _I, _I, _P, _I, _P, _I, _F, _I, _P, _P, _I]
        L.orc_lse_merge.argtypes = [_P, _P, _I, _I64, _I, _P, _P]
        L.orc_paged_decode_ggml_fast.argtypes = [_P, _I, _I, _P, _P, _I, _I, _I, _P, _I, _P, _F, _P, _I]
        L.orc_hardware_threads.restype = _I
        L.orc_quantize_q8_0.argtypes = [_P, _I64, _I, _P, _P]
        L.orc_quantize_q8_0.restype = _I
        L.orc_kv_append_q8.argtypes = [_P, _P, _P, _I, _I64, _I64, _I64, _I, _I, _I, _I, _P, _P, _P, _P, _F, _F, _F,
                                       _P, _P, _P, _P, _I64, _P]
        L.orc_kv_append_q8.restype = _I
        L.orc_paged_attn_q8.argtypes = [_P, _I, _P, _P, _I, _P, _P, _P, _P, _I, _I, _I, _P, _I, _P, _I, _F, _I, _P,
                                        _P, _I]
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(_P) if a is not None else None


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def f32_to_f16_bits(x):
    x = _c(x, np.float32)
    y = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_f16(_ptr(x), _ptr(y), x.size)
    return y


def f16_bits_to_f32(b):
    b = _c(b, np.uint16)
    y = np.empty(b.shape, np.float32)
    lib().orc_f16_to_f32(_ptr(b), _ptr(y), b.size)
    return y


def rms_norm_mul(x, gamma, eps):
    x = _c(x, np.float32)
    y = np.empty_like(x)
    g = _c(gamma, np.float32) if gamma is not None else None
    lib().orc_rms_norm_mul(_ptr(x), _ptr(y), x.size // x.shape[-1], x.shape[-1], _ptr(g), eps)
    return y


def rope_cache(pos, n_dims, freq_base, freq_scale=1.0):
    cs = np.empty(n_dims, np.float32)
    lib().orc_rope_cache(int(pos), n_dims, freq_base, freq_scale, _ptr(cs))
    return cs


def rope_neox(x, pos, freq_base, freq_scale=1.0):
    """x: [T][H][D] f32 (copied); returns the rotated copy."""
    x = np.array(x, dtype=np.float32, order="C", copy=True)
    pos = _c(pos, np.int32)
    T, H, D = x.shape
    lib().orc_rope_neox(_ptr(x), T, H, D, _ptr(pos), D, freq_base, freq_scale)
    return x


def kv_append(q_in, k_in, v_in, positions, cells, k_cache, v_cache, q_gamma=None, k_gamma=None, eps=1e-6,
              freq_base=1e6, freq_scale=1.0, in_dtype="f32"):
    """attn_block steps 2-4 on the CPU. q_in [T][Hq][D], k_in/v_in [T][Hkv][D] as f32 arrays, or
    uint16 bf16 bit patterns when in_dtype == "bf16". k_cache / v_cache: uint16 f16 bit arrays
    [n_cells][Hkv][D], updated in place. Returns q_out [T][Hq][D] f32."""
    dt = np.uint16 if in_dtype == "bf16" else np.float32
    q_in, k_in, v_in = _c(q_in, dt), _c(k_in, dt), _c(v_in, dt)
    T, Hq, D = q_in.shape
    Hkv = k_in.shape[1]
    positions, cells = _c(positions, np.int32), _c(cells, np.int64)
    assert k_cache.dtype == np.uint16 and k_cache.flags.c_contiguous
    assert v_cache.dtype == np.uint16 and v_cache.flags.c_contiguous
    qg = _c(q_gamma, np.float32) if q_gamma is not None else None
    kg = _c(k_gamma, np.float32) if k_gamma is not None else None
    q_out = np.empty((T, Hq, D), np.float32)
    rc = lib().orc_kv_append(_ptr(q_in), _ptr(k_in), _ptr(v_in), 2 if in_dtype == "bf16" else 0, Hq * D, Hkv * D,
                             Hkv * D, T, Hq, Hkv, D, _ptr(positions), _ptr(cells), _ptr(qg), _ptr(kg), eps,
                             freq_base, freq_scale, _ptr(k_cache), _ptr(v_cache), k_cache.shape[0], _ptr(q_out))
    if rc != 0:
        raise ValueError("oracle kv_append: cell index out of range")
    return q_out


def quantize_q8_0(x):
    """ggml q8_0 of each row of x [..., D] f32 (D a multiple of 32): (qs int8 [..., D],
    d uint16 f16 bits [..., D // 32]); ties round to even (the ARM NEON form)."""
    x = _c(x, np.float32)
    D = x.shape[-1]
    n_rows = x.size // D
    qs = np.empty(x.shape, np.int8)
    d = np.empty(x.shape[:-1] + (D // 32,), np.uint16)
    if lib().orc_quantize_q8_0(_ptr(x), n_rows, D, _ptr(qs), _ptr(d)) != 0:
        raise ValueError("row length must be a multiple of 32")
    return qs, d


def dequantize_q8_0(qs, d):
    """f32 values d * q of q8_0 planes (qs [..., D] int8, d [..., D // 32] f16 bits)."""
    scale = f16_bits_to_f32(np.asarray(d, np.uint16))
    return (np.repeat(scale, 32, axis=-1) * qs.astype(np.float32)).astype(np.float32)


def kv_append_q8(q_in, k_in, v_in, positions, cells, k_qs, k_d, v_qs, v_d, q_gamma=None, k_gamma=None, eps=1e-6,
                 freq_base=1e6, freq_scale=1.0, in_dtype="f32"):
    """kv_append with K and V stored as q8_0 planes: k_qs / v_qs int8 [n_cells][Hkv][D] and
    k_d / v_d uint16 f16 bits [n_cells][Hkv][D // 32], updated in place. Returns q_out f32."""
    dt = np.uint16 if in_dtype == "bf16" else np.float32
    q_in, k_in, v_in = _c(q_in, dt), _c(k_in, dt), _c(v_in, dt)
    T, Hq, D = q_in.shape
    Hkv = k_in.shape[1]
    positions, cells = _c(positions, np.int32), _c(cells, np.int64)
    for a, t in ((k_qs, np.int8), (v_qs, np.int8), (k_d, np.uint16), (v_d, np.uint16)):
        assert a.dtype == t and a.flags.c_contiguous
    qg = _c(q_gamma, np.float32) if q_gamma is not None else None
    kg = _c(k_gamma, np.float32) if k_gamma is not None else None
    q_out = np.empty((T, Hq, D), np.float32)
    rc = lib().orc_kv_append_q8(_ptr(q_in), _ptr(k_in), _ptr(v_in), 2 if in_dtype == "bf16" else 0, Hq * D,
                                Hkv * D, Hkv * D, T, Hq, Hkv, D, _ptr(positions), _ptr(cells), _ptr(qg), _ptr(kg), eps,
                                freq_base, freq_scale, _ptr(k_qs), _ptr(k_d), _ptr(v_qs), _ptr(v_d), k_qs.shape[0],
                                _ptr(q_out))
    if rc != 0:
        raise ValueError("oracle kv_append_q8: cell index out of range")
    return q_out


def paged_attn_q8(q, q_seq, q_pos, k_qs, k_d, v_qs, v_d, block_tables, kv_lens, scale, causal=True, mode=MODE_GGML,
                  block_size=32, n_threads=0, want_lse=False):
    """paged_attn over a q8_0 cache (planes as in kv_append_q8). MODE_GGML: ggml's CPU semantics
    for a q8_0 cache (query quantised to q8_0, integer block dots, f32 V accumulation);
    MODE_EXACT: f32 query against the dequantised cache, in double."""
    q = _c(q, np.float32)
    n_q, Hq, D = q.shape
    Hkv = k_qs.shape[1]
    q_seq, q_pos = _c(q_seq, np.int32), _c(q_pos, np.int32)
    bt = _c(block_tables, np.int32)
    kv_lens = _c(kv_lens, np.int32)
    k_qs, v_qs = _c(k_qs, np.int8), _c(v_qs, np.int8)
    k_d, v_d = _c(k_d, np.uint16), _c(v_d, np.uint16)
    out = np.empty_like(q)
    lse = np.empty((n_q, Hq), np.float32) if want_lse else None
    lib().orc_paged_attn_q8(_ptr(q), n_q, _ptr(q_seq), _ptr(q_pos), Hq, _ptr(k_qs), _ptr(k_d), _ptr(v_qs), _ptr(v_d),
                            Hkv, D, block_size, _ptr(bt), bt.shape[1], _ptr(kv_lens), 1 if causal else 0, scale, mode,
                            _ptr(out), _ptr(lse), n_threads)
    return (out, lse) if want_lse else out


def flash_attn_ext(q, k_cache, v_cache, n_kv, mask, scale, mode=MODE_EXACT, n_threads=0):
    """Dense masked attention over cells [0, n_kv) as ggml_flash_attn_ext (src/qwen3.cpp:165)."""
    q = _c(q, np.float32)
    T, Hq, D = q.shape
    Hkv = k_cache.shape[1]
    mask = _c(mask, np.uint16) if mask is not None else None
    out = np.empty_like(q)
    lib().orc_flash_attn_ext(_ptr(q), T, Hq, _ptr(k_cache), _ptr(v_cache), Hkv, D, n_kv, _ptr(mask), scale, mode,
                             _ptr(out), n_threads)
    return out


def paged_attn(q, q_seq, q_pos, k_cache, v_cache, block_tables, kv_lens, scale, causal=True, mode=MODE_EXACT,
               block_size=32, n_threads=0, want_lse=False):
    """Page-table attention. q [n_q][Hq][D]; q_seq/q_pos [n_q]; block_tables [B][max_blocks]."""
    q = _c(q, np.float32)
    n_q, Hq, D = q.shape
    Hkv = k_cache.shape[1]
    q_seq, q_pos = _c(q_seq, np.int32), _c(q_pos, np.int32)
    bt = _c(block_tables, np.int32)
    kv_lens = _c(kv_lens, np.int32)
    out = np.empty_like(q)
    lse = np.empty((n_q, Hq), np.float32) if want_lse else None
    lib().orc_paged_attn(_ptr(q), n_q, _ptr(q_seq), _ptr(q_pos), Hq, _ptr(k_cache), _ptr(v_cache), Hkv, D,
                         block_size, _ptr(bt), bt.shape[1], _ptr(kv_lens), 1 if causal else 0, scale, mode,
                         _ptr(out), _ptr(lse), n_threads)
    return (out, lse) if want_lse else out


def lse_merge(o_parts, lse_parts):
    o_parts = _c(o_parts, np.float32)
    lse_parts = _c(lse_parts, np.float32)
    R, n_rows, D = o_parts.shape
    out = np.empty((n_rows, D), np.float32)
    lse = np.empty(n_rows, np.float32)
    lib().orc_lse_merge(_ptr(o_parts), _ptr(lse_parts), R, n_rows, D, _ptr(out), _ptr(lse))
    return out, lse


def paged_decode_ggml_fast(q, k_cache, v_cache, block_tables, kv_lens, scale, block_size=32, n_threads=0):
    """Timed CPU baseline (ggml CPU precision model), one query per sequence. q [B][Hq][D]."""
    q = _c(q, np.float32)
    B, Hq, D = q.shape
    Hkv = k_cache.shape[1]
    bt = _c(block_tables, np.int32)
    kv_lens = _c(kv_lens, np.int32)
    out = np.empty_like(q)
    lib().orc_paged_decode_ggml_fast(_ptr(q), B, Hq, _ptr(k_cache), _ptr(v_cache), Hkv, D, block_size, _ptr(bt),
                                     bt.shape[1], _ptr(kv_lens), scale, _ptr(out), n_threads)
    return out


def hardware_threads():
    return lib().orc_hardware_threads()


# ---------------------------------------------------------------------------------------------
# The reference's own KvCache (src/kv_cache.h:24-62), compiled unchanged against ref_shim.


def ref_available():
    return os.path.exists(REF_LIB_PATH)


def ref_lib():
    global _ref
    if _ref is None:
        if not ref_available():
            raise FileNotFoundError("oracle/_ref/libref_kv_cache.so not built (reference sources absent)")
        L = ctypes.CDLL(REF_LIB_PATH)
        U32, I32 = ctypes.c_uint32, ctypes.c_int32
        L.refkv_create.argtypes = [U32, U32, U32]
        L.refkv_create.restype = _P
        L.refkv_destroy.argtypes = [_P]
        L.refkv_set_free_blocks.argtypes = [_P, _P, _I]
        L.refkv_alloc.argtypes = [_P, I32, _I, _P, _P]
        L.refkv_alloc.restype = _I
        L.refkv_remove_seq.argtypes = [_P, I32]
        L.refkv_truncate_seq.argtypes = [_P, I32, I32]
        L.refkv_length.argtypes = [_P, I32]
        L.refkv_length.restype = I32
        L.refkv_used_hwm.argtypes = [_P]
        L.refkv_used_hwm.restype = U32
        L.refkv_n_free_cells.argtypes = [_P]
        L.refkv_n_free_cells.restype = U32
        L.refkv_cells.argtypes = [_P, _P, _P]
        L.refkv_free_blocks.argtypes = [_P, _P, _I]
        L.refkv_free_blocks.restype = _I
        L.refkv_seq_blocks.argtypes = [_P, I32, _P, _I]
        L.refkv_seq_blocks.restype = _I
        L.refkv_fill_mask.argtypes = [_P, I32, _P, _I, _I, _P]
        _ref = L
    return _ref


class RefKvCache:
    """The reference's KvCache driven through ctypes (bookkeeping only; host tensors are dummies)."""

    def __init__(self, size, n_embd_gqa=8, n_layer=1):
        self.size = size
        self.h = ref_lib().refkv_create(n_layer, n_embd_gqa, size)
        if not self.h:
            raise RuntimeError("KvCache::init failed")

    def __del__(self):
        if getattr(self, "h", None):
            ref_lib().refkv_destroy(self.h)
            self.h = None

    def set_free_blocks(self, blocks):
        b = _c(blocks, np.uint32)
        ref_lib().refkv_set_free_blocks(self.h, _ptr(b), b.size)

    def alloc(self, seq, n_tokens):
        cells = np.empty(n_tokens, np.int64)
        pos = np.empty(n_tokens, np.int32)
        ok = ref_lib().refkv_alloc(self.h, seq, n_tokens, _ptr(cells), _ptr(pos))
        return (cells, pos) if ok else None

    def remove_seq(self, seq):
        ref_lib().refkv_remove_seq(self.h, seq)

    def truncate_seq(self, seq, keep):
        ref_lib().refkv_truncate_seq(self.h, seq, keep)

    def length(self, seq):
        return ref_lib().refkv_length(self.h, seq)

    @property
    def used_hwm(self):
        return ref_lib().refkv_used_hwm(self.h)

    def n_free_cells(self):
        return ref_lib().refkv_n_free_cells(self.h)

    def cells(self):
        cs = np.empty(self.size, np.int32)
        cp = np.empty(self.size, np.int32)
        ref_lib().refkv_cells(self.h, _ptr(cs), _ptr(cp))
        return cs, cp

    def free_blocks(self):
        out = np.empty(self.size // 32 + 1, np.uint32)
        n = ref_lib().refkv_free_blocks(self.h, _ptr(out), out.size)
        return out[:n].copy()

    def seq_blocks(self, seq):
        out = np.empty(self.size // 32 + 1, np.uint32)
        n = ref_lib().refkv_seq_blocks(self.h, seq, _ptr(out), out.size)
        return out[:n].copy()

    def fill_mask(self, seq, pos, n_kv):
        pos = _c(pos, np.int32)
        mask = np.empty((pos.size, n_kv), np.uint16)
        ref_lib().refkv_fill_mask(self.h, seq, _ptr(pos), pos.size, n_kv, _ptr(mask))
        return mask
