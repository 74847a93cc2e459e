"""Loader for liblstk_attn.so, the sm_100a kernels behind include/lstk_cuda_attn.h.

The library is built in-tree (localstack_b200/liblstk_attn.so) by `build()`. There is no
fallback: if the library is missing or fails to load, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "liblstk_attn.so")
HEADER = os.path.join(ROOT, "include", "lstk_cuda_attn.h")

LSTK_OK = 0
LSTK_ERR_INVALID_ARG = -1
LSTK_ERR_CAPACITY = -2
LSTK_ERR_TIMEOUT = -3
LSTK_ERR_CUDA = -4
LSTK_ERR_UNSUPPORTED = -5
LSTK_ERR_DEVICE_INDEX = -6

DTYPE_F32 = 0
DTYPE_F16 = 1
DTYPE_BF16 = 2


class KvLayout(ctypes.Structure):
    """lstk_kv_layout: geometry of one layer's K (or V) cache tensor."""

    _fields_ = [
        ("n_cells", ctypes.c_int64),
        ("n_head_kv", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
    ]


class LstkError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"lstk error {code}: {msg}")
        self.code = code


def build(verbose=False):
    """Compile liblstk_attn.so for sm_100a with nvcc (no GPU needed)."""
    out = subprocess.run(["make", "-C", os.path.join(HERE, "csrc")], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("building liblstk_attn.so failed:\n" + out.stdout + out.stderr)
    if verbose:
        print(out.stdout)


_lib = None

_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F = ctypes.c_float
_SZ = ctypes.c_size_t
_LP = ctypes.POINTER(KvLayout)


class KvPages(ctypes.Structure):
    """lstk_kv_pages (include/lstk_cuda_attn.h): device-side KvCache state."""
    _fields_ = [("free_blocks", ctypes.c_void_p), ("free_top", ctypes.c_void_p), ("block_tables", ctypes.c_void_p),
                ("seq_lens", ctypes.c_void_p), ("used_hwm", ctypes.c_void_p), ("n_slots", ctypes.c_int32),
                ("max_blocks", ctypes.c_int32), ("block_size", ctypes.c_int32)]


def declared_symbols():
    """Names of every function declared in include/lstk_cuda_attn.h."""
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"\b(lstk_[a-z0-9_]+)\s*\(", text)))


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise FileNotFoundError(f"{LIB_PATH} is not built; run localstack_b200._lib.build()")
    L = ctypes.CDLL(LIB_PATH)
    L.lstk_cuda_last_error.restype = ctypes.c_char_p
    L.lstk_cuda_status.argtypes = [_P]
    L.lstk_rope_table_bytes.argtypes = [_I32, _I32]
    L.lstk_rope_table_bytes.restype = _SZ
    L.lstk_rope_table_fill.argtypes = [_P, _I32, _I32, _F, _F]
    L.lstk_cuda_set_wait_policy.argtypes = [ctypes.c_uint64, _P]
    L.lstk_cuda_kv_append.argtypes = [_LP, _P, _P, _P, _P, _P, _I32, _I64, _I64, _I64, _I32, _I32, _P, _P, _P, _P,
                                      _F, _P, _I32, _P, _I32, _P]
    L.lstk_cuda_attn_decode_workspace_size.argtypes = [_I32, _I32, _I32, _I32]
    L.lstk_cuda_attn_decode_workspace_size.restype = _SZ
    L.lstk_cuda_attn_decode.argtypes = [_LP, _P, _P, _P, _I32, _I32, _I32, _P, _I32, _P, _I32, _F, _P, _P, _P, _SZ,
                                        _I32, _P]
    L.lstk_cuda_attn_decode_partial.argtypes = [_P, _P, _P, _P, _I32, _I32, _I32, _P, _I32, _P, _I32, _I32, _I32,
                                                ctypes.c_float, _P, _P, _P, _SZ, _I32, _P]
    L.lstk_cuda_attn_merge.argtypes = [_P, _P, _I32, _I64, _I32, _I64, _I64, _P, _P, _P]
    L.lstk_cuda_kv_append_q8.argtypes = [_LP, _P, _P, _P, _P, _P, _P, _P, _I32, _I64, _I64, _I64, _I32, _I32, _P, _P,
                                         _P, _P, _F, _P, _I32, _P, _I32, _P]
    L.lstk_cuda_q8_prefill_scratch_size.argtypes = [_I32, _I32, _I32]
    L.lstk_cuda_q8_prefill_scratch_size.restype = _SZ
    L.lstk_cuda_attn_prefill_q8.argtypes = [_LP, _P, _P, _P, _P, _P, _I32, _I32, _I32, _P, _I32, _I64, _P, _P, _P,
                                            _I32, _F, _P, _P, _SZ, _P, _SZ, _P]
    L.lstk_cuda_q8_from_ggml_blocks.argtypes = [_P, _I64, _P, _P, _P]
    L.lstk_cuda_q8_to_ggml_blocks.argtypes = [_P, _P, _I64, _P, _P]
    L.lstk_cuda_attn_decode_q8.argtypes = [_LP, _P, _P, _P, _P, _P, _I32, _I32, _I32, _P, _I32, _P, _I32, _F, _P, _P,
                                           _P, _SZ, _I32, _P]
    L.lstk_cuda_mailbox_bytes.restype = _SZ
    L.lstk_cuda_mailbox_bytes.argtypes = [_I32, _I64, _I32]
    L.lstk_cuda_mailbox_alloc.argtypes = [_SZ, _P, _P]
    L.lstk_cuda_mailbox_free.argtypes = [_P]
    L.lstk_cuda_mailbox_open.argtypes = [_P, _P]
    L.lstk_cuda_mailbox_close.argtypes = [_P]
    L.lstk_cuda_attn_exchange_merge.argtypes = [_P, _I32, _I32, _P, _P, _I64, _I32, ctypes.c_uint64, _P, _P, _P]
    L.lstk_cuda_attn_decode_exchange.argtypes = [_LP, _P, _P, _P, _I32, _I32, _I32, _P, _I32, _P, _I32, _F, _P, _P,
                                                 _P, _SZ, _I32, _P, _I32, _I32, ctypes.c_uint64, _P]
    L.lstk_cuda_attn_prefill_workspace_size.argtypes = [_I32, _I32, _I32, _I32, _I32, _I32, _I64, _I32]
    L.lstk_cuda_attn_prefill_workspace_size.restype = _SZ
    L.lstk_cuda_attn_prefill.argtypes = [_LP, _P, _P, _P, _I32, _I32, _I32, _P, _I32, _I64, _P, _P, _P, _I32, _F, _P,
                                         _P, _SZ, _P]
    L.lstk_cuda_proj.argtypes = [_P, _I64, _P, _I64, _I32, _I32, _I32, _P, _I64, _P, _I32, _I64, _P]
    L.lstk_cuda_proj_workspace_size.argtypes = [_I32, _I32, _I32]
    L.lstk_cuda_proj_workspace_size.restype = _SZ
    L.lstk_cuda_proj_ws.argtypes = [_P, _I64, _P, _I64, _I32, _I32, _I32, _P, _I64, _P, _I32, _I64, _P, _SZ, _P]
    L.lstk_cuda_rms_norm.argtypes = [_P, _I32, _I64, _P, _F, _P, _I64, _I32, _I32, _P]
    L.lstk_cuda_to_bf16.argtypes = [_P, _I64, _P, _I64, _I32, _I32, _P]
    L.lstk_cuda_kv_alloc.argtypes = [_P, _P, _P, _I32, _I32, _P, _P, _P, _P]
    L.lstk_cuda_kv_release.argtypes = [_P, _I32, _I32, _P]
    _lib = L
    return L


def last_error():
    return lib().lstk_cuda_last_error().decode()


def check(rc):
    if rc != LSTK_OK:
        raise LstkError(rc, last_error())
    return rc
