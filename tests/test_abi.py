"""The C-ABI library loads, exports every function its headers declare, and rejects bad
arguments with the documented status codes before touching a GPU."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

import localstack_b200 as L
from localstack_b200 import _lib

INCLUDE = os.path.join(_lib.ROOT, "include")


def _declared(header):
    with open(os.path.join(INCLUDE, header)) as f:
        return sorted(set(re.findall(r"\b(lstk_[a-z0-9_]+)\s*\(", f.read())))


def test_every_declared_symbol_is_exported():
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True, check=True)
    exported = set(re.findall(r" T (lstk_\w+)", out.stdout))
    for header in sorted(os.listdir(INCLUDE)):
        if header.endswith(".h"):
            missing = [s for s in _declared(header) if s not in exported]
            assert not missing, f"{header}: not exported: {missing}"
    lib = L.lib()
    for s in _declared("lstk_cuda_attn.h"):
        assert hasattr(lib, s)


def test_library_is_built_for_sm100a_only():
    # ptxas's own report of the build (-Xptxas -v): every kernel entry was compiled for sm_100a
    log = os.path.join(_lib.ROOT, "localstack_b200", "csrc", "_build", "ptxas.log")
    if not os.path.exists(log):
        pytest.skip("no ptxas log (library built elsewhere)")
    with open(log) as f:
        targets = set(re.findall(r"Compiling entry function '\w+' for '(\w+)'", f.read()))
    assert targets == {"sm_100a"}, targets


def _layout(n_cells=64, hkv=8, hd=128, bs=32):
    return _lib.KvLayout(n_cells, hkv, hd, bs)


NULL = None


def test_validation_errors_without_gpu():
    lib = L.lib()
    fake = ctypes.c_void_p(0x10000)  # never dereferenced: validation fails first
    lay = _layout()
    # head_dim other than 128 is unsupported
    rc = lib.lstk_cuda_attn_decode(ctypes.byref(_layout(hd=64)), fake, fake, fake, 0, 1, 16, fake, 1, fake, 0, 0.1,
                                   fake, NULL, fake, 1 << 30, 0, NULL)
    assert rc == _lib.LSTK_ERR_UNSUPPORTED and "head_dim" in _lib.last_error()
    # GQA group above 8
    rc = lib.lstk_cuda_attn_decode(ctypes.byref(_layout(hkv=1)), fake, fake, fake, 0, 1, 16, fake, 1, fake, 0, 0.1,
                                   fake, NULL, fake, 1 << 30, 0, NULL)
    assert rc == _lib.LSTK_ERR_UNSUPPORTED
    # workspace too small
    rc = lib.lstk_cuda_attn_decode(ctypes.byref(lay), fake, fake, fake, 0, 4, 16, fake, 1, fake, 0, 0.1, fake, NULL,
                                   fake, 16, 0, NULL)
    assert rc == _lib.LSTK_ERR_CAPACITY
    # null layout, null pointers, n_head not a multiple of n_head_kv
    assert lib.lstk_cuda_attn_decode(None, fake, fake, fake, 0, 1, 16, fake, 1, fake, 0, 0.1, fake, NULL, fake,
                                     1 << 30, 0, NULL) == _lib.LSTK_ERR_INVALID_ARG
    assert lib.lstk_cuda_attn_decode(ctypes.byref(lay), NULL, fake, fake, 0, 1, 16, fake, 1, fake, 0, 0.1, fake, NULL,
                                     fake, 1 << 30, 0, NULL) == _lib.LSTK_ERR_INVALID_ARG
    assert lib.lstk_cuda_attn_decode(ctypes.byref(lay), fake, fake, fake, 0, 1, 12, fake, 1, fake, 0, 0.1, fake, NULL,
                                     fake, 1 << 30, 0, NULL) == _lib.LSTK_ERR_INVALID_ARG
    # kv_append: bad dtype, short stride, unaligned pointer
    args = lambda dt=0, qs=16 * 128, ptr=fake: (ctypes.byref(lay), ptr, fake, fake, fake, fake, dt, qs, 8 * 128,
                                                8 * 128, 1, 16, fake, fake, NULL, NULL, 1e-6, fake, 10, fake, 0, NULL)
    assert lib.lstk_cuda_kv_append(*args(dt=1)) == _lib.LSTK_ERR_UNSUPPORTED
    assert lib.lstk_cuda_kv_append(*args(qs=100)) == _lib.LSTK_ERR_INVALID_ARG
    # bf16 rows must start on 16-byte boundaries: a stride of 8-element multiples
    assert lib.lstk_cuda_kv_append(*args(dt=_lib.DTYPE_BF16, qs=16 * 128 + 4)) == _lib.LSTK_ERR_INVALID_ARG
    assert lib.lstk_cuda_kv_append(*args(ptr=ctypes.c_void_p(0x10002))) == _lib.LSTK_ERR_INVALID_ARG
    # prefill: GQA group 3 cannot tile 128 rows
    rc = lib.lstk_cuda_attn_prefill(ctypes.byref(_layout(hkv=4)), fake, fake, fake, 1, 1, 12, fake, 1, 1, fake, fake,
                                    fake, 1, 0.1, fake, NULL, 0, NULL)
    assert rc == _lib.LSTK_ERR_UNSUPPORTED
    # merge: no parts
    assert lib.lstk_cuda_attn_merge(fake, fake, 0, 1, 128, 0, 0, fake, NULL, NULL) == _lib.LSTK_ERR_INVALID_ARG
    assert lib.lstk_cuda_attn_merge(fake, fake, 2, 4, 128, 100, 0, fake, NULL, NULL) == _lib.LSTK_ERR_INVALID_ARG
    # a zero-sized call is a no-op that succeeds without a device
    rc = lib.lstk_cuda_kv_append(ctypes.byref(lay), fake, fake, fake, fake, fake, 0, 16 * 128, 8 * 128, 8 * 128, 0, 16,
                                 fake, fake, NULL, NULL, 1e-6, fake, 10, fake, 0, NULL)
    assert rc == _lib.LSTK_OK


def test_kv_pages_validation_without_gpu():
    lib = L.lib()
    fake = 0x10000
    st = lambda bs=32, n_slots=4: _lib.KvPages(fake, fake, fake, fake, fake, n_slots, 8, bs)
    alloc = lambda state, slots=fake, n=1, cap=1, cells=fake: lib.lstk_cuda_kv_alloc(state, slots, NULL, n, cap, cells,
                                                                                     fake, fake, NULL)
    assert alloc(None) == _lib.LSTK_ERR_INVALID_ARG
    assert alloc(ctypes.byref(st(bs=16))) == _lib.LSTK_ERR_UNSUPPORTED
    assert alloc(ctypes.byref(st(n_slots=0))) == _lib.LSTK_ERR_INVALID_ARG
    assert alloc(ctypes.byref(st()), slots=NULL) == _lib.LSTK_ERR_INVALID_ARG
    assert alloc(ctypes.byref(st()), n=-1) == _lib.LSTK_ERR_INVALID_ARG
    assert alloc(ctypes.byref(st()), cap=-1) == _lib.LSTK_ERR_INVALID_ARG
    assert alloc(ctypes.byref(st()), cells=NULL) == _lib.LSTK_ERR_INVALID_ARG
    assert alloc(ctypes.byref(st()), n=2049, cap=2049) == _lib.LSTK_ERR_CAPACITY
    assert alloc(ctypes.byref(st()), n=0) == _lib.LSTK_OK
    assert lib.lstk_cuda_kv_release(ctypes.byref(st()), 4, 0, NULL) == _lib.LSTK_ERR_INVALID_ARG
    assert lib.lstk_cuda_kv_release(ctypes.byref(st()), -1, 0, NULL) == _lib.LSTK_ERR_INVALID_ARG


def test_decode_partial_validates_range():
    lib = L.lib()
    lay = _layout()
    fake = ctypes.c_void_p(1 << 20)
    args = lambda b, e: (ctypes.byref(lay), fake, fake, fake, _lib.DTYPE_F32, 1, 16, fake, 2, fake, 64, b, e,
                         ctypes.c_float(0.1), fake, NULL, fake, 1 << 30, 0, NULL)
    assert lib.lstk_cuda_attn_decode_partial(*args(16, 64)) == _lib.LSTK_ERR_INVALID_ARG  # not a page multiple
    assert lib.lstk_cuda_attn_decode_partial(*args(64, 32)) == _lib.LSTK_ERR_INVALID_ARG  # end before begin
    assert lib.lstk_cuda_attn_decode_partial(*args(-32, 32)) == _lib.LSTK_ERR_INVALID_ARG


def test_exchange_entry_points_validate():
    lib = L.lib()
    assert lib.lstk_cuda_mailbox_bytes(2, 32, 128) > 2 * 2 * 32 * 129 * 4
    assert lib.lstk_cuda_mailbox_bytes(0, 32, 128) == 0 and lib.lstk_cuda_mailbox_bytes(2, 32, 64) == 0
    fake = ctypes.c_void_p(1 << 20)
    h = (ctypes.c_char * 64)()
    assert lib.lstk_cuda_mailbox_alloc(0, ctypes.byref(ctypes.c_void_p()), h) == _lib.LSTK_ERR_INVALID_ARG
    assert lib.lstk_cuda_mailbox_open(NULL, ctypes.byref(ctypes.c_void_p())) == _lib.LSTK_ERR_INVALID_ARG
    assert lib.lstk_cuda_mailbox_free(NULL) == _lib.LSTK_OK
    # rank out of range, bad head_dim
    assert lib.lstk_cuda_attn_exchange_merge(fake, 2, 2, fake, fake, 32, 128, 0, fake, NULL, NULL) == \
        _lib.LSTK_ERR_INVALID_ARG
    assert lib.lstk_cuda_attn_exchange_merge(fake, 0, 2, fake, fake, 32, 64, 0, fake, NULL, NULL) == \
        _lib.LSTK_ERR_UNSUPPORTED


def test_workspace_sizes():
    lib = L.lib()
    a = lib.lstk_cuda_attn_decode_workspace_size(64, 32, 4, 128)
    b = lib.lstk_cuda_attn_decode_workspace_size(4096, 32, 4, 128)
    assert 0 < a < b
    # f16 queries need no scratch; f32 queries need their f16 copy
    assert lib.lstk_cuda_attn_prefill_workspace_size(1, 16, 8, 128, 2048, 64, 2048, _lib.DTYPE_F16) == 0
    assert lib.lstk_cuda_attn_prefill_workspace_size(1, 16, 8, 128, 2048, 64, 2048, _lib.DTYPE_F32) == \
        2048 * 16 * 128 * 2


def test_rope_table_host_fill():
    t = L.rope_table_host(4).numpy()
    assert t.shape == (4, 64, 2)
    assert np.all(t[0, :, 0] == 1.0) and np.all(t[0, :, 1] == 0.0)
    lib = L.lib()
    assert lib.lstk_rope_table_fill(None, 4, 128, 1e6, 1.0) == _lib.LSTK_ERR_INVALID_ARG
    assert lib.lstk_rope_table_bytes(4, 128) == 4 * 64 * 2 * 4


def test_ggml_front_end_links_the_reference_graph_builder():
    """Where the reference sources were present at build time, the ggml-compatible front end
    exists and contains the reference's own graph builder and KvCache next to its entry points."""
    lib = os.path.join(_lib.ROOT, "localstack_b200", "ggml_node", "_build", "libggml_node.so")
    if not os.path.exists(lib):
        pytest.skip("front end not built (reference sources absent)")
    out = subprocess.run(["nm", "-D", "--defined-only", "-C", lib], capture_output=True, text=True, check=True).stdout
    for sym in ("lstk_node_create", "lstk_node_create_gguf", "lstk_node_step", "lstk_node_truncate",
                "lstk_node_destroy", "lstk_node_last_error",
                "qwen3_build_graph(", "KvCache::alloc(", "KvCache::fill_mask(", "ggml_flash_attn_ext("):
        assert sym in out, sym


def test_python_wrappers_validate_before_launch():
    # Wrong index dtypes, shapes or strided tensors are refused in Python, before any launch.
    import torch
    kc = torch.zeros(64, 8, 128, dtype=torch.float16)
    q = torch.zeros(4, 16, 128, dtype=torch.float16)
    i32 = lambda *v: torch.tensor(v, dtype=torch.int32)
    bt = torch.zeros(1, 2, dtype=torch.int32)
    with pytest.raises(ValueError):  # q_seq_start int64
        L.attn_prefill(kc, kc, q, torch.tensor([0, 4]), i32(0), i32(4), bt, 4)
    with pytest.raises(ValueError):  # q_seq_start must have B + 1 entries
        L.attn_prefill(kc, kc, q, i32(0, 2, 4), i32(0), i32(4), bt, 4)
    with pytest.raises(ValueError):  # strided q
        L.attn_prefill(kc, kc, torch.zeros(4, 32, 128, dtype=torch.float16)[:, ::2], i32(0, 4), i32(0), i32(4), bt, 4)
    with pytest.raises(ValueError):  # bf16 q is not a prefill input
        L.attn_prefill(kc, kc, q.bfloat16(), i32(0, 4), i32(0), i32(4), bt, 4)
    with pytest.raises(ValueError):  # int64 block tables
        L.attn_decode(kc, kc, q[:1], bt.long(), i32(4))
    with pytest.raises(ValueError):  # strided block tables
        L.attn_decode(kc, kc, q[:1], torch.zeros(1, 4, dtype=torch.int32)[:, ::2], i32(4))


def test_wait_policy_validation_without_gpu():
    lib = L.lib()
    assert lib.lstk_cuda_set_wait_policy(0, ctypes.c_void_p(0x10002)) == _lib.LSTK_ERR_INVALID_ARG
    assert "aligned" in _lib.last_error()
    assert lib.lstk_cuda_set_wait_policy(1000, ctypes.c_void_p(0x10000)) == _lib.LSTK_OK
    assert lib.lstk_cuda_set_wait_policy(0, None) == _lib.LSTK_OK  # back to the default: 4 s, no gate
