"""GGUF files the front end must refuse before touching a GPU: a wrong magic and a tensor type
the loader does not convert (runs on the CPU; skipped where the front end is not built)."""
import ctypes
import os
import struct
import sys

import numpy as np
import pytest

from localstack_b200 import _lib

sys.path.insert(0, os.path.dirname(__file__))
import gguf_file as G  # noqa: E402

LIB = os.path.join(_lib.ROOT, "localstack_b200", "ggml_node", "_build", "libggml_node.so")
pytestmark = pytest.mark.skipif(not os.path.exists(LIB) or not os.path.exists(_lib.LIB_PATH),
                                reason="front end not built")


def _lib_node():
    _lib.lib()
    lib = ctypes.CDLL(LIB)
    lib.lstk_node_create_gguf.restype = ctypes.c_void_p
    lib.lstk_node_create_gguf.argtypes = [ctypes.c_char_p, ctypes.c_int]
    lib.lstk_node_last_error.restype = ctypes.c_char_p
    return lib


def test_refuses_non_gguf_and_unsupported_types(tmp_path):
    lib = _lib_node()
    bad = tmp_path / "bad.gguf"
    G.write(str(bad), {"general.architecture": "qwen3"}, [], magic=b"GGUX")
    assert not lib.lstk_node_create_gguf(str(bad).encode(), 64)
    assert "not a GGUF" in lib.lstk_node_last_error().decode()
    assert not lib.lstk_node_create_gguf(str(tmp_path / "absent.gguf").encode(), 64)
    assert "cannot open" in lib.lstk_node_last_error().decode()
    # a Q4_K (ggml type 12) tensor: refused with its type id, before any device allocation
    q4k = tmp_path / "q4k.gguf"
    G.write(str(q4k), {"general.architecture": "qwen3", "qwen3.block_count": 1},
            [("token_embd.weight", [256, 4], 12, bytes(144 * 4))])
    assert not lib.lstk_node_create_gguf(str(q4k).encode(), 64)
    assert "ggml type 12" in lib.lstk_node_last_error().decode()
    # truncated metadata
    trunc = tmp_path / "trunc.gguf"
    trunc.write_bytes(b"GGUF" + struct.pack("<IQQ", 3, 0, 5) + b"\x01")
    assert not lib.lstk_node_create_gguf(str(trunc).encode(), 64)
    assert "malformed" in lib.lstk_node_last_error().decode()


def test_q8_0_and_bf16_encodings_round_trip():
    x = np.random.default_rng(0).standard_normal((8, 64)).astype(np.float32)
    raw, vals = G.quantize_q8_0(x)
    assert len(raw) == 8 * 2 * 34 and np.max(np.abs(vals - x)) <= np.max(np.abs(x)) / 127
    raw, vals = G.to_bf16(x)
    assert len(raw) == x.size * 2 and np.max(np.abs(vals - x) / np.abs(x)) <= 2 ** -8
