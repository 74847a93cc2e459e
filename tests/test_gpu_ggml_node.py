"""The reference's own model graph on this backend.

localstack_b200/ggml_node builds libggml_node.so from the reference's src/qwen3.cpp and
src/kv_cache.cpp, compiled unchanged against the front end's ggml declarations: the reference's
qwen3_build_graph records the model (attn_block's rms_norm / rope_ext / set_rows /
flash_attn_ext nodes included), its KvCache hands out the cells and builds the mask, and the
graph runs on the GPU with the attention node on this library's C ABI. The logits of a prompt
chunk followed by decode steps are compared with a numpy restatement of the same dense Qwen3
forward pass (f16 K/V cache, exact softmax). The library is built where the reference sources
exist; elsewhere the test is skipped.
"""
import ctypes
import math
import os

import numpy as np
import pytest

from localstack_b200 import _lib

pytestmark = pytest.mark.gpu
LIB = os.path.join(_lib.ROOT, "localstack_b200", "ggml_node", "_build", "libggml_node.so")
D = 128


def _rms(x, eps):
    x64 = x.astype(np.float64)
    return (x64 / np.sqrt(np.mean(x64 * x64, axis=-1, keepdims=True) + eps)).astype(np.float32)


def _rope(x, pos, base):
    # NEOX: pairs (i, i + 64), theta_i = pos * base^(-2i/128)
    half = D // 2
    inv = base ** (-2.0 * np.arange(half) / D)
    ang = pos[:, None].astype(np.float64) * inv[None, :]
    c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    a, b = x[..., :half].astype(np.float64), x[..., half:].astype(np.float64)
    return np.concatenate([a * c - b * s, a * s + b * c], -1).astype(np.float32)


class RefModel:
    """The dense Qwen3 forward pass of src/qwen3.cpp:128-259 in numpy (f32, f16 KV cache)."""

    def __init__(self, W, n_layer, n_head, n_head_kv, base, eps):
        self.W, self.L, self.hq, self.hkv, self.base, self.eps = W, n_layer, n_head, n_head_kv, base, eps
        self.k = [np.zeros((0, n_head_kv, D), np.float16) for _ in range(n_layer)]
        self.v = [np.zeros((0, n_head_kv, D), np.float16) for _ in range(n_layer)]

    def step(self, tokens):
        W, T = self.W, len(tokens)
        pos = np.arange(self.k[0].shape[0], self.k[0].shape[0] + T)
        x = W["tok_embd"][tokens]
        for l in range(self.L):
            P = W["layers"][l]
            h = _rms(x, self.eps) * P["attn_norm"]
            q = (h @ P["wq"].T).reshape(T, self.hq, D)
            k = (h @ P["wk"].T).reshape(T, self.hkv, D)
            v = (h @ P["wv"].T).reshape(T, self.hkv, D)
            q = _rope(_rms(q, self.eps) * P["q_norm"], pos, self.base)
            k = _rope(_rms(k, self.eps) * P["k_norm"], pos, self.base)
            self.k[l] = np.concatenate([self.k[l], k.astype(np.float16)])
            self.v[l] = np.concatenate([self.v[l], v.astype(np.float16)])
            K, V = self.k[l].astype(np.float64), self.v[l].astype(np.float64)
            G = self.hq // self.hkv
            o = np.zeros((T, self.hq, D))
            for t in range(T):
                n = pos[t] + 1
                for hh in range(self.hq):
                    s = K[:n, hh // G] @ q[t, hh].astype(np.float64) / math.sqrt(D)
                    p = np.exp(s - s.max())
                    o[t, hh] = (p / p.sum()) @ V[:n, hh // G]
            x = (o.reshape(T, -1).astype(np.float32) @ P["wo"].T) + x
            if l == self.L - 1:
                x = x[-1:]
            hn = _rms(x, self.eps) * P["ffn_norm"]
            g, u = hn @ P["ffn_gate"].T, hn @ P["ffn_up"].T
            x = ((g / (1 + np.exp(-g))) * u) @ P["ffn_down"].T + x
        x = _rms(x, self.eps) * W["output_norm"]
        return (x @ W["output"].T)[0]


def _weights(rng, n_layer, n_embd, n_ff, hq, hkv, n_vocab):
    r = lambda *s, sd=0.05: (rng.standard_normal(s) * sd).astype(np.float32)
    norm = lambda n: (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    W = {"tok_embd": r(n_vocab, n_embd, sd=1.0), "output_norm": norm(n_embd), "output": r(n_vocab, n_embd),
         "layers": []}
    for _ in range(n_layer):
        W["layers"].append({"attn_norm": norm(n_embd), "wq": r(hq * D, n_embd), "wk": r(hkv * D, n_embd),
                            "wv": r(hkv * D, n_embd), "wo": r(n_embd, hq * D), "q_norm": norm(D),
                            "k_norm": norm(D), "ffn_norm": norm(n_embd), "ffn_gate": r(n_ff, n_embd),
                            "ffn_up": r(n_ff, n_embd), "ffn_down": r(n_embd, n_ff)})
    order = [W["tok_embd"], W["output_norm"], W["output"]]
    for P in W["layers"]:
        order += [P[k] for k in ("attn_norm", "wq", "wk", "wv", "wo", "q_norm", "k_norm", "ffn_norm", "ffn_gate",
                                 "ffn_up", "ffn_down")]
    return W, [np.ascontiguousarray(a) for a in order]


@pytest.mark.skipif(not os.path.exists(LIB), reason="libggml_node.so not built (needs the reference sources)")
@pytest.mark.parametrize("hq,hkv,prompt", [(4, 2, 40), (8, 1, 130)])
def test_reference_graph_runs_on_the_backend(hq, hkv, prompt):
    _lib.lib()  # liblstk_attn.so first, so the front end finds it
    lib = ctypes.CDLL(LIB)
    lib.lstk_node_create.restype = ctypes.c_void_p
    lib.lstk_node_create.argtypes = [ctypes.c_int] * 7 + [ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                                          ctypes.POINTER(ctypes.c_void_p)]
    lib.lstk_node_step.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    lib.lstk_node_destroy.argtypes = [ctypes.c_void_p]
    lib.lstk_node_last_error.restype = ctypes.c_char_p
    rng = np.random.default_rng(hq * 10 + hkv)
    n_layer, n_embd, n_ff, n_vocab, kv_size = 2, 256, 512, 512, 1024
    base, eps = 1e6, 1e-6
    W, order = _weights(rng, n_layer, n_embd, n_ff, hq, hkv, n_vocab)
    ptrs = (ctypes.c_void_p * len(order))(*[a.ctypes.data for a in order])
    m = lib.lstk_node_create(n_layer, n_embd, n_ff, hq, hkv, n_vocab, kv_size, base, eps, 1, ptrs)
    assert m, lib.lstk_node_last_error().decode()
    ref = RefModel(W, n_layer, hq, hkv, base, eps)
    try:
        steps = [rng.integers(0, n_vocab, prompt)] + [rng.integers(0, n_vocab, 1) for _ in range(3)]
        for i, toks in enumerate(steps):
            toks = np.ascontiguousarray(toks, np.int32)
            logits = np.empty(n_vocab, np.float32)
            rc = lib.lstk_node_step(m, 7, toks.ctypes.data, len(toks), logits.ctypes.data)
            assert rc == 0, lib.lstk_node_last_error().decode()
            want = ref.step(toks)
            err = np.max(np.abs(logits - want))
            assert err <= 2e-2 * np.max(np.abs(want)) + 2e-3, (i, err, np.max(np.abs(want)))
            assert int(np.argmax(logits)) == int(np.argmax(want)), i
    finally:
        lib.lstk_node_destroy(m)


@pytest.mark.skipif(not os.path.exists(LIB), reason="libggml_node.so not built (needs the reference sources)")
def test_prefix_reuse_through_the_reference_cache():
    """The server's prefix reuse (src/server.cpp:212-219): prompt A, then the reference's own
    KvCache::truncate_seq to the prefix A shares with prompt B, then the rest of B. The logits must
    match a fresh model stepping all of B, and the numpy forward pass of B."""
    _lib.lib()
    lib = ctypes.CDLL(LIB)
    lib.lstk_node_create.restype = ctypes.c_void_p
    lib.lstk_node_create.argtypes = [ctypes.c_int] * 7 + [ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                                          ctypes.POINTER(ctypes.c_void_p)]
    lib.lstk_node_step.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    lib.lstk_node_truncate.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32]
    lib.lstk_node_destroy.argtypes = [ctypes.c_void_p]
    lib.lstk_node_last_error.restype = ctypes.c_char_p
    rng = np.random.default_rng(21)
    hq, hkv, n_layer, n_embd, n_ff, n_vocab, kv_size = 8, 2, 2, 256, 512, 512, 1024
    W, order = _weights(rng, n_layer, n_embd, n_ff, hq, hkv, n_vocab)
    ptrs = (ctypes.c_void_p * len(order))(*[a.ctypes.data for a in order])
    a_toks = rng.integers(0, n_vocab, 70).astype(np.int32)
    b_toks = np.concatenate([a_toks[:37], rng.integers(0, n_vocab, 30)]).astype(np.int32)  # shares 37 tokens
    reuse = lib.lstk_node_create(n_layer, n_embd, n_ff, hq, hkv, n_vocab, kv_size, 1e6, 1e-6, 1, ptrs)
    fresh = lib.lstk_node_create(n_layer, n_embd, n_ff, hq, hkv, n_vocab, kv_size, 1e6, 1e-6, 1, ptrs)
    assert reuse and fresh, lib.lstk_node_last_error().decode()
    try:
        logits = np.empty(n_vocab, np.float32)
        assert lib.lstk_node_step(reuse, 3, a_toks.ctypes.data, len(a_toks), logits.ctypes.data) == 0
        lib.lstk_node_truncate(reuse, 3, 37)
        rest = np.ascontiguousarray(b_toks[37:])
        got = np.empty(n_vocab, np.float32)
        assert lib.lstk_node_step(reuse, 3, rest.ctypes.data, len(rest), got.ctypes.data) == 0, \
            lib.lstk_node_last_error().decode()
        want = np.empty(n_vocab, np.float32)
        assert lib.lstk_node_step(fresh, 3, b_toks.ctypes.data, len(b_toks), want.ctypes.data) == 0
        ref = RefModel(W, n_layer, hq, hkv, 1e6, 1e-6).step(b_toks)
        scale = np.max(np.abs(ref))
        assert np.max(np.abs(got - want)) <= 1e-3 * scale + 1e-4, np.max(np.abs(got - want))
        assert np.max(np.abs(got - ref)) <= 2e-2 * scale + 2e-3
        assert int(np.argmax(got)) == int(np.argmax(ref))
        # then one more decode step on the reused sequence
        nxt = np.array([int(np.argmax(got))], np.int32)
        assert lib.lstk_node_step(reuse, 3, nxt.ctypes.data, 1, got.ctypes.data) == 0
        assert lib.lstk_node_step(fresh, 3, nxt.ctypes.data, 1, want.ctypes.data) == 0
        assert np.max(np.abs(got - want)) <= 1e-3 * scale + 1e-4
    finally:
        lib.lstk_node_destroy(reuse)
        lib.lstk_node_destroy(fresh)



def _gguf_model(tmp_path, rng, hq, hkv, n_layer, n_embd, n_ff, n_vocab, drop=None):
    """A dense Qwen3 written as a GGUF file with mixed tensor types; returns (path, the f32 weights
    the file holds, for the numpy model)."""
    import gguf_file as G
    W, _ = _weights(rng, n_layer, n_embd, n_ff, hq, hkv, n_vocab)
    meta = {"general.architecture": "qwen3", "general.alignment": 32, "qwen3.block_count": n_layer,
            "qwen3.embedding_length": n_embd, "qwen3.feed_forward_length": n_ff,
            "qwen3.attention.head_count": hq, "qwen3.attention.head_count_kv": hkv,
            "qwen3.attention.key_length": D, "qwen3.context_length": 4096,
            "qwen3.attention.layer_norm_rms_epsilon": 1e-6, "qwen3.rope.freq_base": 1e6}
    tensors, Wq = [], {"layers": []}

    def add(name, a, ty):
        raw, vals = G.encode(a, ty)
        if name != drop:
            tensors.append((name, list(a.shape[::-1]), ty, raw))
        return vals

    Wq["tok_embd"] = add("token_embd.weight", W["tok_embd"], G.F32)
    Wq["output_norm"] = add("output_norm.weight", W["output_norm"], G.F32)
    Wq["output"] = add("output.weight", W["output"], G.F16)
    types = {"wq": G.Q8_0, "wk": G.F16, "wv": G.BF16, "wo": G.Q8_0, "ffn_gate": G.F16, "ffn_up": G.BF16,
             "ffn_down": G.Q8_0}
    names = {"attn_norm": "attn_norm", "wq": "attn_q", "wk": "attn_k", "wv": "attn_v", "wo": "attn_output",
             "q_norm": "attn_q_norm", "k_norm": "attn_k_norm", "ffn_norm": "ffn_norm", "ffn_gate": "ffn_gate",
             "ffn_up": "ffn_up", "ffn_down": "ffn_down"}
    for l, P in enumerate(W["layers"]):
        Wq["layers"].append({k: add(f"blk.{l}.{names[k]}.weight", P[k], types.get(k, G.F32)) for k in names})
    path = str(tmp_path / "model.gguf")
    G.write(path, meta, tensors)
    return path, Wq


def _node_lib():
    _lib.lib()
    lib = ctypes.CDLL(LIB)
    lib.lstk_node_create_gguf.restype = ctypes.c_void_p
    lib.lstk_node_create_gguf.argtypes = [ctypes.c_char_p, ctypes.c_int]
    lib.lstk_node_step.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    lib.lstk_node_destroy.argtypes = [ctypes.c_void_p]
    lib.lstk_node_last_error.restype = ctypes.c_char_p
    return lib


@pytest.mark.skipif(not os.path.exists(LIB), reason="libggml_node.so not built (needs the reference sources)")
def test_gguf_model_file(tmp_path):
    """A GGUF file (F32 / F16 / BF16 / Q8_0 tensors) read by the front end's GGUF reader through
    the reference's own qwen3_load_hparams / qwen3_map_weights, then a prompt and decode steps:
    logits match the numpy model on the weights as the file stores them."""
    import sys
    sys.path.insert(0, os.path.dirname(__file__))
    rng = np.random.default_rng(31)
    hq, hkv, n_layer, n_embd, n_ff, n_vocab = 8, 2, 2, 256, 512, 512
    path, Wq = _gguf_model(tmp_path, rng, hq, hkv, n_layer, n_embd, n_ff, n_vocab)
    lib = _node_lib()
    m = lib.lstk_node_create_gguf(path.encode(), 1024)
    assert m, lib.lstk_node_last_error().decode()
    ref = RefModel(Wq, n_layer, hq, hkv, 1e6, 1e-6)
    try:
        for i, toks in enumerate([rng.integers(0, n_vocab, 50)] + [rng.integers(0, n_vocab, 1) for _ in range(2)]):
            toks = np.ascontiguousarray(toks, np.int32)
            logits = np.empty(n_vocab, np.float32)
            assert lib.lstk_node_step(m, 0, toks.ctypes.data, len(toks), logits.ctypes.data) == 0, \
                lib.lstk_node_last_error().decode()
            want = ref.step(toks)
            assert np.max(np.abs(logits - want)) <= 2e-2 * np.max(np.abs(want)) + 2e-3, i
            assert int(np.argmax(logits)) == int(np.argmax(want)), i
    finally:
        lib.lstk_node_destroy(m)
    # a file missing a required tensor: the reference's own error
    (tmp_path / "missing").mkdir()
    path2, _ = _gguf_model(tmp_path / "missing", np.random.default_rng(32), hq, hkv, n_layer, n_embd, n_ff,
                           n_vocab, drop="blk.1.ffn_down.weight")
    assert not lib.lstk_node_create_gguf(path2.encode(), 1024)
    assert "missing tensor blk.1.ffn_down.weight" in lib.lstk_node_last_error().decode()
