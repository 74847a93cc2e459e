"""The BASELINE configurations at their full sizes, end to end, against the CPU oracle.

* Config 1: 513 keys, Hq 16 / Hkv 8.
* Config 2 as one chain: bf16 N(0,1) Q/K/V -> lstk_cuda_kv_append (QK-RMSNorm, NEOX RoPE 1e6, f16
  pages at seeded random page ids; pages and Q bit-exact against the oracle's append) ->
  lstk_cuda_attn_prefill over the pages the append wrote (causal, 2048 tokens, Hq 16 / Hkv 8).
* Config 3 with all 64 sequences (ctx U[1024, 32768], Hq 32 / Hkv 4, one global page permutation).
* Config 4: one 131072-token context (4096 pages at random places).

Gate (the tolerance of the north star, on f32 outputs): |gpu - exact| <= 2e-3 + 1e-2 |exact|,
where exact is the oracle with f32 accumulation - the precision the reference's call site asks
for (GGML_PREC_F32, src/qwen3.cpp:165-167). Against the oracle's model of ggml's CPU kernel (Q
rounded to f16 for the dot, an f16 V accumulator) the GPU must be no further than the exact answer
itself is, plus the same tolerance: that model already sits up to ~2.6e-3 from the exact result
at these sizes, so a plain 2e-3 band around it cannot be met by any f32-accumulating kernel.
"""
import numpy as np
import pytest

from tests import config_cases as C
from tests.helpers import max_err, within

pytestmark = pytest.mark.gpu


def _check_both_modes(out, ex, gg):
    assert within(out, ex), f"max |gpu - exact| = {max_err(out, ex)}"
    gap = np.abs(ex.astype(np.float64) - gg)
    assert np.all(np.abs(out.astype(np.float64) - gg) <= gap + 2e-3 + 1e-2 * np.abs(gg)), max_err(out, gg)


def test_config1_513_keys():
    _check_both_modes(*C.config1())


def test_config2_chain_bf16_append_then_prefill():
    _check_both_modes(*C.config2_chain())


def test_config3_full_batch_64_sequences():
    _check_both_modes(*C.config3())


def test_config4_131072_keys():
    out, ex, gg, lse, lse_ex = C.config4(want_lse=True)
    _check_both_modes(out, ex, gg)
    assert np.allclose(lse, lse_ex, atol=1e-3, rtol=1e-4)
