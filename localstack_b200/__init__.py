"""localstack_b200 - B200 (sm_100a) backend for the Qwen3 attention node of ludehsar/localstack.

The product is liblstk_attn.so (CUDA kernels + the C ABI in include/lstk_cuda_attn.h).
This package loads it and exposes thin Python bindings over torch device tensors.
"""
from ._lib import LstkError, build, lib  # noqa: F401
from .attn import (  # noqa: F401
    DecodeWorkspace,
    alloc_cache,
    attn_decode,
    attn_merge,
    attn_prefill,
    check_status,
    kv_append,
    layout_of,
    rope_table,
    rope_table_host,
)
from .pages import DevicePages  # noqa: F401,E402
from .proj import proj, rms_norm, to_bf16  # noqa: F401,E402
from .q8 import Q8Cache, alloc_cache_q8, attn_decode_q8, attn_prefill_q8, kv_append_q8  # noqa: F401,E402
