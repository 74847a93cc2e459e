"""A minimal GGUF (llama.cpp model file, version 3) writer for tests, written from the published
format: magic, version, tensor and metadata counts; typed metadata; the tensor index (name,
dimensions innermost first, ggml type, offset); tensor data aligned to 32 bytes. Also the Q8_0
block format (32 values: an f16 scale, then 32 int8) and bf16 rounding, with their f32 values."""
import struct

import numpy as np

F32, F16, Q8_0, BF16 = 0, 1, 8, 30
_U32, _I32, _F32, _STRING, _U64 = 4, 5, 6, 8, 10


def _str(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def quantize_q8_0(x):
    """x f32 [..., n] (n % 32 == 0) -> (bytes of the blocks, the f32 values they decode to)."""
    blocks = x.astype(np.float32).reshape(-1, 32)
    amax = np.max(np.abs(blocks), axis=1)
    d = amax / 127.0
    inv = np.where(d > 0, 1.0 / np.where(d > 0, d, 1), 0.0)
    q = np.clip(np.round(blocks * inv[:, None]), -127, 127).astype(np.int8)
    d16 = d.astype(np.float16)
    raw = np.zeros((blocks.shape[0], 34), np.uint8)
    raw[:, :2] = d16.view(np.uint8).reshape(-1, 2)
    raw[:, 2:] = q.view(np.uint8)
    return raw.tobytes(), (q.astype(np.float32) * d16.astype(np.float32)[:, None]).reshape(x.shape)


def to_bf16(x):
    """x f32 -> (bf16 bytes, round to nearest even, the f32 values they hold)."""
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return r.tobytes(), (r.astype(np.uint32) << 16).view(np.float32).reshape(x.shape)


def encode(x, ggml_type):
    """(bytes, f32 values as stored) of array x in ggml_type."""
    if ggml_type == F32:
        v = np.ascontiguousarray(x, np.float32)
        return v.tobytes(), v
    if ggml_type == F16:
        v = x.astype(np.float16)
        return v.tobytes(), v.astype(np.float32)
    if ggml_type == BF16:
        return to_bf16(x)
    if ggml_type == Q8_0:
        return quantize_q8_0(x)
    raise ValueError(ggml_type)


def write(path, metadata, tensors, version=3, magic=b"GGUF"):
    """metadata: {key: int | float | str}; tensors: [(name, ne (innermost first), ggml_type,
    raw bytes)]."""
    out = bytearray(magic + struct.pack("<IQQ", version, len(tensors), len(metadata)))
    for k, v in metadata.items():
        out += _str(k)
        if isinstance(v, str):
            out += struct.pack("<I", _STRING) + _str(v)
        elif isinstance(v, float):
            out += struct.pack("<If", _F32, v)
        else:
            out += struct.pack("<II", _U32, v)
    offsets, at = [], 0
    for _, _, _, raw in tensors:
        offsets.append(at)
        at += (len(raw) + 31) // 32 * 32
    for (name, ne, ty, _), off in zip(tensors, offsets):
        out += _str(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", n) for n in ne)
        out += struct.pack("<IQ", ty, off)
    out += b"\0" * ((32 - len(out) % 32) % 32)
    for (_, _, _, raw), off in zip(tensors, offsets):
        out += raw + b"\0" * ((len(raw) + 31) // 32 * 32 - len(raw))
    with open(path, "wb") as f:
        f.write(bytes(out))
