"""ORACLE — test infrastructure only.

A numpy restatement of the KV-cache wire format of
inference_benchmark/kv_manager.py:

* serialize_kv_cache (lines 43-63): struct.pack("<IIIIH", num_layers,
  num_kv_heads, seq_len, head_dim, 0) followed by, per layer, K then V as
  contiguous [kv_heads][seq_len][head_dim] float16 bytes.  Tensors of other
  dtypes are converted to float16 first (.to(torch.float16), which rounds to
  nearest even; numpy's float32 -> float16 cast rounds the same way).
* deserialize_kv_cache (lines 66-95): the inverse for dtype id 0.

Only tests/ import this module; the product never does.
"""
from __future__ import annotations

import struct

import numpy as np

HEADER_FMT = "<IIIIH"
HEADER_SIZE = struct.calcsize(HEADER_FMT)


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """bfloat16 bit patterns (uint16) as float32 values (exact)."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def serialize(pairs) -> bytes:
    """pairs: [(K, V)] per layer, numpy arrays [heads, seq, dim] of float16
    or float32 (bfloat16 callers pass bf16_to_f32 of the bits)."""
    heads, seq, dim = pairs[0][0].shape
    out = [struct.pack(HEADER_FMT, len(pairs), heads, seq, dim, 0)]
    with np.errstate(over="ignore"):        # overflow to inf is the rule
        for k, v in pairs:
            for t in (k, v):
                out.append(np.ascontiguousarray(t).astype(np.float16).tobytes())
    return b"".join(out)


def deserialize(data: bytes):
    """[(K, V)] per layer as float16 arrays [heads, seq, dim]."""
    layers, heads, seq, dim, dtype_id = struct.unpack(
        HEADER_FMT, bytes(data[:HEADER_SIZE]))
    assert dtype_id == 0, dtype_id
    per = heads * seq * dim
    vals = np.frombuffer(bytes(data[HEADER_SIZE:HEADER_SIZE + 4 * layers * per]),
                         dtype=np.float16)
    return [(vals[(2 * l) * per:(2 * l + 1) * per].reshape(heads, seq, dim),
             vals[(2 * l + 1) * per:(2 * l + 2) * per].reshape(heads, seq, dim))
            for l in range(layers)]
