"""The KV-cache wire format of kv_manager.serialize_kv_cache /
deserialize_kv_cache (inference_benchmark/kv_manager.py:11-95), on the GPU.

The reference's KVCacheStore.store (kv_manager.py:116-127) moves every
layer's K and V to the host (`.cpu()`), joins the bytes behind an 18-byte
"<IIIIH" header (layers, kv_heads, seq_len, head_dim, dtype id 0 = FP16) and
puts that blob; load (kv_manager.py:135-156) copies the blob back and
rebuilds the tensors on the GPU.  Here the same bytes are built and split by
one kernel launch each, straight from and into device tensors, so a KV cache
goes from `past_key_values` to the HBM pool and back without a host copy:

    wire = kvwire.serialize_kv_cache(past_key_values)     # CUDA uint8
    store.put(prefix_hash, wire)                           # CascadeStore
    found, size = store.get(prefix_hash, buf)              # CUDA uint8 buf
    past_key_values = kvwire.deserialize_kv_cache(buf[:size])

The bytes are the reference's exactly, so blocks stored by the reference's
host path and by this one read back through either.  A store with
kv_compression quantises a blob whole, header included (the reference's
KVCompressor does the same), so a cache read back from INT8 storage is split
by a shape the caller knows (load_kv_caches, or `header=`).
"""
from __future__ import annotations

import ctypes
import struct
from typing import Sequence

from . import _lib
from ._lib import check

HEADER_FMT = "<IIIIH"              # kv_manager.py:11
HEADER_SIZE = struct.calcsize(HEADER_FMT)
FP16_ID = 0                        # DTYPE_MAP[torch.float16], kv_manager.py:14
ROW_ALIGN = 256                    # row pitch of batched wire buffers


class _KvTensor(ctypes.Structure):
    """cascade_kv_tensor_t."""
    _fields_ = [("ptr", ctypes.c_uint64), ("stride_head", ctypes.c_int64),
                ("stride_seq", ctypes.c_int64)]


_vp, _sz, _u32, _int = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_uint32, \
    ctypes.c_int
_lib.register("cascade_kv_wire_bytes", ctypes.c_uint64, [_u32, _u32, _u32,
                                                         _u32])
_lib.register("cascade_kv_serialize_batch", _int,
              [_vp, _int, _u32, _u32, _u32, _u32, _vp, _sz, _vp])
_lib.register("cascade_kv_deserialize_batch", _int,
              [_vp, _u32, _u32, _u32, _u32, _vp, _sz, _vp])
_lib.register("cascade_store_put_kv_batch", _int,
              [_vp, _sz, _vp, _u32, _u32, _u32, _u32, _vp, _int, _vp, _vp,
               _vp, ctypes.POINTER(ctypes.c_uint64)])
_lib.register("cascade_store_get_kv_batch", _int,
              [_vp, _sz, _vp, _u32, _u32, _u32, _u32, _vp, _vp, _vp,
               ctypes.POINTER(ctypes.c_uint64)])


def wire_bytes(layers: int, heads: int, seq: int, head_dim: int) -> int:
    """Bytes of one serialised cache: header + 2 x layers FP16 tensors."""
    return HEADER_SIZE + 4 * layers * heads * seq * head_dim


def extract_kv_pairs(past_key_values) -> list:
    """[(K, V) per layer], as kv_manager.extract_kv_pairs (kv_manager.py:
    22-34): a cache with key_cache/value_cache lists, or a sequence of
    (K, V) pairs; also a cache with .layers[i].keys / .values."""
    if hasattr(past_key_values, "key_cache"):
        return list(zip(past_key_values.key_cache,
                        past_key_values.value_cache))
    if hasattr(past_key_values, "layers") and not isinstance(
            past_key_values, (tuple, list)):
        return [(l.keys, l.values) for l in past_key_values.layers]
    out = []
    for layer in past_key_values:
        if isinstance(layer, (tuple, list)):
            out.append((layer[0], layer[1]))
        else:
            raise ValueError(f"Unexpected layer type: {type(layer)}")
    return out


def _dtype_code(dt):
    import torch
    codes = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}
    if dt not in codes:
        raise TypeError(f"KV tensors must be float16, bfloat16 or float32, "
                        f"not {dt}")
    return codes[dt]


def _heads_seq_dim(t):
    """(tensor as [heads, seq, dim], strides in elements) for a [1, heads,
    seq, dim] or [heads, seq, dim] tensor with contiguous head_dim."""
    if t.dim() == 4:
        if t.shape[0] != 1:
            raise ValueError("a KV tensor's batch dimension must be 1 "
                             f"(got shape {tuple(t.shape)})")
        t = t[0]
    if t.dim() != 3:
        raise ValueError(f"KV tensors are [1, heads, seq, dim]; got "
                         f"{tuple(t.shape)}")
    if t.shape[2] > 1 and t.stride(2) != 1:
        raise ValueError("head_dim must be contiguous (stride 1)")
    return t


def _geometry(pairs):
    if not pairs:
        raise ValueError("a KV cache needs at least one layer")
    k0 = _heads_seq_dim(pairs[0][0])
    heads, seq, dim = (int(x) for x in k0.shape)
    dev, dt = k0.device, k0.dtype
    if dev.type != "cuda":
        raise ValueError("serialize_kv_cache takes CUDA tensors")
    for k, v in pairs:
        for t in (k, v):
            t3 = _heads_seq_dim(t)
            if tuple(t3.shape) != (heads, seq, dim):
                raise ValueError("every layer's K and V must have the first "
                                 f"K's shape {(heads, seq, dim)}; got "
                                 f"{tuple(t3.shape)}")
            if t3.device != dev or t3.dtype != dt:
                raise ValueError("every K and V must share one device and "
                                 "dtype")
    return len(pairs), heads, seq, dim, dev, dt


def _descriptors(tensors, device):
    """cascade_kv_tensor_t rows for [heads, seq, dim] views, on `device`."""
    import numpy as np
    import torch
    rows = np.empty((len(tensors), 3), dtype=np.int64)
    for i, t in enumerate(tensors):
        rows[i, 0] = t.data_ptr()
        rows[i, 1] = t.stride(0)
        rows[i, 2] = t.stride(1)
    return torch.from_numpy(rows).to(device)


def _stream(device) -> int:
    import torch
    return torch.cuda.current_stream(device).cuda_stream


def serialize_kv_caches(caches: Sequence, out=None) -> list:
    """Serialises n KV caches of one shape in one launch.  Returns n CUDA
    uint8 tensors of wire_bytes() each: rows of one allocation whose pitch
    is rounded up to 256 bytes (or views of `out`, a 2-D CUDA uint8 tensor
    of n rows at least that long).  Each row equals
    kv_manager.serialize_kv_cache of that cache, byte for byte."""
    import torch
    n = len(caches)
    if n == 0:
        return []
    per = [extract_kv_pairs(c) for c in caches]
    geo = [_geometry(p) for p in per]
    L, H, S, D, dev, dt = geo[0]
    if any(g != geo[0] for g in geo):
        raise ValueError("serialize_kv_caches: every cache must have one "
                         "shape, dtype and device")
    nbytes = wire_bytes(L, H, S, D)
    if out is None:
        pitch = -(-nbytes // ROW_ALIGN) * ROW_ALIGN
        out = torch.empty((n, pitch), dtype=torch.uint8, device=dev)
    elif (out.dtype != torch.uint8 or out.dim() != 2 or out.shape[0] < n
          or out.shape[1] < nbytes or out.device != dev
          or out.stride(1) != 1):
        raise ValueError(f"out must be a CUDA uint8 [n, >= {nbytes}] tensor "
                         "with contiguous rows on the caches' device")
    views = [_heads_seq_dim(t) for p in per for kv in p for t in kv]
    src = _descriptors(views, dev)
    dst = torch.tensor([out[i].data_ptr() for i in range(n)],
                       dtype=torch.int64).to(dev)
    check(_lib.load().cascade_kv_serialize_batch(
        src.data_ptr(), _dtype_code(dt), L, H, S, D, dst.data_ptr(), n,
        _stream(dev)))
    # src and dst may be freed now: the caching allocator hands their memory
    # out again only to work ordered after this launch on the same stream.
    return [out[i, :nbytes] for i in range(n)]


def serialize_kv_cache(past_key_values, out=None):
    """kv_manager.serialize_kv_cache on the device: the wire bytes as a
    1-D CUDA uint8 tensor (16-byte aligned)."""
    if out is not None:
        out = out.view(1, -1)
    return serialize_kv_caches([past_key_values], out=out)[0]


def read_header(data) -> tuple:
    """(layers, heads, seq, head_dim, dtype id) of a wire block (host bytes,
    a numpy array or a CUDA tensor: 18 bytes come to the host)."""
    import numpy as np
    if hasattr(data, "is_cuda") and data.is_cuda:
        head = bytes(data[:HEADER_SIZE].cpu().numpy())
    else:
        head = bytes(np.asarray(data[:HEADER_SIZE], dtype=np.uint8))
    if len(head) < HEADER_SIZE:
        raise ValueError("a wire block is at least 18 bytes")
    return struct.unpack(HEADER_FMT, head)


def deserialize_kv_caches(blocks: Sequence, header=None) -> list:
    """Splits n wire blocks of one shape (CUDA uint8 tensors) into n tuples
    of per-layer (K, V) FP16 tensors [1, heads, seq, dim] on the blocks'
    device, in one launch: kv_manager.deserialize_kv_cache for each.  The
    shape comes from the first block's header, or from `header` (the
    5-tuple read_header returns) when the caller knows it; every block
    must be that long."""
    import torch
    n = len(blocks)
    if n == 0:
        return []
    L, H, S, D, dtype_id = header if header is not None else \
        read_header(blocks[0])
    if dtype_id != FP16_ID:
        raise ValueError(f"wire dtype id {dtype_id}: the reference writes "
                         "FP16 (id 0) only")
    nbytes = wire_bytes(L, H, S, D)
    dev = blocks[0].device
    for b in blocks:
        if (not b.is_cuda or b.dtype != torch.uint8 or b.dim() != 1
                or b.numel() < nbytes or b.device != dev
                or (b.numel() > 1 and b.stride(0) != 1)):
            raise ValueError(f"wire blocks must be contiguous CUDA uint8 "
                             f"tensors of at least {nbytes} bytes on one "
                             "device")
    outs = torch.empty((n, L, 2, 1, H, S, D), dtype=torch.float16,
                       device=dev)
    views = [outs[i, l, kv, 0] for i in range(n) for l in range(L)
             for kv in range(2)]
    dst = _descriptors(views, dev)
    src = torch.tensor([b.data_ptr() for b in blocks],
                       dtype=torch.int64).to(dev)
    check(_lib.load().cascade_kv_deserialize_batch(
        src.data_ptr(), L, H, S, D, dst.data_ptr(), n, _stream(dev)))
    return [tuple((outs[i, l, 0], outs[i, l, 1]) for l in range(L))
            for i in range(n)]


def deserialize_kv_cache(data, header=None) -> tuple:
    """kv_manager.deserialize_kv_cache on the device, for a CUDA uint8 wire
    block: a tuple of per-layer (K, V) FP16 tensors [1, heads, seq, dim]."""
    return deserialize_kv_caches([data], header=header)[0]


def _sources(caches):
    """(layers, heads, seq, head_dim, device, dtype, descriptor tensor) of a
    batch of caches of one shape."""
    per = [extract_kv_pairs(c) for c in caches]
    geo = [_geometry(p) for p in per]
    if any(g != geo[0] for g in geo):
        raise ValueError("every cache must have one shape, dtype and device")
    L, H, S, D, dev, dt = geo[0]
    views = [_heads_seq_dim(t) for p in per for kv in p for t in kv]
    return L, H, S, D, dev, dt, _descriptors(views, dev)


def store_kv_caches(store, block_ids: Sequence, caches: Sequence,
                    is_prefix=None):
    """KVCacheStore.store (kv_manager.py:116-127) for a batch, without host
    copies.  ``store``: a CascadeStore.  When every wire block fits the HBM
    pool as a raw payload, one store call (cascade_store_put_kv_batch)
    serialises each cache straight into its pool slot; otherwise the caches
    are serialised in one launch and put with put_batch.  Returns the
    per-block put status codes."""
    import numpy as np
    if len(block_ids) != len(caches):
        raise ValueError("one id per cache")
    n = len(caches)
    if n == 0:
        return []
    L, H, S, D, dev, dt, src = _sources(caches)
    keys = np.frombuffer(b"".join(store._key(b) for b in block_ids),
                         dtype=np.uint8).copy()
    pf = (np.array([1 if p else 0 for p in is_prefix], dtype=np.uint8)
          if is_prefix is not None else None)
    status = np.zeros(n, np.uint8)
    nst = ctypes.c_uint64(0)
    rc = _lib.load().cascade_store_put_kv_batch(
        store._h, n, keys.ctypes.data, L, H, S, D, src.data_ptr(),
        _dtype_code(dt), pf.ctypes.data if pf is not None else None,
        status.ctypes.data, _stream(dev), ctypes.byref(nst))
    if rc != _lib.CASCADE_ERR_UNSUPPORTED:
        check(rc)
        return status
    rows = serialize_kv_caches(caches)
    return store.put_batch(rows, keys=list(block_ids), is_prefix=is_prefix,
                           return_status=True)[1]


def load_kv_caches(store, block_ids: Sequence, layers: int, heads: int,
                   seq: int, head_dim: int) -> list:
    """KVCacheStore.load (kv_manager.py:135-156) for a batch of caches of a
    known shape, without host copies, in one store call
    (cascade_store_get_kv_batch): raw blocks in HBM are split straight out
    of the pool into fresh per-layer tensors.  Returns, per id, the tuple of
    (K, V) FP16 tensors [1, heads, seq, dim] per layer, or None when the
    store does not hold that id with the wire size of that shape."""
    import numpy as np
    import torch
    n = len(block_ids)
    if n == 0:
        return []
    dev = torch.device(f"cuda:{store._device}")
    L, H, S, D = layers, heads, seq, head_dim
    outs = torch.empty((n, L, 2, 1, H, S, D), dtype=torch.float16,
                       device=dev)
    views = [outs[i, l, kv, 0] for i in range(n) for l in range(L)
             for kv in range(2)]
    dst = _descriptors(views, dev)
    keys = np.frombuffer(b"".join(store._key(b) for b in block_ids),
                         dtype=np.uint8).copy()
    found = np.zeros(n, np.uint8)
    nf = ctypes.c_uint64(0)
    check(_lib.load().cascade_store_get_kv_batch(
        store._h, n, keys.ctypes.data, L, H, S, D, dst.data_ptr(),
        found.ctypes.data, _stream(dev), ctypes.byref(nf)))
    return [tuple((outs[i, l, 0], outs[i, l, 1]) for l in range(L))
            if found[i] else None for i in range(n)]
