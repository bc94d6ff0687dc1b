"""Drop-in replacement for the reference's pybind11 module ``cascade_cpp``
(cascade_code/cpp/python/bindings.cpp:9-244), backed by the B200 C ABI.

Same names, arguments, defaults and return values as the reference:
``CascadeConfig``, ``CascadeStats``, ``CascadeStore.put/get/contains/
get_stats/clear/flush``, ``compute_block_id``, ``GPUBackend``,
``ShmBackend``, ``LustreBackend`` and ``AggregatedLustreBackend``.  Every
block operation runs on the GPU through libcascade_b200.so; there is no CPU
path, and a machine without a CUDA device gets a CascadeError from the
store's constructor.

Additive extensions (absent from the reference module, so no caller depends
on them): torch CUDA tensors are accepted wherever a numpy buffer is, and
``CascadeStore.put_batch / put_batch_host / get_batch`` and
``compute_block_ids`` process many blocks per call.
"""
from __future__ import annotations

import ctypes
from typing import Iterable, Optional, Sequence

import numpy as np

from . import _lib
from ._lib import CascadeError, check

_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_u64 = ctypes.c_uint64
_int = ctypes.c_int
_u8p = ctypes.POINTER(ctypes.c_uint8)


class _CConfig(ctypes.Structure):
    """Layout of cascade_config_t (include/cascade_b200.h)."""
    _fields_ = [
        ("gpu_capacity_bytes", ctypes.c_uint64),
        ("gpu_device_id", ctypes.c_int32),
        ("use_gpu", ctypes.c_int32),
        ("shm_capacity_bytes", ctypes.c_uint64),
        ("shm_path", ctypes.c_char_p),
        ("lustre_path", ctypes.c_char_p),
        ("lustre_stripe_size", ctypes.c_uint64),
        ("lustre_stripe_count", ctypes.c_int32),
        ("dedup_enabled", ctypes.c_int32),
        ("compression_enabled", ctypes.c_int32),
        ("num_io_threads", ctypes.c_int32),
        ("semantic_eviction", ctypes.c_int32),
        ("promotion_enabled", ctypes.c_int32),
        ("prefetch_enabled", ctypes.c_int32),
        ("prefetch_threads", ctypes.c_int32),
        ("prefetch_queue_size", ctypes.c_uint64),
        ("kv_compression", ctypes.c_int32),
        ("aggregated_lustre", ctypes.c_int32),
        ("agg_file_size", ctypes.c_uint64),
        ("gpu_q8", ctypes.c_int32),
        ("reserved0", ctypes.c_int32),
        ("index_slots", ctypes.c_uint64),
        ("dram_chunk_bytes", ctypes.c_uint64),
    ]


_STAT_FIELDS = ("gpu_used", "shm_used", "gpu_hits", "shm_hits", "lustre_hits",
                "misses", "dedup_hits", "gpu_evictions", "shm_evictions",
                "promotions_to_gpu", "promotions_to_shm", "prefetch_completed",
                "compression_savings_bytes", "shm_puts", "lustre_puts")


class _CStats(ctypes.Structure):
    _fields_ = [(f, ctypes.c_uint64) for f in _STAT_FIELDS]


_lib.register("cascade_config_init", None, [ctypes.POINTER(_CConfig)])
_lib.register("cascade_struct_sizes", None, [ctypes.POINTER(_sz),
                                             ctypes.POINTER(_sz)])
_lib.register("cascade_store_create", _int, [ctypes.POINTER(_CConfig),
                                             ctypes.POINTER(_vp)])
_lib.register("cascade_store_destroy", _int, [_vp])
_lib.register("cascade_store_put", _int, [_vp, ctypes.c_char_p, _vp, _u64,
                                          _int, ctypes.POINTER(_int)])
_lib.register("cascade_store_get", _int, [_vp, ctypes.c_char_p, _vp, _u64,
                                          ctypes.POINTER(_int),
                                          ctypes.POINTER(_u64)])
_lib.register("cascade_store_contains", _int, [_vp, ctypes.c_char_p,
                                               ctypes.POINTER(_int)])
_lib.register("cascade_store_get_stats", _int, [_vp, ctypes.POINTER(_CStats)])
_lib.register("cascade_store_clear", _int, [_vp])
_lib.register("cascade_store_flush", _int, [_vp])
_lib.register("cascade_store_key_of", _int, [_vp, ctypes.c_char_p, _vp])
_lib.register("cascade_store_put_batch", _int,
              [_vp, _sz, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
               ctypes.POINTER(_u64)])
_lib.register("cascade_store_put_batch_host", _int,
              [_vp, _sz, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.POINTER(_u64)])
_lib.register("cascade_store_get_batch", _int,
              [_vp, _sz, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.POINTER(_u64)])


# ------------------------------------------------------------------ config
class CascadeConfig:
    """cascade::CascadeConfig (cascade.hpp:25-60) with its defaults.

    The 18 fields bound at bindings.cpp:15-35, plus ``num_io_threads`` and
    three B200 extensions: ``gpu_q8`` (HBM holds the INT8 form when
    ``kv_compression`` is on), ``index_slots`` and ``dram_chunk_bytes``.
    """

    _INT_FIELDS = ("gpu_capacity_bytes", "gpu_device_id", "shm_capacity_bytes",
                   "lustre_stripe_size", "lustre_stripe_count",
                   "num_io_threads", "prefetch_threads", "prefetch_queue_size",
                   "agg_file_size", "index_slots", "dram_chunk_bytes")
    _BOOL_FIELDS = ("use_gpu", "dedup_enabled", "compression_enabled",
                    "semantic_eviction", "promotion_enabled",
                    "prefetch_enabled", "kv_compression", "aggregated_lustre",
                    "gpu_q8")
    _STR_FIELDS = ("shm_path", "lustre_path")

    def __init__(self):
        c = _CConfig()
        _lib.load().cascade_config_init(ctypes.byref(c))
        for f in self._INT_FIELDS:
            object.__setattr__(self, f, int(getattr(c, f)))
        for f in self._BOOL_FIELDS:
            object.__setattr__(self, f, bool(getattr(c, f)))
        for f in self._STR_FIELDS:
            object.__setattr__(self, f, getattr(c, f).decode())

    def __setattr__(self, name, value):
        if name in self._INT_FIELDS:
            value = int(value)
            if value < 0:
                raise TypeError(f"{name} must be non-negative")
        elif name in self._BOOL_FIELDS:
            value = bool(value)
        elif name in self._STR_FIELDS:
            value = str(value)
        else:
            raise AttributeError(f"CascadeConfig has no field {name!r}")
        object.__setattr__(self, name, value)

    def _to_c(self):
        """(cascade_config_t, encoded strings the struct points into)."""
        c = _CConfig()
        _lib.load().cascade_config_init(ctypes.byref(c))
        for f in self._INT_FIELDS + self._BOOL_FIELDS:
            setattr(c, f, int(getattr(self, f)))
        keep = (self.shm_path.encode(), self.lustre_path.encode())
        c.shm_path, c.lustre_path = keep
        return c, keep


class CascadeStats:
    """CascadeStore::Stats (cascade.hpp:439-456), read-only, with the
    reference's __repr__ (bindings.cpp:57-66)."""

    __slots__ = _STAT_FIELDS

    def __init__(self, c: _CStats):
        for f in _STAT_FIELDS:
            object.__setattr__(self, f, int(getattr(c, f)))

    def __setattr__(self, name, value):
        raise AttributeError("CascadeStats is read-only")

    def __repr__(self):
        mb = 1024 * 1024
        return ("CascadeStats(gpu=" + str(self.gpu_used // mb) + "MB"
                ", shm=" + str(self.shm_used // mb) + "MB"
                ", hits=" + str(self.gpu_hits + self.shm_hits + self.lustre_hits)
                + ", dedup=" + str(self.dedup_hits)
                + ", evictions=" + str(self.gpu_evictions + self.shm_evictions)
                + ", promotions=" + str(self.promotions_to_gpu
                                        + self.promotions_to_shm)
                + ", prefetch=" + str(self.prefetch_completed)
                + ", compression_saved="
                + str(self.compression_savings_bytes // mb) + "MB)")


# --------------------------------------------------------------- buffers
def _is_cuda_tensor(x) -> bool:
    return type(x).__module__.startswith("torch") and getattr(x, "is_cuda", False)


def _host_u8(data) -> np.ndarray:
    """A contiguous uint8 view of host data, cast the way pybind11's
    py::array_t<uint8_t> (forcecast) converts its argument."""
    if isinstance(data, (bytes, bytearray, memoryview)):
        return np.frombuffer(data, dtype=np.uint8)
    if type(data).__module__.startswith("torch"):
        data = data.numpy()
    return np.ascontiguousarray(np.asarray(data, dtype=np.uint8))


def _cuda_u8(t):
    """The bytes of a contiguous CUDA tensor as a flat uint8 view."""
    import torch
    if not t.is_contiguous():
        raise ValueError("CUDA tensors must be contiguous")
    return t.reshape(-1).view(torch.uint8)


def _torch_stream_of(t) -> int:
    import torch
    return torch.cuda.current_stream(t.device).cuda_stream


# ------------------------------------------------------------------ store
class CascadeStore:
    """cascade::CascadeStore (cascade.hpp:420-502) on a B200."""

    def __init__(self, config: CascadeConfig):
        if not isinstance(config, CascadeConfig):
            raise TypeError("CascadeStore(config: CascadeConfig)")
        self._cfg, self._cfg_strings = config._to_c()
        h = _vp()
        check(_lib.load().cascade_store_create(ctypes.byref(self._cfg),
                                               ctypes.byref(h)))
        self._h = h
        self._device = config.gpu_device_id

    # bindings.cpp:73-76
    def put(self, block_id: str, data, is_prefix: bool = False) -> bool:
        if _is_cuda_tensor(data):
            key = self._key(block_id)
            t = _cuda_u8(data)
            st = self.put_batch([t], keys=[key], is_prefix=[bool(is_prefix)],
                                return_status=True)[1]
            return int(st[0]) != _lib.PUT_FAILED
        arr = _host_u8(data)
        stored = _int(0)
        check(_lib.load().cascade_store_put(self._h, block_id.encode(),
                                            arr.ctypes.data, arr.size,
                                            int(bool(is_prefix)),
                                            ctypes.byref(stored)))
        return bool(stored.value)

    # bindings.cpp:77-82
    def get(self, block_id: str, out_data):
        if _is_cuda_tensor(out_data):
            t = _cuda_u8(out_data)
            key = self._key(block_id)
            found, sizes = self.get_batch([key], [t])
            return bool(found[0]), int(sizes[0])
        if not (isinstance(out_data, np.ndarray) and out_data.dtype == np.uint8
                and out_data.flags.c_contiguous and out_data.flags.writeable):
            raise TypeError("out_data must be a writable C-contiguous "
                            "numpy uint8 array")
        found = _int(0)
        size = _u64(0)
        check(_lib.load().cascade_store_get(self._h, block_id.encode(),
                                            out_data.ctypes.data,
                                            out_data.size, ctypes.byref(found),
                                            ctypes.byref(size)))
        return bool(found.value), int(size.value)

    def contains(self, block_id: str) -> bool:
        present = _int(0)
        check(_lib.load().cascade_store_contains(self._h, block_id.encode(),
                                                 ctypes.byref(present)))
        return bool(present.value)

    def get_stats(self) -> CascadeStats:
        c = _CStats()
        check(_lib.load().cascade_store_get_stats(self._h, ctypes.byref(c)))
        return CascadeStats(c)

    def clear(self) -> None:
        check(_lib.load().cascade_store_clear(self._h))

    def flush(self) -> None:
        check(_lib.load().cascade_store_flush(self._h))

    # -------------------------------------------------- batched extensions
    def _key(self, block_id) -> bytes:
        if isinstance(block_id, (bytes, bytearray)) and len(block_id) == 16:
            return bytes(block_id)
        buf = (ctypes.c_uint8 * 16)()
        check(_lib.load().cascade_store_key_of(self._h, str(block_id).encode(),
                                               buf))
        return bytes(buf)

    def key_of(self, block_id: str) -> bytes:
        """The 16-byte key the store uses for ``block_id``."""
        return self._key(block_id)

    def put_batch(self, blocks, keys=None, is_prefix=None,
                  return_status: bool = False):
        """Stores device-resident blocks in one call.

        ``blocks``: a list of CUDA uint8 tensors, or one 2-D CUDA tensor
        whose rows are blocks.  ``keys``: block ids (str) or 16-byte keys;
        None content-addresses every block (id = compute_block_id).
        Returns the number of blocks stored or deduplicated; with
        ``return_status`` also the per-block status codes and, when
        content-addressed, the 32-byte digests.
        """
        import torch
        if isinstance(blocks, torch.Tensor) and blocks.dim() == 2:
            rows = blocks.contiguous()
            n = rows.shape[0]
            base, stride = rows.data_ptr(), rows.stride(0) * rows.element_size()
            ptrs = np.arange(n, dtype=np.uint64) * np.uint64(stride) + np.uint64(base)
            sizes = np.full(n, rows.shape[1] * rows.element_size(), np.uint64)
            keepalive = rows
            stream = _torch_stream_of(rows)
        else:
            blocks = [_cuda_u8(b) for b in blocks]
            n = len(blocks)
            ptrs = np.array([b.data_ptr() for b in blocks], dtype=np.uint64)
            sizes = np.array([b.numel() for b in blocks], dtype=np.uint64)
            keepalive = blocks
            stream = _torch_stream_of(blocks[0]) if n else 0
        return self._put_batch_raw(n, ptrs, sizes, keys, is_prefix,
                                   return_status, stream, keepalive)

    def _put_batch_raw(self, n, ptrs, sizes, keys, is_prefix, return_status,
                       stream, keepalive=None):
        kbuf = None
        if keys is not None:
            kbuf = np.frombuffer(b"".join(self._key(k) for k in keys),
                                 dtype=np.uint8).copy()
            if kbuf.size != 16 * n:
                raise ValueError("one key per block")
        pf = None
        if is_prefix is not None:
            pf = np.array([1 if p else 0 for p in is_prefix], dtype=np.uint8)
        status = np.zeros(n, np.uint8)
        digests = np.zeros(32 * n, np.uint8) if keys is None else None
        stored = _u64(0)
        check(_lib.load().cascade_store_put_batch(
            self._h, n, ptrs.ctypes.data, sizes.ctypes.data,
            kbuf.ctypes.data if kbuf is not None else None,
            pf.ctypes.data if pf is not None else None,
            status.ctypes.data,
            digests.ctypes.data if digests is not None else None,
            stream, ctypes.byref(stored)))
        del keepalive
        if return_status:
            return int(stored.value), status, (
                digests.reshape(n, 32) if digests is not None else None)
        return int(stored.value)

    def put_batch_host(self, blocks: Sequence, keys=None, is_prefix=None,
                       return_status: bool = False):
        """Stores host blocks (numpy uint8 arrays, pinned or not) in one call;
        the library moves them to the GPU.  Same results as put_batch.
        ``blocks``: a sequence of arrays, or one 2-D uint8 array with a
        block per row (described without a per-block Python step)."""
        if (isinstance(blocks, np.ndarray) and blocks.ndim == 2
                and blocks.dtype == np.uint8 and blocks.strides[1] == 1):
            n = blocks.shape[0]
            ptrs = (np.arange(n, dtype=np.uint64)
                    * np.uint64(blocks.strides[0])
                    + np.uint64(blocks.ctypes.data))
            sizes = np.full(n, blocks.shape[1], np.uint64)
            arrs = blocks                   # keeps the rows alive
        else:
            arrs = [_host_u8(b) for b in blocks]
            n = len(arrs)
            ptrs = np.array([a.ctypes.data for a in arrs], dtype=np.uint64)
            sizes = np.array([a.size for a in arrs], dtype=np.uint64)
        kbuf = None
        if keys is not None:
            kbuf = np.frombuffer(b"".join(self._key(k) for k in keys),
                                 dtype=np.uint8).copy()
        pf = None
        if is_prefix is not None:
            pf = np.array([1 if p else 0 for p in is_prefix], dtype=np.uint8)
        status = np.zeros(n, np.uint8)
        digests = np.zeros(32 * n, np.uint8) if keys is None else None
        stored = _u64(0)
        check(_lib.load().cascade_store_put_batch_host(
            self._h, n, ptrs.ctypes.data, sizes.ctypes.data,
            kbuf.ctypes.data if kbuf is not None else None,
            pf.ctypes.data if pf is not None else None,
            status.ctypes.data,
            digests.ctypes.data if digests is not None else None,
            ctypes.byref(stored)))
        if return_status:
            return int(stored.value), status, (
                digests.reshape(n, 32) if digests is not None else None)
        return int(stored.value)

    def get_batch(self, keys: Sequence, outs: Sequence):
        """Reads blocks into CUDA uint8 tensors ``outs``.  Returns
        (found[n] uint8, sizes[n] uint64); a block larger than its output is
        reported found with its size and not written."""
        outs = [_cuda_u8(o) for o in outs]
        n = len(outs)
        kbuf = np.frombuffer(b"".join(self._key(k) for k in keys),
                             dtype=np.uint8).copy()
        if kbuf.size != 16 * n:
            raise ValueError("one key per output")
        ptrs = np.array([o.data_ptr() for o in outs], dtype=np.uint64)
        caps = np.array([o.numel() for o in outs], dtype=np.uint64)
        stream = _torch_stream_of(outs[0]) if n else 0
        return self._get_batch_raw(n, kbuf, ptrs, caps, stream)

    def _get_batch_raw(self, n, keys16, ptrs, caps, stream):
        """get_batch on prepared arrays: keys16 uint8[n*16], ptrs / caps
        uint64[n] (device addresses and their capacities)."""
        sizes = np.zeros(n, np.uint64)
        found = np.zeros(n, np.uint8)
        nf = _u64(0)
        check(_lib.load().cascade_store_get_batch(
            self._h, n, keys16.ctypes.data, ptrs.ctypes.data,
            caps.ctypes.data, sizes.ctypes.data, found.ctypes.data, stream,
            ctypes.byref(nf)))
        return found, sizes

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.load().cascade_store_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------- compute_block_id
def compute_block_id(data) -> str:
    """bindings.cpp:173-176: lowercase hex of SHA-256 digest bytes 0..15,
    computed on the GPU."""
    if _is_cuda_tensor(data):
        return compute_block_ids([data])[0]
    arr = _host_u8(data)
    out = ctypes.create_string_buffer(33)
    check(_lib.load().cascade_compute_block_id(arr.ctypes.data, arr.size, out))
    return out.value.decode()


def sha256_batch(blocks) -> "torch.Tensor":
    """32-byte SHA-256 digests (CUDA uint8 tensor [n, 32]) of CUDA blocks."""
    import torch
    blocks = [_cuda_u8(b) for b in blocks]
    n = len(blocks)
    dev = blocks[0].device
    ptrs = torch.tensor([b.data_ptr() for b in blocks], dtype=torch.int64,
                        device=dev)
    sizes = torch.tensor([b.numel() for b in blocks], dtype=torch.int64,
                         device=dev)
    out = torch.empty((n, 32), dtype=torch.uint8, device=dev)
    _lib.call("cascade_sha256_batch", ptrs.data_ptr(), sizes.data_ptr(), n,
              out.data_ptr(), _torch_stream_of(out))
    torch.cuda.current_stream(dev).synchronize()
    del ptrs, sizes, blocks
    return out


def compute_block_ids(blocks) -> list:
    """compute_block_id for many CUDA blocks in one launch."""
    d = sha256_batch(blocks).cpu().numpy()
    return [row[:16].tobytes().hex() for row in d]


# ------------------------------------------------------------ raw tiers
class _TierBase:
    _store: CascadeStore

    def put(self, id: str, data) -> bool:
        return self._store.put(id, data)

    def get(self, id: str, out):
        return self._store.get(id, out)

    def contains(self, id: str) -> bool:
        return self._store.contains(id)

    def clear(self) -> None:
        self._store.clear()


class GPUBackend(_TierBase):
    """cascade::GPUBackend (cascade.hpp:129-206; bindings.cpp:178-192): the
    HBM pool alone, raw bytes, no dedup counting."""

    def __init__(self, capacity_bytes: int, device_id: int = 0):
        cfg = CascadeConfig()
        cfg.use_gpu = True
        cfg.gpu_capacity_bytes = capacity_bytes
        cfg.gpu_device_id = device_id
        cfg.shm_capacity_bytes = 0
        cfg.dedup_enabled = False
        cfg.kv_compression = False
        self._store = CascadeStore(cfg)

    def used_bytes(self) -> int:
        return self._store.get_stats().gpu_used


class ShmBackend(_TierBase):
    """cascade::ShmBackend (cascade.hpp:209-274; bindings.cpp:194-208): the
    DRAM tier alone (pinned host memory; ``path`` is accepted for
    compatibility and not used)."""

    def __init__(self, capacity_bytes: int, path: str = "/dev/shm/cascade"):
        cfg = CascadeConfig()
        cfg.use_gpu = False
        cfg.shm_capacity_bytes = capacity_bytes
        cfg.shm_path = path
        cfg.dedup_enabled = False
        cfg.kv_compression = False
        self._store = CascadeStore(cfg)

    def used_bytes(self) -> int:
        return self._store.get_stats().shm_used


class LustreBackend:
    """Name kept for ``from cascade_cpp import ... LustreBackend``
    (cascade/__init__.py:1).  The parallel-filesystem cold tier
    (cascade_core.cpp:572-691) is not part of this library."""

    def __init__(self, path: str, stripe_size: int = 4 * 1024 * 1024,
                 stripe_count: int = 4):
        raise NotImplementedError(
            "LustreBackend: the Lustre cold tier is not part of cascade_b200")


class AggregatedLustreBackend:
    """See LustreBackend (cascade_core.cpp:694-816)."""

    def __init__(self, path: str, max_file_size: int = 256 * 1024 * 1024,
                 stripe_size: int = 4 * 1024 * 1024, stripe_count: int = 16):
        raise NotImplementedError(
            "AggregatedLustreBackend: the Lustre cold tier is not part of "
            "cascade_b200")


__all__ = ["CascadeConfig", "CascadeStats", "CascadeStore", "compute_block_id",
           "compute_block_ids", "sha256_batch", "GPUBackend", "ShmBackend",
           "LustreBackend", "AggregatedLustreBackend", "CascadeError"]
