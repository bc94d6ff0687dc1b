"""The allocation-free compression entry point.

cascade_kv_compress_batch_noalloc exists for callers that cannot let the
library allocate device memory (an engine that has already reserved almost
all of HBM for its own KV cache, or an ingest loop that cannot risk an
allocator call mid-step).  It must produce exactly the bytes of
cascade_kv_compress_batch and allocate nothing (the device's stream-ordered
pool and its free memory are checked around the calls); it shares one fixed
scratch array across calls, so two calls in a row also check that the
second does not see the first's leftovers.  This file is collected last on purpose, and also passes when
run alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from cascade_b200 import _lib
from cascade_b200 import workloads

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
MAX_BLOCKS = 65536


def _blocks(seed, n_kv, n_rand):
    rng = np.random.default_rng(seed)
    xs = list(workloads.kv_blocks_np(n_kv, seed, layers=2))
    for _ in range(n_rand):
        lo = int(rng.integers(-32768, 32767))
        hi = int(rng.integers(lo, 32768))
        n = int(rng.integers(1, 40000))
        xs.append(rng.integers(lo, hi + 1, n).astype(np.int16).view(np.uint8))
    xs.append(rng.integers(0, 256, 101, dtype=np.uint8))    # odd size
    return xs


def _compress(entry, xs):
    src = [torch.from_numpy(np.ascontiguousarray(x)).to(DEV) for x in xs]
    dst = [torch.full((8 + x.size // 2,), 0xAB, dtype=torch.uint8, device=DEV)
           for x in xs]
    ps = torch.tensor([t.data_ptr() for t in src], dtype=torch.int64, device=DEV)
    pd = torch.tensor([t.data_ptr() for t in dst], dtype=torch.int64, device=DEV)
    sz = torch.tensor([x.size for x in xs], dtype=torch.int64, device=DEV)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    _lib.call(entry, ps.data_ptr(), sz.data_ptr(), pd.data_ptr(), len(xs),
              max(x.size for x in xs), stream)
    torch.cuda.synchronize()
    return [d.cpu().numpy() for d in dst]


def _cudart():
    """The CUDA runtime the library links (libcudart.so.12), for reading
    the device's stream-ordered memory pool."""
    return ctypes.CDLL("libcudart.so.12")


_USED_HIGH, _RESERVED_HIGH = 8, 6     # cudaMemPoolAttrUsedMemHigh / ...High


def _pool_high(rt, pool):
    out = []
    for attr in (_USED_HIGH, _RESERVED_HIGH):
        v = ctypes.c_uint64(0)
        assert rt.cudaMemPoolGetAttribute(pool, attr, ctypes.byref(v)) == 0
        out.append(v.value)
    return out


def _reset_pool_high(rt, pool):
    for attr in (_USED_HIGH, _RESERVED_HIGH):
        z = ctypes.c_uint64(0)
        assert rt.cudaMemPoolSetAttribute(pool, attr, ctypes.byref(z)) == 0


def test_noalloc_allocates_nothing():
    # The set-up call (n = 0) places the scratch array on the GPU; after
    # it, a call must leave the device's stream-ordered pool untouched and
    # the device's free memory unchanged.
    L = _lib.load()
    stream = torch.cuda.current_stream(DEV).cuda_stream
    assert L.cascade_kv_compress_batch_noalloc(None, None, None, 0, 0,
                                               ctypes.c_void_p(stream)) == 0
    xs = _blocks(3, 4, 8)
    src = [torch.from_numpy(np.ascontiguousarray(x)).to(DEV) for x in xs]
    dst = [torch.empty(8 + x.size // 2, dtype=torch.uint8, device=DEV)
           for x in xs]
    ps = torch.tensor([t.data_ptr() for t in src], dtype=torch.int64, device=DEV)
    pd = torch.tensor([t.data_ptr() for t in dst], dtype=torch.int64, device=DEV)
    sz = torch.tensor([x.size for x in xs], dtype=torch.int64, device=DEV)
    torch.cuda.synchronize()
    rt = _cudart()
    pool = ctypes.c_void_p()
    assert rt.cudaDeviceGetDefaultMemPool(ctypes.byref(pool), 0) == 0
    # The probe has teeth: a stream-ordered allocation shows in the pool.
    _reset_pool_high(rt, pool)
    p = ctypes.c_void_p()
    assert rt.cudaMallocAsync(ctypes.byref(p), 1 << 20,
                              ctypes.c_void_p(stream)) == 0
    assert rt.cudaFreeAsync(p, ctypes.c_void_p(stream)) == 0
    torch.cuda.synchronize()
    assert _pool_high(rt, pool)[0] >= 1 << 20
    _reset_pool_high(rt, pool)
    free0, _ = torch.cuda.mem_get_info(DEV)
    for _ in range(2):
        _lib.call("cascade_kv_compress_batch_noalloc", ps.data_ptr(),
                  sz.data_ptr(), pd.data_ptr(), len(xs),
                  max(x.size for x in xs), stream)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(DEV)
    assert _pool_high(rt, pool) == [0, 0]
    assert free1 == free0


def test_noalloc_matches_allocating_entry_point_on_two_calls():
    # The first call sees a wide mix of value ranges; the second, smaller
    # call uses narrow ranges, so scratch left over from the first call
    # would change its scales.
    for seed, n_kv, n_rand in ((1, 8, 40), (2, 2, 5)):
        xs = _blocks(seed, n_kv, n_rand)
        want = _compress("cascade_kv_compress_batch", xs)
        got = _compress("cascade_kv_compress_batch_noalloc", xs)
        for i, (g, w) in enumerate(zip(got, want)):
            assert np.array_equal(g, w), (seed, i)


def test_noalloc_rejects_batches_over_its_limit():
    L = _lib.load()
    dummy = ctypes.c_void_p(16)  # never dereferenced: the size check is first
    rc = L.cascade_kv_compress_batch_noalloc(dummy, dummy, dummy,
                                             MAX_BLOCKS + 1, 64, None)
    assert rc == 1
    assert b"65536" in L.cascade_last_error()
