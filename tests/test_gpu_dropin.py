"""The reference's Python callers, replayed against the drop-in module.

``import cascade_cpp`` is resolved through cascade_b200/dropin (the path a
user puts first on PYTHONPATH).  The calls below are the ones
inference_benchmark/kv_manager.py (KVCacheStore.store/load,
serialize_kv_cache / deserialize_kv_cache, lines 43-156) and
script_example/benchmark/adapters/cascade_adapter.py (CascadeAdapter.put/
get, lines 112-151) make, with their argument types: a KV cache
serialised to bytes with an 18-byte "<IIIIH" header, put as a numpy uint8
array made from the K+V byte halves, read back into a reusable numpy
buffer and split into halves again.
"""
import importlib
import os
import struct
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DROPIN = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "cascade_b200", "dropin")
HEADER_FMT = "<IIIIH"     # num_layers, num_kv_heads, seq_len, head_dim, dtype


@pytest.fixture()
def cascade_cpp():
    sys.path.insert(0, DROPIN)
    try:
        yield importlib.import_module("cascade_cpp")
    finally:
        sys.path.remove(DROPIN)
        sys.modules.pop("cascade_cpp", None)


def serialize(kv):
    """[(k, v)] of [1, heads, seq, dim] tensors -> bytes, header first."""
    _, heads, seq, dim = kv[0][0].shape
    out = [struct.pack(HEADER_FMT, len(kv), heads, seq, dim, 0)]
    for k, v in kv:
        out.append(k.squeeze(0).contiguous().to(torch.float16).cpu().numpy()
                   .view(np.uint8).tobytes())
        out.append(v.squeeze(0).contiguous().to(torch.float16).cpu().numpy()
                   .view(np.uint8).tobytes())
    return b"".join(out)


def deserialize(data, device):
    n, heads, seq, dim, _ = struct.unpack(HEADER_FMT, data[:18])
    payload = data[18:]
    tb = heads * seq * dim * 2
    kv, off = [], 0
    for _ in range(n):
        k = torch.from_numpy(np.frombuffer(payload[off:off + tb], np.float16).copy())
        off += tb
        v = torch.from_numpy(np.frombuffer(payload[off:off + tb], np.float16).copy())
        off += tb
        kv.append((k.view(1, heads, seq, dim).to(device),
                   v.view(1, heads, seq, dim).to(device)))
    return kv


class Adapter:
    """The calls CascadeAdapter makes on the store it wraps."""

    def __init__(self, cascade_cpp, use_gpu):
        cfg = cascade_cpp.CascadeConfig()
        if use_gpu:
            cfg.gpu_capacity_bytes = int(0.25 * 1024 ** 3)
            cfg.shm_capacity_bytes = int(0.5 * 1024 ** 3)
            cfg.dedup_enabled = True
            cfg.use_gpu = True
        else:            # cascade.create_login_node_store()
            cfg.use_gpu = False
            cfg.shm_capacity_bytes = 1 * 1024 * 1024 * 1024
            cfg.shm_path = "/dev/shm/cascade_login"
        self.store = cascade_cpp.CascadeStore(cfg)
        self._get_buf = np.empty(64 * 1024 * 1024, dtype=np.uint8)

    def put(self, block_id, key_data, value_data):
        data = np.frombuffer(key_data + value_data, dtype=np.uint8)
        return self.store.put(block_id, data, is_prefix=False)

    def get(self, block_id):
        found, size = self.store.get(block_id, self._get_buf)
        if found and size > len(self._get_buf):
            self._get_buf = np.empty(int(size * 1.1), dtype=np.uint8)
            found, size = self.store.get(block_id, self._get_buf)
        if not found or size == 0:
            return None
        data = self._get_buf[:size]
        mid = len(data) // 2
        return (data[:mid], data[mid:])


@pytest.mark.parametrize("use_gpu", [True, False])
def test_kv_manager_store_load_roundtrip(cascade_cpp, use_gpu):
    import hashlib
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(3)
    kv = [(torch.randn(1, 8, 37, 128, generator=g, device=dev).half(),
           torch.randn(1, 8, 37, 128, generator=g, device=dev).half())
          for _ in range(4)]
    token_ids = torch.arange(37, device=dev).view(1, -1)
    prefix_hash = hashlib.sha256(
        token_ids[0, :37].cpu().numpy().tobytes()).hexdigest()[:32]
    adapter = Adapter(cascade_cpp, use_gpu)
    blob = serialize(kv)
    mid = len(blob) // 2
    assert adapter.put(prefix_hash, blob[:mid], blob[mid:])
    assert adapter.store.contains(prefix_hash)
    res = adapter.get(prefix_hash)
    assert res is not None
    back = deserialize(bytes(res[0]) + bytes(res[1]), dev)
    for (k0, v0), (k1, v1) in zip(kv, back):
        assert torch.equal(k0, k1) and torch.equal(v0, v1)
    assert adapter.get("0" * 32) is None
    s = adapter.store.get_stats()
    assert (s.gpu_hits if use_gpu else s.shm_hits) == 1 and s.misses == 1
    assert adapter.put(prefix_hash, blob[:mid], blob[mid:])   # dedup hit
    assert adapter.store.get_stats().dedup_hits == 1
    assert "dedup=1" in repr(adapter.store.get_stats())


def test_package_import_line(cascade_cpp):
    # cascade/__init__.py:1 of the reference
    from cascade_cpp import (CascadeConfig, CascadeStore, GPUBackend,  # noqa
                             LustreBackend, ShmBackend, compute_block_id)
    import hashlib
    assert compute_block_id(np.frombuffer(b"abc", np.uint8)) == \
        hashlib.sha256(b"abc").hexdigest()[:32]
