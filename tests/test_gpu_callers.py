"""The reference's own Python callers of this path, unchanged, on the
drop-in module.

``make -C oracle callers`` (run by ``__graft_entry__.build()`` where the
reference tree is present) copies the reference's files, byte for byte,
into the git-ignored baseline/_ref/callers:

* cascade/__init__.py (the package that imports ``cascade_cpp``, line 1);
* inference_benchmark/{__init__,config,kv_manager}.py (KVCacheStore.store
  / load, serialize_kv_cache / deserialize_kv_cache, kv_manager.py:43-156);
* script_example/benchmark/adapters/{base,cascade_adapter}.py
  (CascadeAdapter, cascade_adapter.py:28-189).

Here they are imported as they are, with cascade_b200/dropin first on the
path so that their ``import cascade_cpp`` resolves to the drop-in, and run
through a KV-cache store / load round trip on the GPU store and on the
CPU-tier ("login node") store.  The tests skip only when the copies are
absent.
"""
import hashlib
import importlib
import os
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DROPIN = os.path.join(ROOT, "cascade_b200", "dropin")
CALLERS = os.path.join(ROOT, "baseline", "_ref", "callers")
ADAPTERS = os.path.join(CALLERS, "script_example", "benchmark", "adapters")
MODULES = ("cascade_cpp", "cascade", "base", "cascade_adapter",
           "inference_benchmark", "inference_benchmark.config",
           "inference_benchmark.kv_manager")


@pytest.fixture()
def callers():
    if not os.path.exists(os.path.join(CALLERS, "inference_benchmark",
                                       "kv_manager.py")):
        pytest.skip("the reference's callers were not staged "
                    "(make -C oracle callers)")
    paths = [DROPIN, CALLERS, ADAPTERS]
    saved = list(sys.path)
    for p in reversed(paths):
        sys.path.insert(0, p)
    try:
        yield {
            "cascade": importlib.import_module("cascade"),
            "adapter": importlib.import_module("cascade_adapter"),
            "kv": importlib.import_module("inference_benchmark.kv_manager"),
            "config": importlib.import_module("inference_benchmark.config"),
        }
    finally:
        # cascade_adapter.py puts its own repository root on the path too
        sys.path[:] = saved
        for m in MODULES:
            sys.modules.pop(m, None)


def _kv_cache(seed, layers=4, heads=8, seq=37, dim=128):
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return tuple((torch.randn(1, heads, seq, dim, generator=g, device=dev).half(),
                  torch.randn(1, heads, seq, dim, generator=g, device=dev).half())
                 for _ in range(layers))


@pytest.mark.parametrize("use_gpu", [True, False])
def test_kv_cache_store_load_through_cascade_adapter(callers, use_gpu):
    ca, kv, conf = callers["adapter"], callers["kv"], callers["config"]
    # the drop-in module is the one the callers imported
    assert sys.modules["cascade_cpp"].__file__.startswith(DROPIN)
    adapter = ca.CascadeAdapter({"use_gpu": use_gpu, "gpu_capacity_gb": 0.25,
                                 "shm_capacity_gb": 0.5})
    assert adapter.initialize()
    store = kv.KVCacheStore(adapter, conf.ModelConfig())
    past = _kv_cache(5)
    token_ids = torch.arange(37, device="cuda:0").view(1, -1)
    prefix_hash = kv.compute_prefix_hash(token_ids, 37)
    assert store.store(prefix_hash, past)
    assert store.contains(prefix_hash)
    back = store.load(prefix_hash, device=torch.device("cuda:0"))
    assert back is not None and len(back) == len(past)
    for (k0, v0), (k1, v1) in zip(past, back):
        assert torch.equal(k0, k1) and torch.equal(v0, v1)
    assert store.load("0" * 32) is None
    assert store.stats["hits"] == 1 and store.stats["misses"] == 1
    # a second store of the same id is a dedup hit; a prefix block is kept
    assert store.store(prefix_hash, past)
    blob = kv.serialize_kv_cache(_kv_cache(6))
    mid = len(blob) // 2
    assert adapter.put_prefix("f" * 32, blob[:mid], blob[mid:])
    got = adapter.get("f" * 32)
    assert bytes(got[0]) + bytes(got[1]) == blob
    stats = adapter.get_stats()
    assert stats["dedup_hits"] == 1 and stats["misses"] == 1
    hits = stats["gpu_hits"] if use_gpu else stats["shm_hits"]
    assert hits == 2
    adapter.clear()
    assert not store.contains(prefix_hash)
    adapter.close()


def test_cascade_package_helpers(callers):
    cascade = callers["cascade"]
    data = b"the reference's cascade package, unchanged"
    assert cascade.compute_block_id_from_bytes(data) == \
        hashlib.sha256(data).hexdigest()[:32]
    store = cascade.create_login_node_store()
    x = np.frombuffer(data * 100, dtype=np.uint8)
    bid = cascade.compute_block_id(x)
    assert store.put(bid, x)
    out = np.empty(x.size, np.uint8)
    assert store.get(bid, out) == (True, x.size)
    assert np.array_equal(out, x)


def test_reference_store_device_load_and_back(callers):
    """The reference's KVCacheStore.store (host serialisation) and this
    library's device path on one store: kvwire.load_kv_caches reads what
    the reference stored, and the reference's load reads what
    kvwire.store_kv_caches stored."""
    from cascade_b200 import kvwire
    ca, kv, conf = callers["adapter"], callers["kv"], callers["config"]
    adapter = ca.CascadeAdapter({"use_gpu": True, "gpu_capacity_gb": 0.25,
                                 "shm_capacity_gb": 0.5})
    assert adapter.initialize()
    store = kv.KVCacheStore(adapter, conf.ModelConfig())
    past = _kv_cache(11)
    assert store.store("a" * 32, past)
    got = kvwire.load_kv_caches(adapter.store, ["a" * 32], 4, 8, 37, 128)[0]
    for (k0, v0), (k1, v1) in zip(past, got):
        assert torch.equal(k0, k1) and torch.equal(v0, v1)
    other = _kv_cache(12)
    st = kvwire.store_kv_caches(adapter.store, ["b" * 32], [other])
    assert int(st[0]) == 0
    back = store.load("b" * 32, device=torch.device("cuda:0"))
    for (k0, v0), (k1, v1) in zip(other, back):
        assert torch.equal(k0, k1) and torch.equal(v0, v1)
    adapter.close()
