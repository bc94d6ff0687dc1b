"""Pins the store model's demotion counters to the reference itself: the
compiled reference CascadeStore with its GPU tier (oracle/_ref, GPUBackend
on device 0: cudaMalloc'd pool and copies, no kernels of its own) against
oracle/store_model.py and this library's store, on random put sequences
that overflow the GPU tier.

Blocks are all one size and raw (kv_compression off), so the reference's
victim choice (the LRU tail of its largest index shard) and this library's
(the least recent block of the whole tier) demote the same number of blocks
and the same bytes: gpu_used, shm_used, gpu_evictions, shm_puts, dedup_hits
and every put's result must agree among the three.  Which blocks were
demoted differs, so reads are not compared here (tests/test_gpu_store.py
checks them against the model)."""
import tempfile

import numpy as np
import pytest

import oracle
from cascade_b200 import cascade_cpp as cc
from oracle.store_model import StoreModel

pytestmark = pytest.mark.gpu

COUNTERS = ("gpu_used", "shm_used", "gpu_evictions", "shm_puts", "dedup_hits")


@pytest.mark.parametrize("seed", range(4))
@pytest.mark.parametrize("semantic", [True, False], ids=["prefix", "lru"])
def test_demotion_counters_match_compiled_reference(seed, semantic):
    if oracle.ref() is None:
        pytest.skip("oracle/_ref not built")
    S, cap_blocks = 4096, 16
    rng = np.random.default_rng(500 + seed + 10 * semantic)
    universe = [rng.integers(0, 256, S, dtype=np.uint8) for _ in range(48)]
    ids = [f"{k:032x}" if k % 2 else f"block_{k}" for k in range(48)]
    ops = [(int(rng.integers(0, 48)), bool(rng.random() < 0.3))
           for _ in range(160)]
    cfg = cc.CascadeConfig()
    cfg.use_gpu = True
    cfg.gpu_capacity_bytes = cap_blocks * S
    cfg.shm_capacity_bytes = 64 << 20
    cfg.semantic_eviction = semantic
    cfg.promotion_enabled = False
    cfg.dram_chunk_bytes = 16 << 20
    ours = cc.CascadeStore(cfg)
    model = StoreModel(use_gpu=True, gpu_capacity=cap_blocks * S,
                       shm_capacity=64 << 20, semantic_eviction=semantic)
    with tempfile.TemporaryDirectory(dir="/dev/shm") as d:
        ref = oracle.RefStore(d + "/s", 64 << 20, gpu_bytes=cap_blocks * S,
                              semantic_eviction=semantic)
        try:
            for step, (k, pre) in enumerate(ops):
                r = ref.put(ids[k], universe[k], pre)
                assert model.put(ids[k], universe[k], pre) == r, step
                assert ours.put(ids[k], universe[k], is_prefix=pre) == r, step
                if step % 20 == 19:
                    rs = ref.stats()
                    os_ = ours.get_stats()
                    for f in COUNTERS:
                        assert model.stats[f] == rs[f], (step, f)
                        assert getattr(os_, f) == rs[f], (step, f)
            assert ref.stats()["gpu_evictions"] > 0
            for k in range(48):
                assert ours.contains(ids[k]) == ref.contains(ids[k])
        finally:
            ref.close()
            ours.close()
