"""Pins the sequential store model (oracle/store_model.py) against the
reference CascadeStore runs recorded in tests/golden/store_scenarios.json,
and checks the dedup count rule the sharded index relies on."""
import hashlib

import numpy as np
import pytest

from conftest import scenarios
from make_golden import scenario_blocks
from oracle.store_model import StoreModel


@pytest.mark.parametrize("sc", scenarios(), ids=lambda s: s["name"])
def test_model_replays_reference(sc):
    ids, blocks, pre = scenario_blocks(sc["kind"], sc["seed"])
    assert ids == sc["ids"]
    m = StoreModel(use_gpu=False, shm_capacity=sc["shm_capacity"],
                   kv_compression=sc["kv_compression"],
                   dedup_enabled=sc["dedup_enabled"])
    assert [m.put(i, b, p) for i, b, p in zip(ids, blocks, pre)] == sc["puts"]
    for bid, found, size, digest in sc["gets"]:
        f, data = m.get(bid)
        assert f == found
        if found:
            assert data.size == size
            assert hashlib.sha256(data.tobytes()).hexdigest() == digest
    assert [m.contains(i) for i in ids] == sc["contains"]
    assert m.stats == sc["stats"]


def test_dedup_hits_equal_n_minus_distinct():
    sc = [s for s in scenarios() if s["name"] == "dedup_plain"][0]
    assert sc["stats"]["dedup_hits"] == len(sc["ids"]) - len(set(sc["ids"]))


def _random_ops(seed, kv_compression):
    """A random put/get/contains sequence over a small id pool (so ids
    repeat), within the DRAM tier's capacity."""
    rng = np.random.default_rng(seed)
    sizes = [64, 65, 100, 127, 4096, 4097, 65536] + \
        ([] if kv_compression else [0, 1, 2, 63])
    pool = []
    for k in range(24):
        n = int(rng.choice(sizes))
        if k % 3 == 0:      # KV-like int16 data with a narrow range
            lo = int(rng.integers(-32768, 32000))
            b = rng.integers(lo, lo + int(rng.integers(1, 700)), (n + 1) // 2,
                             dtype=np.int64).astype(np.int16).view(np.uint8)[:n]
        else:
            b = rng.integers(0, 256, n, dtype=np.uint8)
        pool.append((f"{k:032x}" if k % 2 else f"block_{k}", b.copy()))
    ops = []
    for _ in range(160):
        r = rng.random()
        bid, data = pool[int(rng.integers(0, len(pool)))]
        if r < 0.55:
            ops.append(("put", bid, data, bool(rng.random() < 0.3)))
        elif r < 0.9:
            ops.append(("get", bid, None, False))
        else:
            ops.append(("contains", bid, None, False))
    return ops


@pytest.mark.parametrize("seed", range(6))
@pytest.mark.parametrize("kv_compression,dedup", [(False, True), (True, True),
                                                  (False, False)])
def test_model_matches_compiled_reference_random(seed, kv_compression, dedup,
                                                 tmp_path):
    """The model against the reference CascadeStore (use_gpu=False) itself,
    on random operation sequences: every result and every counter."""
    import tempfile

    import oracle
    if oracle.ref() is None:
        pytest.skip("oracle/_ref not built")
    with tempfile.TemporaryDirectory(dir="/dev/shm") as d:
        ref = oracle.RefStore(d + "/s", 64 << 20, kv_compression=kv_compression,
                              dedup_enabled=dedup)
        m = StoreModel(use_gpu=False, shm_capacity=64 << 20,
                       kv_compression=kv_compression, dedup_enabled=dedup)
        buf = np.zeros(70000, np.uint8)
        for op, bid, data, pre in _random_ops(100 * seed + 7, kv_compression):
            if op == "put":
                assert m.put(bid, data, pre) == ref.put(bid, data, pre), bid
            elif op == "get":
                found, size = ref.get(bid, buf)
                mf, mdata = m.get(bid)
                assert mf == found, bid
                if found:
                    assert mdata.size == size
                    assert np.array_equal(mdata, buf[:size]), bid
            else:
                assert m.contains(bid) == ref.contains(bid)
        assert m.stats == ref.stats()
        ref.close()
