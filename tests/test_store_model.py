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
