"""The device KV-cache wire format (cascade_b200.kvwire over
cascade_kv_serialize_batch / cascade_kv_deserialize_batch) against the
reference's own bytes: the golden cases made by kv_manager.serialize_kv_cache
(inference_benchmark/kv_manager.py:43-63), the oracle's restatement for
larger and strided shapes, and a store round trip through CascadeStore."""
import struct

import numpy as np
import pytest
import torch

from cascade_b200 import cascade_cpp as cc
from cascade_b200 import kvwire
from conftest import load_npz
from oracle import kvwire as okv

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
TORCH_DT = {0: torch.float16, 1: torch.bfloat16, 2: torch.float32}


def _golden_cache(d, name):
    L, H, S, D = (int(x) for x in d[name + "_shape"])
    dt = TORCH_DT[int(d[name + "_dtype"])]
    raw = torch.from_numpy(d[name + "_src"].copy()).to(DEV)
    vals = raw.view(torch.int16 if dt == torch.bfloat16 else dt)
    if dt == torch.bfloat16:
        vals = vals.view(torch.bfloat16)
    per = H * S * D
    return tuple((vals[2 * l * per:(2 * l + 1) * per].view(1, H, S, D),
                  vals[(2 * l + 1) * per:(2 * l + 2) * per].view(1, H, S, D))
                 for l in range(L))


def _bytes(t):
    return t.cpu().numpy().tobytes()


def test_serialize_equals_the_reference_golden():
    d = load_npz("kvwire_cases.npz")
    for name in d["names"]:
        name = str(name)
        wire = kvwire.serialize_kv_cache(_golden_cache(d, name))
        assert _bytes(wire) == d[name + "_wire"].tobytes(), name


def test_deserialize_of_the_reference_golden():
    d = load_npz("kvwire_cases.npz")
    for name in d["names"]:
        name = str(name)
        want = okv.deserialize(d[name + "_wire"].tobytes())
        blob = torch.from_numpy(d[name + "_wire"].copy()).to(DEV)
        back = kvwire.deserialize_kv_cache(blob)
        assert len(back) == len(want)
        for (k, v), (k0, v0) in zip(back, want):
            assert k.shape == (1,) + k0.shape and k.dtype == torch.float16
            assert np.array_equal(k[0].cpu().numpy().view(np.uint16),
                                  k0.view(np.uint16)), name
            assert np.array_equal(v[0].cpu().numpy().view(np.uint16),
                                  v0.view(np.uint16)), name


def _cache(seed, L, H, S, D, dtype=torch.float16):
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    return tuple((torch.randn(1, H, S, D, generator=g, device=DEV).to(dtype),
                  torch.randn(1, H, S, D, generator=g, device=DEV).to(dtype))
                 for _ in range(L))


def _oracle_bytes(cache):
    return okv.serialize([(k[0].float().cpu().numpy(), v[0].float().cpu().numpy())
                          for k, v in cache])


@pytest.mark.parametrize("shape", [(32, 8, 16, 128), (4, 8, 37, 128),
                                   (2, 3, 5, 64), (3, 2, 9, 24),
                                   (2, 1, 3, 7), (1, 1, 1, 1)])
def test_serialize_matches_oracle_and_round_trips(shape):
    cache = _cache(sum(shape), *shape)
    wire = kvwire.serialize_kv_cache(cache)
    assert wire.numel() == kvwire.wire_bytes(*shape)
    assert _bytes(wire) == _oracle_bytes(cache)
    back = kvwire.deserialize_kv_cache(wire)
    for (k, v), (k0, v0) in zip(back, cache):
        assert torch.equal(k, k0) and torch.equal(v, v0)


def test_strided_sources():
    # a slice of a longer static cache (seq stride > seq * dim, offset
    # start) and a [seq, heads, dim] buffer permuted to [heads, seq, dim]
    L, H, S, D = 3, 4, 11, 64
    big = torch.randn(L, 2, 1, H, 40, D, device=DEV).half()
    sliced = tuple((big[l, 0, :, :, 5:5 + S], big[l, 1, :, :, 5:5 + S])
                   for l in range(L))
    perm = torch.randn(L, 2, S, H, D, device=DEV).half()
    permuted = tuple((perm[l, 0].permute(1, 0, 2).unsqueeze(0),
                      perm[l, 1].permute(1, 0, 2).unsqueeze(0))
                     for l in range(L))
    for cache in (sliced, permuted):
        assert not cache[0][0].is_contiguous()
        assert _bytes(kvwire.serialize_kv_cache(cache)) == _oracle_bytes(cache)


def test_unaligned_sources_and_blocks():
    # sources that start 2 bytes off a 16-byte boundary, outputs written at
    # an odd byte offset, and a wire block read from an odd offset
    L, H, S, D = 2, 2, 6, 16
    flat = torch.randn(2 * L * H * S * D + 1, device=DEV).half()
    per = H * S * D
    cache = tuple((flat[1 + 2 * l * per:1 + (2 * l + 1) * per].view(1, H, S, D),
                   flat[1 + (2 * l + 1) * per:1 + (2 * l + 2) * per]
                   .view(1, H, S, D)) for l in range(L))
    want = _oracle_bytes(cache)
    n = len(want)
    buf = torch.zeros((1, n + 64), dtype=torch.uint8, device=DEV)
    out = buf[:, 3:3 + n]
    kvwire.serialize_kv_caches([cache], out=out)
    assert _bytes(out[0]) == want
    assert int(buf[0, :3].sum()) == 0 and int(buf[0, 3 + n:].sum()) == 0
    back = kvwire.deserialize_kv_cache(out[0])
    for (k, v), (k0, v0) in zip(back, cache):
        assert torch.equal(k, k0) and torch.equal(v, v0)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_conversions_round_like_torch(dtype):
    cache = _cache(7, 3, 4, 9, 32, dtype)
    cache[0][0].view(-1)[:6] = torch.tensor(
        [70000.0, -1e6, 65520.0, 3e-8, float("inf"), -0.0]).to(dtype)
    want = tuple((k.to(torch.float16), v.to(torch.float16)) for k, v in cache)
    assert _bytes(kvwire.serialize_kv_cache(cache)) == \
        _bytes(kvwire.serialize_kv_cache(want))


def test_batch_of_caches_in_one_launch():
    caches = [_cache(100 + i, 4, 8, 16, 128) for i in range(37)]
    rows = kvwire.serialize_kv_caches(caches)
    assert len(rows) == 37
    for row, c in zip(rows, caches):
        assert row.data_ptr() % 256 == 0
        assert _bytes(row) == _oracle_bytes(c)
    backs = kvwire.deserialize_kv_caches(rows)
    for back, c in zip(backs, caches):
        for (k, v), (k0, v0) in zip(back, c):
            assert torch.equal(k, k0) and torch.equal(v, v0)


def test_large_batch_round_trip():
    """256 caches of llama3-8b geometry (32 layers x (K, V) x [8][16][128]
    FP16 = 2 MiB each, 512 MiB in all, larger than L2) in one launch each
    way: every header, every payload byte and the round trip."""
    n, L, H, S, D = 256, 32, 8, 16, 128
    src = torch.randn(n, L, 2, 1, H, S, D, device=DEV).half()
    caches = [tuple((src[i, l, 0], src[i, l, 1]) for l in range(L))
              for i in range(n)]
    rows = kvwire.serialize_kv_caches(caches)
    wire = torch.stack(rows)
    head = np.frombuffer(struct.pack("<IIIIH", L, H, S, D, 0), np.uint8)
    assert (wire[:, :18].cpu().numpy() == head).all()
    assert torch.equal(wire[:, 18:], src.view(n, -1).view(torch.uint8))
    backs = kvwire.deserialize_kv_caches(rows)
    back = torch.stack([torch.stack([torch.stack(kv) for kv in b])
                        for b in backs])
    assert torch.equal(back, src)


def test_store_round_trip_without_host_copies():
    """KVCacheStore.store / load (kv_manager.py:116-156) with the device
    wire format: the block the store holds is the reference's blob."""
    cfg = cc.CascadeConfig()
    cfg.gpu_capacity_bytes = 64 << 20
    cfg.shm_capacity_bytes = 16 << 20
    store = cc.CascadeStore(cfg)
    try:
        cache = _cache(3, 4, 8, 29, 128)
        wire = kvwire.serialize_kv_cache(cache)
        assert store.put("prefix-0", wire)
        buf = torch.empty(wire.numel() + 100, dtype=torch.uint8, device=DEV)
        found, size = store.get("prefix-0", buf)
        assert found and size == wire.numel()
        back = kvwire.deserialize_kv_cache(buf[:size])
        for (k, v), (k0, v0) in zip(back, cache):
            assert torch.equal(k, k0) and torch.equal(v, v0)
        # a host reader gets the reference's bytes
        host = np.empty(size, np.uint8)
        assert store.get("prefix-0", host) == (True, size)
        assert host.tobytes() == _oracle_bytes(cache)
    finally:
        store.close()


def test_rejects_bad_shapes():
    with pytest.raises(ValueError):
        kvwire.serialize_kv_cache(((torch.zeros(2, 2, 3, 8, device=DEV),) * 2,))
    k = torch.zeros(1, 2, 3, 8, device=DEV).half()
    with pytest.raises(ValueError):
        kvwire.serialize_kv_cache(((k, torch.zeros(1, 2, 4, 8, device=DEV)
                                    .half()),))
    bad = torch.zeros(30, dtype=torch.uint8, device=DEV)
    bad[:18] = torch.tensor(list(b"\x01\0\0\0\x01\0\0\0\x01\0\0\0\x08\0\0\0"
                                 b"\x02\0"), dtype=torch.uint8)
    with pytest.raises(ValueError):           # dtype id 2 is not written
        kvwire.deserialize_kv_cache(bad)


def test_store_and_load_batches_of_caches():
    """store_kv_caches / load_kv_caches: KVCacheStore.store / load for a
    batch; a blob the reference's host path put reads back too."""
    cfg = cc.CascadeConfig()
    cfg.gpu_capacity_bytes = 64 << 20
    cfg.shm_capacity_bytes = 16 << 20
    store = cc.CascadeStore(cfg)
    try:
        shape = (4, 8, 13, 128)
        caches = [_cache(40 + i, *shape) for i in range(5)]
        st = kvwire.store_kv_caches(store, [f"p{i}" for i in range(5)], caches)
        assert (np.asarray(st) == 0).all()
        host = np.frombuffer(_oracle_bytes(caches[0]), np.uint8).copy()
        assert store.put("from-host", host)
        got = kvwire.load_kv_caches(store, ["p3", "missing", "from-host", "p0"],
                                    *shape)
        assert got[1] is None
        for g, c in ((got[0], caches[3]), (got[2], caches[0]),
                     (got[3], caches[0])):
            for (k, v), (k0, v0) in zip(g, c):
                assert torch.equal(k, k0) and torch.equal(v, v0)
        # another shape under an id: not this wire size, so not loaded
        assert kvwire.load_kv_caches(store, ["p1"], 4, 8, 12, 128) == [None]
    finally:
        store.close()


def test_load_through_the_dram_tier_and_int8():
    """load_kv_caches for blocks the fused pool path cannot split: raw
    blocks demoted to the DRAM tier (exact), and INT8 blocks in HBM (equal
    to what get + deserialize return)."""
    shape = (4, 8, 16, 128)                      # 256 KiB + 18 per cache
    caches = [_cache(70 + i, *shape) for i in range(6)]
    ids = [f"c{i}" for i in range(6)]
    cfg = cc.CascadeConfig()
    cfg.gpu_capacity_bytes = 3 * (kvwire.wire_bytes(*shape) + 4096)
    cfg.shm_capacity_bytes = 16 << 20
    store = cc.CascadeStore(cfg)
    try:
        kvwire.store_kv_caches(store, ids, caches)
        assert store.get_stats().gpu_evictions > 0
        got = kvwire.load_kv_caches(store, ids, *shape)
        for g, c in zip(got, caches):
            for (k, v), (k0, v0) in zip(g, c):
                assert torch.equal(k, k0) and torch.equal(v, v0)
        s = store.get_stats()
        assert s.gpu_hits + s.shm_hits == 6 and s.shm_hits > 0
    finally:
        store.close()
    cfg = cc.CascadeConfig()
    cfg.gpu_capacity_bytes = 64 << 20
    cfg.shm_capacity_bytes = 16 << 20
    cfg.kv_compression = True
    cfg.gpu_q8 = True
    store = cc.CascadeStore(cfg)
    try:
        kvwire.store_kv_caches(store, ids[:3], caches[:3])
        got = kvwire.load_kv_caches(store, ids[:3], *shape)
        buf = torch.empty(kvwire.wire_bytes(*shape), dtype=torch.uint8,
                          device=DEV)
        for i in range(3):
            assert store.get(ids[i], buf)[0]
            # INT8 storage quantises the header with the payload (as the
            # reference's KVCompressor does): the shape comes from the caller
            want = kvwire.deserialize_kv_cache(buf, header=shape + (0,))
            for (k, v), (k0, v0) in zip(got[i], want):   # bits (NaNs too)
                assert torch.equal(k.view(torch.int16), k0.view(torch.int16))
                assert torch.equal(v.view(torch.int16), v0.view(torch.int16))
    finally:
        store.close()


def test_fused_put_dedup_and_slot_retry():
    """cascade_store_put_kv_batch: first of a batch wins, a known id is a
    dedup hit, and caches whose pool slot cannot be allocated (a pool sized
    by bytes, 144 KiB size classes for 128 KiB + 18-byte blocks) are placed
    in the DRAM tier through the staging buffer; every cache reads back."""
    shape = (2, 8, 16, 128)
    wb = kvwire.wire_bytes(*shape)
    caches = [_cache(90 + i, *shape) for i in range(16)]
    cfg = cc.CascadeConfig()
    cfg.gpu_capacity_bytes = 16 * wb
    cfg.shm_capacity_bytes = 16 << 20
    store = cc.CascadeStore(cfg)
    try:
        ids = [f"k{i}" for i in range(16)]
        st = kvwire.store_kv_caches(store, ids, caches)
        assert (np.asarray(st) == 0).all()
        s = store.get_stats()
        assert s.shm_puts >= 1 and s.gpu_used + s.shm_used > 0
        got = kvwire.load_kv_caches(store, ids, *shape)
        for g, c in zip(got, caches):
            for (k, v), (k0, v0) in zip(g, c):
                assert torch.equal(k, k0) and torch.equal(v, v0)
    finally:
        store.close()
    cfg = cc.CascadeConfig()
    cfg.gpu_capacity_bytes = 64 << 20
    cfg.shm_capacity_bytes = 0
    store = cc.CascadeStore(cfg)
    try:
        st = kvwire.store_kv_caches(store, ["x", "y", "x"],
                                    [caches[0], caches[1], caches[2]])
        assert list(np.asarray(st)) == [0, 0, 2]
        st = kvwire.store_kv_caches(store, ["y"], [caches[3]])
        assert list(np.asarray(st)) == [1]
        assert store.get_stats().dedup_hits == 2
        got = kvwire.load_kv_caches(store, ["x", "y"], *shape)
        for g, c in zip(got, (caches[0], caches[1])):
            for (k, v), (k0, v0) in zip(g, c):
                assert torch.equal(k, k0) and torch.equal(v, v0)
    finally:
        store.close()


@pytest.mark.parametrize("dedup", [True, False])
def test_fused_put_matches_put_batch(dedup):
    """The one-call put and serialise + put_batch give the same statuses
    and counters, with repeated ids, prefix flags and BF16 sources."""
    shape = (3, 4, 9, 64)
    caches = [_cache(200 + i, *shape, dtype=torch.bfloat16) for i in range(6)]
    ids = ["a", "b", "a", "c", "b", "d"]
    pre = [True, False, True, False, False, True]
    results = []
    for fused in (True, False):
        cfg = cc.CascadeConfig()
        cfg.gpu_capacity_bytes = 64 << 20
        cfg.shm_capacity_bytes = 16 << 20
        cfg.dedup_enabled = dedup
        store = cc.CascadeStore(cfg)
        try:
            if fused:
                st = kvwire.store_kv_caches(store, ids, caches, is_prefix=pre)
            else:
                rows = kvwire.serialize_kv_caches(caches)
                st = store.put_batch(rows, keys=ids, is_prefix=pre,
                                     return_status=True)[1]
            s = store.get_stats()
            got = kvwire.load_kv_caches(store, ["a", "b", "c", "d"], *shape)
            counters = {f: getattr(s, f) for f in cc._STAT_FIELDS}
            results.append((list(np.asarray(st)), counters, got))
        finally:
            store.close()
    (st0, s0, g0), (st1, s1, g1) = results
    assert st0 == st1 and s0 == s1
    for a, b in zip(g0, g1):
        for (k, v), (k0, v0) in zip(a, b):
            assert torch.equal(k, k0) and torch.equal(v, v0)
    # the stored caches are the first of each id, rounded to FP16
    for g, c in zip(g0, (caches[0], caches[1], caches[3], caches[5])):
        for (k, v), (k0, v0) in zip(g, c):
            assert torch.equal(k, k0.half()) and torch.equal(v, v0.half())
