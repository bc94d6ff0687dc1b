"""CascadeStore on the GPU against the reference's recorded runs (golden)
and the pinned sequential model: put/get/contains results, returned bytes
and every CascadeStats counter."""
import hashlib
import threading

import numpy as np
import pytest
import torch

import oracle
from cascade_b200 import cascade_cpp as cc
from cascade_b200 import workloads
from conftest import scenarios
from gpu_util import DEV
from make_golden import scenario_blocks
from oracle.store_model import StoreModel

pytestmark = pytest.mark.gpu


def make_store(use_gpu=False, gpu_cap=64 << 20, shm_cap=64 << 20,
               kv_compression=False, dedup=True, gpu_q8=False,
               promotion=True, semantic=True):
    cfg = cc.CascadeConfig()
    cfg.semantic_eviction = semantic
    cfg.use_gpu = use_gpu
    cfg.gpu_capacity_bytes = gpu_cap
    cfg.shm_capacity_bytes = shm_cap
    cfg.kv_compression = kv_compression
    cfg.dedup_enabled = dedup
    cfg.gpu_q8 = gpu_q8
    cfg.promotion_enabled = promotion
    cfg.dram_chunk_bytes = 16 << 20
    return cc.CascadeStore(cfg)


def stats_dict(s):
    return {f: getattr(s, f) for f in cc._STAT_FIELDS}


def replay(store, sc, ids, blocks, pre):
    puts = [store.put(i, b, p) for i, b, p in zip(ids, blocks, pre)]
    buf = np.zeros(1 << 20, np.uint8)
    gets = []
    order = list(range(len(ids)))[::-1] + ["missing_block"]
    for k in order:
        bid = ids[k] if k != "missing_block" else "ffffffffffffffffffffffffffffff00"
        found, size = store.get(bid, buf)
        gets.append([bid, bool(found), int(size),
                     hashlib.sha256(buf[:size].tobytes()).hexdigest()
                     if found else None])
    contains = [store.contains(i) for i in ids]
    return puts, gets, contains


@pytest.mark.parametrize("sc", scenarios(), ids=lambda s: s["name"])
def test_dram_tier_matches_reference_runs(sc):
    """use_gpu=False: the configuration the reference itself ran."""
    ids, blocks, pre = scenario_blocks(sc["kind"], sc["seed"])
    st = make_store(use_gpu=False, shm_cap=sc["shm_capacity"],
                    kv_compression=sc["kv_compression"],
                    dedup=sc["dedup_enabled"])
    puts, gets, contains = replay(st, sc, ids, blocks, pre)
    assert puts == sc["puts"]
    assert gets == sc["gets"]
    assert contains == sc["contains"]
    assert stats_dict(st.get_stats()) == sc["stats"]


@pytest.mark.parametrize("gpu_q8", [False, True])
@pytest.mark.parametrize("sc", scenarios(), ids=lambda s: s["name"])
def test_hbm_tier_matches_model(sc, gpu_q8):
    ids, blocks, pre = scenario_blocks(sc["kind"], sc["seed"])
    st = make_store(use_gpu=True, shm_cap=sc["shm_capacity"],
                    kv_compression=sc["kv_compression"],
                    dedup=sc["dedup_enabled"], gpu_q8=gpu_q8)
    m = StoreModel(use_gpu=True, gpu_capacity=64 << 20,
                   shm_capacity=sc["shm_capacity"],
                   kv_compression=sc["kv_compression"],
                   dedup_enabled=sc["dedup_enabled"], gpu_q8=gpu_q8)
    puts, gets, contains = replay(st, sc, ids, blocks, pre)
    mp = [m.put(i, b, p) for i, b, p in zip(ids, blocks, pre)]
    assert puts == mp
    for bid, found, size, digest in gets:
        f, data = m.get(bid)
        assert f == found
        if f:
            assert size == data.size
            assert digest == hashlib.sha256(data.tobytes()).hexdigest()
    assert contains == [m.contains(i) for i in ids]
    assert stats_dict(st.get_stats()) == m.stats


def test_tier_spill_and_capacity_exhaustion():
    rng = np.random.default_rng(1)
    blocks = [rng.integers(0, 256, 4096, dtype=np.uint8) for _ in range(10)]
    ids = [oracle.block_id(b) for b in blocks]
    st = make_store(use_gpu=True, gpu_cap=3 * 4096, shm_cap=4 * 4096)
    m = StoreModel(use_gpu=True, gpu_capacity=3 * 4096, shm_capacity=4 * 4096)
    res = [st.put(i, b) for i, b in zip(ids, blocks)]
    assert res == [m.put(i, b) for i, b in zip(ids, blocks)]
    assert res == [True] * 7 + [False] * 3
    buf = np.zeros(8192, np.uint8)
    for i, b in zip(ids[:7], blocks[:7]):
        f, n = st.get(i, buf)
        assert f and n == 4096 and np.array_equal(buf[:n], b)
    for i in ids[7:]:
        assert st.get(i, buf) == (False, 0)
    s = st.get_stats()
    assert s.gpu_used == 3 * 4096 and s.shm_used == 4 * 4096


def test_get_into_small_buffer_reports_size():
    st = make_store(use_gpu=True)
    x = np.arange(5000, dtype=np.uint8)
    assert st.put("named", x)
    small = np.zeros(100, np.uint8)
    assert st.get("named", small) == (True, 5000)
    assert not small.any()                      # nothing written
    big = np.zeros(8000, np.uint8)
    assert st.get("named", big) == (True, 5000)
    assert np.array_equal(big[:5000], x)


def test_device_batch_put_get_content_addressed():
    n = 32
    blocks = workloads.kv_blocks_torch(n, 4, DEV, layers=2)     # 64 KiB each
    st = make_store(use_gpu=True, gpu_cap=256 << 20)
    stored, status, digests = st.put_batch(blocks, return_status=True)
    assert stored == n and (status == 0).all()
    host = blocks.cpu().numpy()
    for i in range(n):
        assert digests[i].tobytes() == hashlib.sha256(host[i].tobytes()).digest()
    # a second put of the same blocks: all dedup hits
    stored, status, _ = st.put_batch(blocks, return_status=True)
    assert stored == n and (status == 1).all()
    assert st.get_stats().dedup_hits == n
    ids = [d[:16].tobytes().hex() for d in digests]
    outs = [torch.zeros(host.shape[1], dtype=torch.uint8, device=DEV)
            for _ in range(n)]
    found, sizes = st.get_batch(ids, outs)
    assert found.all() and (sizes == host.shape[1]).all()
    for i in range(n):
        assert torch.equal(outs[i], blocks[i])
    # the host API sees the same blocks under the same ids
    buf = np.zeros(host.shape[1], np.uint8)
    assert st.get(ids[3], buf) == (True, host.shape[1])
    assert np.array_equal(buf, host[3])


@pytest.mark.parametrize("side_stream", [False, True])
def test_batch_put_waits_for_callers_stream(side_stream):
    """The blocks' final bytes are written on the caller's stream behind a
    long sleep kernel; the put must hash and store those bytes, whether the
    caller's stream is torch's default stream (handle 0, the legacy default
    stream) or a stream of its own."""
    n = 8
    want = workloads.kv_blocks_torch(n, 11, DEV, layers=2)
    blocks = torch.zeros_like(want)
    torch.cuda.synchronize()
    side = torch.cuda.Stream(DEV) if side_stream else None
    st = make_store(use_gpu=True, gpu_cap=64 << 20)
    with torch.cuda.stream(side) if side is not None else torch.cuda.device(DEV):
        torch.cuda._sleep(200_000_000)          # ~0.1 s at 1.9 GHz
        blocks.copy_(want)
        stored, status, digests = st.put_batch(blocks, return_status=True)
    assert stored == n and (status == 0).all()
    host = want.cpu().numpy()
    for i in range(n):
        assert digests[i].tobytes() == hashlib.sha256(host[i].tobytes()).digest()


def test_device_batch_q8_roundtrip_matches_oracle():
    blocks = workloads.kv_blocks_torch(8, 9, DEV)                # 2 MiB each
    st = make_store(use_gpu=True, gpu_cap=256 << 20, kv_compression=True,
                    gpu_q8=True)
    stored, status, digests = st.put_batch(blocks, return_status=True)
    assert stored == 8
    host = blocks.cpu().numpy()
    ids = [d[:16].tobytes().hex() for d in digests]
    outs = [torch.zeros(host.shape[1], dtype=torch.uint8, device=DEV)
            for _ in range(8)]
    found, sizes = st.get_batch(ids, outs)
    for i in range(8):
        want = oracle.kv_decompress(oracle.kv_compress(host[i]), host.shape[1])
        assert np.array_equal(outs[i].cpu().numpy(), want)
    s = st.get_stats()
    assert s.gpu_used == 8 * host.shape[1] // 2     # HBM holds the INT8 half
    assert s.compression_savings_bytes == 8 * (host.shape[1] - (8 + host.shape[1] // 2))


def test_dedup_count_is_n_minus_distinct():
    seq, pre = workloads.dedup_sequence(2048, 17, pool=64, sessions=32,
                                        prefix_min=4, prefix_max=32)
    rng = np.random.default_rng(17)
    pool = torch.from_numpy(rng.integers(0, 256, (64, 8192), dtype=np.uint8)).to(DEV)
    uniq = torch.from_numpy(rng.integers(0, 256, (2048, 8192), dtype=np.uint8)).to(DEV)
    blocks = [pool[k] if k < 64 else uniq[k - 64] for k in seq]
    st = make_store(use_gpu=True, gpu_cap=256 << 20)
    stored, status, digests = st.put_batch(blocks, is_prefix=list(pre),
                                           return_status=True)
    distinct = len(np.unique(seq))
    assert stored == len(seq)
    assert (status == 0).sum() == distinct
    s = st.get_stats()
    assert s.dedup_hits == len(seq) - distinct
    assert s.gpu_used == distinct * 8192
    # first occurrence in sequence order is the stored one
    first = {}
    for i, k in enumerate(seq):
        first.setdefault(int(k), i)
    assert set(np.nonzero(status == 0)[0].tolist()) == set(first.values())


def test_host_batch_api_pinned_and_pageable():
    rng = np.random.default_rng(2)
    pageable = [rng.integers(0, 256, 70000, dtype=np.uint8) for _ in range(6)]
    pinned_t = [torch.from_numpy(b.copy()).pin_memory() for b in pageable[:3]]
    blocks = [t.numpy() for t in pinned_t] + pageable[3:]
    st = make_store(use_gpu=True)
    stored, status, digests = st.put_batch_host(blocks, return_status=True)
    assert stored == 6 and (status == 0).all()
    for b, d in zip(blocks, digests):
        assert d.tobytes() == hashlib.sha256(b.tobytes()).digest()
    buf = np.zeros(70000, np.uint8)
    for b, d in zip(blocks, digests):
        assert st.get(d[:16].tobytes().hex(), buf) == (True, 70000)
        assert np.array_equal(buf, b)


def test_raw_tier_classes():
    g = cc.GPUBackend(1 << 20)
    x = np.arange(300, dtype=np.uint8)
    assert g.put("a", x) and g.contains("a") and g.used_bytes() == 300
    buf = np.zeros(300, np.uint8)
    assert g.get("a", buf) == (True, 300) and np.array_equal(buf, x)
    g.clear()
    assert not g.contains("a") and g.used_bytes() == 0
    s = cc.ShmBackend(1 << 20)
    assert s.put("b", x) and s.used_bytes() == 300
    assert s.get("b", buf) == (True, 300) and np.array_equal(buf, x)


def test_clear_resets_everything():
    st = make_store(use_gpu=True)
    x = np.ones(1000, np.uint8)
    st.put("k1", x)
    st.put("k1", x)
    st.clear()
    s = st.get_stats()
    assert all(getattr(s, f) == 0 for f in cc._STAT_FIELDS)
    assert not st.contains("k1")
    assert st.put("k1", x) and st.get_stats().dedup_hits == 0


def test_threads_share_one_store():
    st = make_store(use_gpu=True)
    rng = np.random.default_rng(8)
    blocks = [rng.integers(0, 256, 3000, dtype=np.uint8) for _ in range(64)]
    errors = []

    def worker(lo):
        try:
            for i in range(lo, 64, 4):
                assert st.put(f"t{i}", blocks[i])
        except Exception as e:  # pragma: no cover
            errors.append(e)

    ts = [threading.Thread(target=worker, args=(k,)) for k in range(4)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errors
    buf = np.zeros(3000, np.uint8)
    for i in range(64):
        assert st.get(f"t{i}", buf) == (True, 3000)
        assert np.array_equal(buf, blocks[i])


def test_cuda_tensor_put_get_by_name():
    st = make_store(use_gpu=True)
    t = torch.arange(4096, device=DEV, dtype=torch.int16)
    assert st.put("tensor_block", t)
    out = torch.zeros(4096, device=DEV, dtype=torch.int16)
    assert st.get("tensor_block", out) == (True, 8192)
    assert torch.equal(out, t)


@pytest.mark.parametrize("form", ["rows", "2d"])
@pytest.mark.parametrize("size", [1000, 65536 + 100, (2 << 20) + 100])
def test_host_batch_striped_uniform_pinned(size, form):
    """Equal-size blocks in one pinned array stream to the GPU in stripes
    while SHA-256 advances stripe by stripe; the result must equal hashing
    whole blocks (OpenSSL) and store the same bytes.  The blocks are passed
    as a list of rows or as the 2-D array itself."""
    n = 24
    rng = np.random.default_rng(size)
    host = torch.from_numpy(rng.integers(0, 256, (n, size), dtype=np.uint8)).pin_memory()
    rows = [host.numpy()[i] for i in range(n)]
    rows[5] = rows[2]                       # a duplicate inside the batch
    host.numpy()[5] = host.numpy()[2]
    st = make_store(use_gpu=True, gpu_cap=256 << 20)
    stored, status, digests = st.put_batch_host(
        rows if form == "rows" else host.numpy(), return_status=True)
    assert stored == n
    assert status[5] == 2 and (np.delete(status, 5) == 0).all()
    for i in range(n):
        assert digests[i].tobytes() == hashlib.sha256(rows[i].tobytes()).digest()
    buf = np.zeros(size, np.uint8)
    for i in (0, 5, n - 1):
        assert st.get(digests[i][:16].tobytes().hex(), buf) == (True, size)
        assert np.array_equal(buf, rows[i])
    assert st.get_stats().dedup_hits == 1


@pytest.mark.parametrize("with_dram", [False, True])
def test_hbm_allocation_failure_falls_back(with_dram):
    """4097-byte blocks use 4608-byte pool classes: a pool sized by byte
    count cannot hold all of them.  The blocks that get no HBM slot go to the
    DRAM tier (as the reference falls back to SHM), or fail without one."""
    n = 16
    rng = np.random.default_rng(4)
    blocks = torch.from_numpy(rng.integers(0, 256, (n, 4097), dtype=np.uint8)).to(DEV)
    st = make_store(use_gpu=True, gpu_cap=n * 4097 + 100,
                    shm_cap=(1 << 20) if with_dram else 0)
    stored, status, digests = st.put_batch(blocks, return_status=True)
    in_hbm = (n * 4097 + 100) // 4608
    s = st.get_stats()
    assert s.gpu_used == in_hbm * 4097
    if with_dram:
        assert stored == n and (status == 0).all()
        assert s.shm_used == (n - in_hbm) * 4097 and s.shm_puts == n - in_hbm
    else:
        assert stored == in_hbm
        assert (status == 0).sum() == in_hbm and (status == 3).sum() == n - in_hbm
    buf = np.zeros(4097, np.uint8)
    host = blocks.cpu().numpy()
    for i in range(n):
        found, size = st.get(digests[i][:16].tobytes().hex(), buf)
        assert found == (status[i] == 0)
        if found:
            assert np.array_equal(buf, host[i])


def _stats(st):
    return stats_dict(st.get_stats())


def test_demotion_lru_with_prefix_protection():
    """HBM holds 8 blocks; 4 more evict the 4 least recently used non-prefix
    blocks to DRAM (raw bytes), prefix blocks and a recently read block stay."""
    S = 4096
    rng = np.random.default_rng(31)
    blocks = [rng.integers(0, 256, S, dtype=np.uint8) for _ in range(12)]
    ids = [oracle.block_id(b) for b in blocks]
    st = make_store(use_gpu=True, gpu_cap=8 * S, shm_cap=1 << 20,
                    promotion=False)
    for i in range(8):
        assert st.put(ids[i], blocks[i], is_prefix=i < 2)
    buf = np.zeros(S, np.uint8)
    assert st.get(ids[2], buf) == (True, S)          # touch block 2
    for i in range(8, 12):
        assert st.put(ids[i], blocks[i])
    s = _stats(st)
    assert s["gpu_evictions"] == 4
    assert s["gpu_used"] == 8 * S and s["shm_used"] == 4 * S
    hits = []
    for i in range(12):
        before = _stats(st)
        assert st.get(ids[i], buf) == (True, S)
        assert np.array_equal(buf, blocks[i])
        after = _stats(st)
        hits.append("gpu" if after["gpu_hits"] > before["gpu_hits"] else "shm")
    assert [i for i, h in enumerate(hits) if h == "shm"] == [3, 4, 5, 6]


def test_overflowing_batch_leaves_serial_end_state():
    """A batch of 12 blocks into an HBM tier that holds 8: the blocks left in
    HBM are the ones serial puts (each demoting the least recently used,
    prefix blocks last) would leave there, i.e. the batch's prefix blocks and
    its latest blocks, and every counter equals the serial puts' (4 GPU
    evictions: the batch's blocks that serial puts would have stored and
    demoted go to DRAM directly and count as evictions)."""
    S = 4096
    rng = np.random.default_rng(41)
    blocks = [rng.integers(0, 256, S, dtype=np.uint8) for _ in range(12)]
    ids = [oracle.block_id(b) for b in blocks]
    pre = [i in (0, 5) for i in range(12)]

    def tiers(st):
        buf = np.zeros(S, np.uint8)
        out = []
        for i in range(12):
            before = _stats(st)
            assert st.get(ids[i], buf) == (True, S)
            assert np.array_equal(buf, blocks[i])
            out.append("gpu" if _stats(st)["gpu_hits"] > before["gpu_hits"]
                       else "shm")
        return out

    serial = make_store(use_gpu=True, gpu_cap=8 * S, shm_cap=1 << 20,
                        promotion=False)
    for i in range(12):
        assert serial.put(ids[i], blocks[i], is_prefix=pre[i])
    assert _stats(serial)["gpu_evictions"] == 4
    batch = make_store(use_gpu=True, gpu_cap=8 * S, shm_cap=1 << 20,
                       promotion=False)
    rows = torch.from_numpy(np.stack(blocks)).to(DEV)
    stored, status, _ = batch.put_batch(rows, is_prefix=pre, return_status=True)
    assert stored == 12 and (status == 0).all()
    s = _stats(batch)
    assert s["gpu_used"] == 8 * S and s["shm_used"] == 4 * S
    assert s == _stats(serial)
    want = ["shm" if i in (1, 2, 3, 4) else "gpu" for i in range(12)]
    assert tiers(serial) == want
    assert tiers(batch) == want


@pytest.mark.parametrize("gpu_q8", [False, True])
def test_demotion_to_int8_dram_and_promotion(gpu_q8):
    """With kv_compression the DRAM tier holds INT8: demoted blocks come back
    dequantised (bit-exact with KVCompressor), and a DRAM hit is promoted
    back to HBM, demoting another block to make room."""
    blocks = workloads.kv_blocks_np(6, 77, layers=2)          # 128 KiB each
    S = blocks.shape[1]
    ids = [oracle.block_id(b) for b in blocks]
    hbm_per_block = S // 2 if gpu_q8 else S
    st = make_store(use_gpu=True, gpu_cap=4 * hbm_per_block, shm_cap=8 << 20,
                    kv_compression=True, gpu_q8=gpu_q8)
    for i in range(6):
        assert st.put(ids[i], blocks[i])
    s = _stats(st)
    assert s["gpu_evictions"] == 2 and s["gpu_used"] == 4 * hbm_per_block
    assert s["shm_used"] == 2 * (8 + S // 2)
    buf = np.zeros(S, np.uint8)
    for i in range(6):
        assert st.get(ids[i], buf) == (True, S)
        lossy = oracle.kv_decompress(oracle.kv_compress(blocks[i]), S)
        if i < 2 or gpu_q8:        # went through the INT8 form
            assert np.array_equal(buf, lossy), i
        else:
            # each promotion demotes the then least recently used HBM block,
            # so a later block may have been through the INT8 form as well
            assert np.array_equal(buf, blocks[i]) or np.array_equal(buf, lossy), i
    s = _stats(st)
    assert s["promotions_to_gpu"] >= 2
    assert s["gpu_used"] <= 4 * hbm_per_block


@pytest.mark.parametrize("semantic", [True, False], ids=["prefix", "lru"])
@pytest.mark.parametrize("kv_compression,gpu_q8",
                         [(False, False), (True, False), (True, True)],
                         ids=["raw", "int8-dram", "int8-hbm"])
def test_overflowing_batches_match_serial_model(kv_compression, gpu_q8,
                                                semantic):
    """Rounds of content-addressed batches (new blocks, repeats of earlier
    ones, prefix blocks) into an HBM tier of 16 blocks, each followed by
    single gets (which touch, and promote DRAM hits): after every round the
    counters, and every block's bytes and tier, equal the serial model's
    (oracle/store_model.py: each put demotes least recently used blocks,
    prefix blocks last, until it fits)."""
    S = 8192
    rng = np.random.default_rng(97 + 10 * kv_compression + gpu_q8 + 7 * semantic)
    universe = [rng.integers(0, 256, S, dtype=np.uint8) for _ in range(120)]
    ids = [oracle.block_id(b) for b in universe]
    hbm_per_block = S // 2 if gpu_q8 else S
    st = make_store(use_gpu=True, gpu_cap=16 * hbm_per_block, shm_cap=32 << 20,
                    kv_compression=kv_compression, gpu_q8=gpu_q8,
                    semantic=semantic)
    m = StoreModel(use_gpu=True, gpu_capacity=16 * hbm_per_block,
                   shm_capacity=32 << 20, kv_compression=kv_compression,
                   gpu_q8=gpu_q8, semantic_eviction=semantic)
    is_prefix = rng.random(120) < 0.2
    seen = []
    buf = np.zeros(S, np.uint8)
    for rnd in range(10):
        k = int(rng.integers(6, 26))
        fresh = list(range(12 * rnd, 12 * rnd + 12))
        picks = [int(rng.choice(fresh)) if (not seen or rng.random() < 0.7)
                 else int(rng.choice(seen)) for _ in range(k)]
        rows = torch.from_numpy(np.stack([universe[p] for p in picks])).to(DEV)
        pre = [bool(is_prefix[p]) for p in picks]
        stored, status, _ = st.put_batch(rows, is_prefix=pre,
                                         return_status=True)
        want = [m.put(ids[p], universe[p], is_prefix=q)
                for p, q in zip(picks, pre)]
        assert stored == sum(want), rnd
        seen.extend(picks)
        assert _stats(st) == m.stats, ("after put", rnd)
        for p in rng.choice(sorted(set(seen)), 5):
            got = st.get(ids[p], buf)
            mf, mdata = m.get(ids[p])
            assert got == (mf, S), (rnd, p)
            assert np.array_equal(buf, mdata), (rnd, p)
        assert _stats(st) == m.stats, ("after get", rnd)
    # every block: found, its bytes, and which tier answered
    for p in sorted(set(seen)):
        before = _stats(st)
        got = st.get(ids[p], buf)
        mf, mdata = m.get(ids[p])
        assert got == (mf, S) and np.array_equal(buf, mdata), p
        after = _stats(st)
        assert {f: after[f] - before[f] for f in ("gpu_hits", "shm_hits")} == \
            {f: m.stats[f] - before[f] for f in ("gpu_hits", "shm_hits")}, p
    assert _stats(st) == m.stats
