"""Sharded dedup on real GPUs (one process per GPU, NCCL): statuses equal
serial puts in (rank, block) order, hits total N - #distinct, and each rank
keeps exactly the bytes of the blocks it stored.  Then every rank reads
every block, most of them held in the other GPU's pool (peer reads over
NVLink), and gets the stored bytes back: exactly, or, with INT8 HBM
blocks, the oracle's compress -> decompress of them.  Needs two GPUs."""
import hashlib
import json
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _blocks(rank, batch):
    rng = np.random.default_rng(2000 + 10 * batch + rank)
    pool = np.random.default_rng(9).integers(0, 256, (48, 65536), dtype=np.uint8)
    picks = rng.integers(0, 48 + 64, 96)
    own = rng.integers(0, 256, (96, 65536), dtype=np.uint8)
    return [pool[p] if p < 48 else own[p - 48] for p in picks]


def _get_ids(world):
    ids = []
    for r in range(world):
        for b in _blocks(r, 0):
            ids.append(hashlib.sha256(b.tobytes()).hexdigest()[:32])
    return ids + ["cd" * 16]


def _rank_main(rank, world, port, out_dir, q8):
    import datetime

    import torch.distributed as dist

    from cascade_b200 import cascade_cpp as cc
    from cascade_b200.sharded import ShardedCascadeStore
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        cfg = cc.CascadeConfig()
        cfg.gpu_device_id = rank
        cfg.gpu_capacity_bytes = 256 << 20
        cfg.shm_capacity_bytes = 0
        cfg.kv_compression = q8
        cfg.gpu_q8 = q8
        store = ShardedCascadeStore(cfg)
        res = []
        for batch in range(2):
            if batch == 0:       # device blocks
                blocks = torch.from_numpy(np.stack(_blocks(rank, batch))).to(dev)
                stored, status, digests = store.put_batch(
                    [blocks[i] for i in range(blocks.shape[0])],
                    return_status=True)
            else:                # pinned host rows: striped copy + hash
                rows = torch.from_numpy(np.stack(_blocks(rank, batch))).pin_memory()
                stored, status, digests = store.put_batch_host(
                    rows.numpy(), return_status=True)
            res.append({"stored": stored, "status": status.tolist(),
                        "digests": [d.tobytes().hex() for d in digests]})
        s = store.get_stats()
        res.append({"gpu_used": s.gpu_used, "dedup_hits": s.dedup_hits})
        ids = _get_ids(world)
        # first read: a list of outputs (one of them too small) and hex ids;
        # second read: one 2-D output tensor and the keys as an (n, 16) array
        outs = [torch.zeros(65536, dtype=torch.uint8, device=dev)
                for _ in ids]
        outs[rank] = torch.zeros(100, dtype=torch.uint8, device=dev)
        found, sizes = store.get_batch(ids, outs)
        res.append({"found": found.tolist(), "sizes": sizes.tolist(),
                    "sha": [hashlib.sha256(o.cpu().numpy().tobytes())
                            .hexdigest() for o in outs]})
        keys = np.frombuffer(b"".join(bytes.fromhex(k) for k in ids),
                             np.uint8).reshape(-1, 16)
        rows = torch.zeros((len(ids), 65536), dtype=torch.uint8, device=dev)
        found, sizes = store.get_batch(keys, rows)
        res.append({"found": found.tolist(), "sizes": sizes.tolist(),
                    "sha": [hashlib.sha256(r.cpu().numpy().tobytes())
                            .hexdigest() for r in rows]})
        s = store.get_stats()
        res.append({"gpu_hits": s.gpu_hits, "misses": s.misses})
        store.close()
        with open(os.path.join(out_dir, f"r{rank}.json"), "w") as f:
            json.dump(res, f)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
@pytest.mark.parametrize("q8", [False, True], ids=["raw", "int8"])
def test_sharded_put_get_two_gpus(tmp_path, q8):
    import torch.multiprocessing as mp

    import oracle
    mp.spawn(_rank_main, args=(WORLD, _free_port(), str(tmp_path), q8),
             nprocs=WORLD, join=True)
    res = [json.load(open(tmp_path / f"r{r}.json")) for r in range(WORLD)]
    known = set()
    total_hits = 0
    stored_bytes = [0] * WORLD
    for batch in range(2):
        for r in range(WORLD):
            got = res[r][batch]
            blocks = _blocks(r, batch)
            for i, b in enumerate(blocks):
                d = hashlib.sha256(b.tobytes()).digest()
                assert got["digests"][i] == d.hex()
                hit = d[:16] in known
                known.add(d[:16])
                assert (got["status"][i] != 0) == hit
                total_hits += hit
                stored_bytes[r] += 0 if hit else b.size
            assert got["stored"] == len(blocks)
    assert sum(r[2]["dedup_hits"] for r in res) == total_hits
    want_used = [b // 2 for b in stored_bytes] if q8 else stored_bytes
    assert [r[2]["gpu_used"] for r in res] == want_used
    # reads: every block of batch 0 from both ranks, plus a missing id
    ids = _get_ids(WORLD)
    blocks = {hashlib.sha256(b.tobytes()).hexdigest()[:32]: b
              for r in range(WORLD) for b in _blocks(r, 0)}
    for rank in range(WORLD):
        for rep, got in enumerate(res[rank][3:5]):
            assert got["found"] == [1] * (len(ids) - 1) + [0]
            assert got["sizes"] == [65536] * (len(ids) - 1) + [0]
            for i, k in enumerate(ids[:-1]):
                if i == rank and rep == 0:   # 100-byte buffer: untouched
                    assert got["sha"][i] == hashlib.sha256(bytes(100)).hexdigest()
                    continue
                b = blocks[k]
                want = oracle.kv_decompress(oracle.kv_compress(b), b.size) \
                    if q8 else b
                assert got["sha"][i] == hashlib.sha256(
                    np.ascontiguousarray(want).tobytes()).hexdigest(), (rank, i)
        hits = res[rank][5]      # the block that did not fit is no hit
        assert hits["gpu_hits"] == 2 * (len(ids) - 1) - 1
        assert hits["misses"] == 2


def _demote_blocks(rank, rnd):
    rng = np.random.default_rng(5000 + 10 * rnd + rank)
    shared = np.random.default_rng(77).integers(0, 256, (16, 65536),
                                                dtype=np.uint8)
    own = rng.integers(0, 256, (12, 65536), dtype=np.uint8)
    picks = [shared[int(p)] for p in rng.integers(0, 16, 4)]
    return list(own) + picks


def _demote_main(rank, world, port, out_dir, q8, fail_round=None):
    import datetime

    import torch.distributed as dist

    from cascade_b200 import cascade_cpp as cc
    from cascade_b200.sharded import ShardedCascadeStore
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        cfg = cc.CascadeConfig()
        cfg.gpu_device_id = rank
        hbm = 32768 if q8 else 65536
        cfg.gpu_capacity_bytes = 20 * hbm          # 20 blocks per GPU
        cfg.shm_capacity_bytes = 64 << 20
        cfg.dram_chunk_bytes = 4 << 20
        cfg.kv_compression = True
        cfg.gpu_q8 = q8
        store = ShardedCascadeStore(cfg)
        moves = []
        if fail_round is not None and rank == 1:
            # host-side injection: rank 1's begin raises in one round, after
            # its prepare demoted payloads whose keys rank 0 owns
            prepare, begin = store.ops.prepare, store.ops.begin
            state = {"rnd": 0}

            def counted_prepare(*a):
                m = prepare(*a)
                moves.append(m)
                return m

            def failing_begin(*a):
                if state["rnd"] == fail_round:
                    raise RuntimeError("injected begin failure")
                return begin(*a)
            store.ops.prepare, store.ops.begin = counted_prepare, failing_begin
        res = []
        for rnd in range(4):
            blocks = torch.from_numpy(np.stack(_demote_blocks(rank, rnd))).to(dev)
            try:
                stored, status, _ = store.put_batch(blocks, return_status=True)
                res.append({"stored": stored, "status": status.tolist()})
            except RuntimeError as e:
                res.append({"error": str(e)})
            if fail_round is not None and rank == 1:
                state["rnd"] += 1
        s = store.get_stats()
        res.append({"gpu_used": s.gpu_used, "gpu_evictions": s.gpu_evictions,
                    "shm_used": s.shm_used, "moves": moves})
        ids = []
        for r in range(world):
            for rnd in range(4):
                if (r, rnd) == (1, fail_round):
                    continue
                for b in _demote_blocks(r, rnd):
                    ids.append(hashlib.sha256(b.tobytes()).hexdigest()[:32])
        outs = torch.zeros((len(ids), 65536), dtype=torch.uint8, device=dev)
        found, sizes = store.get_batch(ids, outs)
        res.append({"found": found.tolist(), "sizes": sizes.tolist(),
                    "sha": [hashlib.sha256(o.cpu().numpy().tobytes())
                            .hexdigest() for o in outs]})
        store.close()
        with open(os.path.join(out_dir, f"d{rank}.json"), "w") as f:
            json.dump(res, f)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
@pytest.mark.parametrize("q8", [False, True], ids=["raw-hbm", "int8-hbm"])
def test_sharded_demotion_two_gpus(tmp_path, q8):
    """Pools of 20 blocks per GPU take 4 rounds of 16 blocks per rank: each
    rank demotes its least recently put payloads to its DRAM tier before a
    round (cascade_shard_put_prepare), the owners' entries follow them, and
    every rank then reads every block, from HBM or from the holder's DRAM
    tier (its own, or the other rank's shared arena), as the oracle's
    compress -> decompress of the stored bytes; the statuses still equal
    serial puts in (round, rank, block) order."""
    import torch.multiprocessing as mp

    import oracle
    mp.spawn(_demote_main, args=(WORLD, _free_port(), str(tmp_path), q8),
             nprocs=WORLD, join=True)
    res = [json.load(open(tmp_path / f"d{r}.json")) for r in range(WORLD)]
    known = set()
    for rnd in range(4):
        for r in range(WORLD):
            got = res[r][rnd]
            assert got["stored"] == 16
            for b, s in zip(_demote_blocks(r, rnd), got["status"]):
                d = hashlib.sha256(b.tobytes()).digest()[:16]
                assert (s != 0) == (d in known)
                known.add(d)
    assert sum(r[4]["gpu_evictions"] for r in res) > 0
    hbm = 32768 if q8 else 65536
    for r in res:
        assert r[4]["gpu_used"] <= 20 * hbm
    # INT8 in HBM, or demoted to the INT8 DRAM tier: the lossy form; a raw
    # HBM block that stayed in HBM: its own bytes
    want = {}
    for r in range(WORLD):
        for rnd in range(4):
            for b in _demote_blocks(r, rnd):
                k = hashlib.sha256(b.tobytes()).hexdigest()[:32]
                want[k] = {hashlib.sha256(np.ascontiguousarray(
                    oracle.kv_decompress(oracle.kv_compress(b), b.size))
                    .tobytes()).hexdigest()}
                if not q8:
                    want[k].add(hashlib.sha256(b.tobytes()).hexdigest())
    ids = [hashlib.sha256(b.tobytes()).hexdigest()[:32]
           for r in range(WORLD) for rnd in range(4)
           for b in _demote_blocks(r, rnd)]
    for rank in range(WORLD):
        got = res[rank][5]
        assert got["found"] == [1] * len(ids)
        assert got["sizes"] == [65536] * len(ids)
        for i, k in enumerate(ids):
            assert got["sha"][i] in want[k], (rank, i)
    # both ranks read the same bytes for every block
    assert res[0][5]["sha"] == res[1][5]["sha"]


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_sharded_demotion_survives_a_failed_begin(tmp_path):
    """As the demotion test, but rank 1's begin raises in round 2, after its
    prepare demoted payloads whose keys rank 0 owns.  Rank 1 still sends
    those relocation records in the failed round's exchange, so rank 0's
    entries follow the payloads to rank 1's DRAM tier before rank 1's later
    puts reuse the freed HBM: every block that was put reads back as the
    oracle's compress -> decompress of its bytes, on both ranks, and the
    statuses equal serial puts without rank 1's failed batch."""
    import torch.multiprocessing as mp

    import oracle
    fail_round = 2
    mp.spawn(_demote_main, args=(WORLD, _free_port(), str(tmp_path), True,
                                 fail_round), nprocs=WORLD, join=True)
    res = [json.load(open(tmp_path / f"d{r}.json")) for r in range(WORLD)]
    assert res[1][fail_round] == {"error": "injected begin failure"}
    assert res[1][4]["moves"][fail_round] > 0
    known = set()
    puts = [(r, rnd) for rnd in range(4) for r in range(WORLD)
            if (r, rnd) != (1, fail_round)]
    for r, rnd in puts:
        got = res[r][rnd]
        assert got["stored"] == 16
        for b, s in zip(_demote_blocks(r, rnd), got["status"]):
            d = hashlib.sha256(b.tobytes()).digest()[:16]
            assert (s != 0) == (d in known)
            known.add(d)
    want = {}
    for r, rnd in puts:
        for b in _demote_blocks(r, rnd):
            k = hashlib.sha256(b.tobytes()).hexdigest()[:32]
            want[k] = hashlib.sha256(np.ascontiguousarray(
                oracle.kv_decompress(oracle.kv_compress(b), b.size))
                .tobytes()).hexdigest()
    ids = [hashlib.sha256(b.tobytes()).hexdigest()[:32]
           for r in range(WORLD) for rnd in range(4)
           if (r, rnd) != (1, fail_round) for b in _demote_blocks(r, rnd)]
    for rank in range(WORLD):
        got = res[rank][5]
        assert got["found"] == [1] * len(ids)
        for i, k in enumerate(ids):
            assert got["sha"][i] == want[k], (rank, i)


def _sliced_main(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    from cascade_b200 import cascade_cpp as cc
    from cascade_b200.sharded import ShardedCascadeStore
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        cfg = cc.CascadeConfig()
        cfg.gpu_device_id = rank
        cfg.gpu_capacity_bytes = 20 * 32768        # 20 INT8 blocks per GPU
        cfg.shm_capacity_bytes = 64 << 20
        cfg.dram_chunk_bytes = 4 << 20
        cfg.kv_compression = True
        cfg.gpu_q8 = True
        store = ShardedCascadeStore(cfg)
        res = []
        # rank 0: one batch of 48 blocks (three pools' worth of slices), then
        # 16; rank 1: 16 blocks, then 48
        plan = [[0, 1, 2], [3]] if rank == 0 else [[0], [1, 2, 3]]
        for rnds in plan:
            mine = [b for rnd in rnds for b in _demote_blocks(rank, rnd)]
            blocks = torch.from_numpy(np.stack(mine)).to(dev)
            cuts, _ = store.ops.slices(blocks, False)
            stored, status, digests = store.put_batch(blocks,
                                                      return_status=True)
            res.append({"rnds": rnds, "cuts": cuts, "stored": stored,
                        "status": status.tolist(),
                        "digests": [bytes(d).hex() for d in digests]})
        s = store.get_stats()
        res.append({"gpu_used": s.gpu_used, "gpu_evictions": s.gpu_evictions})
        ids = [hashlib.sha256(b.tobytes()).hexdigest()[:32]
               for r in range(world) for rnd in range(4)
               for b in _demote_blocks(r, rnd)]
        outs = torch.zeros((len(ids), 65536), dtype=torch.uint8, device=dev)
        found, sizes = store.get_batch(ids, outs)
        res.append({"found": found.tolist(), "sizes": sizes.tolist(),
                    "sha": [hashlib.sha256(o.cpu().numpy().tobytes())
                            .hexdigest() for o in outs]})
        store.close()
        with open(os.path.join(out_dir, f"s{rank}.json"), "w") as f:
            json.dump(res, f)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_sharded_put_of_batches_larger_than_the_pool(tmp_path):
    """A batch of three pools' worth of blocks goes in slices that fit
    (cascade_shard_put_slices), hashed once in one launch and put with the
    digests (cascade_shard_put_begin_digests), one exchange round per
    slice; the other rank puts empty batches until it is done.  Statuses
    equal serial puts in (round, rank, block) order, digests are the
    blocks' SHA-256, and every block reads back, from HBM or a DRAM tier,
    as the oracle's compress -> decompress of its bytes."""
    import torch.multiprocessing as mp

    import oracle
    mp.spawn(_sliced_main, args=(WORLD, _free_port(), str(tmp_path)),
             nprocs=WORLD, join=True)
    res = [json.load(open(tmp_path / f"s{r}.json")) for r in range(WORLD)]
    assert res[0][0]["cuts"] == [0, 16, 32, 48] and res[1][0]["cuts"] == [0, 16]
    known = set()
    for put in range(2):
        blocks = [[b for rnd in res[r][put]["rnds"]
                   for b in _demote_blocks(r, rnd)] for r in range(WORLD)]
        cuts = [res[r][put]["cuts"] for r in range(WORLD)]
        want = [[None] * len(blocks[r]) for r in range(WORLD)]
        for k in range(max(len(c) - 1 for c in cuts)):
            for r in range(WORLD):
                if k + 1 < len(cuts[r]):
                    for i in range(cuts[r][k], cuts[r][k + 1]):
                        d = hashlib.sha256(blocks[r][i].tobytes()).digest()[:16]
                        want[r][i] = d in known
                        known.add(d)
        for r in range(WORLD):
            got = res[r][put]
            assert got["stored"] == len(blocks[r])
            assert [s != 0 for s in got["status"]] == want[r]
            assert got["digests"] == [hashlib.sha256(b.tobytes()).hexdigest()
                                      for b in blocks[r]]
    assert sum(r[2]["gpu_evictions"] for r in res) > 0
    for r in res:
        assert r[2]["gpu_used"] <= 20 * 32768
    want = {}
    for r in range(WORLD):
        for rnd in range(4):
            for b in _demote_blocks(r, rnd):
                k = hashlib.sha256(b.tobytes()).hexdigest()[:32]
                want[k] = hashlib.sha256(np.ascontiguousarray(
                    oracle.kv_decompress(oracle.kv_compress(b), b.size))
                    .tobytes()).hexdigest()
    ids = [hashlib.sha256(b.tobytes()).hexdigest()[:32]
           for r in range(WORLD) for rnd in range(4)
           for b in _demote_blocks(r, rnd)]
    for rank in range(WORLD):
        got = res[rank][3]
        assert got["found"] == [1] * len(ids)
        assert got["sizes"] == [65536] * len(ids)
        for i, k in enumerate(ids):
            assert got["sha"][i] == want[k], (rank, i)


def _single_main(rank, world, port, out_dir, sliced=False):
    import datetime

    import torch.distributed as dist

    from cascade_b200 import cascade_cpp as cc
    from cascade_b200.sharded import ShardedCascadeStore
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        cfg = cc.CascadeConfig()
        cfg.gpu_capacity_bytes = 20 * 32768        # 20 INT8 blocks
        cfg.shm_capacity_bytes = 64 << 20
        cfg.dram_chunk_bytes = 4 << 20
        cfg.kv_compression = True
        cfg.gpu_q8 = True
        store = ShardedCascadeStore(cfg)
        res = []
        if sliced:     # all four rounds' blocks in one batch of 4 slices
            mine = [b for rnd in range(4) for b in _demote_blocks(0, rnd)]
            blocks = torch.from_numpy(np.stack(mine)).to(dev)
            # a batch that fits the empty pool stays one round, even above
            # the 4/5 that slices fill; one that does not fit is cut
            assert store.ops.slices(blocks[:18], False)[0] == [0, 18]
            assert store.ops.slices(blocks[:21], False)[0] == [0, 16, 21]
            assert store.ops.slices(blocks, False)[0] == [0, 16, 32, 48, 64]
            stored, status, digests = store.put_batch(blocks,
                                                      return_status=True)
            assert stored == 64
            assert [bytes(d) for d in digests] == [
                hashlib.sha256(b.tobytes()).digest() for b in mine]
            for rnd in range(4):
                res.append({"stored": 16,
                            "status": status[16 * rnd:16 * rnd + 16].tolist()})
        else:
            for rnd in range(4):
                blocks = torch.from_numpy(
                    np.stack(_demote_blocks(0, rnd))).to(dev)
                stored, status, _ = store.put_batch(blocks, return_status=True)
                res.append({"stored": stored, "status": status.tolist()})
        s = store.get_stats()
        res.append({"gpu_used": s.gpu_used, "gpu_evictions": s.gpu_evictions})
        ids = [hashlib.sha256(b.tobytes()).hexdigest()[:32]
               for rnd in range(4) for b in _demote_blocks(0, rnd)]
        outs = torch.zeros((len(ids), 65536), dtype=torch.uint8, device=dev)
        found, sizes = store.get_batch(ids, outs)
        res.append({"found": found.tolist(), "sizes": sizes.tolist(),
                    "sha": [hashlib.sha256(o.cpu().numpy().tobytes())
                            .hexdigest() for o in outs]})
        store.close()
        with open(os.path.join(out_dir, "s0.json"), "w") as f:
            json.dump(res, f)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("sliced", [False, True],
                         ids=["four-puts", "one-sliced-put"])
def test_sharded_protocol_one_rank_with_demotion(tmp_path, sliced):
    """The whole sharded C path (prepare, begin, records, resolve, end,
    lookup, reads from HBM and from the DRAM tier) on one GPU as a world of
    one rank: a 20-block pool takes 4 rounds of 16 blocks, demoting before
    each, and every block reads back as the oracle's compress ->
    decompress; statuses equal serial puts.  The rounds are four puts, or
    one put of all 64 blocks that the store cuts into 4 slices, hashed in
    one launch and put with those digests."""
    import torch.multiprocessing as mp

    import oracle
    mp.spawn(_single_main, args=(1, _free_port(), str(tmp_path), sliced),
             nprocs=1, join=True)
    res = json.load(open(tmp_path / "s0.json"))
    known = set()
    for rnd in range(4):
        assert res[rnd]["stored"] == 16
        for b, s in zip(_demote_blocks(0, rnd), res[rnd]["status"]):
            d = hashlib.sha256(b.tobytes()).digest()[:16]
            assert (s != 0) == (d in known)
            known.add(d)
    assert res[4]["gpu_evictions"] > 0 and res[4]["gpu_used"] <= 20 * 32768
    blocks = [b for rnd in range(4) for b in _demote_blocks(0, rnd)]
    assert res[5]["found"] == [1] * len(blocks)
    for i, b in enumerate(blocks):
        want = oracle.kv_decompress(oracle.kv_compress(b), b.size)
        assert res[5]["sha"][i] == hashlib.sha256(want.tobytes()).hexdigest(), i
