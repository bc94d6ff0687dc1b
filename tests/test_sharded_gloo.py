"""The sharded-dedup exchange protocol (ShardedCascadeStore.put_batch) on
two CPU ranks over gloo, with the per-rank steps done by the oracle's CPU
stand-in: every rank's statuses must equal serial puts in (rank, block)
order, and the hit total must be N - #distinct."""
import hashlib
import json
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle.shard_model import DUP_BATCH, DUP_KNOWN, STORED, serial_statuses


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _blocks(rank, batch):
    # 40 blocks per rank per batch from a pool shared by both ranks, so some
    # keys repeat inside a batch, across ranks, and across batches.
    rng = np.random.default_rng(1000 + 10 * batch + rank)
    pool = np.random.default_rng(7).integers(0, 256, (24, 300), dtype=np.uint8)
    picks = rng.integers(0, 24 + 40, 40)
    own = rng.integers(0, 256, (40, 300), dtype=np.uint8)
    return [pool[p] if p < 24 else own[p - 24] for p in picks]


def _get_ids(world):
    ids = []
    for r in range(world):
        for b in _blocks(r, 0):
            ids.append(hashlib.sha256(b.tobytes()).hexdigest()[:32])
    return ids + ["ab" * 16]


def _rank_main(rank, world, port, out_dir):
    import torch.distributed as dist
    from cascade_b200.sharded import ShardedCascadeStore
    from oracle.shard_model import CpuShardOps
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        store = ShardedCascadeStore(ops=CpuShardOps(shared_dir=out_dir))
        res = []
        for batch in range(2):   # the second batch through the host form
            put = store.put_batch if batch == 0 else store.put_batch_host
            stored, status, digests = put(_blocks(rank, batch),
                                          return_status=True)
            res.append({"stored": stored, "status": status.tolist()})
        # every rank reads every block of batch 0 (held on any rank), an id
        # that was never stored, and one block into a too-small buffer
        ids = _get_ids(world)
        outs = [np.zeros(300, np.uint8) for _ in ids]
        outs[rank] = np.zeros(10, np.uint8)
        found, sizes = store.get_batch(ids, outs)
        res.append({"found": found.tolist(), "sizes": sizes.tolist(),
                    "sha": [hashlib.sha256(o.tobytes()).hexdigest()
                            for o in outs]})
        store.close()
        with open(os.path.join(out_dir, f"r{rank}.json"), "w") as f:
            json.dump(res, f)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_exchange_matches_serial_puts(tmp_path, world):
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path)),
             nprocs=world, join=True)
    results = [json.load(open(tmp_path / f"r{r}.json")) for r in range(world)]
    known_total = 0
    all_keys = set()
    for batch in range(2):
        blocks = [_blocks(r, batch) for r in range(world)]
        # serial outcome across batches: earlier batches count as known
        want = []
        known = set(all_keys)
        for r in range(world):
            st = []
            for b in blocks[r]:
                d = hashlib.sha256(b.tobytes()).digest()[:16]
                st.append(1 if d in known else 0)
                known.add(d)
            want.append(st)
        for r in range(world):
            got = results[r][batch]["status"]
            assert results[r][batch]["stored"] == len(got)
            # stored where the serial order stores; a hit otherwise (known
            # from an earlier batch or earlier in this one)
            assert [0 if s == STORED else 1 for s in got] == want[r]
            for s, w in zip(got, want[r]):
                if w:
                    assert s in (DUP_KNOWN, DUP_BATCH)
        all_keys = known
    n_total = sum(len(_blocks(r, b)) for r in range(world) for b in range(2))
    hits = sum(1 for r in range(world) for b in range(2)
               for s in results[r][b]["status"] if s != STORED)
    assert hits == n_total - len(all_keys)


def test_serial_model_helper():
    a = [np.zeros(4, np.uint8), np.ones(4, np.uint8)]
    b = [np.ones(4, np.uint8), np.full(4, 2, np.uint8)]
    assert serial_statuses([a, b]) == [[STORED, STORED], [DUP_KNOWN, STORED]]


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_get_reads_blocks_held_on_any_rank(tmp_path, world):
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path)),
             nprocs=world, join=True)
    ids = _get_ids(world)
    blocks = {hashlib.sha256(b.tobytes()).hexdigest()[:32]: b
              for r in range(world) for b in _blocks(r, 0)}
    for rank in range(world):
        got = json.load(open(tmp_path / f"r{rank}.json"))[-1]
        assert got["found"] == [1] * (len(ids) - 1) + [0]
        for i, k in enumerate(ids[:-1]):
            assert got["sizes"][i] == 300
            if i == rank:      # 10-byte buffer: reported, left untouched
                assert got["sha"][i] == hashlib.sha256(bytes(10)).hexdigest()
            else:
                assert got["sha"][i] == hashlib.sha256(blocks[k].tobytes()).hexdigest()
        assert got["sizes"][-1] == 0


def _uneven_main(rank, world, port, out_dir):
    import torch.distributed as dist
    from cascade_b200.sharded import ShardedCascadeStore
    from oracle.shard_model import CpuShardOps
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        store = ShardedCascadeStore(ops=CpuShardOps(shared_dir=out_dir))
        # rank 0 puts 20 blocks, every other rank an empty batch
        mine = _blocks(0, 0)[:20] if rank == 0 else []
        stored, status, _ = store.put_batch(mine, return_status=True)
        # rank 0 reads nothing; the others read rank 0's blocks plus ids that
        # were never stored
        if rank == 0:
            ids, outs = [], []
        else:
            ids = [hashlib.sha256(b.tobytes()).hexdigest()[:32]
                   for b in _blocks(0, 0)[:20]] + ["00" * 16, "ff" * 16]
            outs = [np.zeros(300, np.uint8) for _ in ids]
        found, sizes = store.get_batch(ids, outs)
        res = {"stored": stored, "status": status.tolist(),
               "found": found.tolist(), "sizes": sizes.tolist(),
               "sha": [hashlib.sha256(o.tobytes()).hexdigest() for o in outs]}
        store.close()
        with open(os.path.join(out_dir, f"u{rank}.json"), "w") as f:
            json.dump(res, f)
    finally:
        dist.destroy_process_group()


def test_sharded_uneven_and_empty_batches(tmp_path):
    world = 3
    mp.spawn(_uneven_main, args=(world, _free_port(), str(tmp_path)),
             nprocs=world, join=True)
    blocks = _blocks(0, 0)[:20]
    distinct = len({hashlib.sha256(b.tobytes()).digest()[:16] for b in blocks})
    r0 = json.load(open(tmp_path / "u0.json"))
    assert r0["stored"] == 20 and r0["status"].count(STORED) == distinct
    assert r0["found"] == [] and r0["sizes"] == []
    for rank in (1, 2):
        r = json.load(open(tmp_path / f"u{rank}.json"))
        assert r["stored"] == 0 and r["status"] == []
        assert r["found"] == [1] * 20 + [0, 0]
        assert r["sizes"] == [300] * 20 + [0, 0]
        for i, b in enumerate(blocks):
            assert r["sha"][i] == hashlib.sha256(b.tobytes()).hexdigest()
        assert r["sha"][20] == r["sha"][21] == hashlib.sha256(bytes(300)).hexdigest()


# ------------------------------------------------------------ failures
# Host-side fault injection: a rank's own step raises (a stand-in for an
# error code from the device), or a rank never joins.  Nothing here touches
# a GPU.

def _failing_ops(fail_step, fail_batch, out_dir):
    from oracle.shard_model import CpuShardOps

    class FailingOps(CpuShardOps):
        batch = 0

        def begin(self, *a):
            if fail_step == "begin" and self.batch == fail_batch:
                self.batch += 1
                raise RuntimeError("injected begin failure")
            return super().begin(*a)

        def records(self, cap):
            if fail_step == "records" and self.batch == fail_batch:
                self.batch += 1
                raise RuntimeError("injected records failure")
            return super().records(cap)

        def resolve(self, recv):
            if fail_step == "resolve" and self.batch == fail_batch:
                self.batch += 1          # end() does not run for this batch
                raise RuntimeError("injected resolve failure")
            return super().resolve(recv)

        def end(self, back):
            self.batch += 1
            return super().end(back)

    return FailingOps(shared_dir=out_dir)


def _failure_main(rank, world, port, out_dir, fail_step):
    import datetime

    import torch.distributed as dist
    from cascade_b200.sharded import ShardedCascadeStore
    from oracle.shard_model import CpuShardOps
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        ops = (_failing_ops(fail_step, 0, out_dir) if rank == 1
               else CpuShardOps(shared_dir=out_dir))
        store = ShardedCascadeStore(ops=ops)
        res = []
        for batch in range(2):
            try:
                stored, status, _ = store.put_batch(_blocks(rank, batch),
                                                    return_status=True)
                res.append({"status": status.tolist()})
            except RuntimeError as e:
                res.append({"error": str(e)})
        store.close()
        with open(os.path.join(out_dir, f"f{rank}.json"), "w") as f:
            json.dump(res, f)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fail_step", ["begin", "records", "resolve"])
def test_sharded_put_survives_a_failing_rank(tmp_path, fail_step):
    """Rank 1 fails in its first batch: it raises after both exchanges, the
    other ranks finish that batch (their blocks that rank 1 owns come back
    FAILED when rank 1 could not resolve them), and every rank's next batch
    works."""
    world = 3
    mp.spawn(_failure_main, args=(world, _free_port(), str(tmp_path),
                                  fail_step), nprocs=world, join=True)
    from oracle.shard_model import FAILED, owner_of
    res = [json.load(open(tmp_path / f"f{r}.json")) for r in range(world)]
    assert res[1][0] == {"error": f"injected {fail_step} failure"}
    for r in (0, 2):
        status = res[r][0]["status"]
        for b, s in zip(_blocks(r, 0), status):
            owner = owner_of(hashlib.sha256(b.tobytes()).digest(), world)
            if fail_step == "resolve" and owner == 1:
                assert s == FAILED
            else:
                assert s != FAILED
    for r in range(world):
        assert "status" in res[r][1]
        assert FAILED not in res[r][1]["status"]


def _absent_main(rank, world, port, out_dir):
    import datetime
    import time

    import torch.distributed as dist
    from cascade_b200.sharded import ShardedCascadeStore
    from oracle.shard_model import CpuShardOps
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    store = ShardedCascadeStore(ops=CpuShardOps(shared_dir=out_dir))
    if rank == 1:
        # leaves between steps: never calls put_batch
        with open(os.path.join(out_dir, "a1.json"), "w") as f:
            json.dump({"left": True}, f)
        time.sleep(8)
        return
    t0 = time.monotonic()
    try:
        store.put_batch(_blocks(rank, 0))
        outcome = "returned"
    except RuntimeError as e:
        outcome = "raised: " + str(e)[:80]
    with open(os.path.join(out_dir, "a0.json"), "w") as f:
        json.dump({"outcome": outcome, "seconds": time.monotonic() - t0}, f)


def test_sharded_put_raises_when_a_rank_never_joins(tmp_path):
    """A rank that leaves makes its peers' next collective end with the
    process group's timeout error instead of waiting for it."""
    mp.spawn(_absent_main, args=(2, _free_port(), str(tmp_path)), nprocs=2,
             join=True)
    got = json.load(open(tmp_path / "a0.json"))
    assert got["outcome"].startswith("raised"), got
    assert got["seconds"] < 30


def _sliced_main(rank, world, port, out_dir, per):
    import torch.distributed as dist
    from cascade_b200.sharded import ShardedCascadeStore
    from oracle.shard_model import CpuShardOps
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        store = ShardedCascadeStore(ops=CpuShardOps(shared_dir=out_dir,
                                                    slice_blocks=per[rank]))
        res = []
        for batch in range(2):
            put = store.put_batch if batch == 0 else store.put_batch_host
            stored, status, digests = put(_blocks(rank, batch),
                                          return_status=True)
            res.append({"stored": stored, "status": status.tolist(),
                        "digests": [bytes(d).hex() for d in digests]})
        store.close()
        with open(os.path.join(out_dir, f"s{rank}.json"), "w") as f:
            json.dump(res, f)
    finally:
        dist.destroy_process_group()


def test_sharded_sliced_puts_resolve_round_by_round(tmp_path):
    """Ranks whose batches do not fit their pools put them in slices, one
    exchange round per slice, and ranks with fewer slices (or none) put
    empty batches until the last rank is done: statuses equal serial puts
    in (round, rank, block) order, digests come back in block order, and
    the hit total is N - #distinct."""
    world, per = 3, [7, 16, None]
    mp.spawn(_sliced_main, args=(world, _free_port(), str(tmp_path), per),
             nprocs=world, join=True)
    res = [json.load(open(tmp_path / f"s{r}.json")) for r in range(world)]
    known, n_total = set(), 0
    for batch in range(2):
        blocks = [_blocks(r, batch) for r in range(world)]
        cuts = [list(range(0, len(blocks[r]), per[r] or len(blocks[r])))
                + [len(blocks[r])] for r in range(world)]
        want = [[None] * len(blocks[r]) for r in range(world)]
        for k in range(max(len(c) - 1 for c in cuts)):
            for r in range(world):
                if k + 1 >= len(cuts[r]):
                    continue
                for i in range(cuts[r][k], cuts[r][k + 1]):
                    d = hashlib.sha256(blocks[r][i].tobytes()).digest()[:16]
                    want[r][i] = 1 if d in known else 0
                    known.add(d)
        for r in range(world):
            got = res[r][batch]
            assert got["stored"] == len(blocks[r])
            assert [0 if s == STORED else 1 for s in got["status"]] == want[r]
            assert got["digests"] == [
                hashlib.sha256(b.tobytes()).hexdigest() for b in blocks[r]]
            n_total += len(blocks[r])
    hits = sum(1 for r in range(world) for b in range(2)
               for s in res[r][b]["status"] if s != STORED)
    assert hits == n_total - len(known)
