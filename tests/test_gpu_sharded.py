"""Sharded dedup on real GPUs (one process per GPU, NCCL): statuses equal
serial puts in (rank, block) order, hits total N - #distinct, and each rank
keeps exactly the bytes of the blocks it stored.  Needs two GPUs."""
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


def _rank_main(rank, world, port, out_dir):
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
        store = ShardedCascadeStore(cfg)
        res = []
        for batch in range(2):
            blocks = torch.from_numpy(np.stack(_blocks(rank, batch))).to(dev)
            stored, status, digests = store.put_batch(
                [blocks[i] for i in range(blocks.shape[0])], return_status=True)
            res.append({"stored": stored, "status": status.tolist(),
                        "digests": [d.tobytes().hex() for d in digests]})
        s = store.get_stats()
        res.append({"gpu_used": s.gpu_used, "dedup_hits": s.dedup_hits})
        with open(os.path.join(out_dir, f"r{rank}.json"), "w") as f:
            json.dump(res, f)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs 2 GPUs")
def test_sharded_put_two_gpus(tmp_path):
    import hashlib

    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(WORLD, _free_port(), str(tmp_path)),
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
    assert sum(r[-1]["dedup_hits"] for r in res) == total_hits
    assert [r[-1]["gpu_used"] for r in res] == stored_bytes
