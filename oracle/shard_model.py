"""ORACLE — test infrastructure only.

CPU stand-in for the three per-rank steps of the sharded PUT
(cascade_b200.sharded.CudaShardOps), with the same 64-byte record and
8-byte reply layouts, so the exchange protocol of ShardedCascadeStore can
be run on CPU ranks (gloo).  The dedup decision restates the reference's
rule (CascadeStore::put, cascade_core.cpp:1077-1080, applied to puts in
global (rank, block) order): a key already stored is a hit; among new keys
the first put stores and later ones are hits.
"""
from __future__ import annotations

import hashlib

import numpy as np

STORED, DUP_KNOWN, DUP_BATCH, FAILED = 0, 1, 2, 3
REC = np.dtype([("k0", "<u8"), ("k1", "<u8"), ("seq", "<u8"),
                ("offset", "<u8"), ("size", "<u8"), ("flags", "<u4"),
                ("holder", "<u4"), ("src_idx", "<u4"), ("hdr_scale", "<u4"),
                ("hdr_zp", "<u4"), ("pad", "<u4")])
REPLY = np.dtype([("src_idx", "<u4"), ("status", "<u4")])
assert REC.itemsize == 64 and REPLY.itemsize == 8


def owner_of(digest: bytes, world: int) -> int:
    return (digest[0] * world) >> 8


class CpuShardOps:
    def __init__(self):
        import torch
        self.device = torch.device("cpu")
        self.index = {}        # this rank's key slice: key -> seq of storer
        self._digests = None
        self.store = None

    def begin(self, blocks, is_prefix, world, rank, seq_base):
        import torch
        n = len(blocks)
        digests = [hashlib.sha256(np.ascontiguousarray(b).tobytes()).digest()
                   for b in blocks]
        recs = np.zeros(n, REC)
        owners = np.zeros(n, np.int64)
        for i, d in enumerate(digests):
            recs[i]["k0"] = int.from_bytes(d[:8], "little")
            recs[i]["k1"] = int.from_bytes(d[8:16], "little")
            recs[i]["seq"] = seq_base + i
            recs[i]["offset"] = i
            recs[i]["size"] = len(blocks[i])
            recs[i]["holder"] = rank
            recs[i]["src_idx"] = i
            owners[i] = owner_of(d, world)
        order = np.argsort(owners, kind="stable")
        counts = np.bincount(owners, minlength=world).tolist()
        send = torch.from_numpy(recs[order].view(np.uint8).reshape(n, 64).copy())
        self._digests = digests
        return send, counts

    def resolve(self, recv):
        import torch
        recs = recv.numpy().reshape(-1).view(REC) if recv.numel() else np.zeros(0, REC)
        m = len(recs)
        status = np.full(m, FAILED, np.uint32)
        seen = {}
        for j in np.argsort(recs["seq"], kind="stable"):
            key = (int(recs[j]["k0"]), int(recs[j]["k1"]))
            if key in self.index:
                status[j] = DUP_KNOWN
            elif key in seen:
                status[j] = DUP_BATCH
            else:
                seen[key] = int(recs[j]["seq"])
                status[j] = STORED
        self.index.update(seen)
        rep = np.zeros(m, REPLY)
        rep["src_idx"] = recs["src_idx"]
        rep["status"] = status
        return torch.from_numpy(rep.view(np.uint8).reshape(m, 8).copy())

    def end(self, back):
        rep = back.numpy().reshape(-1).view(REPLY) if back.numel() else np.zeros(0, REPLY)
        n = len(self._digests)
        status = np.full(n, FAILED, np.uint8)
        status[rep["src_idx"]] = rep["status"]
        digests = np.frombuffer(b"".join(self._digests), np.uint8).reshape(n, 32) \
            if n else np.zeros((0, 32), np.uint8)
        stored = int((status != FAILED).sum())
        return stored, status, digests


def serial_statuses(blocks_by_rank):
    """Reference outcome: puts in (rank, block) order against one set."""
    known, out = set(), []
    for blocks in blocks_by_rank:
        st = []
        for b in blocks:
            d = hashlib.sha256(np.ascontiguousarray(b).tobytes()).digest()[:16]
            st.append(DUP_KNOWN if d in known else STORED)
            known.add(d)
        out.append(st)
    return out
