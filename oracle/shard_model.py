"""ORACLE — test infrastructure only.

CPU stand-in for the per-rank steps of the sharded PUT and GET
(cascade_b200.sharded.CudaShardOps), with the same 64-byte record, 8-byte
reply, 32-byte query and 48-byte location layouts, so the exchange protocol
of ShardedCascadeStore can be run on CPU ranks (gloo).  The dedup decision
restates the reference's rule (CascadeStore::put, cascade_core.cpp:1077-1080,
applied to puts in global (rank, block) order): a key already stored is a
hit; among new keys the first put stores and later ones are hits.  For the
GET, a directory shared by the ranks stands in for the holders' HBM pools
(each holder writes the blocks it stored there, one file per key).
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
QUERY = np.dtype([("k0", "<u8"), ("k1", "<u8"), ("src_idx", "<u4"),
                  ("pad0", "<u4"), ("pad1", "<u8")])
LOCATION = np.dtype([("src_idx", "<u4"), ("found", "<u4"), ("flags", "<u4"),
                     ("holder", "<u4"), ("offset", "<u8"), ("size", "<u8"),
                     ("hdr_scale", "<u4"), ("hdr_zp", "<u4"), ("pad", "<u8")])
assert REC.itemsize == 64 and REPLY.itemsize == 8
assert QUERY.itemsize == 32 and LOCATION.itemsize == 48
TIER_HBM, FLAG_REMOTE = 1 << 2, 1 << 4


UNUSED = 0xffffffff     # src_idx of a padded entry that carries nothing


def owner_of(digest: bytes, world: int) -> int:
    return (digest[0] * world) >> 8


def _padded(entries, owners, world, cap):
    """`world` segments of `cap` entries, entries grouped by owner rank;
    the rest all 0xff bytes."""
    out = np.full(world * cap * entries.itemsize, 0xff, np.uint8)
    view = out.view(entries.dtype)
    for o in range(world):
        mine = entries[owners == o]
        assert len(mine) <= cap
        view[o * cap:o * cap + len(mine)] = mine
    return out.reshape(world * cap, entries.itemsize)


class CpuShardOps:
    def __init__(self, shared_dir=None, slice_blocks=None):
        import torch
        self.slice_blocks = slice_blocks
        self.device = torch.device("cpu")
        self.index = {}        # this rank's key slice: key -> (seq, holder, size)
        self._digests = None
        self._blocks = None
        self._rank = None
        self._world = None
        self._get_keys = None
        self.shared_dir = shared_dir
        self.store = None

    def slices(self, blocks, host):
        """Cut points of a put: slices of `slice_blocks` blocks when set
        (the stand-in for an HBM pool that holds that many), else one."""
        n = len(blocks)
        if not self.slice_blocks:
            return [0, n], None
        return list(range(0, n, self.slice_blocks)) + [n], None

    @staticmethod
    def part(blocks, desc, a, b, host):
        return blocks[a:b]

    def begin(self, blocks, is_prefix, world, rank):
        n = len(blocks)
        digests = [hashlib.sha256(np.ascontiguousarray(b).tobytes()).digest()
                   for b in blocks]
        recs = np.zeros(n, REC)
        owners = np.zeros(n, np.int64)
        for i, d in enumerate(digests):
            recs[i]["k0"] = int.from_bytes(d[:8], "little")
            recs[i]["k1"] = int.from_bytes(d[8:16], "little")
            recs[i]["seq"] = (rank << 32) + i + 1
            recs[i]["offset"] = i
            recs[i]["size"] = len(blocks[i])
            recs[i]["holder"] = rank
            recs[i]["src_idx"] = i
            owners[i] = owner_of(d, world)
        self._digests = digests
        self._blocks = [np.ascontiguousarray(b) for b in blocks]
        self._recs, self._owners, self._world = recs, owners, world

    def begin_host(self, blocks, is_prefix, world, rank):
        return self.begin(blocks, is_prefix, world, rank)

    def records(self, cap):
        import torch
        return torch.from_numpy(_padded(self._recs, self._owners,
                                        self._world, cap))

    def resolve(self, recv):
        import torch
        recs = recv.numpy().reshape(-1).view(REC) if recv.numel() else np.zeros(0, REC)
        m = len(recs)
        status = np.full(m, FAILED, np.uint32)
        seen = {}
        for j in np.argsort(recs["seq"], kind="stable"):
            if recs[j]["src_idx"] == UNUSED:
                status[j] = UNUSED
                continue
            key = (int(recs[j]["k0"]), int(recs[j]["k1"]))
            if key in self.index:
                status[j] = DUP_KNOWN
            elif key in seen:
                status[j] = DUP_BATCH
            else:
                seen[key] = (int(recs[j]["seq"]), int(recs[j]["holder"]),
                             int(recs[j]["size"]))
                status[j] = STORED
        self.index.update(seen)
        rep = np.zeros(m, REPLY)
        rep["src_idx"] = recs["src_idx"]
        rep["status"] = status
        return torch.from_numpy(rep.view(np.uint8).reshape(m, 8).copy())

    def end(self, back):
        rep = back.numpy().reshape(-1).view(REPLY) if back.numel() else np.zeros(0, REPLY)
        rep = rep[rep["src_idx"] != UNUSED]
        n = len(self._digests)
        assert sorted(rep["src_idx"].tolist()) == list(range(n)), \
            "every block gets one reply"
        status = np.full(n, FAILED, np.uint8)
        status[rep["src_idx"]] = rep["status"]
        digests = np.frombuffer(b"".join(self._digests), np.uint8).reshape(n, 32) \
            if n else np.zeros((0, 32), np.uint8)
        stored = int((status != FAILED).sum())
        if self.shared_dir is not None:   # this rank now holds these
            import os
            for i in np.nonzero(status == STORED)[0]:
                name = self._digests[i][:16].hex() + ".bin"
                with open(os.path.join(self.shared_dir, name), "wb") as f:
                    f.write(self._blocks[i].tobytes())
        self._blocks = None
        return stored, status, digests

    # ---------------------------------------------------------------- get
    def key(self, block_id) -> bytes:
        if isinstance(block_id, (bytes, bytearray)) and len(block_id) == 16:
            return bytes(block_id)
        return bytes.fromhex(block_id)

    def pool_handle(self) -> bytes:
        import torch.distributed as dist
        return bytes([dist.get_rank()]) * 64

    def prepare(self, blocks, host, world, rank):
        return 0              # no DRAM tier: nothing to demote, no moves

    def dram_name(self) -> bytes:
        return bytes(64)

    def attach(self, world, rank, handles: bytes, dram_names: bytes = None):
        assert handles == b"".join(bytes([r]) * 64 for r in range(world))
        self._world, self._rank = world, rank

    def detach(self):
        self._world = self._rank = None

    def get_begin(self, keys: bytes, world, cap):
        import torch
        n = len(keys) // 16
        q = np.zeros(n, QUERY)
        owners = np.zeros(n, np.int64)
        for i in range(n):
            k = keys[16 * i:16 * i + 16]
            q[i]["k0"] = int.from_bytes(k[:8], "little")
            q[i]["k1"] = int.from_bytes(k[8:], "little")
            q[i]["src_idx"] = i
            owners[i] = owner_of(k, world)
        self._get_keys = [keys[16 * i:16 * i + 16] for i in range(n)]
        return torch.from_numpy(_padded(q, owners, world, cap))

    def lookup(self, recv):
        import torch
        q = recv.numpy().reshape(-1).view(QUERY) if recv.numel() else np.zeros(0, QUERY)
        loc = np.zeros(len(q), LOCATION)
        for j, r in enumerate(q):
            loc[j]["src_idx"] = r["src_idx"]
            if r["src_idx"] == UNUSED:
                continue
            hit = self.index.get((int(r["k0"]), int(r["k1"])))
            if hit is None:
                continue
            _, holder, size = hit
            loc[j]["found"] = 1
            loc[j]["holder"] = holder
            loc[j]["size"] = size
            loc[j]["flags"] = TIER_HBM | (FLAG_REMOTE if holder != self._rank else 0)
        return torch.from_numpy(loc.view(np.uint8).reshape(len(q), 48).copy())

    def get_end(self, back, outs):
        import os
        loc = back.numpy().reshape(-1).view(LOCATION) if back.numel() else np.zeros(0, LOCATION)
        loc = loc[loc["src_idx"] != UNUSED]
        n = len(outs)
        found = np.zeros(n, np.uint8)
        sizes = np.zeros(n, np.uint64)
        assert sorted(loc["src_idx"].tolist()) == list(range(n))
        for r in loc:
            i = int(r["src_idx"])
            if not r["found"]:
                continue
            found[i] = 1
            sizes[i] = r["size"]
            if r["size"] > len(outs[i]):
                continue
            name = self._get_keys[i].hex() + ".bin"
            with open(os.path.join(self.shared_dir, name), "rb") as f:
                data = np.frombuffer(f.read(), np.uint8)
            assert len(data) == r["size"]
            outs[i][:len(data)] = data
        return found, sizes


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
