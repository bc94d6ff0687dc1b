"""ORACLE — test infrastructure only.

A sequential Python model of the observable behaviour of the reference's
CascadeStore put/get (cascade_core.cpp:1074-1189) for the tiers this
library has: the GPU tier (raw bytes, GPUBackend::put/get,
gpu_backend.cu:266-344) and the DRAM tier (ShmBackend, cascade_core.cpp:
411-449, holding KVCompressor output when kv_compression is on).

It restates the reference's decisions step by step:
  put: dedup check against the known set (1077-1080) -> compress when
       kv_compression and size >= 64, counting the savings (1086-1092) ->
       GPU tier while used + size <= capacity (1097-1105; an id the tier
       already holds is "stored" without a copy, gpu_backend.cu:268-270) ->
       DRAM tier while used + stored size <= capacity (1108-1118) ->
       record known / prefix ids when dedup is on (1127-1132).
  get: GPU hit (1139-1143) -> DRAM hit, decompressed when kv_compression,
       promoted to the GPU tier when promotion is on (1145-1164) -> miss.

Where the reference has a defect this model states the corrected
behaviour the product implements, and says so:
  * a DRAM block stored raw (size < 64, or compression off when it was
    put) is returned raw; the reference "decompresses" any DRAM block when
    kv_compression is on (1149-1156), garbling those.
Demotion (evict_gpu_to_shm, 998-1018, from put 1100-1103 and promote_to_gpu
1039-1056) is modelled with this library's victim order, which differs from
the reference's: the least recently put or read GPU block first over the
whole tier (the reference takes the LRU tail of its largest index shard),
prefix blocks last when semantic_eviction and dedup are on; a demoted block
goes to the DRAM tier in the DRAM tier's format (KVCompressor output when
kv_compression applies; the reference demotes raw bytes), and a demotion
that finds the DRAM tier full ends that put's demotions (the reference
would push on to its Lustre tier, which is not modelled).

Pinned by tests/test_store_model.py against the compiled reference
(oracle/_ref) on the configurations the reference can run here
(use_gpu=False).
"""
from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field

import numpy as np

from . import kv_compress, kv_decompress

STAT_FIELDS = ("gpu_used", "shm_used", "gpu_hits", "shm_hits", "lustre_hits",
               "misses", "dedup_hits", "gpu_evictions", "shm_evictions",
               "promotions_to_gpu", "promotions_to_shm", "prefetch_completed",
               "compression_savings_bytes", "shm_puts", "lustre_puts")


@dataclass
class StoreModel:
    use_gpu: bool = True
    gpu_capacity: int = 32 << 30
    shm_capacity: int = 64 << 30
    kv_compression: bool = False
    dedup_enabled: bool = True
    promotion_enabled: bool = True
    semantic_eviction: bool = True
    gpu_q8: bool = False  # B200 extension: HBM keeps the INT8 form too
    # id -> bytes returned by get, least recently used first
    gpu: OrderedDict = field(default_factory=OrderedDict)
    gpu_comp: dict = field(default_factory=dict)  # id -> INT8 form (gpu_q8)
    shm: dict = field(default_factory=dict)     # id -> (payload, is_q8, orig)
    known: set = field(default_factory=set)
    prefix: set = field(default_factory=set)
    stats: dict = field(default_factory=lambda: {f: 0 for f in STAT_FIELDS})

    def _q8(self, size: int) -> bool:
        return self.kv_compression and size >= 64

    def _hbm_bytes(self, size: int) -> int:
        """GPU-tier bytes of a block: its size (the reference's raw tier), or
        the INT8 payload size/2 in the gpu_q8 extension."""
        return size // 2 if (self.gpu_q8 and self._q8(size)) else size

    def _gpu_store(self, block_id, data, comp):
        """Puts a block into the GPU tier (most recently used end)."""
        if self.gpu_q8 and comp is not None:
            self.gpu[block_id] = kv_decompress(comp, 2 * (data.size // 2))
            self.gpu_comp[block_id] = comp
        else:
            self.gpu[block_id] = data.copy()
        self.stats["gpu_used"] += self._hbm_bytes(data.size)

    def _victim(self):
        """The GPU block to demote next: least recently used first, prefix
        blocks last when prefix protection is on."""
        protect = self.semantic_eviction and self.dedup_enabled
        for bid in self.gpu:
            if not (protect and bid in self.prefix):
                return bid
        return next(iter(self.gpu), None)

    def _evict_gpu_to_shm(self, needed: int):
        """Demotes GPU blocks until `needed` GPU bytes are freed, while the
        DRAM tier has room (evict_gpu_to_shm, cascade_core.cpp:998-1018)."""
        if self.shm_capacity <= 0:
            return
        s = self.stats
        freed = 0
        while freed < needed:
            bid = self._victim()
            if bid is None:
                return
            data = self.gpu[bid]
            size = data.size
            if self._q8(size):
                payload = self.gpu_comp.get(bid)
                if payload is None:
                    payload = kv_compress(data)
                entry = (payload, True, size)
            else:
                entry = (data.copy(), False, size)
            if s["shm_used"] + entry[0].size > self.shm_capacity:
                return
            del self.gpu[bid]
            self.gpu_comp.pop(bid, None)
            hbm = self._hbm_bytes(size)
            s["gpu_used"] -= hbm
            freed += hbm
            self.shm[bid] = entry
            s["shm_used"] += entry[0].size
            s["gpu_evictions"] += 1

    def put(self, block_id: str, data: np.ndarray, is_prefix=False) -> bool:
        data = np.ascontiguousarray(data, dtype=np.uint8)
        size = data.size
        s = self.stats
        if self.dedup_enabled and block_id in self.known:
            s["dedup_hits"] += 1
            return True
        comp = None
        if self._q8(size):
            comp = kv_compress(data)
            s["compression_savings_bytes"] += size - comp.size
        stored = False
        if self.use_gpu and self.gpu_capacity > 0:
            hbm = self._hbm_bytes(size)
            if s["gpu_used"] + hbm > self.gpu_capacity:
                self._evict_gpu_to_shm(hbm)
            if s["gpu_used"] + hbm <= self.gpu_capacity:
                if block_id in self.gpu or block_id in self.shm:
                    stored = True
                else:
                    self._gpu_store(block_id, data, comp)
                    stored = True
        if not stored and self.shm_capacity > 0:
            acc = comp.size if comp is not None else size
            if block_id in self.shm:
                # ShmBackend::put answers true for an id it holds, and the
                # store counts that as an SHM put (cascade_core.cpp:1110-1111)
                stored = True
                s["shm_puts"] += 1
            elif block_id in self.gpu:
                stored = True
            elif s["shm_used"] + acc <= self.shm_capacity:
                self.shm[block_id] = (comp if comp is not None else data.copy(),
                                      comp is not None, size)
                s["shm_used"] += acc
                s["shm_puts"] += 1
                stored = True
        if stored and self.dedup_enabled:
            self.known.add(block_id)
            if is_prefix:
                self.prefix.add(block_id)
        return stored

    def get(self, block_id: str):
        """(found, bytes or None)."""
        s = self.stats
        if block_id in self.gpu:
            s["gpu_hits"] += 1
            self.gpu.move_to_end(block_id)
            return True, self.gpu[block_id]
        if block_id in self.shm:
            s["shm_hits"] += 1
            payload, q8, orig = self.shm[block_id]
            out = kv_decompress(payload, 2 * (orig // 2)) if q8 else payload
            if self.promotion_enabled and self.use_gpu and self.gpu_capacity > 0:
                hbm = self._hbm_bytes(out.size)
                if s["gpu_used"] + hbm > self.gpu_capacity:
                    self._evict_gpu_to_shm(hbm)
                if s["gpu_used"] + hbm <= self.gpu_capacity:
                    comp = kv_compress(out) if self._q8(out.size) else None
                    del self.shm[block_id]
                    s["shm_used"] -= payload.size
                    self._gpu_store(block_id, out, comp)
                    s["promotions_to_gpu"] += 1
            return True, out
        s["misses"] += 1
        return False, None

    def contains(self, block_id: str) -> bool:
        return block_id in self.gpu or block_id in self.shm
