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
Eviction (1001-1018) and the Lustre tier are not modelled: scenarios that
use the model stay within capacity or expect the put to fail.

Pinned by tests/test_store_model.py against the compiled reference
(oracle/_ref) on the configurations the reference can run here
(use_gpu=False).
"""
from __future__ import annotations

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
    gpu_q8: bool = False  # B200 extension: HBM keeps the INT8 form too
    gpu: dict = field(default_factory=dict)     # id -> bytes returned by get
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
            if s["gpu_used"] + hbm <= self.gpu_capacity:
                if block_id in self.gpu or block_id in self.shm:
                    stored = True
                else:
                    if self.gpu_q8 and comp is not None:
                        self.gpu[block_id] = kv_decompress(comp, 2 * (size // 2))
                    else:
                        self.gpu[block_id] = data.copy()
                    s["gpu_used"] += hbm
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
            return True, self.gpu[block_id]
        if block_id in self.shm:
            s["shm_hits"] += 1
            payload, q8, orig = self.shm[block_id]
            out = kv_decompress(payload, 2 * (orig // 2)) if q8 else payload
            if self.promotion_enabled and self.use_gpu and self.gpu_capacity > 0:
                hbm = self._hbm_bytes(out.size)
                if s["gpu_used"] + hbm <= self.gpu_capacity:
                    if self.gpu_q8 and self._q8(out.size):
                        self.gpu[block_id] = kv_decompress(
                            kv_compress(out), 2 * (out.size // 2))
                    else:
                        self.gpu[block_id] = out.copy()
                    s["gpu_used"] += hbm
                    s["promotions_to_gpu"] += 1
                    del self.shm[block_id]
                    s["shm_used"] -= payload.size
            return True, out
        s["misses"] += 1
        return False, None

    def contains(self, block_id: str) -> bool:
        return block_id in self.gpu or block_id in self.shm
