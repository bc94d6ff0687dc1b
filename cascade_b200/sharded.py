"""Content-addressed PUT with the dedup index sharded across the GPUs of one
box (one process per GPU, torch.distributed for the exchange).

The reference's multi-node store keeps a replicated dedup set per rank and
reconciles it with MPI_Allgatherv (DistributedStore::put and
sync_metadata, distributed_backend.cpp:583-590, 1269-1324).  Here every key
has exactly one owner rank (the top bits of SHA-256 digest byte 0) and a
batch is exact at once:

1. every rank hashes its blocks and stores them speculatively in its own
   HBM pool (``cascade_shard_put_begin``); while the hash runs, one small
   all-gather of the batch sizes gives ``cap``, the largest batch of any
   rank, and ``cascade_shard_put_records`` then writes one 64-byte record
   per block into its owner rank's segment of a padded send buffer
   (``world`` segments of ``cap`` entries);
2. the records go to their owners in one all-to-all with equal splits
   (NCCL on GPUs), with no host round trip for counts;
3. each owner resolves the records it received against its slice of the
   index (``cascade_shard_resolve``): a key already stored is a dedup hit,
   and among new keys the smallest sequence number ((rank, block) packed in
   64 bits) stores, which is what serial puts in (rank, block) order would
   do;
4. the 8-byte replies return in a second all-to-all and each rank frees the
   slots of its duplicates (``cascade_shard_put_end``).

Block payloads never leave the rank that produced them until they are read.
``get_batch`` reads any block from any rank (the reference's remote read,
DistributedStore::get, distributed_backend.cpp:673-767): keys go to their
owners in one all-to-all, each owner answers with the block's location
(holder rank, pool offset, size, INT8 header), and each rank copies or
dequantises the payloads straight out of the holders' HBM pools, which every
rank maps at construction (CUDA IPC; the reads cross NVLink).

Every rank must call ``put_batch``, ``get_batch``, ``clear`` and ``close``
the same number of times, in the same order.
"""
from __future__ import annotations

import ctypes
import threading
from typing import Optional, Sequence

import numpy as np

from . import _lib
from ._lib import check
from .cascade_cpp import CascadeConfig, CascadeStore, _cuda_u8

RECORD_BYTES = 64
REPLY_BYTES = 8
QUERY_BYTES = 32
LOCATION_BYTES = 48
IPC_HANDLE_BYTES = 64
DRAM_NAME_BYTES = 64

_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_u64 = ctypes.c_uint64
_int = ctypes.c_int
_lib.register("cascade_shard_put_begin", _int,
              [_vp, _sz, _vp, _vp, _vp, _int, _int, _vp])
_lib.register("cascade_shard_put_begin_host", _int,
              [_vp, _sz, _vp, _vp, _vp, _int, _int, _vp])
_lib.register("cascade_shard_put_begin_digests", _int,
              [_vp, _sz, _vp, _vp, _vp, _vp, _int, _int, _vp])
_lib.register("cascade_shard_put_slices", _int,
              [_vp, _sz, _vp, _vp, ctypes.POINTER(_u64)])
_lib.register("cascade_shard_put_records", _int, [_vp, _sz, _vp, _vp])
_lib.register("cascade_shard_resolve", _int, [_vp, _vp, _sz, _vp, _vp])
_lib.register("cascade_shard_put_end", _int,
              [_vp, _vp, _sz, _sz, _vp, _vp, ctypes.POINTER(_u64), _vp])
_lib.register("cascade_shard_pool_handle", _int, [_vp, _vp])
_lib.register("cascade_shard_attach_pools", _int,
              [_vp, _int, _int, _vp, _vp])
_lib.register("cascade_shard_dram_name", _int, [_vp, _vp])
_lib.register("cascade_shard_put_prepare", _int,
              [_vp, _sz, _vp, _int, _int, ctypes.POINTER(_u64)])
_lib.register("cascade_shard_detach_pools", _int, [_vp])
_lib.register("cascade_shard_get_begin", _int, [_vp, _sz, _vp, _sz, _vp, _vp])
_lib.register("cascade_shard_lookup", _int, [_vp, _vp, _sz, _vp, _vp])
_lib.register("cascade_shard_get_end", _int,
              [_vp, _vp, _sz, _sz, _vp, _vp, _vp, _vp, ctypes.POINTER(_u64),
               _vp])

# Byte offset of src_idx in a record (the first 32-bit field after k0, k1,
# seq, offset, size, flags, holder).
_RECORD_SRC = 48
_PUT_FAILED = 3


def unused(rows: int, width: int, device):
    """A padded exchange buffer of `rows` entries that carry nothing."""
    import torch
    return torch.full((rows, width), 0xff, dtype=torch.uint8, device=device)


def failed_replies(recv):
    """The replies an owner sends when it could not resolve `recv`: every
    record it received fails (the holders free those blocks' slots)."""
    import torch
    reply = unused(recv.shape[0], REPLY_BYTES, recv.device)
    src = recv[:, _RECORD_SRC:_RECORD_SRC + 4]
    used = (src != 0xff).any(dim=1)
    reply[:, 0:4] = src
    code = torch.tensor([_PUT_FAILED, 0, 0, 0], dtype=torch.uint8,
                        device=recv.device)
    reply[used, 4:8] = code
    return reply


class CudaShardOps:
    """The three per-rank steps on this rank's GPU, through the C ABI."""

    def __init__(self, store: CascadeStore):
        import torch
        self.store = store
        self.device = torch.device("cuda", store._device)
        self._n = 0

    def _stream(self):
        import torch
        return torch.cuda.current_stream(self.device).cuda_stream

    @staticmethod
    def _describe(blocks):
        """Device blocks -> (addresses, sizes, what to keep alive)."""
        import torch
        if isinstance(blocks, tuple):    # (device addresses, sizes)
            ptrs = np.ascontiguousarray(blocks[0], dtype=np.uint64)
            sizes = np.ascontiguousarray(blocks[1], dtype=np.uint64)
            return ptrs, sizes, None     # the caller keeps the blocks alive
        if isinstance(blocks, torch.Tensor) and blocks.dim() == 2:
            rows = blocks.contiguous()   # one block per row
            n = rows.shape[0]
            stride = rows.stride(0) * rows.element_size()
            ptrs = (np.arange(n, dtype=np.uint64) * np.uint64(stride)
                    + np.uint64(rows.data_ptr()))
            sizes = np.full(n, rows.shape[1] * rows.element_size(), np.uint64)
            return ptrs, sizes, rows
        blocks = [_cuda_u8(b) for b in blocks]
        ptrs = np.array([b.data_ptr() for b in blocks], dtype=np.uint64)
        sizes = np.array([b.numel() for b in blocks], dtype=np.uint64)
        return ptrs, sizes, blocks

    @staticmethod
    def _describe_host(blocks):
        """Host blocks -> (addresses, sizes, what to keep alive)."""
        if isinstance(blocks, np.ndarray) and blocks.ndim == 2:
            n = blocks.shape[0]
            ptrs = (np.arange(n, dtype=np.uint64) * np.uint64(blocks.strides[0])
                    + np.uint64(blocks.ctypes.data))
            return ptrs, np.full(n, blocks.shape[1], np.uint64), blocks
        arrs = [np.ascontiguousarray(b, dtype=np.uint8).reshape(-1)
                for b in blocks]
        ptrs = np.array([a.ctypes.data for a in arrs], dtype=np.uint64)
        sizes = np.array([a.size for a in arrs], dtype=np.uint64)
        return ptrs, sizes, arrs

    def prepare(self, blocks, host, world, rank):
        """Room in this rank's pool for the batch (demoting to the DRAM
        tier); returns how many relocation records the records step sends,
        those a failed put left pending included.  Without a DRAM tier
        there is nothing to do."""
        self._desc = (self._describe_host if host else self._describe)(blocks)
        self._n, self._world = 0, world
        if not self.store._cfg.shm_capacity_bytes:
            return 0
        sizes = self._desc[1]
        n = len(sizes)
        moves = _u64(0)
        check(_lib.load().cascade_shard_put_prepare(
            self.store._h, n, sizes.ctypes.data if n else None, world, rank,
            ctypes.byref(moves)))
        return int(moves.value)

    def _begin(self, fn, desc, is_prefix, world, rank, digests=None):
        ptrs, sizes, keep = desc
        n = len(ptrs)
        pf = (np.array([1 if p else 0 for p in is_prefix], dtype=np.uint8)
              if is_prefix is not None else None)
        self._keep = keep
        self._n = 0
        extra = () if digests is None else (
            digests.data_ptr() if n else None,)
        check(fn(self.store._h, n, ptrs.ctypes.data if n else None,
                 sizes.ctypes.data if n else None,
                 pf.ctypes.data if pf is not None else None, *extra, world,
                 rank, self._stream()))
        self._n = n
        self._world = world

    def slices(self, blocks, host):
        """Cut points of a batch that is put in slices, each fitting the
        HBM pool (over a DRAM tier), and the batch's description.  Without
        a DRAM tier a batch is one slice."""
        if not self.store._cfg.shm_capacity_bytes:
            return [0, len(blocks[0]) if isinstance(blocks, tuple)
                    else len(blocks)], None
        desc = (self._describe_host if host else self._describe)(blocks)
        sizes = desc[1]
        n = len(sizes)
        cuts = np.zeros(max(n, 1) + 1, np.uint64)
        k = _u64(0)
        check(_lib.load().cascade_shard_put_slices(
            self.store._h, n, sizes.ctypes.data if n else None,
            cuts.ctypes.data, ctypes.byref(k)))
        return [int(c) for c in cuts[:k.value + 1]], desc

    @staticmethod
    def part(blocks, desc, a, b, host):
        """Blocks a..b-1 of a batch that slices() described."""
        if host:
            return blocks[a:b]
        return desc[0][a:b], desc[1][a:b]

    def digests(self, desc):
        """SHA-256 of a described device batch in one launch (all its
        chains at once), as a (n, 32) uint8 tensor on this GPU."""
        import torch
        ptrs, sizes, _ = desc
        n = len(ptrs)
        d_ptrs = torch.from_numpy(ptrs.view(np.int64)).to(self.device)
        d_sizes = torch.from_numpy(sizes.view(np.int64)).to(self.device)
        out = torch.empty((n, 32), dtype=torch.uint8, device=self.device)
        check(_lib.load().cascade_sha256_batch(
            d_ptrs.data_ptr(), d_sizes.data_ptr(), n, out.data_ptr(),
            self._stream()))
        return out

    def _described(self, blocks, describe):
        """prepare's description of these blocks, or a new one."""
        desc, self._desc = getattr(self, "_desc", None), None
        return desc if desc is not None else describe(blocks)

    def begin(self, blocks, is_prefix, world, rank, digests=None):
        """Hashes (unless `digests` holds the batch's digests, a device
        tensor) and stores the batch speculatively (returns at once)."""
        if digests is None:
            self._begin(_lib.load().cascade_shard_put_begin,
                        self._described(blocks, self._describe), is_prefix,
                        world, rank)
        else:
            self._begin(_lib.load().cascade_shard_put_begin_digests,
                        self._described(blocks, self._describe), is_prefix,
                        world, rank, digests)

    def begin_host(self, blocks, is_prefix, world, rank):
        """begin for host blocks: a list of uint8 numpy arrays, or one 2-D
        uint8 array (pinned rows are staged fastest)."""
        self._begin(_lib.load().cascade_shard_put_begin_host,
                    self._described(blocks, self._describe_host), is_prefix,
                    world, rank)

    def records(self, cap):
        """The batch's records for `world` segments of `cap` entries (a
        device tensor, ready on the current stream)."""
        import torch
        send = torch.empty((self._world * cap, RECORD_BYTES),
                           dtype=torch.uint8, device=self.device)
        check(_lib.load().cascade_shard_put_records(
            self.store._h, cap, send.data_ptr(), self._stream()))
        return send

    def resolve(self, recv):
        import torch
        m = recv.shape[0]
        reply = torch.empty((m, REPLY_BYTES), dtype=torch.uint8,
                            device=self.device)
        check(_lib.load().cascade_shard_resolve(
            self.store._h, recv.data_ptr() if m else None, m,
            reply.data_ptr() if m else None, self._stream()))
        return reply

    def end(self, back):
        n, m = self._n, back.shape[0]
        status = np.zeros(n, np.uint8)
        digests = np.zeros((n, 32), np.uint8)
        stored = _u64(0)
        self._n = 0
        try:
            check(_lib.load().cascade_shard_put_end(
                self.store._h, back.data_ptr() if m else None, m, n,
                status.ctypes.data if n else None,
                digests.ctypes.data if n else None, ctypes.byref(stored),
                self._stream()))
        finally:
            self._keep = None
        return int(stored.value), status, digests

    # ---------------------------------------------------------------- get
    def key(self, block_id) -> bytes:
        return self.store._key(block_id)

    def pool_handle(self) -> bytes:
        buf = (ctypes.c_uint8 * IPC_HANDLE_BYTES)()
        check(_lib.load().cascade_shard_pool_handle(self.store._h, buf))
        return bytes(buf)

    def dram_name(self) -> bytes:
        buf = (ctypes.c_uint8 * DRAM_NAME_BYTES)()
        check(_lib.load().cascade_shard_dram_name(self.store._h, buf))
        return bytes(buf)

    def attach(self, world, rank, handles: bytes, dram_names: bytes = None):
        check(_lib.load().cascade_shard_attach_pools(
            self.store._h, world, rank, handles, dram_names))

    def detach(self):
        check(_lib.load().cascade_shard_detach_pools(self.store._h))

    def get_begin(self, keys: bytes, world, cap):
        import torch
        n = len(keys) // 16
        send = torch.empty((world * cap, QUERY_BYTES), dtype=torch.uint8,
                           device=self.device)
        kbuf = np.frombuffer(keys, np.uint8) if n else None
        check(_lib.load().cascade_shard_get_begin(
            self.store._h, n, kbuf.ctypes.data if n else None, cap,
            send.data_ptr(), self._stream()))
        return send

    def lookup(self, recv):
        import torch
        m = recv.shape[0]
        reply = torch.empty((m, LOCATION_BYTES), dtype=torch.uint8,
                            device=self.device)
        check(_lib.load().cascade_shard_lookup(
            self.store._h, recv.data_ptr() if m else None, m,
            reply.data_ptr() if m else None, self._stream()))
        return reply

    def get_end(self, back, outs):
        import torch
        if isinstance(outs, torch.Tensor) and outs.dim() == 2:
            if not outs.is_contiguous() or outs.device != self.device:
                raise ValueError("outs: a contiguous 2-D tensor on this GPU")
            n = outs.shape[0]
            row = outs.stride(0) * outs.element_size()
            ptrs = (np.arange(n, dtype=np.uint64) * np.uint64(row)
                    + np.uint64(outs.data_ptr()))
            caps = np.full(n, outs.shape[1] * outs.element_size(), np.uint64)
        else:
            outs = [_cuda_u8(o) for o in outs]
            n = len(outs)
            ptrs = np.array([o.data_ptr() for o in outs], dtype=np.uint64)
            caps = np.array([o.numel() for o in outs], dtype=np.uint64)
        sizes = np.zeros(n, np.uint64)
        found = np.zeros(n, np.uint8)
        nf = _u64(0)
        m = back.shape[0]
        check(_lib.load().cascade_shard_get_end(
            self.store._h, back.data_ptr() if m else None, m, n,
            ptrs.ctypes.data if n else None, caps.ctypes.data if n else None,
            sizes.ctypes.data if n else None, found.ctypes.data if n else None,
            ctypes.byref(nf), self._stream()))
        return found, sizes


class ShardedCascadeStore:
    """One rank's view of a store whose dedup index is sharded by key over
    the ranks of ``group``.  ``ops`` defaults to the GPU implementation."""

    def __init__(self, config: Optional[CascadeConfig] = None, group=None,
                 ops=None):
        import torch.distributed as dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if ops is None:
            self.store = CascadeStore(config)
            ops = CudaShardOps(self.store)
        self.ops = ops
        self._lock = threading.Lock()
        self._attached = False
        self._attach()

    def _attach(self):
        """Collective: every rank maps the other ranks' pools and DRAM
        tiers."""
        import torch
        import torch.distributed as dist
        if not hasattr(self.ops, "attach"):
            return
        rec = self.ops.pool_handle() + self.ops.dram_name()
        mine = torch.frombuffer(bytearray(rec),
                                dtype=torch.uint8).to(self.ops.device)
        every = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(every, mine, group=self.group)
        recs = [bytes(t.cpu().numpy().tobytes()) for t in every]
        handles = b"".join(r[:IPC_HANDLE_BYTES] for r in recs)
        names = b"".join(r[IPC_HANDLE_BYTES:] for r in recs)
        self.ops.attach(self.world, self.rank, handles, names)
        self._attached = True

    def put_batch(self, blocks: Sequence, is_prefix=None,
                  return_status: bool = False):
        """Collective: every rank calls it with its own blocks (a list of
        CUDA tensors, one 2-D CUDA tensor with a block per row, or a tuple
        (device addresses, sizes) of uint64 arrays for blocks on this rank's
        GPU that the caller keeps alive until the call returns).  Returns
        the number of this rank's blocks stored or deduplicated (and, with
        ``return_status``, per-block status codes and 32-byte digests)."""
        n = len(blocks[0]) if isinstance(blocks, tuple) else len(blocks)
        return self._put(False, blocks, n, is_prefix, return_status)

    def put_batch_host(self, blocks, is_prefix=None,
                       return_status: bool = False):
        """put_batch for blocks in host memory (a list of uint8 numpy arrays,
        or one 2-D uint8 array with a block per row).  Pinned rows of one
        size are copied to the GPU in stripes and hashed as they land."""
        return self._put(True, blocks, len(blocks), is_prefix, return_status)

    def _sizes(self, n, extra=0, more=0):
        """Collective: every rank's (batch size, extra records, more slices
        to come), in one small all-gather."""
        import torch
        import torch.distributed as dist
        mine = torch.tensor([n, extra, more], dtype=torch.int64,
                            device=self.ops.device)
        every = torch.zeros(3 * self.world, dtype=torch.int64,
                            device=self.ops.device)
        dist.all_gather_into_tensor(every, mine, group=self.group)
        v = [int(x) for x in every.tolist()]
        return list(zip(v[0::3], v[1::3], v[2::3]))

    def _put(self, host, blocks, n, is_prefix, return_status):
        """A put in one or more rounds of the exchange.  A batch whose
        payloads do not fit this rank's HBM pool (over a DRAM tier) goes in
        slices that do, one round each; a device batch is hashed in one
        launch first, so that all its chains run at once.  Every round's
        size all-gather carries a flag for more slices to come, and the
        ranks run rounds (with empty batches once theirs is done) until no
        rank has more.  Keys resolve in (round, rank, block) order.

        A rank whose own step fails still takes part in every exchange and
        raises once the rounds are over, so its peers never wait on it."""
        with self._lock:
            cuts, desc, digests = [0, n], None, None
            if n and hasattr(self.ops, "slices"):
                cuts, desc = self.ops.slices(blocks, host)
            error = None
            if len(cuts) > 2 and not host and hasattr(self.ops, "digests"):
                try:
                    digests = self.ops.digests(desc)
                except Exception as e:   # noqa: BLE001 (re-raised below)
                    error = e
            parts, k = [], 0
            while True:
                a, b = (cuts[k], cuts[k + 1]) if k + 1 < len(cuts) else (n, n)
                if a == b:
                    part = []            # this rank's slices are done
                elif len(cuts) == 2:
                    part = blocks
                else:
                    part = self.ops.part(blocks, desc, a, b, host)
                more = error is None and k + 2 < len(cuts)
                r, others, err = self._round(
                    host, part, b - a,
                    is_prefix[a:b] if is_prefix is not None else None,
                    digests[a:b] if digests is not None else None, more,
                    skip=error is not None)
                error = error or err
                if r is not None and a < b:
                    parts.append(r)
                k += 1
                if not others:
                    break
            if error is not None:
                raise error
        stored = sum(p[0] for p in parts)
        if not return_status:
            return stored
        if not parts:
            return 0, np.zeros(0, np.uint8), np.zeros((0, 32), np.uint8)
        return (stored, np.concatenate([p[1] for p in parts]),
                np.concatenate([p[2] for p in parts]))

    def _round(self, host, blocks, n, is_prefix, digests, more, skip=False):
        """One round of the put exchange for this rank's `blocks` (none
        with `skip`, after an earlier round failed here).  Returns (result
        or None, whether any rank has more slices, this rank's error)."""
        import torch
        import torch.distributed as dist
        dev = self.ops.device
        error, moves = None, 0
        if skip:
            n = 0
        else:
            try:    # room in this rank's pool; relocation records to send
                moves = self.ops.prepare(blocks, host, self.world, self.rank)
                if host:
                    self.ops.begin_host(blocks, is_prefix, self.world,
                                        self.rank)
                elif digests is not None:
                    self.ops.begin(blocks, is_prefix, self.world, self.rank,
                                   digests=digests)
                else:
                    self.ops.begin(blocks, is_prefix, self.world, self.rank)
            except Exception as e:       # noqa: BLE001 (returned below)
                error = e
        # while the hash runs: every rank's batch, relocation count and
        # whether it has more slices
        sizes = self._sizes(n, moves, 1 if more else 0)
        others = any(m for _, _, m in sizes)
        cap = max(c + m for c, m, _ in sizes)
        if cap == 0:
            if error is not None or skip:
                return None, others, error
            return ((0, np.zeros(0, np.uint8), np.zeros((0, 32), np.uint8)),
                    others, None)
        send = None
        if not skip and (error is None or moves):
            # after a failed begin: the relocation records alone
            try:
                send = self.ops.records(cap)
            except Exception as e:       # noqa: BLE001
                error = error or e
        if send is None:
            send = unused(self.world * cap, RECORD_BYTES, dev)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        try:
            reply = self.ops.resolve(recv)
        except Exception as e:           # noqa: BLE001
            error = error or e
            reply = failed_replies(recv)
        back = torch.empty_like(reply)
        dist.all_to_all_single(back, reply, group=self.group)
        if error is not None or skip:
            return None, others, error
        try:
            return self.ops.end(back), others, None
        except Exception as e:           # noqa: BLE001
            return None, others, e

    def get_batch(self, ids, outs):
        """Collective: every rank reads its own list of blocks (any rank may
        hold them) into its output buffers on this rank's GPU: a list of
        CUDA tensors, or one 2-D CUDA tensor with a block per row.  Returns
        (found[n] uint8, sizes[n] uint64) as CascadeStore.get_batch: a block
        larger than its output is reported with its size and not written.
        ``ids``: content ids (32 hex characters) or 16-byte keys, or all the
        keys at once as a uint8 array of shape (n, 16).  A rank whose own
        step fails still takes part in both exchanges and raises afterwards;
        its peers' reads of keys it owns then raise too."""
        import torch
        import torch.distributed as dist
        if isinstance(ids, np.ndarray) and ids.dtype == np.uint8 \
                and ids.ndim == 2 and ids.shape[1] == 16:
            keys = np.ascontiguousarray(ids).tobytes()
        else:
            keys = b"".join(self.ops.key(k) for k in ids)
        n_out = outs.shape[0] if isinstance(outs, torch.Tensor) else len(outs)
        if len(keys) // 16 != n_out:
            raise ValueError("one output per id")
        with self._lock:
            dev = self.ops.device
            cap = max(c for c, _, _ in self._sizes(n_out))
            if cap == 0:
                return np.zeros(0, np.uint8), np.zeros(0, np.uint64)
            error = None
            try:
                send = self.ops.get_begin(keys, self.world, cap)
            except Exception as e:       # noqa: BLE001 (re-raised below)
                error = e
                send = unused(self.world * cap, QUERY_BYTES, dev)
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send, group=self.group)
            try:
                reply = self.ops.lookup(recv)
            except Exception as e:       # noqa: BLE001
                error = error or e
                reply = unused(recv.shape[0], LOCATION_BYTES, dev)
            back = torch.empty_like(reply)
            dist.all_to_all_single(back, reply, group=self.group)
            if error is not None:
                raise error
            # Synchronous: the reads of the peers' pools are complete when
            # this returns, and clear() / close() start with a barrier, so
            # no pool is reset or unmapped while another rank reads it.
            found, sizes = self.ops.get_end(back, outs)
        return found, sizes

    def close(self):
        """Collective: unmaps the other ranks' pools on every rank, then
        synchronises, so that no rank frees a pool another rank can read."""
        import torch.distributed as dist
        if self._attached:
            self.ops.detach()
            self._attached = False
        dist.barrier(group=self.group)

    def get_stats(self):
        return self.ops.store.get_stats()

    def clear(self):
        """Collective: every rank empties its store."""
        import torch.distributed as dist
        dist.barrier(group=self.group)
        self.ops.store.clear()
