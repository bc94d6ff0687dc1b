"""PUT throughput of the block-ingest path: SHA-256 content addressing +
FP16->INT8 compression + store into the HBM pool, for the Llama-3-8B-shape
KV workload (4096 blocks x 2 MiB = 16 tokens x 32 layers x 8 KV heads x
128 dims x {K,V} FP16; N(0,1) with 0.1 % outlier channels x20; seeded,
generated on the GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One JSON line on rank 0.  A step is one content-addressed put_batch of the
whole workload into an emptied store (CascadeStore.clear() + put_batch).
`value` is device-resident throughput (inputs already in HBM); `e2e` is the
same PUT through the public host-buffer API (put_batch_host) with the
inputs in pinned host memory, host->device copies and the digests/status
read-back inside the timed region.  Multi-GPU runs are weak-scaled: each
rank ingests its own 4096 blocks.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "PUT GB/s of FP16 KV (SHA-256+INT8+store)"
UNIT = "GB/s"
N_BLOCKS = 4096
SEED = 2024
SAMPLE_BLOCKS = 256          # CPU baseline sample: 512 MiB of the workload
CPU_MIN_SECONDS = 5.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--blocks", type=int, default=N_BLOCKS)
    ap.add_argument("--layers", type=int, default=32,
                    help="layers per KV block (32 = 2 MiB; smaller for "
                         "profiling captures)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--headline-only", action="store_true",
                    help="skip the 1 MiB round trip, the block-size sweep "
                         "and the prefix-dedup mix (for profiling captures)")
    ap.add_argument("--workload", default="llama3-8b",
                    choices=["llama3-8b", "llama3-70b-zipf"],
                    help="llama3-8b: the headline line (it also carries the "
                         "1 MiB round trip, the block-size sweep and the "
                         "prefix-dedup mix); llama3-70b-zipf: 8192 x 5 MiB "
                         "blocks per GPU, 30%% Zipf copies of a pool shared "
                         "by all GPUs")
    ap.add_argument("--cap-gib", type=float, default=120.0,
                    help="llama3-70b-zipf: HBM pool per GPU (GiB); below the "
                         "stored bytes, 1-GPU runs demote to the DRAM tier")
    return ap.parse_args()


def workload_config(args, block_bytes):
    return {
        "workload": "llama3-8b-kv-" + (
            f"{block_bytes >> 20}MiB" if block_bytes % (1 << 20) == 0
            else f"{block_bytes >> 10}KiB") + f"-x{args.blocks}",
        "blocks_per_gpu": args.blocks,
        "block_bytes": block_bytes,
        "block_shape": f"[{args.layers} layers][K,V][8 heads][16 tokens]"
                       "[128 dim] fp16",
        "values": "N(0,1), 0.1% channels x20, seeded (synthetic)",
        "content_addressed": True,
        "kv_compression": True,
        "hbm_format": "int8 codes + per-block header in the index",
        "dedup": True,
        "l2": f"inputs ({args.blocks * block_bytes / 2**30:.2f} GiB/GPU) "
              "exceed the 126 MB L2; no flush needed",
        "parallelism": f"weak x{args.gpus} (each rank its own blocks)",
    }


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,"
         "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.idx), "--query-gpu=" + self.Q,
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        import time
        for line in self.proc.stdout:
            self.lines.append((time.perf_counter(), line.strip()))

    def mark(self, name):
        import time
        setattr(self, name, time.perf_counter())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        mhz, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                 "sw_power_cap"]
        t0 = getattr(self, "t_begin", None)
        t1 = getattr(self, "t_end", None)
        for when, ln in self.lines:
            if t0 is not None and not (t0 - 0.15 <= when <= t1 + 0.15):
                continue
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                mhz.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(mhz) if mhz else None,
                "sm_max_mhz": mx, "samples": len(mhz),
                "reasons": sorted(reasons)}


# -------------------------------------------------------------- reference
def cpu_reference(blocks_np, threads, min_seconds, steps=0, warmup=1,
                  lib=""):
    """Times a build of the reference's own code (oracle/_ref) in a child
    process."""
    import numpy as np
    fd, path = tempfile.mkstemp(suffix=".npy", dir="/dev/shm")
    os.close(fd)
    try:
        np.save(path, blocks_np)
        cmd = [sys.executable, "-m", "oracle.ref_bench", "--input", path,
               "--threads", str(threads), "--min-seconds", str(min_seconds),
               "--steps", str(steps), "--warmup", str(warmup)]
        if lib:
            cmd += ["--lib", lib]
        out = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True,
                             timeout=600)
        if out.returncode != 0:
            raise RuntimeError(out.stderr[-2000:])
        return json.loads(out.stdout.strip().splitlines()[-1])
    finally:
        os.unlink(path)


def reference_build():
    """(path, description) of the reference build to time on this host: the
    -march=native build when it was made for exactly this host's options,
    else the portable -march=x86-64-v3 build."""
    import oracle
    if oracle.native_build_matches_host():
        return oracle.REF_NATIVE_SO, ("-O3 -march=native (built with this "
                                      "host's exact -march=native options)")
    return oracle.REF_SO, ("-O3 -march=x86-64-v3 (portable build; this "
                           "host's -march=native differs from the native "
                           "build's)")


def host_cpu():
    import oracle
    return {"model": oracle.cpu_model(), "nproc": os.cpu_count()}


def run_reference(args):
    """--impl reference: the reference's CPU path on all host threads."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from cascade_b200 import workloads
    threads = os.cpu_count() or 1
    sample = workloads.kv_blocks_np(SAMPLE_BLOCKS, SEED)
    bb = sample.shape[1]
    lib, build = reference_build()
    # Each step = one put_batch of the sample into an emptied store: W
    # untimed steps, then exactly K timed ones.
    res = cpu_reference(sample, threads, 0.0, steps=args.steps,
                        warmup=args.warmup, lib=lib)
    value = res["gbps"]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": res["passes"], "warmup": args.warmup,
        "ms_per_step": 1e3 * res["seconds"] / res["passes"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u32 (SHA-256), f32 (INT8 scale math)", "data": "synthetic",
        "config": workload_config(args, bb),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads,
                         "kind": "reference", "build": build,
                         "cpu": host_cpu(),
                         "sample": f"{SAMPLE_BLOCKS} blocks x {bb} B per step, "
                                   f"{res['passes']} steps"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------- ours
class Ctx:
    """Rank, device and the collective helpers of one bench process."""

    def __init__(self):
        import torch
        import torch.distributed as dist
        self.torch, self.dist = torch, dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            from datetime import timedelta
            dist.init_process_group("nccl", device_id=self.dev,
                                    timeout=timedelta(seconds=120))
        self.stream = torch.cuda.current_stream(self.dev).cuda_stream

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max(self, x):
        if self.world == 1:
            return x
        t = self.torch.tensor([x], dtype=self.torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def all_true(self, ok):
        if self.world == 1:
            return bool(ok)
        t = self.torch.tensor([1 if ok else 0], dtype=self.torch.int32,
                              device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MIN)
        return bool(t.item())

    def gather_rows(self, t):
        """Every rank's int64 vector t, stacked (numpy, on every rank)."""
        if self.world == 1:
            return t.cpu().numpy()[None]
        every = [self.torch.empty_like(t) for _ in range(self.world)]
        self.dist.all_gather(every, t)
        return self.torch.stack(every).cpu().numpy()

    def timed(self, fn, warm, steps):
        """fn() W times untimed, then `steps` times between CUDA events on
        the current stream; ms per call, max over ranks."""
        torch = self.torch
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        self.barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            out = fn()
        b.record()
        torch.cuda.synchronize()
        return self.max(a.elapsed_time(b) / steps), out


def _addr_table(torch, rows, dev, stride=None):
    n = rows.shape[0]
    stride = stride or rows.stride(0) * rows.element_size()
    return (torch.arange(n, dtype=torch.int64, device=dev) * stride
            + rows.data_ptr())


def compress_roundtrip(ctx, rows):
    """The stateless compress -> decompress of CUDA rows [n, S] (the bytes
    a GET of INT8-stored blocks must return)."""
    from cascade_b200 import _lib
    torch = ctx.torch
    n, bb = rows.shape
    cb = 8 + bb // 2
    cstride = (cb + 255) // 256 * 256
    comp = torch.empty(n * cstride, dtype=torch.uint8, device=ctx.dev)
    out = torch.empty_like(rows)
    sizes = torch.full((n,), bb, dtype=torch.int64, device=ctx.dev)
    src = _addr_table(torch, rows, ctx.dev)
    mid = torch.arange(n, dtype=torch.int64, device=ctx.dev) * cstride + comp.data_ptr()
    dst = _addr_table(torch, out, ctx.dev)
    _lib.call("cascade_kv_compress_batch", src.data_ptr(), sizes.data_ptr(),
              mid.data_ptr(), n, bb, ctx.stream)
    _lib.call("cascade_kv_decompress_batch", mid.data_ptr(), sizes.data_ptr(),
              dst.data_ptr(), n, bb, ctx.stream)
    torch.cuda.synchronize()
    return out


def make_cfg(cc, local, cap_bytes, q8=True, shm=0, slots=1 << 16):
    cfg = cc.CascadeConfig()
    cfg.gpu_device_id = local
    cfg.gpu_capacity_bytes = cap_bytes
    cfg.shm_capacity_bytes = shm
    cfg.kv_compression = q8
    cfg.gpu_q8 = q8
    cfg.index_slots = slots
    return cfg


def section_cfg1(ctx, args):
    """The reference's CPU-runnable workload on one GPU: 256 x 1 MiB of
    seeded uniform bytes, is_prefix on blocks 0..127, content-addressed PUT
    into a default (raw-format) store, then GET of every block.  Digests
    are checked against hashlib (OpenSSL) and the round trip byte for byte."""
    import hashlib

    import numpy as np
    from cascade_b200 import cascade_cpp as cc
    from cascade_b200 import workloads
    torch = ctx.torch
    n, size = 256, 1 << 20
    host = workloads.random_bytes(n, size, SEED)
    rows = torch.from_numpy(host).to(ctx.dev)
    cfg = cc.CascadeConfig()                    # the reference's defaults
    cfg.gpu_device_id = ctx.local
    cfg.gpu_capacity_bytes = 1 << 30
    cfg.shm_capacity_bytes = 0
    store = cc.CascadeStore(cfg)
    ptrs = np.arange(n, dtype=np.uint64) * np.uint64(size) + np.uint64(rows.data_ptr())
    sizes = np.full(n, size, np.uint64)
    prefix = [i < n // 2 for i in range(n)]

    def put():
        store.clear()
        return store._put_batch_raw(n, ptrs, sizes, None, prefix, True,
                                    ctx.stream)

    ms, (stored, status, dig) = ctx.timed(put, 2, 5)
    want = [hashlib.sha256(host[i].tobytes()).digest() for i in range(n)]
    digests_ok = all(dig[i].tobytes() == want[i] for i in range(n))
    outs = torch.zeros_like(rows)
    keys16 = np.ascontiguousarray(dig[:, :16]).reshape(-1)
    optrs = np.arange(n, dtype=np.uint64) * np.uint64(size) + np.uint64(outs.data_ptr())
    caps = np.full(n, size, np.uint64)
    gms, (found, gsz) = ctx.timed(
        lambda: store._get_batch_raw(n, keys16, optrs, caps, ctx.stream), 1, 3)
    roundtrip_ok = bool(found.all()) and bool((gsz == size).all()) and \
        bool(torch.equal(outs, rows))
    s = store.get_stats()
    store.close()
    assert digests_ok and roundtrip_ok and stored == n, (digests_ok, roundtrip_ok)
    return {"workload": "256 x 1 MiB seeded uniform bytes, is_prefix on "
                        "blocks 0..127, content-addressed put_batch + "
                        "get_batch, default (raw) store",
            "put_gbps": n * size / (ms * 1e-3) / 1e9, "put_ms": ms,
            "get_gbps": n * size / (gms * 1e-3) / 1e9, "get_ms": gms,
            "digests_equal_hashlib": digests_ok,
            "roundtrip_bit_exact": roundtrip_ok,
            "gpu_used": int(s.gpu_used), "gpu_hits": int(s.gpu_hits),
            "note": "256 serial SHA-256 chains of 1 MiB: the per-chain "
                    "issue rate bounds this workload (8 warps)"}


def section_sweep(ctx, args, sha_peak):
    """Block-size sweep on one GPU: 64 KiB .. 16 MiB KV blocks, 1 GiB per
    size, content-addressed INT8 PUT."""
    import numpy as np
    from cascade_b200 import cascade_cpp as cc
    from cascade_b200 import workloads
    torch = ctx.torch
    hbm = hbm_peak()[0]
    res = []
    for layers in (1, 4, 16, 64, 256):
        bb = workloads.kv_block_bytes(layers, 8, 16, 128)
        n = (1 << 30) // bb
        blocks = workloads.kv_blocks_torch(n, SEED + layers, ctx.dev,
                                           layers=layers)
        store = cc.CascadeStore(make_cfg(cc, ctx.local,
                                         int(n * bb // 2 * 1.1) + (64 << 20)))
        ptrs = np.arange(n, dtype=np.uint64) * np.uint64(bb) + np.uint64(blocks.data_ptr())
        sizes = np.full(n, bb, np.uint64)

        def put():
            store.clear()
            return store._put_batch_raw(n, ptrs, sizes, None, None, False,
                                        ctx.stream)

        ms, stored = ctx.timed(put, 2, 3)
        assert stored == n
        store.close()
        del store, blocks
        torch.cuda.empty_cache()
        gbps = n * bb / (ms * 1e-3) / 1e9
        # Bounds: the serial chains (each chain's consumer warp issues
        # 1408 cycles per 64-byte chunk; at most 64 x SMs chains run at
        # once, beyond that the measured all-scheduler SHA peak) and HBM
        # (hash read + compress 1.5 S + payload write: 3.5 S).
        chain = min(n, 64 * 148) * 64 * 1965e6 / 1408 / 1e9
        sha_bound = min(chain, sha_peak)
        hbm_bound = hbm / 3.5
        bound = min(sha_bound, hbm_bound)
        res.append({"block_bytes": bb, "blocks": n, "ms_per_step": ms,
                    "gbps": gbps, "blocks_per_s": n / (ms * 1e-3),
                    "bound_gbps": bound,
                    "bound": "sha chains" if sha_bound < hbm_bound else "hbm",
                    "frac_of_bound": gbps / bound})
    return {"workload": "FP16 N(0,1) KV blocks of 64 KiB, 256 KiB, 1 MiB, "
                        "4 MiB, 16 MiB; 1 GiB per size; content-addressed "
                        "INT8 put_batch", "sizes": res}


def section_dedup(ctx, args):
    """Prefix-dedup workload: 8192 x 2 MiB per GPU, 60% of them Zipf(1.1)
    copies of 512 shared prefix blocks in 256 sessions, every copy in its
    own buffer.  Sharded index across the GPUs at N > 1.  The dedup hit
    count must equal N - #distinct exactly."""
    import numpy as np
    from cascade_b200 import cascade_cpp as cc
    from cascade_b200 import workloads
    torch = ctx.torch
    n = 8192
    seq, pre = workloads.dedup_sequence(n, SEED + ctx.rank, pool=512,
                                        sessions=256)
    pool = workloads.kv_blocks_torch(512, SEED, ctx.dev)        # shared
    uniq_n = int((seq >= 512).sum())
    uniq = workloads.kv_blocks_torch(uniq_n, SEED + 1000 + ctx.rank, ctx.dev)
    rows = workloads.materialise(seq, pool, uniq)
    del pool, uniq
    torch.cuda.empty_cache()
    bb = rows.shape[1]
    cfg = make_cfg(cc, ctx.local, int(n * bb // 2 * 1.1) + (256 << 20))
    if ctx.world > 1:
        from cascade_b200.sharded import ShardedCascadeStore
        store = ShardedCascadeStore(cfg)

        def put():
            store.clear()
            return store.put_batch(rows)
    else:
        store = cc.CascadeStore(cfg)
        ptrs = np.arange(n, dtype=np.uint64) * np.uint64(bb) + np.uint64(rows.data_ptr())
        sizes = np.full(n, bb, np.uint64)

        def put():
            store.clear()
            return store._put_batch_raw(n, ptrs, sizes, None, None, False,
                                        ctx.stream)

    ms, stored = ctx.timed(put, 2, 5)
    hits = int(store.get_stats().dedup_hits)
    store.close()
    del rows
    torch.cuda.empty_cache()
    used = np.zeros(512, np.int64)
    used[np.unique(seq[seq < 512])] = 1
    ev = ctx.gather_rows(torch.tensor(np.concatenate([used, [uniq_n, hits]]),
                                      dtype=torch.int64, device=ctx.dev))
    distinct = int((ev[:, :512].max(axis=0) > 0).sum()) + int(ev[:, 512].sum())
    total_hits = int(ev[:, 513].sum())
    expected = ctx.world * n - distinct
    assert total_hits == expected, (total_hits, expected)
    return {"workload": "prefix-dedup: 8192 x 2 MiB per GPU, 60% Zipf(1.1) "
                        "copies of 512 shared prefix blocks, 256 sessions, "
                        "every copy in its own buffer; content-addressed "
                        "INT8 put_batch" + (", sharded index" if ctx.world > 1
                                            else ""),
            "gbps": ctx.world * n * bb / (ms * 1e-3) / 1e9, "ms_per_step": ms,
            "dedup_hits": total_hits, "expected_hits": expected,
            "hits_exact": total_hits == expected}


def reference_kv_manager_sample(ctx, blocks, wire, L, H, S, D, m=16):
    """The reference's own serialize_kv_cache / deserialize_kv_cache
    (inference_benchmark/kv_manager.py, the copy `make -C oracle callers`
    stages byte for byte) on m of the caches, from and to the GPU as
    KVCacheStore.store / load call them: per-cache time and whether its
    bytes equal the device wire blocks."""
    import importlib
    import time
    callers = os.path.join(ROOT, "baseline", "_ref", "callers")
    if not os.path.exists(os.path.join(callers, "inference_benchmark",
                                       "kv_manager.py")):
        return {"unavailable": "the reference's callers are not staged "
                               "(make -C oracle callers)"}
    sys.path.insert(0, callers)
    try:
        kv = importlib.import_module("inference_benchmark.kv_manager")
    finally:
        sys.path.remove(callers)
    T = H * S * D
    rows = [blocks[i].view(ctx.torch.float16) for i in range(m)]
    caches = [tuple((r[2 * l * T:(2 * l + 1) * T].view(1, H, S, D),
                     r[(2 * l + 1) * T:(2 * l + 2) * T].view(1, H, S, D))
                    for l in range(L)) for r in rows]
    ctx.torch.cuda.synchronize()
    t0 = time.perf_counter()
    blobs = [kv.serialize_kv_cache(c) for c in caches]
    t1 = time.perf_counter()
    for b in blobs:
        kv.deserialize_kv_cache(b, device=ctx.dev)
    ctx.torch.cuda.synchronize()
    t2 = time.perf_counter()
    wb = len(blobs[0])
    equal = all(blobs[i] == bytes(wire[i, :wb].cpu().numpy())
                for i in range(min(4, m)))
    nbytes = m * (wb - 18)
    return {"caches": m, "serialize_ms_per_cache": (t1 - t0) * 1e3 / m,
            "deserialize_ms_per_cache": (t2 - t1) * 1e3 / m,
            "serialize_gbps": nbytes / (t1 - t0) / 1e9,
            "deserialize_gbps": nbytes / (t2 - t1) / 1e9,
            "bytes_equal_device_wire": equal,
            "what": "the reference's kv_manager functions (.cpu() + bytes "
                    "join; numpy copies back to the GPU), host wall clock"}


def section_kvwire(ctx, blocks, hbm, hbm_src):
    """The KV-cache wire format (kv_manager.serialize_kv_cache /
    deserialize_kv_cache) on the device for the headline's blocks: each
    2 MiB block is read as 32 layers x (K, V) x [8 heads][16 tokens][128]
    FP16 tensors, serialised into 18-byte-header wire blocks in one launch
    and split back into the same memory in one launch.  Checked: every
    header, the payload of a sample against its source bytes, and the
    round trip byte for byte."""
    import struct

    import numpy as np
    from cascade_b200 import _lib, kvwire
    torch = ctx.torch
    n, bb = blocks.shape
    L, H, S, D = 32, 8, 16, 128
    assert bb == kvwire.wire_bytes(L, H, S, D) - kvwire.HEADER_SIZE
    T = H * S * D * 2
    wb = kvwire.wire_bytes(L, H, S, D)
    pitch = (wb + 255) // 256 * 256
    wire = torch.empty((n, pitch), dtype=torch.uint8, device=ctx.dev)
    # descriptors: tensor j of block b at blocks[b] + j * T, strides (S*D, D)
    base = np.arange(n, dtype=np.int64)[:, None] * bb + blocks.data_ptr() \
        + np.arange(2 * L, dtype=np.int64)[None, :] * T
    desc = np.stack([base.reshape(-1), np.full(base.size, S * D, np.int64),
                     np.full(base.size, D, np.int64)], axis=1)
    d_desc = torch.from_numpy(np.ascontiguousarray(desc)).to(ctx.dev)
    d_wire = (torch.arange(n, dtype=torch.int64, device=ctx.dev) * pitch
              + wire.data_ptr())
    sample = min(64, n)
    keep = blocks[:sample].clone()

    def ser():
        _lib.call("cascade_kv_serialize_batch", d_desc.data_ptr(), 0, L, H, S,
                  D, d_wire.data_ptr(), n, ctx.stream)

    def de():
        _lib.call("cascade_kv_deserialize_batch", d_wire.data_ptr(), L, H, S,
                  D, d_desc.data_ptr(), n, ctx.stream)

    ser_ms, _ = ctx.timed(ser, 2, 5)
    ref = reference_kv_manager_sample(ctx, blocks, wire, L, H, S, D)
    head = struct.pack(kvwire.HEADER_FMT, L, H, S, D, 0)
    heads_ok = bool((wire[:, :18].cpu().numpy()
                     == np.frombuffer(head, np.uint8)).all())
    payload_ok = bool(torch.equal(wire[:sample, 18:18 + bb], keep))
    blocks[:sample].zero_()
    de_ms, _ = ctx.timed(de, 2, 5)
    torch.cuda.synchronize()
    round_ok = bool(torch.equal(blocks[:sample], keep))

    # KVCacheStore.load of the whole batch from a raw-format store: one
    # cascade_store_get_kv_batch (lookup, then every wire block split
    # straight out of the pool), against get_batch + deserialize.
    from cascade_b200 import cascade_cpp as cc
    # (2 MiB + 18 bytes rounds up to the pool's 2.25 MiB size class)
    store = cc.CascadeStore(make_cfg(cc, ctx.local,
                                     int(n * pitch * 1.13) + (256 << 20),
                                     q8=False, shm=0, slots=1 << 15))
    keys = np.random.default_rng(SEED).integers(
        0, 256, (n, 16), dtype=np.uint8)
    keys[:, 15] = 0x5a                       # clear of the reserved key region
    wptrs = np.arange(n, dtype=np.uint64) * np.uint64(pitch) \
        + np.uint64(wire.data_ptr())
    klist = [bytes(k) for k in keys]
    kflat = np.ascontiguousarray(keys).reshape(-1)
    status = np.zeros(n, np.uint8)
    nst = ctypes.c_uint64(0)

    def put_fused():          # KVCacheStore.store: one store call
        store.clear()
        _lib.call("cascade_store_put_kv_batch", store._h, n,
                  kflat.ctypes.data, L, H, S, D, d_desc.data_ptr(), 0, None,
                  status.ctypes.data, ctx.stream, ctypes.byref(nst))

    def put_two_step():       # serialise, then put_batch of the wire blocks
        store.clear()
        ser()
        store._put_batch_raw(n, wptrs, np.full(n, wb, np.uint64), klist,
                             None, False, ctx.stream)

    two_put_ms, _ = ctx.timed(put_two_step, 1, 3)
    put_ms, _ = ctx.timed(put_fused, 1, 3)
    assert (status == 0).all() and nst.value == n
    found = np.zeros(n, np.uint8)
    nf = ctypes.c_uint64(0)

    def load():
        _lib.call("cascade_store_get_kv_batch", store._h, n,
                  kflat.ctypes.data, L, H, S, D, d_desc.data_ptr(),
                  found.ctypes.data, ctx.stream, ctypes.byref(nf))

    blocks[:sample].zero_()
    load_ms, _ = ctx.timed(load, 2, 5)
    load_ok = bool(found.all()) and bool(torch.equal(blocks[:sample], keep))
    caps = np.full(n, pitch, np.uint64)

    def get_then_split():
        store._get_batch_raw(n, kflat, wptrs, caps, ctx.stream)
        de()

    two_ms, _ = ctx.timed(get_then_split, 2, 5)
    store.close()
    del wire, d_wire, d_desc, keep
    torch.cuda.empty_cache()
    alg = n * (2 * bb + 18)                  # read S, write S + 18 (and back)
    return {
        "workload": f"{n} KV caches of llama3-8b geometry ({L} layers x (K,V) "
                    f"x [{H}][{S}][{D}] FP16, 2 MiB) <-> kv_manager wire "
                    "blocks (18-byte <IIIIH header + payload)",
        "serialize_gbps": n * bb / (ser_ms * 1e-3) / 1e9,
        "serialize_ms": ser_ms,
        "deserialize_gbps": n * bb / (de_ms * 1e-3) / 1e9,
        "deserialize_ms": de_ms,
        "unit": "GB/s of FP16 KV",
        "roofline": {"bound": "hbm", "peak": hbm, "unit": "GB/s",
                     "algorithmic_bytes": "2 x payload + 18 per block",
                     "serialize_frac": alg / (ser_ms * 1e-3) / 1e9 / hbm,
                     "deserialize_frac": alg / (de_ms * 1e-3) / 1e9 / hbm,
                     "peak_source": hbm_src},
        "headers_equal": heads_ok, "payload_equal_sample": payload_ok,
        "round_trip_bit_exact_sample": round_ok,
        "launches_per_call": 1,
        "reference_kv_manager": ref,
        "store": {"what": "KVCacheStore.store of every cache into an "
                          "emptied raw HBM store: cascade_store_put_kv_batch "
                          "(each cache serialised straight into its pool "
                          "slot, keyed index insert)",
                  "gbps": n * bb / (put_ms * 1e-3) / 1e9, "ms": put_ms,
                  "serialize_then_put_batch_ms": two_put_ms},
        "load": {"what": "KVCacheStore.load of every cache from a raw HBM "
                         "store: cascade_store_get_kv_batch (lookup + split "
                         "straight out of the pool)",
                 "gbps": n * bb / (load_ms * 1e-3) / 1e9, "ms": load_ms,
                 "frac": alg / (load_ms * 1e-3) / 1e9 / hbm,
                 "get_then_deserialize_ms": two_ms,
                 "bit_exact_sample": load_ok},
    }


def section_capped(ctx, args):
    """The llama3-70b shape with an HBM pool too small for it (SURVEY cfg5's
    capped variant, scaled to fit a short run at every GPU count): 2048 x 5
    MiB blocks per GPU, 30% Zipf(1.1) copies of a 256-block pool shared by
    all GPUs, into 2 GiB of HBM per GPU (4 GiB at N > 1, where a sharded put
    holds each slice in HBM while its keys resolve) over a DRAM tier, so
    every step demotes to and places in the DRAM tier through the copy
    streams.  Dedup hits must equal N - #distinct exactly."""
    import numpy as np
    from cascade_b200 import cascade_cpp as cc
    from cascade_b200 import workloads
    torch = ctx.torch
    n, pool_n = 2048, 256
    seq, _ = workloads.dedup_sequence(n, SEED + 77 + ctx.rank, pool=pool_n,
                                      sessions=64, shared_frac=0.3)
    geo = workloads.LLAMA3_70B
    pool = workloads.kv_blocks_torch(pool_n, SEED + 77, ctx.dev, **geo)
    uniq_n = int((seq >= pool_n).sum())
    uniq = workloads.kv_blocks_torch(uniq_n, SEED + 2000 + ctx.rank, ctx.dev,
                                     **geo)
    rows = workloads.materialise(seq, pool, uniq)
    del pool, uniq
    torch.cuda.empty_cache()
    bb = rows.shape[1]
    cap = (2 << 30) if ctx.world == 1 else (4 << 30)
    cfg = make_cfg(cc, ctx.local, cap, shm=16 << 30)
    if ctx.world > 1:
        from cascade_b200.sharded import ShardedCascadeStore
        store = ShardedCascadeStore(cfg)
        # the store puts the batch in slices that fit its pool, hashed in
        # one launch first
        cuts = store.ops.slices(rows, False)[0]

        def put():
            store.clear()
            return store.put_batch(rows)
    else:
        store = cc.CascadeStore(cfg)
        cuts = [0, n]
        ptrs = np.arange(n, dtype=np.uint64) * np.uint64(bb) + np.uint64(rows.data_ptr())
        sizes = np.full(n, bb, np.uint64)

        def put():
            store.clear()
            return store._put_batch_raw(n, ptrs, sizes, None, None, False,
                                        ctx.stream)

    ms, stored = ctx.timed(put, 2, 3)
    assert stored == n, stored
    st = store.get_stats()
    store.close()
    del rows
    torch.cuda.empty_cache()
    used = np.zeros(pool_n, np.int64)
    used[np.unique(seq[seq < pool_n])] = 1
    ev = ctx.gather_rows(torch.tensor(
        np.concatenate([used, [uniq_n, int(st.dedup_hits), int(st.gpu_evictions),
                               int(st.shm_used), int(st.gpu_used)]]),
        dtype=torch.int64, device=ctx.dev))
    distinct = int((ev[:, :pool_n].max(axis=0) > 0).sum()) + int(ev[:, pool_n].sum())
    hits = int(ev[:, pool_n + 1].sum())
    expected = ctx.world * n - distinct
    assert hits == expected, (hits, expected)
    return {"workload": "llama3-70b KV, capped HBM: 2048 x 5 MiB per GPU, "
                        "30% Zipf(1.1) copies of a 256-block pool shared by "
                        "all GPUs, every copy in its own buffer; "
                        f"{cap >> 30} GiB HBM pool per GPU over a DRAM tier",
            "gbps": ctx.world * n * bb / (ms * 1e-3) / 1e9, "ms_per_step": ms,
            "dedup_hits": hits, "expected_hits": expected,
            "hits_exact": hits == expected,
            "gpu_evictions_per_step": int(ev[:, pool_n + 2].sum()),
            "dram_tier_bytes_after_step": int(ev[:, pool_n + 3].sum()),
            "hbm_bytes_after_step": int(ev[:, pool_n + 4].sum()),
            "put_slices": len(cuts) - 1}


def hbm_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return (float(json.load(f)["hbm_gbs"]),
                    "MEASURED_PEAKS.json hbm_gbs (of measured)")
    except (OSError, KeyError, ValueError):
        return 6650.0, "profiling-recipe fallback (of fallback)"


def main_ours(args):
    import numpy as np

    from cascade_b200 import _lib
    from cascade_b200 import cascade_cpp as cc
    from cascade_b200 import workloads

    ctx = Ctx()
    torch = ctx.torch
    world, rank, local, dev = ctx.world, ctx.rank, ctx.local, ctx.dev
    stream = ctx.stream
    L = _lib.load()
    blocks = workloads.kv_blocks_torch(args.blocks, SEED + rank, dev,
                                       layers=args.layers)
    n, bb = blocks.shape
    total = n * bb
    cfg = make_cfg(cc, local, int(n * (bb // 2) * 1.1) + (256 << 20),
                   shm=1 << 30, slots=1 << 15)
    ptrs = np.arange(n, dtype=np.uint64) * np.uint64(bb) + np.uint64(blocks.data_ptr())
    sizes = np.full(n, bb, np.uint64)
    if world > 1:
        # the dedup index is sharded over the ranks (NCCL all-to-all)
        from cascade_b200.sharded import ShardedCascadeStore
        sharded = ShardedCascadeStore(cfg)
        store = sharded.store

        def step():
            sharded.clear()
            return sharded.put_batch(blocks)
    else:
        store = cc.CascadeStore(cfg)

        def step():
            store.clear()
            return store._put_batch_raw(n, ptrs, sizes, None, None, False,
                                        stream)

    # ---- the headline: W untimed steps, then exactly K timed ones
    with ClockSampler(local) as clk:   # sampling runs from warm-up on
        for _ in range(args.warmup):
            assert step() == n
        torch.cuda.synchronize()
        ctx.barrier()
        launches0 = L.cascade_diag_launch_count()
        clk.mark("t_begin")
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            stored = step()
        e1.record()
        torch.cuda.synchronize()
        clk.mark("t_end")
        ctx.barrier()
    launches = L.cascade_diag_launch_count() - launches0
    ms = ctx.max(e0.elapsed_time(e1))
    assert stored == n
    s = store.get_stats()
    assert s.gpu_used == total // 2 and s.dedup_hits == 0
    value = world * args.steps * total / (ms * 1e-3) / 1e9

    # ---- per-kernel timing for the roofline (same stream as the launch)
    dptrs = torch.from_numpy(ptrs.view(np.int64)).to(dev)
    dsizes = torch.from_numpy(sizes.view(np.int64)).to(dev)
    digests = torch.empty(n * 32, dtype=torch.uint8, device=dev)
    qdst = torch.empty(n * (bb // 2 + 256), dtype=torch.uint8, device=dev)
    qptrs = (torch.arange(n, dtype=torch.int64, device=dev) * (bb // 2 + 256)
             + qdst.data_ptr())

    def timed(fn, reps):
        fn()
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    sha_ms = timed(lambda: _lib.call("cascade_sha256_batch", dptrs.data_ptr(),
                                     dsizes.data_ptr(), n, digests.data_ptr(),
                                     stream), 3)
    q_ms = timed(lambda: _lib.call("cascade_kv_compress_batch",
                                   dptrs.data_ptr(), dsizes.data_ptr(),
                                   qptrs.data_ptr(), n, bb, stream), 5)
    peak_gbps, peak_ms = ctypes.c_double(), ctypes.c_double()
    _lib.call("cascade_diag_sha_peak", local, 256, ctypes.byref(peak_gbps),
              ctypes.byref(peak_ms))
    del qdst, qptrs
    host = torch.empty((n, bb), dtype=torch.uint8, pin_memory=True)
    host.copy_(blocks)          # the e2e inputs, before GET overwrites blocks

    # ---- GET of every block into device buffers (the blocks' own memory is
    # the output), with a byte-exact check of a sample against the stateless
    # compress -> decompress of the source rows
    sample = min(256, n)
    if world == 1:
        want = compress_roundtrip(ctx, blocks[:sample])
        store.clear()
        _, _, dig = store._put_batch_raw(n, ptrs, sizes, None, None, True,
                                         stream)
        keys16 = np.ascontiguousarray(dig[:, :16]).reshape(-1)
        caps = np.full(n, bb, np.uint64)
        get_ms, (found, gsz) = ctx.timed(
            lambda: store._get_batch_raw(n, keys16, ptrs, caps, stream), 2, 3)
        assert found.all() and (gsz == bb).all()
        exact = bool(torch.equal(blocks[:sample], want))
        get_info = {"value": total / (get_ms * 1e-3) / 1e9, "unit": UNIT,
                    "ms": get_ms, "what": "get_batch of every block: index "
                    "lookup + INT8 dequantise into device buffers (FP16 bytes "
                    "out per second)"}
    else:
        # every rank reads the blocks its neighbour stored: each payload is
        # dequantised straight out of the peer's pool (NVLink reads)
        nb = (rank + 1) % world
        want = compress_roundtrip(
            ctx, workloads.kv_blocks_torch(sample, SEED + nb, dev,
                                           layers=args.layers))
        sharded.clear()
        _, _, dig = sharded.put_batch(blocks, return_status=True)
        mine = torch.from_numpy(np.ascontiguousarray(dig[:, :16])).to(dev)
        every = [torch.empty_like(mine) for _ in range(world)]
        ctx.dist.all_gather(every, mine)
        ids = every[nb].cpu().numpy()      # (n, 16) keys
        get_ms, (found, gsz) = ctx.timed(lambda: sharded.get_batch(ids, blocks),
                                         2, 3)
        assert found.all() and (gsz == bb).all()
        exact = bool(torch.equal(blocks[:sample], want))
        get_info = {"value": world * total / (get_ms * 1e-3) / 1e9,
                    "unit": UNIT, "ms": get_ms,
                    "what": "ShardedCascadeStore.get_batch: every rank reads "
                    "the blocks its neighbour rank stored (owner lookup by "
                    "all-to-all, INT8 dequantise from the peer's pool over "
                    "NVLink); FP16 bytes out per second, all ranks"}
    exact = ctx.all_true(exact)
    assert exact, "GET bytes differ from compress -> decompress of the source"
    get_info["byte_exact_sample"] = {
        "blocks_per_rank": sample, "equal": exact,
        "against": "stateless compress -> decompress of the source rows"
                   + (" (the neighbour rank's blocks, regenerated)"
                      if world > 1 else "")}
    hbm, hbm_src = hbm_peak()
    del want

    # ---- e2e: host buffers through the public API, the same K steps
    kvw = None
    if world == 1 and not args.headline_only and args.layers == 32:
        kvw = section_kvwire(ctx, blocks, hbm, hbm_src)
    del blocks, dptrs, dsizes, digests
    torch.cuda.empty_cache()
    host_np = host.numpy()
    if world > 1:
        def e2e_step():
            sharded.clear()
            return sharded.put_batch_host(host_np)
    else:
        def e2e_step():
            store.clear()
            return store.put_batch_host(host_np)

    e2e_ms, got = ctx.timed(e2e_step, 1, args.steps)
    assert got == n
    e2e_value = world * total / (e2e_ms * 1e-3) / 1e9
    # The roofline under e2e: plain pinned host -> device copies of the same
    # bytes, every rank at once.
    h2d_dst = torch.empty((n, bb), dtype=torch.uint8, device=dev)
    h2d_ms, _ = ctx.timed(lambda: h2d_dst.copy_(host, non_blocking=True), 1, 3)
    del h2d_dst
    torch.cuda.empty_cache()
    h2d_gbps = world * total / (h2d_ms * 1e-3) / 1e9

    # ---- the other reference configurations
    if world > 1:
        sharded.close()       # every rank unmaps the peers' pools first
    store.close()
    del host, host_np
    torch.cuda.empty_cache()
    extra = {}
    if world == 1 and not args.headline_only:
        extra["cfg1"] = section_cfg1(ctx, args)
        extra["sweep"] = section_sweep(ctx, args, peak_gbps.value)
        if kvw is not None:
            extra["kv_wire"] = kvw
    if not args.headline_only:
        extra["dedup"] = section_dedup(ctx, args)
        extra["capped"] = section_capped(ctx, args)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        smp = workloads.kv_blocks_np(SAMPLE_BLOCKS, SEED)
        lib, build = reference_build()
        try:
            res = cpu_reference(smp, os.cpu_count() or 1, CPU_MIN_SECONDS,
                                lib=lib)
            one = cpu_reference(smp[:64], 1, 2.0, lib=lib)
            cpu = {"value": res["gbps"], "unit": UNIT,
                   "cores": res["threads"], "kind": "reference",
                   "build": build, "cpu": host_cpu(),
                   "sample": f"{SAMPLE_BLOCKS} blocks of the same workload "
                             f"({SAMPLE_BLOCKS * bb >> 20} MiB) x "
                             f"{res['passes']} passes",
                   "single_core_value": one["gbps"]}
            import oracle
            if lib != oracle.REF_SO:   # the portable build, for comparison
                port = cpu_reference(smp, os.cpu_count() or 1, 3.0)
                cpu["portable_build_value"] = port["gbps"]
        except Exception as e:  # the line still reports the GPU numbers
            cpu = {"value": None, "unit": UNIT, "cores": None,
                   "kind": "reference", "sample": f"failed: {e}"[:300]}

    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            traffic = json.load(f)

    sha_gbps = total / (sha_ms * 1e-3) / 1e9
    # The ceiling for n serial chains on their own schedulers: a round is
    # 11 integer-ALU + 5 IMAD instructions, each issuing over 2 cycles on a
    # 16-lane pipe, so a 64-byte chunk takes at least 64 x 22 cycles.
    clk_sum = clk.summary()
    mhz = clk_sum["sm_mhz"] or 1965.0
    floor_gbps = min(n, 64 * 148) * 64 * mhz * 1e6 / (64 * 22) / 1e9
    chain_floor = {"gbps": floor_gbps, "frac": sha_gbps / floor_gbps,
                   "sm_mhz": mhz,
                   "basis": "each chain's consumer warp alone on a scheduler: "
                            "64 rounds x 11 ALU (the leanest round: 11 ALU + 5 IMAD) x 2 issue cycles "
                            "= 1408 cycles per 64-byte chunk"}
    q_bytes = total * 1.5 + 8 * n          # read S, write S/2 + header
    q_gbps = q_bytes / (q_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u32 (SHA-256), f32 (INT8 scale math)", "data": "synthetic",
        "config": workload_config(args, bb),
        "blocks_per_s": world * args.steps * n / (ms * 1e-3),
        "roofline": {
            "kernel": "sha256_pipelined", "bound": "int",
            "achieved": sha_gbps, "peak": peak_gbps.value, "unit": "GB/s",
            "frac": sha_gbps / peak_gbps.value,
            "peak_source": "measured live: the same SHA-256 rounds from "
                           "registers with all 64 warp slots/SM busy",
            "traffic": (traffic or {}).get("sha256_pipelined"),
            "note": f"{n} blocks = {n} serial chains = {(n + 31) // 32} "
                    "warps; per-chain issue latency, not the integer pipe, "
                    "bounds 2 MiB blocks",
            "chain_floor": chain_floor},
        "roofline_quantise": {
            "kernel": "compress_fused_kernel (single pass: one HBM read; "
                      "reducer and quantiser warps decoupled by mbarriers, "
                      "clusters of 8 exchanging min/max through DSMEM)",
            "bound": "hbm",
            "achieved": q_gbps, "peak": hbm, "unit": "GB/s",
            "frac": q_gbps / hbm, "peak_source": hbm_src,
            "algorithmic_bytes": "1.5 x block bytes + 8-byte headers",
            "traffic": (traffic or {}).get("compress_fused_kernel")},
        "stage_ms": {"sha256": sha_ms, "compress": q_ms},
        "get": get_info,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": UNIT,
                "h2d_bytes_per_step": total, "d2h_bytes_per_step": n * 33,
                "steps": args.steps,
                "api": ("CascadeStore.put_batch_host (one 2-D pinned host "
                        "array of blocks, striped H2D with hashing under the "
                        "copy)")
                if world == 1 else
                ("ShardedCascadeStore.put_batch_host (pinned host blocks, "
                 "striped H2D with hashing under the copy, per rank)"),
                "roofline": {"bound": "h2d", "achieved": e2e_value,
                             "peak": h2d_gbps, "unit": "GB/s",
                             "frac": e2e_value / h2d_gbps,
                             "peak_source": "measured in this run: plain "
                             "pinned host -> device copies of the same "
                             f"{total >> 30} GiB per rank, all ranks at once"}},
        "gpu_launches": int(launches),
        "clocks": clk_sum,
    }
    line.update(extra)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        ctx.dist.barrier()
        ctx.dist.destroy_process_group()


# ------------------------------------------------------- extra workloads
def run_extra(args):
    """--workload llama3-70b-zipf: 8192 x 5 MiB blocks per GPU, 30% Zipf
    copies of a pool every GPU draws from (one JSON line, not the headline
    line)."""
    import numpy as np
    from cascade_b200 import cascade_cpp as cc
    from cascade_b200 import workloads

    ctx = Ctx()
    torch = ctx.torch
    n, pool_n = 8192, 1024
    seq, pre = workloads.dedup_sequence(n, SEED + ctx.rank, pool=pool_n,
                                        sessions=256, shared_frac=0.3)
    geo = workloads.LLAMA3_70B
    pool = workloads.kv_blocks_torch(pool_n, SEED, ctx.dev, **geo)
    uniq_n = int((seq >= pool_n).sum())
    uniq = workloads.kv_blocks_torch(uniq_n, SEED + 1000 + ctx.rank, ctx.dev,
                                     **geo)
    rows = workloads.materialise(seq, pool, uniq)   # copies in own rows
    del pool, uniq
    torch.cuda.empty_cache()
    bb = rows.shape[1]
    cap = int(args.cap_gib * (1 << 30))
    # A pool smaller than a step's INT8 payload overflows to the DRAM tier.
    capped = n * (bb // 2) > cap
    cfg = make_cfg(cc, ctx.local, cap,
                   shm=(64 << 30) if (ctx.world == 1 or capped) else 0)
    if ctx.world > 1:
        from cascade_b200.sharded import ShardedCascadeStore
        store = ShardedCascadeStore(cfg)
        # A sharded put holds a batch in HBM while the keys resolve
        # (demoting older payloads first), so over a capped pool the store
        # puts the step in slices that fit, hashed in one launch first.
        cuts = store.ops.slices(rows, False)[0]

        def put():
            store.clear()
            return store.put_batch(rows)
    else:
        store = cc.CascadeStore(cfg)
        ptrs = np.arange(n, dtype=np.uint64) * np.uint64(bb) + np.uint64(rows.data_ptr())
        sizes = np.full(n, bb, np.uint64)

        def put():
            store.clear()
            return store._put_batch_raw(n, ptrs, sizes, None, None, False,
                                        ctx.stream)

    ms, stored = ctx.timed(put, args.warmup, args.steps)
    assert stored == n, stored
    st = store.get_stats()
    store.close()
    used = np.zeros(pool_n, np.int64)
    used[np.unique(seq[seq < pool_n])] = 1
    ev = ctx.gather_rows(torch.tensor(
        np.concatenate([used, [uniq_n, int(st.dedup_hits),
                               int(st.gpu_evictions)]]),
        dtype=torch.int64, device=ctx.dev))
    distinct = int((ev[:, :pool_n].max(axis=0) > 0).sum()) + int(ev[:, pool_n].sum())
    hits = int(ev[:, pool_n + 1].sum())
    assert hits == ctx.world * n - distinct, (hits, ctx.world * n, distinct)
    line = {"workload": "llama3-70b KV: 8192 x 5 MiB per GPU, 30% "
                        "Zipf(1.1) copies of a 1024-block pool shared by "
                        "all GPUs, every copy in its own buffer; "
                        "content-addressed INT8 PUT",
            "metric": METRIC, "unit": UNIT, "n_gpus": ctx.world,
            "value": ctx.world * n * bb / (ms * 1e-3) / 1e9,
            "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup,
            "blocks_total": ctx.world * n, "block_bytes": bb,
            "hbm_pool_gib_per_gpu": args.cap_gib,
            "dram_tier": bool(capped or ctx.world == 1),
            "put_slices": (len(cuts) - 1) if ctx.world > 1 else 1,
            "dedup_hits_total": hits,
            "expected_hits": ctx.world * n - distinct,
            "gpu_evictions_total": int(ev[:, pool_n + 2].sum()),
            "parallelism": f"sharded index x{ctx.world}" if ctx.world > 1
            else "1 GPU"}
    if ctx.rank == 0:
        print(json.dumps(line), flush=True)
    if ctx.world > 1:
        ctx.dist.barrier()
        ctx.dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload != "llama3-8b":
        run_extra(args)
    else:
        main_ours(args)


if __name__ == "__main__":
    main()
