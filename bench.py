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
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="llama3-8b",
                    choices=["llama3-8b", "sweep", "dedup", "llama3-70b-zipf"],
                    help="llama3-8b: the headline line; sweep / dedup: the "
                         "block-size sweep and the prefix-dedup mix; "
                         "llama3-70b-zipf: 8192 x 5 MiB blocks per GPU, 30%% "
                         "Zipf copies of a pool shared by all GPUs")
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
def cpu_reference(blocks_np, threads, min_seconds, steps=0, warmup=1):
    """Times oracle/_ref (the reference's own code) in a child process."""
    import numpy as np
    fd, path = tempfile.mkstemp(suffix=".npy", dir="/dev/shm")
    os.close(fd)
    try:
        np.save(path, blocks_np)
        out = subprocess.run(
            [sys.executable, "-m", "oracle.ref_bench", "--input", path,
             "--threads", str(threads), "--min-seconds", str(min_seconds),
             "--steps", str(steps), "--warmup", str(warmup)],
            cwd=ROOT, capture_output=True, text=True, timeout=600)
        if out.returncode != 0:
            raise RuntimeError(out.stderr[-2000:])
        return json.loads(out.stdout.strip().splitlines()[-1])
    finally:
        os.unlink(path)


def run_reference(args):
    """--impl reference: the reference's CPU path on all host threads."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np
    from cascade_b200 import workloads
    threads = os.cpu_count() or 1
    sample = workloads.kv_blocks_np(SAMPLE_BLOCKS, SEED)
    bb = sample.shape[1]
    # Each step = one put_batch of the sample into an emptied store: W
    # untimed steps, then exactly K timed ones.
    res = cpu_reference(sample, threads, 0.0, steps=args.steps,
                        warmup=args.warmup)
    value = res["gbps"]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": res["passes"], "warmup": args.warmup,
        "ms_per_step": 1e3 * res["seconds"] / res["passes"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u32 (SHA-256), f32 (INT8 scale math)", "data": "synthetic",
        "config": workload_config(args, bb),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads,
                         "kind": "reference",
                         "sample": f"{SAMPLE_BLOCKS} blocks x {bb} B per step, "
                                   f"{res['passes']} steps"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------- ours
def main_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from cascade_b200 import _lib
    from cascade_b200 import cascade_cpp as cc
    from cascade_b200 import workloads

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev,
                                timeout=timedelta(seconds=120))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    L = _lib.load()
    blocks = workloads.kv_blocks_torch(args.blocks, SEED + rank, dev,
                                       layers=args.layers)
    n, bb = blocks.shape
    total = n * bb
    cfg = cc.CascadeConfig()
    cfg.gpu_device_id = local
    cfg.gpu_capacity_bytes = int(n * (bb // 2) * 1.1) + (256 << 20)
    cfg.shm_capacity_bytes = 1 << 30
    cfg.kv_compression = True
    cfg.gpu_q8 = True
    cfg.index_slots = 1 << 15
    ptrs = np.arange(n, dtype=np.uint64) * np.uint64(bb) + np.uint64(blocks.data_ptr())
    sizes = np.full(n, bb, np.uint64)
    stream = torch.cuda.current_stream(dev).cuda_stream
    if world > 1:
        # the dedup index is sharded over the ranks (NCCL all-to-all)
        from cascade_b200.sharded import ShardedCascadeStore
        sharded = ShardedCascadeStore(cfg)
        store = sharded.store

        def put_rows(rows):
            return sharded.put_batch(rows)

        def step():
            sharded.clear()
            return put_rows(blocks)
    else:
        store = cc.CascadeStore(cfg)

        def step():
            store.clear()
            return store._put_batch_raw(n, ptrs, sizes, None, None, False,
                                        stream)

    with ClockSampler(local) as clk:   # sampling runs from warm-up on
        for _ in range(args.warmup):
            assert step() == n
        torch.cuda.synchronize()
        barrier()
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
        barrier()
    launches = L.cascade_diag_launch_count() - launches0
    ms = max_over_ranks(e0.elapsed_time(e1))
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
    del qdst
    host = torch.empty((n, bb), dtype=torch.uint8, pin_memory=True)
    host.copy_(blocks)          # the e2e inputs, before GET overwrites blocks
    # ---- GET: lookup + INT8 dequantise of the whole workload into device
    # buffers (the blocks' own memory is the output)
    store.clear() if world == 1 else sharded.clear()
    if world == 1:
        _, _, dig = store._put_batch_raw(n, ptrs, sizes, None, None, True,
                                         stream)
        keys16 = np.ascontiguousarray(dig[:, :16]).reshape(-1)
        caps = np.full(n, bb, np.uint64)
        for _ in range(2):
            store._get_batch_raw(n, keys16, ptrs, caps, stream)
        torch.cuda.synchronize()
        ga = torch.cuda.Event(enable_timing=True)
        gb_ = torch.cuda.Event(enable_timing=True)
        ga.record()
        for _ in range(3):
            found, gsz = store._get_batch_raw(n, keys16, ptrs, caps, stream)
        gb_.record()
        torch.cuda.synchronize()
        assert found.all() and (gsz == bb).all()
        get_ms = ga.elapsed_time(gb_) / 3
        get_info = {"value": total / (get_ms * 1e-3) / 1e9, "unit": UNIT,
                    "ms": get_ms, "what": "get_batch of every block: index "
                    "lookup + INT8 dequantise into device buffers (FP16 bytes "
                    "out per second)"}
    else:
        # every rank reads the 4096 blocks its neighbour stored: each payload
        # is dequantised straight out of the peer's pool (NVLink reads)
        _, _, dig = sharded.put_batch(blocks, return_status=True)
        mine = torch.from_numpy(np.ascontiguousarray(dig[:, :16])).to(dev)
        every = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
        ids = every[(rank + 1) % world].cpu().numpy()      # (n, 16) keys
        outs = blocks                                      # a block per row
        for _ in range(2):
            sharded.get_batch(ids, outs)
        torch.cuda.synchronize()
        barrier()
        ga = torch.cuda.Event(enable_timing=True)
        gb_ = torch.cuda.Event(enable_timing=True)
        ga.record()
        for _ in range(3):
            found, gsz = sharded.get_batch(ids, outs)
        gb_.record()
        torch.cuda.synchronize()
        assert found.all() and (gsz == bb).all()
        get_ms = max_over_ranks(ga.elapsed_time(gb_) / 3)
        get_info = {"value": world * total / (get_ms * 1e-3) / 1e9,
                    "unit": UNIT, "ms": get_ms,
                    "what": "ShardedCascadeStore.get_batch: every rank reads "
                    "the blocks its neighbour rank stored (owner lookup by "
                    "all-to-all, INT8 dequantise from the peer's pool over "
                    "NVLink); FP16 bytes out per second, all ranks"}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            hbm_peak = float(json.load(f)["hbm_gbs"])
        hbm_src = "MEASURED_PEAKS.json hbm_gbs (of measured)"
    except (OSError, KeyError, ValueError):
        hbm_peak, hbm_src = 6650.0, "profiling-recipe fallback (of fallback)"

    # ---- e2e: host buffers through the public API
    del blocks, dptrs, dsizes, digests
    torch.cuda.empty_cache()
    host_np = host.numpy()
    rows = [host_np[i] for i in range(n)]
    e2e_steps = max(1, min(args.e2e_steps, args.steps))
    if world > 1:
        def e2e_step():
            sharded.clear()
            return sharded.put_batch_host(host_np)
    else:
        def e2e_step():
            store.clear()
            return store.put_batch_host(rows)

    e2e_step()
    torch.cuda.synchronize()
    barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(e2e_steps):   # each call returns after its own sync
        assert e2e_step() == n
    b.record()
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(a.elapsed_time(b)) * 1e-3
    e2e_value = world * e2e_steps * total / e2e_s / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sample = host_np[:SAMPLE_BLOCKS].copy()
        try:
            res = cpu_reference(sample, os.cpu_count() or 1, CPU_MIN_SECONDS)
            one = cpu_reference(sample[:64], 1, 2.0)
            cpu = {"value": res["gbps"], "unit": UNIT,
                   "cores": res["threads"], "kind": "reference",
                   "sample": f"{SAMPLE_BLOCKS} of the {n} blocks "
                             f"({SAMPLE_BLOCKS * bb >> 20} MiB) x "
                             f"{res['passes']} passes",
                   "single_core_value": one["gbps"]}
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
                            "64 rounds x (11 ALU + 5 IMAD) x 2 issue cycles "
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
            "kernel": "minmax_kernel+quantize_kernel", "bound": "hbm",
            "achieved": q_gbps, "peak": hbm_peak, "unit": "GB/s",
            "frac": q_gbps / hbm_peak, "peak_source": hbm_src,
            "algorithmic_bytes": "1.5 x block bytes (min/max re-read not counted)",
            "traffic": (traffic or {}).get("quantize_kernel")},
        "stage_ms": {"sha256": sha_ms, "compress": q_ms},
        "get": get_info,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": UNIT,
                "h2d_bytes_per_step": total, "d2h_bytes_per_step": n * 33,
                "steps": e2e_steps,
                "api": ("CascadeStore.put_batch_host (pinned host blocks, "
                        "striped H2D with hashing under the copy)")
                if world == 1 else
                ("ShardedCascadeStore.put_batch_host (pinned host blocks, "
                 "striped H2D with hashing under the copy, per rank)")},
        "gpu_launches": int(launches),
        "clocks": clk_sum,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        sharded.close()       # every rank unmaps the peers' pools first
    store.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------- extra workloads
def run_extra(args):
    """--workload sweep | dedup | llama3-70b-zipf: the other reference
    configurations, one JSON line each (not the headline line)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from cascade_b200 import cascade_cpp as cc
    from cascade_b200 import workloads

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev,
                                timeout=timedelta(seconds=120))
    stream = torch.cuda.current_stream(dev).cuda_stream

    def timed_steps(step, warm, steps):
        for _ in range(warm):
            step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            out = step()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / steps
        if world > 1:
            t = torch.tensor([ms], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms, out

    def make_store(cap_bytes):
        cfg = cc.CascadeConfig()
        cfg.gpu_device_id = local
        cfg.gpu_capacity_bytes = cap_bytes
        cfg.shm_capacity_bytes = 0
        cfg.kv_compression = True
        cfg.gpu_q8 = True
        cfg.index_slots = 1 << 16
        if world > 1:
            from cascade_b200.sharded import ShardedCascadeStore
            return ShardedCascadeStore(cfg)
        return cc.CascadeStore(cfg)

    def put_fn(store, rows_or_list, n, ptrs, sizes):
        if world > 1:
            def step():
                store.clear()
                return store.put_batch(rows_or_list)
        else:
            def step():
                store.clear()
                return store._put_batch_raw(n, ptrs, sizes, None, None, False,
                                            stream)
        return step

    if args.workload == "sweep":
        res = []
        for layers in (1, 4, 16, 64, 256):          # 64 KiB .. 16 MiB
            bb = workloads.kv_block_bytes(layers, 8, 16, 128)
            n = (1 << 30) // bb
            blocks = workloads.kv_blocks_torch(n, SEED + rank + layers, dev,
                                               layers=layers)
            ptrs = np.arange(n, dtype=np.uint64) * np.uint64(bb) + np.uint64(blocks.data_ptr())
            sizes = np.full(n, bb, np.uint64)
            store = make_store(int(n * bb // 2 * 1.1) + (64 << 20))
            ms, stored = timed_steps(put_fn(store, blocks, n, ptrs, sizes),
                                     args.warmup, args.steps)
            assert stored == n
            res.append({"block_bytes": bb, "blocks_per_gpu": n,
                        "ms_per_step": ms,
                        "gbps": world * n * bb / (ms * 1e-3) / 1e9,
                        "blocks_per_s": world * n / (ms * 1e-3)})
            store.close()     # N > 1: every rank unmaps the peers' pools
            del store, blocks
            torch.cuda.empty_cache()
        line = {"workload": "variable block-size sweep, 1 GiB of FP16 KV per "
                            "size per GPU, content-addressed INT8 PUT",
                "metric": METRIC, "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "sweep": res}
    elif args.workload == "llama3-70b-zipf":
        # 65536 x 5 MiB over 8 GPUs (8192 per GPU), 30 % of them Zipf(1.1)
        # copies of a 1024-block pool that every GPU draws from, so copies
        # repeat inside a GPU's batch and across GPUs
        n, pool_n = 8192, 1024
        seq, pre = workloads.dedup_sequence(n, SEED + rank, pool=pool_n,
                                            sessions=256, shared_frac=0.3)
        geo = workloads.LLAMA3_70B
        pool = workloads.kv_blocks_torch(pool_n, SEED, dev, **geo)
        uniq_n = int((seq >= pool_n).sum())
        uniq = workloads.kv_blocks_torch(uniq_n, SEED + 1000 + rank, dev,
                                         **geo)
        rows = workloads.materialise(seq, pool, uniq)   # copies in own rows
        del pool, uniq
        torch.cuda.empty_cache()
        bb = rows.shape[1]
        ptrs = np.arange(n, dtype=np.uint64) * np.uint64(bb) + np.uint64(rows.data_ptr())
        sizes = np.full(n, bb, np.uint64)
        cap = int(args.cap_gib * (1 << 30))
        if world > 1:
            store = make_store(cap)
        else:
            cfg = cc.CascadeConfig()
            cfg.gpu_device_id = local
            cfg.gpu_capacity_bytes = cap
            cfg.shm_capacity_bytes = 64 << 30     # the demotion target
            cfg.kv_compression = True
            cfg.gpu_q8 = True
            cfg.index_slots = 1 << 16
            store = cc.CascadeStore(cfg)
        ms, stored = timed_steps(put_fn(store, rows, n, ptrs, sizes),
                                 args.warmup, args.steps)
        assert stored == n, stored
        st = store.get_stats()
        store.close()
        # expected hits: all blocks minus the distinct ones (the pool blocks
        # used by any GPU, plus every GPU's unique blocks)
        used = np.zeros(pool_n, np.int32)
        used[np.unique(seq[seq < pool_n])] = 1
        t = torch.tensor(np.concatenate([used, [uniq_n, int(st.dedup_hits),
                                                int(st.gpu_evictions)]]),
                         dtype=torch.int64, device=dev)
        if world > 1:
            every = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(every, t)
        else:
            every = [t]
        ev = torch.stack(every).cpu().numpy()
        distinct = int((ev[:, :pool_n].max(axis=0) > 0).sum()) + int(ev[:, pool_n].sum())
        hits = int(ev[:, pool_n + 1].sum())
        assert hits == world * n - distinct, (hits, world * n, distinct)
        line = {"workload": "llama3-70b KV: 8192 x 5 MiB per GPU, 30% "
                            "Zipf(1.1) copies of a 1024-block pool shared by "
                            "all GPUs, every copy in its own buffer; "
                            "content-addressed INT8 PUT",
                "metric": METRIC, "unit": UNIT, "n_gpus": world,
                "value": world * n * bb / (ms * 1e-3) / 1e9,
                "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup,
                "blocks_total": world * n, "block_bytes": bb,
                "hbm_pool_gib_per_gpu": args.cap_gib,
                "dedup_hits_total": hits, "expected_hits": world * n - distinct,
                "gpu_evictions_total": int(ev[:, pool_n + 2].sum()),
                "parallelism": f"sharded index x{world}" if world > 1 else "1 GPU"}
    else:   # dedup: 8192 blocks, 60 % Zipf copies of 512 shared prefixes
        n = 8192
        seq, pre = workloads.dedup_sequence(n, SEED + rank, pool=512,
                                            sessions=256)
        pool = workloads.kv_blocks_torch(512, SEED, dev)        # shared
        uniq_n = int((seq >= 512).sum())
        uniq = workloads.kv_blocks_torch(uniq_n, SEED + 1000 + rank, dev)
        rows = workloads.materialise(seq, pool, uniq)   # copies in own rows
        del pool, uniq
        bb = rows.shape[1]
        ptrs = np.arange(n, dtype=np.uint64) * np.uint64(bb) + np.uint64(rows.data_ptr())
        sizes = np.full(n, bb, np.uint64)
        # room for the whole batch: a put stores every block speculatively
        # while its keys resolve, then frees the duplicates' slots
        store = make_store(int(n * bb // 2 * 1.1) + (256 << 20))
        ms, stored = timed_steps(put_fn(store, rows, n, ptrs, sizes),
                                 args.warmup, args.steps)
        st = store.get_stats()
        store.close()
        hits = int(st.dedup_hits)
        # expected: all blocks minus the distinct ones (pool blocks used by
        # any GPU, plus every GPU's unique blocks)
        used = np.zeros(512, np.int64)
        used[np.unique(seq[seq < 512])] = 1
        t = torch.tensor(np.concatenate([used, [uniq_n, hits]]),
                         dtype=torch.int64, device=dev)
        if world > 1:
            every = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(every, t)
        else:
            every = [t]
        ev = torch.stack(every).cpu().numpy()
        tot_distinct = int((ev[:, :512].max(axis=0) > 0).sum()) + int(ev[:, 512].sum())
        tot_hits = int(ev[:, 513].sum())
        assert tot_hits == world * n - tot_distinct, (tot_hits, world * n, tot_distinct)
        line = {"workload": "prefix-dedup: 8192 x 2 MiB per GPU, 60% Zipf(1.1) "
                            "copies of 512 shared prefix blocks, 256 sessions; "
                            "every copy in its own buffer",
                "metric": METRIC, "unit": UNIT, "n_gpus": world,
                "value": world * n * bb / (ms * 1e-3) / 1e9,
                "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup,
                "dedup_hits_total": tot_hits,
                "expected_hits": world * n - tot_distinct,
                "parallelism": f"sharded index x{world}" if world > 1 else "1 GPU"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


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
