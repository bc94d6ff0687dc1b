"""ORACLE — the timed CPU baseline (test/bench infrastructure only).

Times the reference's own CPU ingest path — compute_block_id (OpenSSL
SHA-256) + KVCompressor::compress + ShmBackend::put, i.e. CascadeStore::put
with use_gpu=False and kv_compression=True (cascade_core.cpp:1074-1135),
driven by the reference's OpenMP put_batch (cascade_core.cpp:1203-1218) —
from oracle/_ref/libcascade_ref.so, on this host's cores.

Run as a separate process so the reference's OpenMP runtime never shares a
process with torch:

    python -m oracle.ref_bench --input /dev/shm/x.npy --threads 16 \
        --min-seconds 3
Prints one JSON object: GB/s of FP16 input hashed+compressed+stored.
"""
from __future__ import annotations

import argparse
import json
import os
import tempfile
import time

import numpy as np


def run(blocks: np.ndarray, threads: int, min_seconds: float,
        max_passes: int = 1000, warmup: int = 1, steps: int = 0,
        lib_path: str = ""):
    """Times put passes over `blocks` (each into an emptied store): exactly
    `steps` passes when steps > 0, else passes until min_seconds."""
    import oracle
    if lib_path:
        oracle.REF_SO = lib_path
    if oracle.ref() is None:
        raise SystemExit(f"{oracle.REF_SO} is not built")
    n, size = blocks.shape
    rows = [blocks[i] for i in range(n)]
    shm_dir = tempfile.mkdtemp(prefix="cascade_ref_", dir="/dev/shm")
    cap = int(n * (8 + size // 2) * 1.05) + (64 << 20)
    store = oracle.RefStore(shm_dir, cap, kv_compression=True,
                            dedup_enabled=True)
    try:
        for _ in range(warmup):
            store.clear()
            assert store.put_path(rows, threads) == n
        passes, total = 0, 0.0
        while (passes < steps) if steps > 0 else (
                passes < max_passes and (total < min_seconds or passes == 0)):
            store.clear()
            t0 = time.perf_counter()
            ok = store.put_path(rows, threads)
            total += time.perf_counter() - t0
            passes += 1
            assert ok == n, (ok, n)
        return dict(gbps=passes * n * size / total / 1e9, passes=passes,
                    seconds=total, blocks=n, block_bytes=size,
                    threads=threads)
    finally:
        store.close()
        try:
            os.unlink(os.path.join(shm_dir, "data.mmap"))
            os.rmdir(shm_dir)
        except OSError:
            pass


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--input", required=True, help=".npy uint8 [n, bytes]")
    ap.add_argument("--threads", type=int, default=os.cpu_count())
    ap.add_argument("--min-seconds", type=float, default=3.0)
    ap.add_argument("--max-passes", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--steps", type=int, default=0)
    ap.add_argument("--lib", default="",
                    help="reference build to time (default oracle/_ref)")
    a = ap.parse_args()
    blocks = np.load(a.input, mmap_mode="r")
    blocks = np.ascontiguousarray(blocks)
    print(json.dumps(run(blocks, a.threads, a.min_seconds, a.max_passes,
                         a.warmup, a.steps, a.lib)))


if __name__ == "__main__":
    main()
