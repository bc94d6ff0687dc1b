"""Generates the golden fixtures in tests/golden/ from the reference itself.

Run in a container that has the reference tree (it builds
oracle/_ref/libcascade_ref.so from the reference's own sources with
`make -C oracle ref`):

    python tests/golden/make_golden.py

Outputs (committed; the tests only read them):
  sha256_cases.npz    message lengths 0..300 and larger, seeded inputs,
                      full digests (hashlib = OpenSSL, the library the
                      reference calls) and the reference's compute_block_id.
  kvq8_cases.npz      KVCompressor::compress / decompress outputs of the
                      reference build for seeded int16 patterns: the full
                      65536-value sweep, random sub-ranges, degenerate and
                      extreme blocks, and decompress inputs whose FMA and
                      non-FMA results differ.
  store_scenarios.json  put/get/contains sequences replayed on the
                      reference CascadeStore (use_gpu=False, the configuration
                      it can run without a GPU), with every result and the
                      final CascadeStats.
"""
from __future__ import annotations

import hashlib
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from cascade_b200 import workloads  # noqa: E402

SHA_LENGTHS = list(range(0, 301)) + [447, 448, 511, 512, 1000, 4095, 4096,
                                     4097, 65535, 65536, 65537, 1 << 20,
                                     (1 << 20) + 3]


STORED_MAX = 4097  # longer inputs are regenerated from sha_input(n)


def sha_input(n: int) -> np.ndarray:
    """The seeded input of length n (the tests regenerate long ones)."""
    return np.random.default_rng(20261201 + n).integers(0, 256, n,
                                                        dtype=np.uint8)


def sha_cases():
    blob, offs, digests, ids = [], [], [], []
    pos = 0
    for n in SHA_LENGTHS:
        d = sha_input(n)
        if n <= STORED_MAX:
            blob.append(d)
            offs.append(pos)
            pos += n
        else:
            offs.append(-1)
        digests.append(np.frombuffer(hashlib.sha256(d.tobytes()).digest(),
                                     np.uint8))
        ids.append(oracle.ref_block_id(d))
        assert ids[-1] == hashlib.sha256(d.tobytes()).hexdigest()[:32]
    np.savez_compressed(os.path.join(HERE, "sha256_cases.npz"),
                        lengths=np.array(SHA_LENGTHS, np.int64),
                        offsets=np.array(offs, np.int64),
                        data=np.concatenate(blob),
                        digests=np.stack(digests),
                        block_ids=np.array(ids))


def _fma_discriminating(rng, want=16):
    """Compressed blocks whose decompression differs between a fused and an
    unfused multiply-add, so the fixture pins which one the reference does."""
    L = oracle.lib()
    found = []
    while len(found) < want:
        lo = int(rng.integers(-32768, 32767))
        hi = int(rng.integers(lo, 32768))
        s, z = oracle.kv_params(lo, hi)
        comp = np.zeros(8 + 256, np.uint8)
        comp[:4] = np.frombuffer(np.float32(s).tobytes(), np.uint8)
        comp[4] = np.uint8(z & 0xFF)
        comp[8:] = np.arange(256, dtype=np.uint8)
        fused = oracle.kv_decompress(comp, 512).view(np.int16)
        minf = float(np.float32(np.float32(z) * np.float32(s)))
        unf = np.array([L.oracle_kv_value_unfused(int(np.int8(np.uint8(c))), s,
                                                  minf) for c in range(256)],
                       np.int16)
        if np.any(fused != unf):
            found.append(comp)
    return found


def kvq8_cases():
    rng = np.random.default_rng(818)
    inputs = [np.arange(-32768, 32768, dtype=np.int16).view(np.uint8)]
    for _ in range(96):
        lo = int(rng.integers(-32768, 32767))
        hi = int(rng.integers(lo, 32768))
        n = int(rng.integers(1, 1000))
        inputs.append(rng.integers(lo, hi + 1, n).astype(np.int16).view(np.uint8))
    inputs += [
        np.full(64, 7, np.uint8),                                  # range 0
        np.array([0x00, 0x80] * 40, np.uint8),                     # all -32768
        np.array([0xFF, 0x7F] * 40, np.uint8),                     # all 32767
        np.array([0x00, 0x80, 0xFF, 0x7F] * 20, np.uint8),         # extremes
        rng.integers(0, 256, 65, dtype=np.uint8),                  # odd size
        rng.integers(0, 256, 2, dtype=np.uint8),                   # one value
        workloads.kv_blocks_np(1, 3, layers=2)[0],                 # KV-shaped
    ]
    comp, dec = [], []
    for x in inputs:
        c = oracle.ref_kv_compress(x)
        comp.append(c)
        dec.append(oracle.ref_kv_decompress(c, 2 * (x.size // 2)))
    fma = _fma_discriminating(rng)
    fma_out = [oracle.ref_kv_decompress(c, 512) for c in fma]

    def pack(arrs):
        lens = np.array([a.size for a in arrs], np.int64)
        offs = np.concatenate([[0], np.cumsum(lens)[:-1]]).astype(np.int64)
        return np.concatenate(arrs), offs, lens

    d_in, o_in, l_in = pack(inputs)
    d_c, o_c, l_c = pack(comp)
    d_d, o_d, l_d = pack(dec)
    d_f, o_f, l_f = pack(fma)
    d_fo, o_fo, l_fo = pack(fma_out)
    np.savez_compressed(os.path.join(HERE, "kvq8_cases.npz"),
                        in_data=d_in, in_off=o_in, in_len=l_in,
                        comp_data=d_c, comp_off=o_c, comp_len=l_c,
                        dec_data=d_d, dec_off=o_d, dec_len=l_d,
                        fma_comp=d_f, fma_comp_off=o_f, fma_comp_len=l_f,
                        fma_out=d_fo, fma_out_off=o_fo, fma_out_len=l_fo)


# ------------------------------------------------------------ store runs
def scenario_blocks(kind: str, seed: int):
    """(ids, blocks, is_prefix) for a named scenario (regenerated by tests)."""
    if kind == "random_1k":        # reference smoke shape, scaled down
        b = workloads.random_bytes(64, 1024, seed)
        pre = [i < 32 for i in range(64)]
        return [oracle.block_id(x) for x in b], list(b), pre
    if kind == "kv_small":         # KV-shaped blocks, 2 layers (16 KiB)
        b = workloads.kv_blocks_np(24, seed, layers=2)
        return [oracle.block_id(x) for x in b], list(b), [False] * 24
    if kind == "dedup":            # prefix-sharing mix, 1 KiB blocks
        seq, pre = workloads.dedup_sequence(384, seed, pool=32, sessions=12,
                                            prefix_min=4, prefix_max=16)
        rng = np.random.default_rng(seed)
        pool = rng.integers(0, 256, (32, 1024), dtype=np.uint8)
        uniq = rng.integers(0, 256, (384, 1024), dtype=np.uint8)
        blocks = [pool[k] if k < 32 else uniq[k - 32] for k in seq]
        return [oracle.block_id(x) for x in blocks], blocks, list(pre)
    if kind == "sizes":            # size edge cases, named ids
        sizes = [0, 1, 2, 7, 63, 64, 65, 127, 128, 255, 256, 257, 4095, 4096,
                 4097]
        rng = np.random.default_rng(seed)
        blocks = [rng.integers(0, 256, s, dtype=np.uint8) for s in sizes]
        return [f"block_{s}" for s in sizes], blocks, [False] * len(sizes)
    raise KeyError(kind)


SCENARIOS = [
    # name, kind, seed, kv_compression, dedup_enabled, shm_capacity
    ("random_1k_plain", "random_1k", 1, False, True, 64 << 20),
    ("random_1k_q8", "random_1k", 1, True, True, 64 << 20),
    ("kv_small_q8", "kv_small", 2, True, True, 64 << 20),
    ("dedup_plain", "dedup", 3, False, True, 64 << 20),
    ("dedup_q8", "dedup", 3, True, True, 64 << 20),
    ("dedup_off", "dedup", 3, False, False, 64 << 20),
    ("sizes_plain", "sizes", 4, False, True, 64 << 20),
]


def run_scenario(name, kind, seed, kvc, dedup, shm_cap, shm_dir):
    ids, blocks, pre = scenario_blocks(kind, seed)
    st = oracle.RefStore(os.path.join(shm_dir, name), shm_cap,
                         kv_compression=kvc, dedup_enabled=dedup)
    puts = [st.put(i, b, p) for i, b, p in zip(ids, blocks, pre)]
    gets = []
    buf = np.zeros(1 << 20, np.uint8)
    order = list(range(len(ids)))[::-1] + ["missing_block"]
    for k in order:
        bid = ids[k] if k != "missing_block" else "ffffffffffffffffffffffffffffff00"
        found, size = st.get(bid, buf)
        gets.append([bid, bool(found), int(size),
                     hashlib.sha256(buf[:size].tobytes()).hexdigest()
                     if found else None])
    contains = [st.contains(i) for i in ids]
    stats = st.stats()
    st.close()
    return dict(name=name, kind=kind, seed=seed, kv_compression=kvc,
                dedup_enabled=dedup, shm_capacity=shm_cap, ids=ids,
                is_prefix=[bool(x) for x in pre], puts=puts, gets=gets,
                contains=contains, stats=stats)


def store_scenarios():
    out = []
    with tempfile.TemporaryDirectory(dir="/dev/shm") as d:
        for sc in SCENARIOS:
            out.append(run_scenario(*sc, shm_dir=d))
    with open(os.path.join(HERE, "store_scenarios.json"), "w") as f:
        json.dump(out, f, indent=1)


def main():
    # The reference's C++ tree: oracle/Makefile's REF, or the directory in
    # CASCADE_REFERENCE_CPP.
    make = ["make", "-s", "-C", os.path.join(ROOT, "oracle")]
    if os.environ.get("CASCADE_REFERENCE_CPP"):
        make.append("REF=" + os.environ["CASCADE_REFERENCE_CPP"])
    if subprocess.run(make + ["-n", "ref"], capture_output=True).returncode:
        sys.exit("needs the reference tree to build oracle/_ref "
                 "(set CASCADE_REFERENCE_CPP)")
    subprocess.check_call(make + ["oracle", "ref"])
    sha_cases()
    kvq8_cases()
    store_scenarios()
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
