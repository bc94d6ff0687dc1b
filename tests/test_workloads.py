"""Synthetic workload generators keep the reference benchmarks' shapes."""
import numpy as np

from cascade_b200 import workloads


def test_llama3_8b_block_is_2mib():
    assert workloads.kv_block_bytes(**workloads.LLAMA3_8B) == 2 * 1024 * 1024
    assert workloads.kv_block_bytes(**workloads.LLAMA3_70B) == 5 * 1024 * 1024


def test_kv_blocks_outliers():
    b = workloads.kv_blocks_np(2, 7, layers=4)
    x = b[0].view(np.float16).astype(np.float32).reshape(4, 2, 8, 16, 128)
    ch = np.abs(x).max(axis=3).ravel()   # per (layer, kv, head, dim) channel
    n_out = int(round(0.001 * ch.size))
    assert n_out >= 1
    assert (ch > 10).sum() >= n_out - 1  # scaled x20: far above N(0,1)
    assert np.isfinite(x).all()


def test_dedup_sequence_mix():
    seq, pre = workloads.dedup_sequence(8192, 1)
    assert seq.size == 8192
    frac = (seq < 512).mean()
    assert abs(frac - 0.6) < 0.01
    assert pre.sum() == (seq < 512).sum()
    # unique blocks are unique
    u = seq[seq >= 512]
    assert len(np.unique(u)) == u.size
