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


def test_materialise_copies_in_own_rows():
    import torch
    seq, _ = workloads.dedup_sequence(600, 3, pool=16, sessions=8,
                                      shared_frac=0.3)
    g = torch.Generator().manual_seed(0)
    pool = torch.randint(0, 256, (16, 64), dtype=torch.uint8, generator=g)
    n_uniq = int((seq >= 16).sum())
    uniq = torch.randint(0, 256, (n_uniq, 64), dtype=torch.uint8, generator=g)
    rows = workloads.materialise(seq, pool, uniq)
    assert rows.shape == (600, 64) and rows.is_contiguous()
    for i, k in enumerate(seq):
        want = pool[k] if k < 16 else uniq[k - 16]
        assert torch.equal(rows[i], want)
    # copies of one pool block are equal bytes in distinct rows
    k = int(seq[seq < 16][0])
    idx = np.nonzero(seq == k)[0]
    assert len(idx) >= 1 and all(torch.equal(rows[j], pool[k]) for j in idx)


def test_dedup_sequence_shared_fraction_parameter():
    seq, pre = workloads.dedup_sequence(8192, 2, pool=1024, sessions=256,
                                        shared_frac=0.3)
    assert abs((seq < 1024).mean() - 0.3) < 0.01
    assert pre.sum() == (seq < 1024).sum()
