"""Seeded synthetic KV-block workloads with the reference benchmarks' shapes.

There is no KV-cache dump or dataset on this machine, so blocks are made up
with the shapes and value distributions the reference's drivers use:

* ``kv_blocks``: FP16 KV blocks laid out [layers][K,V][kv_heads][tokens]
  [head_dim] (the per-layer K,V order of kv_manager.serialize_kv_cache,
  inference_benchmark/kv_manager.py:43-63); values N(0,1) with a fraction
  of (layer, kv, head, dim) channels scaled as outliers across all tokens.
  Llama-3-8B shape: 32 layers x 8 heads x 16 tokens x 128 dims = 2 MiB.
* ``dedup_sequence``: the prefix-sharing mix — sessions whose leading blocks
  are drawn from a pool of shared prefix blocks by a bounded Zipf law, the
  rest unique — as a sequence of block-content indices.
* ``random_bytes``: uniform bytes (the 1 MiB reference smoke workload,
  script_example/05_sensitivity/dedup/dedup_driver.py:46-62 style).
"""
from __future__ import annotations

import numpy as np

LLAMA3_8B = dict(layers=32, kv_heads=8, tokens=16, head_dim=128)
LLAMA3_70B = dict(layers=80, kv_heads=8, tokens=16, head_dim=128)


def kv_block_bytes(layers, kv_heads, tokens, head_dim) -> int:
    """2 (K,V) x layers x heads x tokens x dim x 2 bytes (FP16)."""
    return 2 * layers * kv_heads * tokens * head_dim * 2


def outlier_channels(rng: np.random.Generator, layers, kv_heads, head_dim,
                     frac=0.001) -> np.ndarray:
    n_ch = layers * 2 * kv_heads * head_dim
    k = max(1, int(round(frac * n_ch)))
    return np.sort(rng.choice(n_ch, size=k, replace=False))


def kv_blocks_np(n: int, seed: int, layers=32, kv_heads=8, tokens=16,
                 head_dim=128, outlier_frac=0.001, outlier_scale=20.0):
    """n KV blocks as a uint8 array [n, block_bytes] (host, numpy)."""
    rng = np.random.default_rng(seed)
    ch = outlier_channels(rng, layers, kv_heads, head_dim, outlier_frac)
    out = np.empty((n, kv_block_bytes(layers, kv_heads, tokens, head_dim)),
                   np.uint8)
    for i in range(n):
        x = rng.standard_normal((layers, 2, kv_heads, tokens, head_dim),
                                dtype=np.float32)
        # channel c = ((layer*2 + kv)*heads + head)*dim + d
        x = x.transpose(0, 1, 2, 4, 3).reshape(-1, tokens)
        x[ch] *= outlier_scale
        x = x.reshape(layers, 2, kv_heads, head_dim, tokens).transpose(0, 1, 2, 4, 3)
        out[i] = np.ascontiguousarray(x).astype(np.float16).view(np.uint8).ravel()
    return out


def kv_blocks_torch(n: int, seed: int, device, layers=32, kv_heads=8,
                    tokens=16, head_dim=128, outlier_frac=0.001,
                    outlier_scale=20.0):
    """n KV blocks generated on the GPU: a CUDA uint8 tensor [n, bytes].
    Same distribution as kv_blocks_np (not the same bytes)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    rng = np.random.default_rng(seed)
    ch = torch.as_tensor(outlier_channels(rng, layers, kv_heads, head_dim,
                                          outlier_frac), device=device)
    scale = torch.ones(layers * 2 * kv_heads * head_dim, device=device)
    scale[ch] = outlier_scale
    scale = scale.view(layers, 2, kv_heads, 1, head_dim)
    bb = kv_block_bytes(layers, kv_heads, tokens, head_dim)
    out = torch.empty((n, bb), dtype=torch.uint8, device=device)
    step = max(1, (1 << 30) // (bb * 2))  # ~1 GiB of fp32 at a time
    for s in range(0, n, step):
        m = min(step, n - s)
        x = torch.randn((m, layers, 2, kv_heads, tokens, head_dim),
                        generator=g, device=device, dtype=torch.float32)
        x.mul_(scale)
        out[s:s + m] = x.to(torch.float16).view(m, -1).view(torch.uint8)
    return out


def random_bytes(n: int, size: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).integers(0, 256, (n, size), dtype=np.uint8)


def dedup_sequence(n_blocks: int, seed: int, pool=512, sessions=256,
                   shared_frac=0.6, zipf_s=1.1, prefix_min=4, prefix_max=64):
    """Block-content indices for the prefix-dedup workload.

    Index k < pool names shared prefix block k; index >= pool names a
    unique block.  Each session starts with a shared prefix of
    U{prefix_min..prefix_max} blocks drawn from the pool with
    p(k) ~ (k+1)^-zipf_s, then unique blocks; the mix is trimmed so that
    shared_frac of the n_blocks are pool copies.  Returns (seq, is_prefix).
    """
    rng = np.random.default_rng(seed)
    ranks = np.arange(1, pool + 1, dtype=np.float64)
    p = ranks ** (-zipf_s)
    p /= p.sum()
    per_session = n_blocks // sessions
    n_shared = int(round(shared_frac * n_blocks))
    lens = rng.integers(prefix_min, prefix_max + 1, sessions)
    # scale prefix lengths so their sum is the shared target
    lens = np.maximum(1, np.round(lens * n_shared / lens.sum())).astype(int)
    lens = np.minimum(lens, per_session)
    diff = n_shared - int(lens.sum())
    i = 0
    while diff != 0:
        j = i % sessions
        if diff > 0 and lens[j] < per_session:
            lens[j] += 1
            diff -= 1
        elif diff < 0 and lens[j] > 1:
            lens[j] -= 1
            diff += 1
        i += 1
    seq, pre = [], []
    nxt = pool
    for sidx in range(sessions):
        m = per_session if sidx < sessions - 1 else n_blocks - per_session * (sessions - 1)
        k = int(min(lens[sidx], m))
        seq.extend(rng.choice(pool, size=k, p=p).tolist())
        pre.extend([True] * k)
        for _ in range(m - k):
            seq.append(nxt)
            nxt += 1
            pre.append(False)
    return np.asarray(seq, dtype=np.int64), np.asarray(pre, dtype=bool)


def materialise(seq, pool, uniq):
    """One CUDA row per entry of ``seq`` (``dedup_sequence``): row i is a
    byte copy of pool block seq[i], or unique block seq[i] - len(pool).
    Copies live in their own rows, as the KV blocks of two sessions that
    share a prefix live in two buffers."""
    import torch
    n, npool = len(seq), pool.shape[0]
    out = torch.empty((n, pool.shape[1]), dtype=torch.uint8, device=pool.device)
    idx = torch.as_tensor(np.asarray(seq), device=pool.device)
    shared = torch.nonzero(idx < npool).flatten()
    own = torch.nonzero(idx >= npool).flatten()
    step = 256
    for a in range(0, shared.numel(), step):
        j = shared[a:a + step]
        out[j] = pool[idx[j]]
    for a in range(0, own.numel(), step):
        j = own[a:a + step]
        out[j] = uniq[idx[j] - npool]
    return out
