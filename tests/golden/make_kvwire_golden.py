"""Generates tests/golden/kvwire_cases.npz with the reference's own
kv_manager.serialize_kv_cache (inference_benchmark/kv_manager.py:43-63),
run on CPU tensors.

The reference's Python file is imported from the copy that
``make -C oracle callers`` stages under baseline/_ref/callers (or from the
directory in CASCADE_REFERENCE_CALLERS, which holds inference_benchmark/).
Each case stores the source K/V values (their raw bytes in the source
dtype, layer by layer, K then V, each [heads, seq, dim]) and the wire bytes
the reference produced for them.

    python tests/golden/make_kvwire_golden.py
"""
import importlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

# (name, layers, heads, seq, head_dim, dtype)
CASES = [
    ("fp16_vec", 2, 2, 5, 16, torch.float16),
    ("fp16_dim12", 3, 1, 7, 12, torch.float16),
    ("fp16_ragged", 1, 3, 3, 5, torch.float16),
    ("fp16_one", 1, 1, 1, 8, torch.float16),
    ("bf16", 2, 2, 4, 8, torch.bfloat16),
    ("fp32", 2, 4, 3, 32, torch.float32),
    ("fp32_dim6", 2, 2, 3, 6, torch.float32),
]


def _values(rng, shape, dtype):
    """N(0,1) values, with edge values mixed in for the conversions: ties
    between FP16 neighbours, values past the FP16 range, FP16 subnormals,
    signed zeros and infinities."""
    x = rng.standard_normal(shape).astype(np.float32)
    flat = x.reshape(-1)
    edges = np.array([65504.0, 65520.0, 70000.0, -1e6, 6e-8, 3e-8, -2.9e-8,
                      1.00048828125, 1.0009765625 + 0.00048828125, -0.0,
                      np.inf, -np.inf, 2049.0, 2051.0], dtype=np.float32)
    k = min(len(edges), flat.size // 3)
    flat[rng.choice(flat.size, size=k, replace=False)] = edges[:k]
    t = torch.from_numpy(x)
    return t.to(dtype)


def _raw(t):
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint8).tobytes()
    return t.numpy().view(np.uint8).tobytes()


def main():
    callers = os.environ.get("CASCADE_REFERENCE_CALLERS",
                             os.path.join(ROOT, "baseline", "_ref", "callers"))
    sys.path.insert(0, callers)
    kv = importlib.import_module("inference_benchmark.kv_manager")
    rng = np.random.default_rng(4363)
    out = {}
    for name, L, H, S, D, dt in CASES:
        pairs = tuple((_values(rng, (1, H, S, D), dt),
                       _values(rng, (1, H, S, D), dt)) for _ in range(L))
        wire = kv.serialize_kv_cache(pairs)
        src = b"".join(_raw(t[0]) for p in pairs for t in p)
        out[name + "_shape"] = np.array([L, H, S, D], np.int64)
        out[name + "_dtype"] = np.array(
            {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}[dt])
        out[name + "_src"] = np.frombuffer(src, np.uint8)
        out[name + "_wire"] = np.frombuffer(wire, np.uint8)
    out["names"] = np.array([c[0] for c in CASES])
    np.savez_compressed(os.path.join(HERE, "kvwire_cases.npz"), **out)
    print(f"wrote {len(CASES)} cases")


if __name__ == "__main__":
    main()
