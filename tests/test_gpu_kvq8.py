"""FP16->INT8 KV compression on the GPU: bit-exact codes, scales and
zero points against the reference's KVCompressor (golden outputs of the
compiled reference and the oracle), and bit-exact dequantisation (the
stated tolerance is 0 ulp; north-star allows 1 ulp)."""
import numpy as np
import pytest
import torch

import oracle
from cascade_b200 import _lib
from cascade_b200 import workloads
from conftest import unpack
from gpu_util import DEV, addr_table, size_table, stream, to_dev

pytestmark = pytest.mark.gpu
ULP_TOLERANCE = 0  # dequantised int16 patterns must match exactly


def _compress(xs, misalign=0):
    src = [to_dev(x, pad_front=misalign) for x in xs]
    dst = [torch.zeros(8 + x.size // 2 + 8, dtype=torch.uint8, device=DEV)
           for x in xs]
    ps, pd = addr_table(src), addr_table(dst)
    sz = size_table([x.size for x in xs])
    _lib.call("cascade_kv_compress_batch", ps.data_ptr(), sz.data_ptr(),
              pd.data_ptr(), len(xs), max(x.size for x in xs), stream())
    torch.cuda.synchronize()
    return [d[:8 + x.size // 2].cpu().numpy() for d, x in zip(dst, xs)]


def _decompress(comps, out_sizes, misalign=0):
    src = [to_dev(c, pad_front=misalign) for c in comps]
    dst = [torch.zeros(n + 16, dtype=torch.uint8, device=DEV) for n in out_sizes]
    ps, pd = addr_table(src), addr_table(dst)
    sz = size_table(out_sizes)
    _lib.call("cascade_kv_decompress_batch", ps.data_ptr(), sz.data_ptr(),
              pd.data_ptr(), len(comps), max(out_sizes), stream())
    torch.cuda.synchronize()
    return [d[:n].cpu().numpy() for d, n in zip(dst, out_sizes)]


def _assert_same_comp(got, want):
    # bytes 5..7 of the header are uninitialised padding in the reference
    assert np.array_equal(got[:5], want[:5])
    assert np.array_equal(got[8:], want[8:])


@pytest.mark.parametrize("misalign", [0, 2, 8])
def test_compress_golden(kvq8_cases, misalign):
    d = kvq8_cases
    xs = [unpack(d, "in", i) for i in range(len(d["in_len"]))]
    got = _compress(xs, misalign)
    for i in range(len(xs)):
        _assert_same_comp(got[i], unpack(d, "comp", i))


@pytest.mark.parametrize("misalign", [0, 1, 8])
def test_decompress_golden(kvq8_cases, misalign):
    d = kvq8_cases
    comps = [unpack(d, "comp", i) for i in range(len(d["in_len"]))]
    sizes = [2 * (int(n) // 2) for n in d["in_len"]]
    got = _decompress(comps, sizes, misalign)
    for i in range(len(comps)):
        want = unpack(d, "dec", i).view(np.int16).astype(np.int32)
        diff = np.abs(got[i].view(np.int16).astype(np.int32) - want)
        assert diff.max(initial=0) <= ULP_TOLERANCE, i


def test_decompress_fma_discriminating(kvq8_cases):
    d = kvq8_cases
    n = len(d["fma_comp_len"])
    comps = [d["fma_comp"][d["fma_comp_off"][i]:][:d["fma_comp_len"][i]]
             for i in range(n)]
    got = _decompress(comps, [512] * n)
    for i in range(n):
        want = d["fma_out"][d["fma_out_off"][i]:][:d["fma_out_len"][i]]
        assert np.array_equal(got[i], want)


@pytest.mark.parametrize("scale", [0.003, 1.0, -3.7, 257.0, 8191.75, 8192.0,
                                   8192.5, -8192.0, -9000.25, 20000.125,
                                   1.0e5])
def test_decompress_headers_either_side_of_the_fast_path(scale):
    """Headers of any scale (including ones the compressor never writes:
    negative, or large enough to wrap the 16-bit result) decode like the
    oracle for every code, every zero point sign and values on both sides
    of zero."""
    codes = np.arange(256, dtype=np.uint8)
    comps = []
    for zp in (-128, -77, -1, 0, 1, 64, 127):
        hdr = np.zeros(8, np.uint8)
        hdr[:4] = np.frombuffer(np.float32(scale).tobytes(), np.uint8)
        hdr[4] = np.uint8(zp & 0xff)
        comps.append(np.concatenate([hdr, codes, codes[::-1]]))
    got = _decompress(comps, [1024] * len(comps))
    for c, g in zip(comps, got):
        assert np.array_equal(g, oracle.kv_decompress(c, 1024))


def test_llama_kv_blocks_roundtrip_vs_oracle():
    blocks = workloads.kv_blocks_np(6, 21)          # 6 x 2 MiB, outliers
    got = _compress(list(blocks))
    for b, c in zip(blocks, got):
        want = oracle.kv_compress(b)
        _assert_same_comp(c, want)
    dec = _decompress(got, [b.size for b in blocks])
    for b, c, o in zip(blocks, got, dec):
        assert np.array_equal(o, oracle.kv_decompress(c, b.size))


def test_copy_batch_ragged():
    rng = np.random.default_rng(3)
    xs = [rng.integers(0, 256, n, dtype=np.uint8)
          for n in (0, 1, 15, 16, 17, 4095, 65536 + 7, 1 << 20)]
    for misalign in (0, 3):
        src = [to_dev(x, pad_front=misalign) for x in xs]
        dst = [torch.zeros(x.size + 32, dtype=torch.uint8, device=DEV) for x in xs]
        ps, pd = addr_table(src), addr_table(dst)
        sz = size_table([x.size for x in xs])
        _lib.call("cascade_copy_batch", ps.data_ptr(), pd.data_ptr(),
                  sz.data_ptr(), len(xs), max(x.size for x in xs), stream())
        torch.cuda.synchronize()
        for x, d in zip(xs, dst):
            h = d.cpu().numpy()
            assert np.array_equal(h[:x.size], x)
            assert not h[x.size:].any()   # nothing written past the end


@pytest.mark.parametrize("misalign", [0, 2, 8])
@pytest.mark.parametrize("top", [2 << 20, 512 << 10, 5 << 20],
                         ids=["2MiB", "512KiB", "5MiB"])
def test_single_pass_compress_mixed_batch_vs_oracle(misalign, top):
    # Batches whose largest block is 512 KiB - 6 MiB take the single-pass
    # cluster kernel (clusters of 8, 2 and 16 CTAs here).  Enough blocks
    # that every cluster runs several (so the blocks between the reducer and
    # quantiser warps and the pair exchange reach steady state), of ragged
    # sizes: odd, tiny, empty and not a multiple of the 16-byte groups;
    # misaligned sources take the kernel's direct path.
    rng = np.random.default_rng(40 + misalign + top)
    sizes = [top, top - 2, top // 2 + 6, 0, 1, 100, (3 * top) // 4 + 3,
             top // 2]
    xs = []
    count = {2 << 20: 64, 512 << 10: 400, 5 << 20: 40}[top]
    for i in range(count):
        n = sizes[i % len(sizes)]
        if i % 3 == 0:      # KV-like values with outliers
            x = (rng.standard_normal(n // 2 + 1) * 3).astype(np.float16)
            x[::997] *= 20
            xs.append(x.view(np.uint8)[:n].copy())
        else:               # arbitrary int16 ranges
            lo = int(rng.integers(-32768, 32767))
            hi = int(rng.integers(lo, 32768))
            xs.append(rng.integers(lo, hi + 1, n // 2 + 1)
                      .astype(np.int16).view(np.uint8)[:n].copy())
    got = _compress(xs, misalign)
    for i, x in enumerate(xs):
        _assert_same_comp(got[i], oracle.kv_compress(x))
