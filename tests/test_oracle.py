"""The oracle against OpenSSL (hashlib), the reference's golden outputs and,
when it is built here, the compiled reference itself."""
import hashlib

import numpy as np
import pytest

import oracle
from conftest import unpack
from make_golden import SHA_LENGTHS, STORED_MAX, sha_input


def _sha_input(d, i):
    n = int(d["lengths"][i])
    if n <= STORED_MAX:
        off = int(d["offsets"][i])
        return d["data"][off:off + n]
    return sha_input(n)


def test_sha256_fips_examples():
    # FIPS 180-4 example messages; expected digests come from OpenSSL.
    for msg in (b"abc", b"",
                b"abcdbcdecdefdefgefghfghighijhijkijkljklmklmnlmnomnopnopq",
                b"a" * 1000):
        arr = np.frombuffer(msg, np.uint8)
        assert oracle.sha256(arr) == hashlib.sha256(msg).digest()


def test_sha256_golden_all_lengths(sha_cases):
    d = sha_cases
    assert list(d["lengths"]) == SHA_LENGTHS
    for i in range(len(SHA_LENGTHS)):
        x = _sha_input(d, i)
        assert oracle.sha256(x) == d["digests"][i].tobytes(), int(d["lengths"][i])
        assert oracle.block_id(x) == str(d["block_ids"][i])


def test_kvq8_golden(kvq8_cases):
    d = kvq8_cases
    for i in range(len(d["in_len"])):
        x = unpack(d, "in", i)
        c = oracle.kv_compress(x)
        ref_c = unpack(d, "comp", i)
        assert np.array_equal(c, ref_c), i
        out = oracle.kv_decompress(ref_c, 2 * (x.size // 2))
        assert np.array_equal(out, unpack(d, "dec", i)), i


def test_kvq8_fma_cases(kvq8_cases):
    d = kvq8_cases
    for i in range(len(d["fma_comp_len"])):
        c = d["fma_comp"][d["fma_comp_off"][i]:][:d["fma_comp_len"][i]]
        want = d["fma_out"][d["fma_out_off"][i]:][:d["fma_out_len"][i]]
        assert np.array_equal(oracle.kv_decompress(c, 512), want)


def test_kvq8_zero_point_wraps():
    # min -1000, max -1: scale = 999/255, min/scale = -255.26 -> -255, which
    # the reference's (int8_t) cast wraps to 1 (cascade_core.cpp:832).
    s, z = oracle.kv_params(-1000, -1)
    assert s == float(np.float32(999.0) / np.float32(255.0))
    q = int(np.trunc(np.float32(-1000.0) / np.float32(s)))
    assert q == -255
    assert z == 1


@pytest.mark.skipif(oracle.ref() is None, reason="oracle/_ref not built here")
def test_oracle_matches_compiled_reference_random():
    rng = np.random.default_rng(99)
    for _ in range(300):
        lo = int(rng.integers(-32768, 32767))
        hi = int(rng.integers(lo, 32768))
        n = int(rng.integers(1, 4000))
        x = rng.integers(lo, hi + 1, n).astype(np.int16).view(np.uint8)
        c = oracle.kv_compress(x)
        assert np.array_equal(c, oracle.ref_kv_compress(x))
        assert np.array_equal(oracle.kv_decompress(c, x.size),
                              oracle.ref_kv_decompress(c, x.size))
        assert oracle.block_id(x) == oracle.ref_block_id(x)


def test_quantise_clamp_never_binds():
    """The device quantiser drops the reference's clamp to [0, 255]
    (cascade_core.cpp:842-846): for every int16 range, d = range (the
    largest difference) gives fma(d, RN(1 / RN(range / 255)), 0.5) below
    256, and the code grows with d, so no code exceeds 255."""
    rng = np.arange(1, 65536, dtype=np.float64)
    scale = (rng.astype(np.float32) / np.float32(255.0)).astype(np.float32)
    inv = (np.float32(1.0) / scale).astype(np.float32)
    r = (rng * inv.astype(np.float64) + 0.5).astype(np.float32)  # one rounding
    assert float(r.max()) < 256.0
    assert float(np.floor(r).max()) == 255.0
