"""The KV-cache wire format on a machine without a GPU: the golden cases
(made by the reference's own kv_manager.serialize_kv_cache) against the
oracle's restatement, and the host-side pieces of cascade_b200.kvwire."""
import ctypes
import struct

import numpy as np
import pytest

from cascade_b200 import _lib, kvwire
from conftest import load_npz
from oracle import kvwire as okv


def _pairs(d, name):
    L, H, S, D = (int(x) for x in d[name + "_shape"])
    code = int(d[name + "_dtype"])
    raw = d[name + "_src"].tobytes()
    if code == 0:
        vals = np.frombuffer(raw, np.float16)
    elif code == 1:
        vals = okv.bf16_to_f32(np.frombuffer(raw, np.uint16))
    else:
        vals = np.frombuffer(raw, np.float32)
    per = H * S * D
    return [(vals[2 * l * per:(2 * l + 1) * per].reshape(H, S, D),
             vals[(2 * l + 1) * per:(2 * l + 2) * per].reshape(H, S, D))
            for l in range(L)]


def test_golden_wire_bytes_equal_the_oracle():
    d = load_npz("kvwire_cases.npz")
    for name in d["names"]:
        name = str(name)
        want = d[name + "_wire"].tobytes()
        assert okv.serialize(_pairs(d, name)) == want, name
        L, H, S, D = (int(x) for x in d[name + "_shape"])
        assert len(want) == kvwire.wire_bytes(L, H, S, D)
        assert struct.unpack("<IIIIH", want[:18]) == (L, H, S, D, 0)


def test_golden_covers_the_conversion_edges():
    # FP32 and BF16 sources round to FP16 to nearest even, overflow to inf
    d = load_npz("kvwire_cases.npz")
    wire = d["fp32_wire"].tobytes()
    vals = np.frombuffer(wire[18:], np.float16)
    assert np.isinf(vals).any() and (vals == 65504).any()
    assert (np.abs(vals[np.isfinite(vals)]) < 6.2e-5).any()   # subnormals


@pytest.mark.filterwarnings("ignore:overflow encountered in cast")
def test_oracle_deserialize_inverts_serialize():
    d = load_npz("kvwire_cases.npz")
    for name in d["names"]:
        name = str(name)
        back = okv.deserialize(d[name + "_wire"].tobytes())
        for (k, v), (k0, v0) in zip(back, _pairs(d, name)):
            assert np.array_equal(k.view(np.uint16),
                                  k0.astype(np.float16).view(np.uint16))
            assert np.array_equal(v.view(np.uint16),
                                  v0.astype(np.float16).view(np.uint16))


def test_wire_bytes_matches_the_library():
    L = _lib.load()
    kvwire.wire_bytes(1, 1, 1, 1)          # registers the signatures
    for shape in [(1, 1, 1, 1), (32, 8, 16, 128), (80, 8, 16, 128),
                  (3, 1, 7, 12)]:
        assert L.cascade_kv_wire_bytes(*shape) == kvwire.wire_bytes(*shape)


def test_tensor_descriptor_layout():
    assert ctypes.sizeof(kvwire._KvTensor) == 24


def test_extract_kv_pairs_forms():
    class Legacy:
        key_cache = ["k0", "k1"]
        value_cache = ["v0", "v1"]

    class Layer:
        def __init__(self, i):
            self.keys, self.values = f"k{i}", f"v{i}"

    class Layered:
        layers = [Layer(0), Layer(1)]

    want = [("k0", "v0"), ("k1", "v1")]
    assert kvwire.extract_kv_pairs(Legacy()) == want
    assert kvwire.extract_kv_pairs(Layered()) == want
    assert kvwire.extract_kv_pairs((("k0", "v0"), ["k1", "v1"])) == want
    with pytest.raises(ValueError):
        kvwire.extract_kv_pairs(["not a pair"])


def test_serialize_refuses_host_tensors():
    torch = pytest.importorskip("torch")
    kv = ((torch.zeros(1, 2, 3, 8, dtype=torch.float16),) * 2,)
    with pytest.raises(ValueError):
        kvwire.serialize_kv_cache(kv)


def test_batch_helpers_check_arguments_without_a_gpu():
    class NoStore:
        _device = 0
    assert kvwire.load_kv_caches(NoStore(), [], 1, 1, 1, 8) == []
    assert kvwire.store_kv_caches(NoStore(), [], []) == []
    assert kvwire.serialize_kv_caches([]) == []
    assert kvwire.deserialize_kv_caches([]) == []
    with pytest.raises(ValueError):
        kvwire.store_kv_caches(NoStore(), ["a"], [])


def test_read_header_of_host_bytes():
    head = struct.pack("<IIIIH", 32, 8, 16, 128, 0) + b"\0" * 4
    assert kvwire.read_header(np.frombuffer(head, np.uint8)) == (32, 8, 16,
                                                                128, 0)
    with pytest.raises(ValueError):
        kvwire.read_header(np.zeros(5, np.uint8))
