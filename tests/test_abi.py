"""The C ABI library on a machine without a GPU: it loads, exports every
function include/cascade_b200.h declares, lays its structs out as the
header says, carries the reference's defaults, and refuses to compute
without a CUDA device (there is no CPU path)."""
import ctypes

import numpy as np
import pytest

from cascade_b200 import _lib
from cascade_b200 import cascade_cpp as cc


def test_library_exports_every_declared_function():
    L = _lib.load()
    names = _lib.declared_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_abi_version():
    assert _lib.load().cascade_abi_version() == 1


def test_struct_layouts_match_header():
    a, b = ctypes.c_size_t(), ctypes.c_size_t()
    _lib.load().cascade_struct_sizes(ctypes.byref(a), ctypes.byref(b))
    assert a.value == ctypes.sizeof(cc._CConfig)
    assert b.value == ctypes.sizeof(cc._CStats) == 15 * 8


def test_config_defaults_are_the_references():
    # cascade.hpp:25-60
    c = cc.CascadeConfig()
    assert c.gpu_capacity_bytes == 32 * 1024 ** 3
    assert c.gpu_device_id == 0 and c.use_gpu is True
    assert c.shm_capacity_bytes == 64 * 1024 ** 3
    assert c.shm_path == "/dev/shm/cascade"
    assert c.lustre_path == "cascade_store"
    assert c.lustre_stripe_size == 1024 * 1024 and c.lustre_stripe_count == 16
    assert c.dedup_enabled and c.compression_enabled
    assert c.num_io_threads == 8
    assert c.semantic_eviction and c.promotion_enabled and c.prefetch_enabled
    assert c.prefetch_threads == 2 and c.prefetch_queue_size == 64
    assert c.kv_compression is False and c.aggregated_lustre is False
    assert c.agg_file_size == 256 * 1024 ** 2
    with pytest.raises(AttributeError):
        c.not_a_field = 1


def test_stats_repr_format():
    s = cc._CStats()
    s.gpu_used = 5 << 20
    s.dedup_hits = 3
    s.gpu_hits, s.shm_hits = 2, 1
    r = repr(cc.CascadeStats(s))
    assert r == ("CascadeStats(gpu=5MB, shm=0MB, hits=3, dedup=3, evictions=0, "
                 "promotions=0, prefetch=0, compression_saved=0MB)")


def _no_gpu():
    try:
        import torch
        return not torch.cuda.is_available()
    except Exception:
        return True


@pytest.mark.skipif(not _no_gpu(), reason="checks the no-GPU refusal")
def test_no_cpu_fallback():
    with pytest.raises(_lib.CascadeError) as e:
        cc.CascadeStore(cc.CascadeConfig())
    assert e.value.code == 5
    with pytest.raises(_lib.CascadeError):
        cc.compute_block_id(np.zeros(10, np.uint8))


def test_lustre_tier_not_provided():
    with pytest.raises(NotImplementedError):
        cc.LustreBackend("/tmp/x")
    with pytest.raises(NotImplementedError):
        cc.AggregatedLustreBackend("/tmp/x")


def test_dropin_module_names():
    import importlib
    import os
    import sys
    d = os.path.join(os.path.dirname(_lib.HERE), "cascade_b200", "dropin")
    sys.path.insert(0, d)
    try:
        m = importlib.import_module("cascade_cpp")
        for name in ("CascadeStore", "CascadeConfig", "compute_block_id",
                     "GPUBackend", "ShmBackend", "LustreBackend",
                     "AggregatedLustreBackend"):
            assert hasattr(m, name)
    finally:
        sys.path.remove(d)
        sys.modules.pop("cascade_cpp", None)


def test_ctypes_signatures_match_header_arity():
    """Every entry point the Python layer binds (cascade_cpp, sharded) is
    declared in the header with the same number of parameters, so a
    binding cannot drift from the C ABI."""
    import re

    from cascade_b200 import _lib
    from cascade_b200 import cascade_cpp  # noqa: F401  (registers its entry points)
    from cascade_b200 import sharded  # noqa: F401
    text = open(_lib.HEADER_PATH).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    arity = {}
    for name, params in re.findall(r"\b(cascade_\w+)\s*\(([^;{]*?)\)\s*;",
                                   text, flags=re.S):
        ps = [p for p in params.split(",") if p.strip() not in ("", "void")]
        arity[name] = len(ps)
    assert len(arity) >= 30
    for name, (_, argtypes) in _lib._SIGS.items():
        assert name in arity, name
        assert len(argtypes) == arity[name], (name, len(argtypes), arity[name])
