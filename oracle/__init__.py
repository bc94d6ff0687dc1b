"""ORACLE — test infrastructure only.

ctypes front-ends for the two CPU checkers built by ``oracle/Makefile``:

* ``liboracle.so`` (``oracle/_build``): the plain-C restatement of the
  reference's SHA-256 content addressing (cascade_core.cpp:43-53, which calls
  OpenSSL's SHA256 at line 45) and of KVCompressor
  (cascade_core.cpp:818-872).
* ``libcascade_ref.so`` (``oracle/_ref``): the unmodified reference sources
  behind a small C harness (``oracle/ref_harness.cpp``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
and reference legs may import this package; the product never does.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libcascade_ref.so")
# The same reference sources built with the bench host's -march=native
# expansion (oracle/native_march.txt); the timed CPU baseline there.
REF_NATIVE_SO = os.path.join(HERE, "_ref", "native", "libcascade_ref.so")
NATIVE_MARCH_TXT = os.path.join(HERE, "native_march.txt")


def host_march() -> Optional[str]:
    """The options GCC's -march=native expands to on this host (one line),
    or None when no compiler is available."""
    import subprocess
    try:
        out = subprocess.run(["sh", os.path.join(HERE, "probe_march.sh")],
                             capture_output=True, text=True, timeout=60)
    except (OSError, subprocess.TimeoutExpired):
        return None
    line = out.stdout.strip()
    return line if out.returncode == 0 and line else None


def native_build_matches_host() -> bool:
    """Whether oracle/_ref/native was built with exactly this host's
    -march=native options (so it is the reference's own native build)."""
    if not os.path.exists(REF_NATIVE_SO):
        return False
    here = host_march()
    with open(NATIVE_MARCH_TXT) as f:
        built = f.read().strip()
    return here is not None and here.split() == built.split()


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"

_u8p = ctypes.POINTER(ctypes.c_uint8)
_lib = None
_ref = None


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(_u8p)


def lib() -> ctypes.CDLL:
    """The C restatement; raises if ``make -C oracle`` has not been run."""
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            raise FileNotFoundError(f"{ORACLE_SO} missing: run `make -C oracle`")
        L = ctypes.CDLL(ORACLE_SO)
        L.oracle_sha256.argtypes = [_u8p, ctypes.c_size_t, _u8p]
        L.oracle_block_id.argtypes = [_u8p, ctypes.c_size_t, ctypes.c_char_p]
        L.oracle_kv_compress.argtypes = [_u8p, ctypes.c_size_t, _u8p]
        L.oracle_kv_compress.restype = ctypes.c_size_t
        L.oracle_kv_decompress.argtypes = [_u8p, ctypes.c_size_t, _u8p,
                                           ctypes.c_size_t]
        L.oracle_kv_decompress.restype = ctypes.c_int
        L.oracle_kv_params.argtypes = [ctypes.c_int16, ctypes.c_int16,
                                       ctypes.POINTER(ctypes.c_float),
                                       ctypes.POINTER(ctypes.c_int8)]
        for name in ("oracle_kv_code", "oracle_kv_code_unfused"):
            f = getattr(L, name)
            f.argtypes = [ctypes.c_int16, ctypes.c_float, ctypes.c_float]
            f.restype = ctypes.c_int8
        L.oracle_kv_value_unfused.argtypes = [ctypes.c_int8, ctypes.c_float,
                                              ctypes.c_float]
        L.oracle_kv_value_unfused.restype = ctypes.c_int16
        _lib = L
    return _lib


def ref() -> Optional[ctypes.CDLL]:
    """The compiled reference, or None when ``oracle/_ref`` was not built."""
    global _ref
    if _ref is None and os.path.exists(REF_SO):
        R = ctypes.CDLL(REF_SO)
        R.ref_compute_block_id.argtypes = [_u8p, ctypes.c_size_t,
                                           ctypes.c_char_p]
        R.ref_kv_compress.argtypes = [_u8p, ctypes.c_size_t, _u8p,
                                      ctypes.c_size_t]
        R.ref_kv_compress.restype = ctypes.c_size_t
        R.ref_kv_decompress.argtypes = [_u8p, ctypes.c_size_t, _u8p,
                                        ctypes.c_size_t]
        R.ref_kv_decompress.restype = ctypes.c_int
        R.ref_store_create.argtypes = [ctypes.c_char_p, ctypes.c_size_t,
                                       ctypes.c_int, ctypes.c_int]
        R.ref_store_create.restype = ctypes.c_void_p
        R.ref_store_create_gpu.argtypes = [ctypes.c_char_p, ctypes.c_size_t,
                                           ctypes.c_size_t, ctypes.c_int,
                                           ctypes.c_int, ctypes.c_int]
        R.ref_store_create_gpu.restype = ctypes.c_void_p
        R.ref_store_destroy.argtypes = [ctypes.c_void_p]
        R.ref_store_clear.argtypes = [ctypes.c_void_p]
        R.ref_store_put.argtypes = [ctypes.c_void_p, ctypes.c_char_p, _u8p,
                                    ctypes.c_size_t, ctypes.c_int]
        R.ref_store_put.restype = ctypes.c_int
        R.ref_store_get.argtypes = [ctypes.c_void_p, ctypes.c_char_p, _u8p,
                                    ctypes.POINTER(ctypes.c_size_t)]
        R.ref_store_get.restype = ctypes.c_int
        R.ref_store_contains.argtypes = [ctypes.c_void_p, ctypes.c_char_p]
        R.ref_store_contains.restype = ctypes.c_int
        R.ref_store_stats.argtypes = [ctypes.c_void_p,
                                      ctypes.POINTER(ctypes.c_uint64)]
        R.ref_cpu_put_path.argtypes = [ctypes.c_void_p,
                                       ctypes.POINTER(_u8p),
                                       ctypes.POINTER(ctypes.c_size_t),
                                       ctypes.c_size_t, ctypes.c_int]
        R.ref_cpu_put_path.restype = ctypes.c_size_t
        R.ref_max_threads.restype = ctypes.c_int
        _ref = R
    return _ref


# ---------------------------------------------------------------- helpers
def sha256(data: np.ndarray) -> bytes:
    data = np.ascontiguousarray(data, dtype=np.uint8)
    out = np.zeros(32, np.uint8)
    lib().oracle_sha256(_ptr(data), data.size, _ptr(out))
    return out.tobytes()


def block_id(data: np.ndarray) -> str:
    data = np.ascontiguousarray(data, dtype=np.uint8)
    buf = ctypes.create_string_buffer(33)
    lib().oracle_block_id(_ptr(data), data.size, buf)
    return buf.value.decode()


def kv_compress(data: np.ndarray) -> np.ndarray:
    """8-byte header (scale, zp, 3 zero bytes) + size//2 int8 codes."""
    data = np.ascontiguousarray(data, dtype=np.uint8)
    out = np.empty(8 + data.size // 2, np.uint8)
    n = lib().oracle_kv_compress(_ptr(data), data.size, _ptr(out))
    assert n == out.size
    return out


def kv_decompress(comp: np.ndarray, orig_size: int) -> np.ndarray:
    comp = np.ascontiguousarray(comp, dtype=np.uint8)
    out = np.empty(orig_size, np.uint8)
    if orig_size % 2:
        out[-1] = 0
    ok = lib().oracle_kv_decompress(_ptr(comp), comp.size, _ptr(out),
                                    orig_size)
    if not ok:
        raise ValueError("compressed buffer too small")
    return out


def kv_params(mn: int, mx: int):
    s = ctypes.c_float()
    z = ctypes.c_int8()
    lib().oracle_kv_params(mn, mx, ctypes.byref(s), ctypes.byref(z))
    return s.value, z.value


# ------------------------------------------------------ reference helpers
def ref_block_id(data: np.ndarray) -> str:
    data = np.ascontiguousarray(data, dtype=np.uint8)
    buf = ctypes.create_string_buffer(33)
    ref().ref_compute_block_id(_ptr(data), data.size, buf)
    return buf.value.decode()


def ref_kv_compress(data: np.ndarray) -> np.ndarray:
    data = np.ascontiguousarray(data, dtype=np.uint8)
    out = np.empty(8 + data.size // 2, np.uint8)
    n = ref().ref_kv_compress(_ptr(data), data.size, _ptr(out), out.size)
    assert n == out.size
    out[5:8] = 0  # uninitialised padding in the reference's header
    return out


def ref_kv_decompress(comp: np.ndarray, orig_size: int) -> np.ndarray:
    comp = np.ascontiguousarray(comp, dtype=np.uint8)
    out = np.zeros(orig_size, np.uint8)
    ok = ref().ref_kv_decompress(_ptr(comp), comp.size, _ptr(out), orig_size)
    if not ok:
        raise ValueError("compressed buffer too small")
    return out


STAT_FIELDS = ("gpu_used", "shm_used", "gpu_hits", "shm_hits", "lustre_hits",
               "misses", "dedup_hits", "gpu_evictions", "shm_evictions",
               "promotions_to_gpu", "promotions_to_shm", "prefetch_completed",
               "compression_savings_bytes", "shm_puts", "lustre_puts")


class RefStore:
    """The reference CascadeStore: use_gpu=False (CPU tiers only) unless
    gpu_bytes is given, then with its GPU tier on device 0."""

    def __init__(self, shm_path: str, shm_bytes: int, kv_compression=False,
                 dedup_enabled=True, gpu_bytes=0, semantic_eviction=True):
        self._R = ref()
        if self._R is None:
            raise FileNotFoundError(f"{REF_SO} missing: run `make -C oracle ref`")
        if gpu_bytes:
            self._h = self._R.ref_store_create_gpu(
                shm_path.encode(), shm_bytes, gpu_bytes, int(kv_compression),
                int(dedup_enabled), int(semantic_eviction))
        else:
            self._h = self._R.ref_store_create(shm_path.encode(), shm_bytes,
                                               int(kv_compression),
                                               int(dedup_enabled))

    def put(self, block_id: str, data: np.ndarray, is_prefix=False) -> bool:
        data = np.ascontiguousarray(data, dtype=np.uint8)
        return bool(self._R.ref_store_put(self._h, block_id.encode(),
                                          _ptr(data), data.size,
                                          int(is_prefix)))

    def get(self, block_id: str, out: np.ndarray):
        sz = ctypes.c_size_t(0)
        ok = self._R.ref_store_get(self._h, block_id.encode(), _ptr(out),
                                   ctypes.byref(sz))
        return bool(ok), sz.value

    def contains(self, block_id: str) -> bool:
        return bool(self._R.ref_store_contains(self._h, block_id.encode()))

    def stats(self) -> dict:
        arr = (ctypes.c_uint64 * 15)()
        self._R.ref_store_stats(self._h, arr)
        return dict(zip(STAT_FIELDS, list(arr)))

    def clear(self):
        self._R.ref_store_clear(self._h)

    def put_path(self, blocks, nthreads: int) -> int:
        """compute_block_id + put_batch over `blocks` on `nthreads` threads."""
        n = len(blocks)
        ptrs = (_u8p * n)(*[_ptr(b) for b in blocks])
        sizes = (ctypes.c_size_t * n)(*[b.size for b in blocks])
        return self._R.ref_cpu_put_path(self._h, ptrs, sizes, n, nthreads)

    def close(self):
        if self._h:
            self._R.ref_store_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
