"""ctypes binding of libcascade_b200.so (the C ABI of include/cascade_b200.h).

The library is the only compute path: there is no CPU fallback.  Importing
this module never needs a GPU; calling a compute entry point without one
fails with CascadeError.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcascade_b200.so")
HEADER_PATH = os.path.join(os.path.dirname(HERE), "include", "cascade_b200.h")

CASCADE_OK = 0
CASCADE_ERR_UNSUPPORTED = 6
PUT_STORED, PUT_DUP_KNOWN, PUT_DUP_BATCH, PUT_FAILED = 0, 1, 2, 3

_u8p = ctypes.POINTER(ctypes.c_uint8)
_u64p = ctypes.POINTER(ctypes.c_uint64)
_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_u64 = ctypes.c_uint64
_int = ctypes.c_int


class CascadeError(RuntimeError):
    """A non-zero status from the C ABI, with cascade_last_error()'s text."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[cascade status {code}] {msg}")
        self.code = code


# name -> (restype, argtypes) for every entry point the header declares.
_SIGS = {
    "cascade_last_error": (ctypes.c_char_p, []),
    "cascade_abi_version": (_int, []),
    "cascade_sha256_batch": (_int, [_vp, _vp, _sz, _vp, _vp]),
    "cascade_kv_compress_batch": (_int, [_vp, _vp, _vp, _sz, _u64, _vp]),
    "cascade_kv_compress_batch_noalloc": (_int, [_vp, _vp, _vp, _sz, _u64,
                                                 _vp]),
    "cascade_kv_decompress_batch": (_int, [_vp, _vp, _vp, _sz, _u64, _vp]),
    "cascade_copy_batch": (_int, [_vp, _vp, _vp, _sz, _u64, _vp]),
    "cascade_compute_block_id": (_int, [_vp, _u64, ctypes.c_char_p]),
    "cascade_diag_launch_count": (ctypes.c_uint64, []),
    "cascade_diag_sha_peak": (_int, [_int, ctypes.c_uint32,
                                     ctypes.POINTER(ctypes.c_double),
                                     ctypes.POINTER(ctypes.c_double)]),
}

_lib = None


def declared_functions(header: str = HEADER_PATH) -> list[str]:
    """Names of the functions include/cascade_b200.h declares."""
    text = open(header).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cascade_\w+)\s*\(", text)))


def load() -> ctypes.CDLL:
    """Loads the in-tree library (built by __graft_entry__.build())."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing; build it with "
                "`python -c 'import __graft_entry__ as g; g.build()'`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def register(name: str, restype, argtypes) -> None:
    """Adds a signature (used by modules that bind further entry points)."""
    _SIGS[name] = (restype, argtypes)
    if _lib is not None:
        fn = getattr(_lib, name)
        fn.restype = restype
        fn.argtypes = argtypes


def check(rc: int) -> None:
    if rc != CASCADE_OK:
        msg = load().cascade_last_error()
        raise CascadeError(rc, msg.decode() if msg else "")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))
