"""cascade_b200 — B200-native block-ingest path of CASCADE.

SHA-256 content addressing, the FP16->INT8 KVCompressor and the HBM block
pool run as hand-written sm_100a CUDA behind the C ABI of
include/cascade_b200.h (libcascade_b200.so).  ``cascade_b200.cascade_cpp``
mirrors the reference's pybind11 module ``cascade_cpp``.
"""
__version__ = "0.1.0"
