"""Helpers for the GPU tests: device buffers and descriptor arrays that stay
alive until the work on them has finished."""
import numpy as np
import torch

DEV = torch.device("cuda:0")


def stream():
    return torch.cuda.current_stream(DEV).cuda_stream


def to_dev(a: np.ndarray, pad_front: int = 0) -> torch.Tensor:
    """Upload bytes, optionally starting pad_front bytes into a fresh
    allocation (to place a block at a chosen misalignment)."""
    t = torch.zeros(a.size + pad_front + 16, dtype=torch.uint8, device=DEV)
    if a.size:
        t[pad_front:pad_front + a.size] = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
    return t[pad_front:pad_front + a.size] if a.size else t[pad_front:pad_front]


def addr_table(tensors):
    """int64 device array of data pointers (the caller keeps it alive)."""
    return torch.tensor([t.data_ptr() for t in tensors], dtype=torch.int64,
                        device=DEV)


def size_table(sizes):
    return torch.tensor(list(sizes), dtype=torch.int64, device=DEV)
