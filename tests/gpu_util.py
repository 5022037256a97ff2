"""Helpers of the GPU parity tests: numpy <-> device tensors and the stream."""
from __future__ import annotations

import numpy as np
import torch


def dev(a: np.ndarray, offset_bytes: int = 0) -> torch.Tensor:
    """Copy a numpy array to the GPU.  offset_bytes > 0 places it at an
    unaligned address inside a larger buffer (for the unaligned paths)."""
    a = np.ascontiguousarray(a)
    raw = torch.empty(a.nbytes + offset_bytes + 16, dtype=torch.uint8, device="cuda")
    view = raw[offset_bytes:offset_bytes + a.nbytes]
    if a.nbytes:
        view.copy_(torch.from_numpy(a.view(np.uint8).reshape(-1)))
    view._keep = raw  # keep the buffer alive
    return view


def empty(nbytes: int, offset_bytes: int = 0) -> torch.Tensor:
    raw = torch.zeros(nbytes + offset_bytes + 16, dtype=torch.uint8, device="cuda")
    view = raw[offset_bytes:offset_bytes + nbytes]
    view._keep = raw
    return view


def host(t: torch.Tensor, dtype, shape=None) -> np.ndarray:
    torch.cuda.synchronize()
    a = t.cpu().numpy().view(dtype)
    return a.reshape(shape) if shape is not None else a


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def ptr(t: torch.Tensor) -> int:
    return t.data_ptr()
