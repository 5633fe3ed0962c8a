"""Device plumbing shared by the BOO and PBR front ends: staging host arrays,
raw pointers of torch tensors, the caller's CUDA stream."""

from __future__ import annotations

import numpy as np
import torch


def require_cuda(what: str) -> None:
    if not torch.cuda.is_available():
        raise RuntimeError(f'{what} runs on a CUDA device (sm_100a); no CUDA device is available. '
                           'spmm_b200 has no CPU implementation.')


def default_device() -> torch.device:
    return torch.device('cuda', torch.cuda.current_device())


def to_device(arr, device, dtype=None) -> torch.Tensor:
    """Host array -> device tensor through pinned memory (the reference stages
    the same way, boo.py:50-51)."""
    a = np.ascontiguousarray(arr, dtype=dtype)
    if not a.flags.writeable:
        a = a.copy()
    t = torch.from_numpy(a)
    if t.numel() == 0:
        return torch.empty(t.shape, dtype=t.dtype, device=device)
    return t.pin_memory().to(device, non_blocking=True)


def ptr(t: torch.Tensor | None) -> int | None:
    if t is None or t.numel() == 0:
        return None
    return t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


NP_TO_TORCH = {np.dtype(np.float32): torch.float32, np.dtype(np.float64): torch.float64,
               np.dtype(np.int32): torch.int32, np.dtype(np.int64): torch.int64}
