"""Device plumbing shared by the BOO and PBR front ends: staging host arrays,
raw pointers of torch tensors, the caller's CUDA stream."""

from __future__ import annotations

import threading

import numpy as np
import torch


def require_cuda(what: str) -> None:
    if not torch.cuda.is_available():
        raise RuntimeError(f'{what} runs on a CUDA device (sm_100a); no CUDA device is available. '
                           'spmm_b200 has no CPU implementation.')


def default_device() -> torch.device:
    return torch.device('cuda', torch.cuda.current_device())


STAGE_BYTES = 32 << 20      # one of the two pinned staging buffers per device
_STAGING = {}
_STAGING_LOCK = threading.Lock()


def _staging(device: torch.device):
    """(lock, [two pinned buffers], [their last copies' events]) of `device`,
    allocated on first use and kept for the process."""
    with _STAGING_LOCK:
        if device.index not in _STAGING:
            bufs = [torch.empty(STAGE_BYTES, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
            _STAGING[device.index] = (threading.Lock(), bufs, [None, None])
        return _STAGING[device.index]


def to_device(arr, device, dtype=None) -> torch.Tensor:
    """Host array -> device tensor through pinned memory (the reference stages
    the same way, boo.py:50-51).  Arrays larger than one staging buffer go
    through two reused pinned buffers in turn -- the host copy into one
    overlaps the DMA out of the other -- instead of a fresh pinned copy of
    the whole array (pinning hundreds of MB costs more than moving them).
    The copies are ordered on the device's current stream."""
    a = np.ascontiguousarray(arr, dtype=dtype)
    if not a.flags.writeable:
        a = a.copy()
    t = torch.from_numpy(a)
    if t.numel() == 0:
        return torch.empty(t.shape, dtype=t.dtype, device=device)
    nbytes = t.numel() * t.element_size()
    if nbytes <= STAGE_BYTES:
        return t.pin_memory().to(device, non_blocking=True)
    device = torch.device(device)
    out = torch.empty(t.shape, dtype=t.dtype, device=device)
    src = t.reshape(-1).view(torch.uint8)
    dst = out.reshape(-1).view(torch.uint8)
    lock, bufs, events = _staging(device)
    with lock, torch.cuda.device(device):
        stream = torch.cuda.current_stream(device)
        for i, off in enumerate(range(0, nbytes, STAGE_BYTES)):
            k = i % 2
            if events[k] is not None:
                events[k].synchronize()        # that buffer's previous DMA is done
            m = min(STAGE_BYTES, nbytes - off)
            bufs[k][:m].copy_(src[off:off + m])
            dst[off:off + m].copy_(bufs[k][:m], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(stream)
            events[k] = ev
    return out


def ptr(t: torch.Tensor | None) -> int | None:
    if t is None or t.numel() == 0:
        return None
    return t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


NP_TO_TORCH = {np.dtype(np.float32): torch.float32, np.dtype(np.float64): torch.float64,
               np.dtype(np.int32): torch.int32, np.dtype(np.int64): torch.int64}
