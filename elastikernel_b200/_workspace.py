"""Scratch buffers for the kernels that need them (split-K partials and
tickets, permutation counters).

The C-ABI never allocates; callers pass scratch in. This module keeps one
zero-initialised buffer per (device, stream) and grows it on demand. The GEMM
kernel returns its ticket counters to zero, so a buffer stays valid across
calls on the same stream; distinct streams get distinct buffers so that
concurrent partitions never share scratch.
"""
from __future__ import annotations

import threading

import torch

_BUFS: dict[tuple[int, int, str], torch.Tensor] = {}
_LOCK = threading.Lock()


def get(device: torch.device, stream_handle: int, nbytes: int, kind: str = "gemm") -> torch.Tensor:
    """Zero-filled uint8 buffer of at least `nbytes` for (device, stream, kind)."""
    if nbytes <= 0:
        return None
    dev = device.index if device.index is not None else torch.cuda.current_device()
    key = (dev, stream_handle, kind)
    with _LOCK:
        buf = _BUFS.get(key)
        if buf is None or buf.numel() < nbytes:
            size = max(nbytes, 2 * buf.numel() if buf is not None else 0)
            size = (size + 4095) // 4096 * 4096
            buf = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", dev))
            _BUFS[key] = buf
        return buf


def reset(device: torch.device | None = None) -> None:
    """Drop cached buffers (e.g. after a kernel reported a fault mid-reduction)."""
    with _LOCK:
        if device is None:
            _BUFS.clear()
        else:
            dev = device.index if device.index is not None else torch.cuda.current_device()
            for k in [k for k in _BUFS if k[0] == dev]:
                del _BUFS[k]
