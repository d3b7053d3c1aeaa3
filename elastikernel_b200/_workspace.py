"""Scratch buffers for the kernels that need them (split-K partials and
tickets, padded copies of ragged GEMM operands).

The C-ABI never allocates; callers pass scratch in. This module keeps one
zero-initialised buffer per (device, stream, kind) and grows it on demand.
The GEMM kernel returns its ticket counters to zero, so a buffer stays valid
across calls on the same stream; distinct streams get distinct buffers so
that concurrent partitions never share scratch.

A buffer is never freed once handed out. A CUDA graph captured around a
GEMM (graph.Captured, sm_aware_matmul.GraphMatmul) holds the buffer's raw
address; if a later, larger call on the same stream replaced the buffer and
returned the old one to torch's allocator, replaying that graph would write
partials and tickets into memory that belongs to other tensors. Replaced
buffers therefore stay alive in a retired list (growth doubles, so the
retired ones add at most the size of the live one), and reset() zero-fills
buffers in place instead of dropping them.
"""
from __future__ import annotations

import threading

import torch

_BUFS: dict[tuple[int, int, str], torch.Tensor] = {}
_RETIRED: list[torch.Tensor] = []
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
            if buf is not None:
                _RETIRED.append(buf)  # a captured graph may still hold its address
            buf = torch.zeros(size, dtype=torch.uint8, device=torch.device("cuda", dev))
            _BUFS[key] = buf
        return buf


def reset(device: torch.device | None = None) -> None:
    """Zero-fill the cached buffers in place (ticket counters included), e.g.
    after a kernel reported a bounded-wait timeout in the middle of a split
    reduction and may have left a ticket or a flag set. The buffers keep their
    addresses, so graphs captured over them stay valid."""
    with _LOCK:
        bufs = list(_BUFS.items())
        retired = list(_RETIRED)
    for (dev, _, _), buf in bufs:
        if device is None or dev == (device.index if device.index is not None else torch.cuda.current_device()):
            with torch.cuda.device(dev):
                buf.zero_()
    for buf in retired:
        if device is None or buf.device == device:
            with torch.cuda.device(buf.device):
                buf.zero_()
    for dev in {d for (d, _, _), _ in bufs}:
        torch.cuda.synchronize(dev)


def live_bytes() -> int:
    """Bytes held by current and retired buffers (for tests)."""
    with _LOCK:
        return sum(b.numel() for b in _BUFS.values()) + sum(b.numel() for b in _RETIRED)
