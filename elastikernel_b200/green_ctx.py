"""Green-context SM partitions (drop-in for elastikernel/green_ctx.py).

Same public functions, arguments, rounding and errors as the reference
(green_ctx.py:46-235); the driver work happens in the C++ shim behind
``ek_gctx_create`` (csrc/ek_green_ctx.cpp). Returned streams are
``torch.cuda.ExternalStream`` objects around the partition's CUstream; run
work in a partition with ``with torch.cuda.stream(stream):``.

Differences from the reference, by design:
* the SM count returned is the split result's real ``smCount``;
* green contexts are owned by the library and destroyed by
  :func:`destroy_all_partitions` (the reference never destroys them);
* the stream -> SM-count registry lets the kernels size their grid from the
  current stream (``num_sms=None``).
"""
from __future__ import annotations

import ctypes
from typing import List, Tuple

import torch

from . import _lib
from ._lib import check, lib


def _dev_index(dev) -> int:
    dev = torch.device(dev)
    if dev.type != "cuda":
        raise ValueError(f"green contexts need a CUDA device, got {dev}")
    return dev.index if dev.index is not None else torch.cuda.current_device()


def _sm_info(dev) -> tuple[int, int, int, int, int]:
    vals = [ctypes.c_int(0) for _ in range(5)]
    check(lib().ek_device_sm_info(_dev_index(dev), *[ctypes.byref(v) for v in vals]), "ek_device_sm_info")
    return tuple(v.value for v in vals)


def get_sm_alignment(dev: torch.device) -> Tuple[int, int]:
    """(min_sm_count, sm_alignment) by compute capability (green_ctx.py:46-62):
    CC 7.x (2, 2); CC 8.x (4, 2); CC >= 9 (8, 8)."""
    total, mn, al, major, minor = _sm_info(dev)
    return mn, al


def get_total_sm_count(dev: torch.device) -> int:
    """Total SM count of the device (green_ctx.py:65-67)."""
    return _sm_info(dev)[0]


def _round_up(x: int, alignment: int) -> int:
    return ((x + alignment - 1) // alignment) * alignment


def _create(dev, counts: List[int], disjoint: bool, remainder: bool = False) -> List[Tuple[torch.cuda.Stream, int]]:
    n = len(counts)
    m = n + (1 if remainder else 0)
    arr = (ctypes.c_int * n)(*counts)
    streams = (ctypes.c_void_p * m)()
    actual = (ctypes.c_int * m)()
    idx = _dev_index(dev)
    if remainder:
        check(lib().ek_gctx_create_remainder(idx, arr, n, streams, actual), "ek_gctx_create_remainder")
    else:
        check(lib().ek_gctx_create(idx, arr, n, 1 if disjoint else 0, streams, actual), "ek_gctx_create")
    device = torch.device("cuda", idx)
    return [(torch.cuda.ExternalStream(int(streams[i]), device=device), int(actual[i])) for i in range(m)]


def create_sm_partition(dev: torch.device, sm_count: int) -> Tuple[torch.cuda.Stream, int]:
    """One partition split from the FULL device (green_ctx.py:139-166).

    Repeated calls may return overlapping SM sets; use
    :func:`create_disjoint_partitions` for non-overlapping ones. The request is
    rounded up to the alignment; ValueError if that exceeds the device.
    Returns (stream, actual_sm_count).
    """
    min_sm, alignment = get_sm_alignment(dev)
    rounded = _round_up(max(sm_count, min_sm), alignment)
    total = get_total_sm_count(dev)
    if rounded > total:
        raise ValueError(f"Requested {sm_count} SMs (rounded to {rounded}) exceeds device total of {total} SMs")
    return _create(dev, [rounded], disjoint=False)[0]


def create_disjoint_partitions(dev: torch.device, sm_counts: List[int],
                               with_remainder: bool = False) -> List[Tuple[torch.cuda.Stream, int]]:
    """Partitions with guaranteed disjoint SM sets, chain-split from the
    remainder of each previous split (green_ctx.py:169-235). Each count is
    rounded up to the alignment; ValueError if the rounded total exceeds the
    device.

    with_remainder=True appends one more partition holding every SM the
    requests left over (the remainder the reference splits further but never
    returns, green_ctx.py:110-132): [32] on a 148-SM B200 gives a 32-SM and a
    116-SM partition, where a [32, 116] request fails (116 rounds up to 120)."""
    if not sm_counts:
        return []
    min_sm, alignment = get_sm_alignment(dev)
    total = get_total_sm_count(dev)
    rounded = [_round_up(max(sc, min_sm), alignment) for sc in sm_counts]
    if sum(rounded) > total or (with_remainder and sum(rounded) >= total):
        raise ValueError(
            f"Total requested SMs {sum(rounded)} (after rounding {list(sm_counts)} -> {rounded}) "
            f"exceeds device total of {total} SMs" + (" with SMs left for the remainder" if with_remainder else ""))
    return _create(dev, rounded, disjoint=True, remainder=with_remainder)


def full_device_partition(dev: torch.device) -> Tuple[torch.cuda.Stream, int]:
    """The whole device as a "partition": the current stream and the total SM
    count. A green context cannot hold all SMs when the total is not a
    multiple of the alignment (148 on B200), so the 148-SM level runs here."""
    return torch.cuda.current_stream(torch.device(dev)), get_total_sm_count(dev)


def stream_sm_count(stream) -> int:
    """SM count the registry holds for `stream` (0 if it is not a partition)."""
    v = ctypes.c_int(0)
    check(lib().ek_gctx_stream_sm_count(ctypes.c_void_p(_lib.stream_ptr(stream)), ctypes.byref(v)),
          "ek_gctx_stream_sm_count")
    return v.value


def destroy_all_partitions() -> None:
    """Destroy every partition stream and green context created so far.
    Synchronise the device first; streams must not be used afterwards."""
    check(lib().ek_gctx_destroy_all(), "ek_gctx_destroy_all")
