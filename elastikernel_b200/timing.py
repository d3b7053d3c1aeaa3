"""Device timing helpers: CUDA events on the launching stream, L2 flushed
before every timed repetition (a write larger than the 126 MB L2), as
triton.testing.do_bench does for the reference's benchmarks."""
from __future__ import annotations

import statistics

import torch

L2_FLUSH_BYTES = 256 * 1024 * 1024
_FLUSH: dict[int, torch.Tensor] = {}


def flush_l2(device: torch.device | None = None) -> None:
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    buf = _FLUSH.get(idx)
    if buf is None:
        buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=torch.device("cuda", idx))
        _FLUSH[idx] = buf
    buf.zero_()


def time_on_stream(fn, stream=None, reps: int | None = None, rep_ms: float = 50.0, flush: bool = True,
                   warmup: int = 0) -> dict:
    """Per-rep device time of fn() on `stream` (default: current stream).

    Each rep: flush L2 (untimed), record start, fn(), record end -- all on the
    same stream. `reps` defaults to as many as fit in about rep_ms. `warmup`
    untimed reps are queued right before the timed ones, with no host wait in
    between: a GPU that idled while the host prepared the run (a synchronise,
    a graph capture) brings its clock back up during them instead of during
    the first timed rep.
    """
    stream = stream or torch.cuda.current_stream()
    with torch.cuda.stream(stream):
        if reps is None:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            e.synchronize()
            one = max(s.elapsed_time(e), 1e-3)
            reps = int(max(5, min(200, rep_ms / one)))
        for _ in range(warmup):
            if flush:
                flush_l2()
            fn()
        pairs = []
        for _ in range(reps):
            if flush:
                flush_l2()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            pairs.append((s, e))
        stream.synchronize()
    ms = [s.elapsed_time(e) for s, e in pairs]
    return {"mean_ms": statistics.fmean(ms), "median_ms": statistics.median(ms), "min_ms": min(ms), "reps": reps,
            "all_ms": ms}
