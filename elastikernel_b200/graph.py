"""CUDA-graph capture of a launch sequence on a partition stream.

The hot-path operators issue their launches from Python through the C ABI;
for small problems (a decode step of the MoE layer, a small GEMM) the host
work between launches — planning, tensor-map encoding, allocation, the
ctypes calls — is as long as the kernels. Capturing the sequence once and
replaying it leaves only the kernels. Nothing in the fused operators reads
device data back on the host, so a whole layer captures as one graph.
"""
from __future__ import annotations

import torch


class Captured:
    """`fn()` captured into a CUDA graph on `stream` (default: the current
    stream, e.g. a green-context partition's) after one eager warm-up call
    (kernel attributes, per-stream scratch, tensor maps). `__call__` replays
    it on the same stream and returns what `fn` returned at capture: tensors
    allocated inside `fn` live in the graph's memory pool and are rewritten
    by every replay. Refill the inputs in place between replays."""

    def __init__(self, fn, stream=None, device=None):
        self.stream = stream or torch.cuda.current_stream(device)
        # capture needs a non-default stream: a partition stream is captured
        # on directly, the device's default stream through a side stream
        default = torch.cuda.default_stream(self.stream.device)
        cap = torch.cuda.Stream(self.stream.device) if self.stream == default else self.stream
        cap.wait_stream(self.stream)
        with torch.cuda.stream(cap):
            fn()
        cap.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=cap):
            self.out = fn()

    def __call__(self):
        with torch.cuda.stream(self.stream):
            self.graph.replay()
        return self.out
