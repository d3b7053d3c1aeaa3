"""The reference's own CPU implementations of the hot path, restated for timing.

* gemm_cpu: the GEMM operator body C = torch.matmul(A, B) on CPU tensors
  (sm_aware_agent/definition.py:63-65; the reference's verification op,
  sm_aware_matmul.py:265).
* fused_moe_cpu: the fused-MoE operator body on CPU (definition.py:149-170),
  vectorised per expert (oracle.moe.moe_vec_ref).

Used only by bench.py's cpu_baseline leg and its `--impl reference` arm.
"""
from __future__ import annotations

import os
import time

import torch

from .moe import moe_vec_ref


def set_threads() -> int:
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def gemm_cpu(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return torch.matmul(a, b)


def fused_moe_cpu(x, logits, w1, w2, w3, topk: int) -> torch.Tensor:
    return moe_vec_ref(x, logits, w1, w2, w3, topk)


def time_gemm(M: int, N: int, K: int, reps: int, budget_s: float = 20.0, seed: int = 0) -> dict:
    """Time `reps` bf16 CPU GEMMs of M x N x K (stopping early past budget_s)."""
    g = torch.Generator().manual_seed(seed)
    a = torch.randn((M, K), generator=g).to(torch.bfloat16)
    b = torch.randn((K, N), generator=g).to(torch.bfloat16)
    gemm_cpu(a, b)  # warm-up
    times = []
    t_start = time.perf_counter()
    for _ in range(reps):
        t0 = time.perf_counter()
        gemm_cpu(a, b)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    return {"seconds": times, "flop": 2.0 * M * N * K}


def time_moe(x, logits, w1, w2, w3, topk: int, loop: bool, reps: int = 2, budget_s: float = 10.0) -> dict:
    """Time the fused-MoE operator on CPU tensors: the definition's per-token
    loop (loop=True, definition.py:152-168) or the vectorised per-expert
    restatement (loop=False), `reps` times or until budget_s has passed."""
    from .moe import moe_loop_ref

    fn = moe_loop_ref if loop else fused_moe_cpu
    times = []
    t_start = time.perf_counter()
    for _ in range(reps):
        t0 = time.perf_counter()
        fn(x, logits, w1, w2, w3, topk)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    return {"seconds": times, "tokens": int(x.shape[0])}
