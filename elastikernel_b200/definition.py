"""Operator API in destination-passing style, as the reference's kernel
definitions declare it (sm_aware_agent/definition.py):

* run_gemm(A, B, C, M, N, K, NUM_SMS)              -- definition.py:63-65
* run_fused_moe(hidden_states, gate_logits, w1, w2, w3, out,
                M, K, N, NUM_EXPERTS, TOP_K, NUM_SMS) -- definition.py:149-170

Outputs are written in place into C / out. Shapes follow the definitions:
A [M,K], B [K,N], C [M,N]; hidden_states [M,K], gate_logits [M,E] fp32,
w1, w3 [E,N,K], w2 [E,K,N], out [M,K] (here K is the model hidden size and N
the expert intermediate size).
"""
from __future__ import annotations

import torch

from . import _ops


def run_gemm(A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, M: int, N: int, K: int, NUM_SMS: int) -> None:
    """C = A @ B on a partition of NUM_SMS SMs (definition.py:63-65)."""
    if tuple(A.shape) != (M, K) or tuple(B.shape) != (K, N) or tuple(C.shape) != (M, N):
        raise RuntimeError("run_gemm: shapes do not match (M, N, K)")
    if C.is_contiguous() and C.dtype == A.dtype:
        _ops.gemm(A, B, out=C, num_sms=NUM_SMS)
    else:
        C.copy_(_ops.gemm(A, B, num_sms=NUM_SMS))


def run_fused_moe(hidden_states: torch.Tensor, gate_logits: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                  w3: torch.Tensor, out: torch.Tensor, M: int, K: int, N: int, NUM_EXPERTS: int, TOP_K: int,
                  NUM_SMS: int) -> None:
    """The fused-MoE forward pass (definition.py:149-170) into `out`."""
    if tuple(hidden_states.shape) != (M, K) or tuple(gate_logits.shape) != (M, NUM_EXPERTS):
        raise RuntimeError("run_fused_moe: hidden_states / gate_logits shapes do not match")
    if tuple(w1.shape) != (NUM_EXPERTS, N, K) or tuple(w3.shape) != (NUM_EXPERTS, N, K) or \
            tuple(w2.shape) != (NUM_EXPERTS, K, N):
        raise RuntimeError("run_fused_moe: expert weight shapes do not match")
    if out.is_contiguous() and out.dtype == torch.bfloat16:
        _ops.fused_moe(hidden_states, gate_logits, w1, w2, w3, TOP_K, out=out, num_sms=NUM_SMS)
    else:
        out.copy_(_ops.fused_moe(hidden_states, gate_logits, w1, w2, w3, TOP_K, num_sms=NUM_SMS))


def smoke_moe(dev: torch.device) -> None:
    """One small fused-MoE layer checked against the CPU oracle (used by the smoke entry point)."""
    from oracle.gemm import max_rel_err
    from oracle.moe import moe_ref, route_ref

    from . import _lib

    T, H, I, E, k = 64, 256, 512, 8, 2
    g = torch.Generator().manual_seed(42)
    x = torch.randn((T, H), generator=g).to(torch.bfloat16)
    logits = torch.randn((T, E), generator=g)
    w1 = (torch.randn((E, I, H), generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn((E, H, I), generator=g) * 0.02).to(torch.bfloat16)
    w3 = (torch.randn((E, I, H), generator=g) * 0.02).to(torch.bfloat16)
    out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    run_fused_moe(x.to(dev), logits.to(dev), w1.to(dev), w2.to(dev), w3.to(dev), out, T, H, I, E, k, 148)
    ids, _ = _ops.moe_route(logits.to(dev), k)
    torch.cuda.synchronize()
    err = max_rel_err(out, moe_ref(x, logits, w1, w2, w3, k))
    same_ids = bool((ids.cpu().numpy() == route_ref(logits.numpy(), k)[0]).all())
    status = _lib.device_status(dev.index or 0)
    print(f"smoke fused MoE T={T} H={H} I={I} E={E} k={k}: max rel err {err:.2e}, routing exact {same_ids}, "
          f"status {status}")
    assert status == 0 and err <= 1e-2 and same_ids, "MoE smoke check failed"
