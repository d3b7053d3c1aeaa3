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

