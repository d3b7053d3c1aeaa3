"""Fused-MoE oracle (CPU, numpy; torch only for dtype conversion).

* route_ref      softmax -> top-k -> renormalise      sm_aware_agent/definition.py:152-153
* permute_ref    moe_align_block_size-style layout    (no reference code: defined here)
* moe_ref        SwiGLU experts + weighted combine    sm_aware_agent/definition.py:155-170
* moe_ref_by_expert  the same, one expert's weights fetched at a time (large layers)
* combine_ref    top-k sum of weighted expert rows     sm_aware_agent/definition.py:168 (sum over choices)
* moe_loop_ref   the definition's literal per-token loop in torch (CPU baseline)
* moe_vec_ref    vectorised per-expert torch restatement (CPU baseline at all T)

Top-k selection: the softmax is monotone, so experts are selected on the
logits themselves (exact inputs, no rounding in the comparison), largest
first, ties broken towards the lower expert id. Weights are the fp32 softmax
probabilities of the selected experts divided by their fp32 sum.
"""
from __future__ import annotations

import numpy as np
import torch

from .gemm import to_f32


def softmax_f32(logits: np.ndarray) -> np.ndarray:
    x = np.asarray(logits, dtype=np.float32)
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m, dtype=np.float32)
    return (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)


def route_ref(logits, topk: int) -> tuple[np.ndarray, np.ndarray]:
    """(topk_ids int32 [T,k], topk_weights fp32 [T,k]) as definition.py:152-153."""
    x = to_f32(logits) if not isinstance(logits, np.ndarray) else logits.astype(np.float32)
    T, E = x.shape
    # stable sort of -logit keeps lower ids first among equal logits
    order = np.argsort(-x, axis=-1, kind="stable")[:, :topk].astype(np.int32)
    p = softmax_f32(x)
    w = np.take_along_axis(p, order, axis=-1)
    w = (w / w.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    return order, w


def max_padded_rows(T: int, topk: int, E: int, block_m: int) -> int:
    n = T * topk + E * (block_m - 1)
    return -(-n // block_m) * block_m


def permute_ref(topk_ids, E: int, block_m: int) -> dict:
    """Expert-sorted, block-padded layout of the flattened (token, choice) slots.

    Slot s = t*k + j. Slots are stably sorted by expert id; each expert's run
    is padded to a multiple of block_m with the sentinel T*k. Returns
    sorted_slots [max_rows], block_expert [max_rows/block_m] (-1 past the
    used rows), num_rows_padded and expert_counts [E].
    """
    ids = np.asarray(topk_ids, dtype=np.int64)
    T, k = ids.shape
    flat = ids.reshape(-1)
    sentinel = T * k
    max_rows = max_padded_rows(T, k, E, block_m)
    counts = np.bincount(flat, minlength=E)[:E].astype(np.int64)
    padded = (counts + block_m - 1) // block_m * block_m
    starts = np.concatenate([[0], np.cumsum(padded)[:-1]])
    total = int(padded.sum())
    sorted_slots = np.full(max_rows, sentinel, dtype=np.int32)
    block_expert = np.full(max_rows // block_m, -1, dtype=np.int32)
    order = np.argsort(flat, kind="stable")
    pos = 0
    for e in range(E):
        c = int(counts[e])
        sorted_slots[starts[e]:starts[e] + c] = order[pos:pos + c]
        block_expert[starts[e] // block_m:(starts[e] + padded[e]) // block_m] = e
        pos += c
    return {
        "sorted_slots": sorted_slots,
        "block_expert": block_expert,
        "num_rows_padded": total,
        "expert_counts": counts.astype(np.int32),
    }


def _silu(x: np.ndarray) -> np.ndarray:
    return x / (1.0 + np.exp(-x))


def moe_ref(x, logits, w1, w2, w3, topk: int, ids=None, weights=None) -> np.ndarray:
    """fp32 MoE output [T, H] (definition.py:155-170 math, vectorised by expert).

    x [T,H]; logits [T,E]; w1, w3 [E,I,H]; w2 [E,H,I]. Routing from route_ref
    unless (ids, weights) are given.
    """
    X = to_f32(x)
    if ids is None:
        ids, weights = route_ref(logits, topk)
    W1, W2, W3 = to_f32(w1), to_f32(w2), to_f32(w3)
    T, H = X.shape
    out = np.zeros((T, H), dtype=np.float32)
    for e in range(W1.shape[0]):
        t_idx, j_idx = np.nonzero(ids == e)
        if t_idx.size == 0:
            continue
        h = X[t_idx]
        act = _silu(h @ W1[e].T) * (h @ W3[e].T)
        y = act @ W2[e].T
        wt = weights[t_idx, j_idx][:, None]
        np.add.at(out, t_idx, wt * y)
    return out


def moe_ref_by_expert(x, ids, weights, num_experts: int, expert_weights, act_quant=None):
    """fp32 MoE output [T, H] for tokens x [T, H] with their routing (ids,
    weights [T, k]), the definition.py:155-170 math, fetching one expert's
    weights at a time: expert_weights(e) -> (w1_e [I, H], w2_e [H, I],
    w3_e [I, H]) as fp32 arrays. Used on sampled tokens of layers whose weights
    are too large to hold in fp32 all at once (Mixtral, 256-expert FP8 layers);
    experts no sampled token routes to are never fetched.

    With act_quant (a function of the fp32 SwiGLU activations [rows, I]) a
    second output is computed in the same pass from act_quant(act): the
    reference for a layer that rounds its activations (e.g. to e4m3) before
    the down projection. Returns (plain, quantised) then, else plain."""
    X = to_f32(x)
    ids = np.asarray(ids)
    weights = np.asarray(weights, dtype=np.float32)
    out = np.zeros(X.shape, dtype=np.float32)
    out_q = np.zeros(X.shape, dtype=np.float32) if act_quant is not None else None
    for e in range(num_experts):
        t_idx, j_idx = np.nonzero(ids == e)
        if t_idx.size == 0:
            continue
        w1e, w2e, w3e = expert_weights(e)
        h = X[t_idx]
        act = _silu(h @ w1e.T) * (h @ w3e.T)
        wt = weights[t_idx, j_idx][:, None]
        np.add.at(out, t_idx, wt * (act @ w2e.T))
        if out_q is not None:
            np.add.at(out_q, t_idx, wt * (np.asarray(act_quant(act), dtype=np.float32) @ w2e.T))
    return out if out_q is None else (out, out_q)


def combine_ref(y, T: int, topk: int) -> torch.Tensor:
    """bf16 [T, H]: out[t] = sum_j y[t*k + j], accumulated in fp32 in j order
    (the per-choice sum of definition.py:168 over rows that already carry
    their routing weight), rounded once to bf16."""
    Y = to_f32(y).reshape(T, topk, -1)
    acc = np.zeros((T, Y.shape[2]), dtype=np.float32)
    for j in range(topk):
        acc = acc + Y[:, j]
    return torch.from_numpy(acc).to(torch.bfloat16)


def moe_loop_ref(hidden_states: torch.Tensor, gate_logits: torch.Tensor, w1, w2, w3, topk: int) -> torch.Tensor:
    """The definition's operator body, a per-(token, choice) loop on CPU torch
    (definition.py:152-168), in the inputs' dtype."""
    import torch.nn.functional as F

    topk_weights, topk_ids = torch.topk(gate_logits.softmax(dim=-1), topk, dim=-1)
    topk_weights = topk_weights / topk_weights.sum(dim=-1, keepdim=True)
    result = torch.zeros_like(hidden_states)
    for i in range(hidden_states.shape[0]):
        for j in range(topk):
            e = int(topk_ids[i, j])
            wt = float(topk_weights[i, j])
            h = hidden_states[i]
            hidden = F.silu(w1[e] @ h) * (w3[e] @ h)
            result[i] += wt * (w2[e] @ hidden)
    return result


def moe_vec_ref(hidden_states: torch.Tensor, gate_logits: torch.Tensor, w1, w2, w3, topk: int) -> torch.Tensor:
    """Vectorised per-expert CPU torch restatement of the same operator."""
    import torch.nn.functional as F

    topk_weights, topk_ids = torch.topk(gate_logits.softmax(dim=-1), topk, dim=-1)
    topk_weights = topk_weights / topk_weights.sum(dim=-1, keepdim=True)
    out = torch.zeros(hidden_states.shape, dtype=torch.float32)
    for e in range(w1.shape[0]):
        t_idx, j_idx = torch.nonzero(topk_ids == e, as_tuple=True)
        if t_idx.numel() == 0:
            continue
        h = hidden_states[t_idx]
        act = F.silu(h @ w1[e].T) * (h @ w3[e].T)
        y = (act @ w2[e].T).float() * topk_weights[t_idx, j_idx, None].float()
        out.index_add_(0, t_idx, y)
    return out.to(hidden_states.dtype)
