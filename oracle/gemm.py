"""GEMM oracles (CPU, numpy fp32 accumulate).

* gemm_ref      C = A @ B        (sm_aware_matmul.py:148-216 kernel math;
                                  sm_aware_agent/definition.py:63-65 operator)
* segment_gemm_ref               (sm_aware_benchmark.py:228-290 kernel math)
* gemm_fp8_ref  scaled e4m3 GEMM (no reference code; BASELINE FP8 config)
"""
from __future__ import annotations

import numpy as np
import torch


def to_f32(t) -> np.ndarray:
    """Exact fp32 copy of a torch tensor of any float dtype (bf16/fp16/e4m3)."""
    if isinstance(t, np.ndarray):
        return t.astype(np.float32)
    return t.detach().to("cpu").to(torch.float32).numpy()


def gemm_ref(a, b, b_layout: str = "kn") -> np.ndarray:
    """fp32 C = A @ B. a [M,K]; b [K,N] ("kn") or [N,K] ("nk").

    The reference kernels accumulate in fp32 and round once to the output
    dtype (sm_aware_matmul.py:169-176); this returns the unrounded fp32 value.
    """
    A = to_f32(a)
    B = to_f32(b)
    if b_layout == "nk":
        B = B.T
    return A @ B


def segment_gemm_ref(hs, weights, offsets, N: int, K: int) -> np.ndarray:
    """Reference segment GEMM (sm_aware_benchmark.py:242-290).

    For expert e, rows [offsets[e], offsets[e+1]) of hs [M,K] are multiplied by
    the expert's weight block addressed as weights_flat[e*N*K + k*K + n]
    (sm_aware_benchmark.py:273 with stride_bk = K, stride_bn = 1), i.e. rows
    e*N .. e*N+K-1, columns 0..N-1 of the [E*N, K] weight matrix. Rows not
    covered by any segment are returned as NaN (the reference leaves them
    uninitialised).
    """
    H = to_f32(hs)
    W = to_f32(weights)
    off = np.asarray(offsets.cpu() if hasattr(offsets, "cpu") else offsets).astype(np.int64)
    M = H.shape[0]
    out = np.full((M, N), np.nan, dtype=np.float32)
    Wflat = W.reshape(-1)
    for e in range(len(off) - 1):
        s0, s1 = int(off[e]), int(off[e + 1])
        if s1 <= s0:
            continue
        base = e * N * K
        idx = base + np.arange(K)[:, None] * K + np.arange(N)[None, :]
        blk = Wflat[np.clip(idx, 0, Wflat.size - 1)]
        out[s0:s1] = H[s0:s1] @ blk
    return out


def gemm_fp8_ref(a_q, w_q, a_scale, w_scale) -> np.ndarray:
    """fp32 (a_q * a_scale[:,None]) @ (w_q * w_scale[:,None])^T from e4m3 codes."""
    A = to_f32(a_q) * to_f32(a_scale)[:, None]
    W = to_f32(w_q) * to_f32(w_scale)[:, None]
    return A @ W.T


def max_rel_err(out, ref) -> float:
    """max |out - ref| / max |ref| (the tolerance measure used by the tests)."""
    o = to_f32(out)
    r = np.asarray(ref, dtype=np.float32)
    mask = np.isfinite(r)
    denom = float(np.max(np.abs(r[mask]))) if mask.any() else 1.0
    return float(np.max(np.abs(o[mask] - r[mask]))) / max(denom, 1e-30)
