"""FP8 e4m3 quantisation oracle (no reference code: the reference has no FP8
path; this is the definition the GPU kernels are tested against).

scale = amax(block) / 448 in fp32 (1.0 for an all-zero block);
q = e4m3(x / scale) with IEEE fp32 division and round-to-nearest-even
(torch's float8_e4m3fn cast); |x / scale| <= 448 by construction.

pow2=True: the scale is rounded up to the next power of two (kept if it is
one), the UE8M0 form the block-scaled tensor-core MMA applies itself; the
division is then an exact rescaling.
"""
from __future__ import annotations

import numpy as np
import torch

E4M3_MAX = np.float32(448.0)


def _f32(x) -> np.ndarray:
    if isinstance(x, np.ndarray):
        return x.astype(np.float32)
    return x.detach().cpu().to(torch.float32).numpy()


def pow2_up(s) -> np.ndarray:
    """fp32 scales rounded up to the next power of two (unchanged if one): the
    biased exponent is incremented and the mantissa cleared, capped at 2^127."""
    b = np.ascontiguousarray(s, dtype=np.float32).view(np.uint32).copy()
    frac = (b & np.uint32(0x007FFFFF)) != 0
    b[frac] = (b[frac] & np.uint32(0x7F800000)) + np.uint32(0x00800000)
    b = np.minimum(b, np.uint32(0x7F000000))
    return b.view(np.float32)


def _cast(v: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32)).to(torch.float8_e4m3fn)


def quant_rows(x, pow2: bool = False) -> tuple[torch.Tensor, np.ndarray]:
    X = _f32(x)
    amax = np.abs(X).max(axis=1)
    s = np.where(amax > 0, amax / E4M3_MAX, np.float32(1.0)).astype(np.float32)
    if pow2:
        s = pow2_up(s)
    return _cast(X / s[:, None]), s


def quant_blocks(x, br: int, bc: int, pow2: bool = False) -> tuple[torch.Tensor, np.ndarray]:
    X = _f32(x)
    R, C = X.shape
    nbr, nbc = -(-R // br), -(-C // bc)
    s = np.ones((nbr, nbc), dtype=np.float32)
    Q = np.empty_like(X)
    for i in range(nbr):
        for j in range(nbc):
            blk = X[i * br:(i + 1) * br, j * bc:(j + 1) * bc]
            a = np.abs(blk).max()
            sc = np.float32(a / E4M3_MAX) if a > 0 else np.float32(1.0)
            if pow2:
                sc = pow2_up(np.array([sc], dtype=np.float32))[0]
            s[i, j] = sc
            Q[i * br:(i + 1) * br, j * bc:(j + 1) * bc] = blk / sc
    return _cast(Q), s


def dequant_blocks(q: torch.Tensor, s: np.ndarray, br: int, bc: int) -> np.ndarray:
    Q = q.to(torch.float32).numpy()
    S = np.repeat(np.repeat(s, br, axis=0), bc, axis=1)[:Q.shape[0], :Q.shape[1]]
    return Q * S


def dequant_block_rows(q: torch.Tensor, s: np.ndarray, block: int = 128) -> np.ndarray:
    """fp32 values of e4m3 codes q [R, C] with block x block scales s
    [R/block, C/block] (R and C multiples of block): the same values as
    dequant_blocks, by broadcasting instead of materialising the scale grid."""
    Q = q.to(torch.float32).numpy()
    R, C = Q.shape
    S = np.asarray(s, dtype=np.float32).reshape(R // block, 1, C // block, 1)
    return (Q.reshape(R // block, block, C // block, block) * S).reshape(R, C)
