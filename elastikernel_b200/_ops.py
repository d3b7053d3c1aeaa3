"""Torch-tensor front end of the C-ABI: argument checks, scratch management and
stream plumbing. Every launch goes to the *current* torch stream, which is
how a green-context partition stream reaches the kernels (the reference
relies on the same mechanism, sm_aware_matmul.py:270).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib, _workspace
from ._lib import check, lib

_DTYPES = {torch.bfloat16: _lib.EK_DTYPE_BF16, torch.float16: _lib.EK_DTYPE_FP16}
_FP8 = getattr(torch, "float8_e4m3fn", None)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _require_cuda(*ts: torch.Tensor) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("elastikernel_b200 operators take CUDA tensors only (no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} vs {t.device}")
    return dev


def _contig(name: str, t: torch.Tensor) -> None:
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def plan(M: int, N: int, K: int, num_sms: int, dtype=torch.bfloat16, b_layout: str = "kn", force_bn: int = 0,
         force_split: int = 0) -> dict:
    """Tile schedule the kernel would use for this shape on `num_sms` SMs (CPU-only call)."""
    p = _lib.GemmPlan()
    dt = _lib.EK_DTYPE_E4M3 if (_FP8 is not None and dtype == _FP8) else _DTYPES[dtype]
    bl = _lib.EK_B_KN if b_layout == "kn" else _lib.EK_B_NK
    check(lib().ek_gemm_plan_make(int(M), int(N), int(K), int(num_sms), dt, bl, int(force_bn), int(force_split),
                                  ctypes.byref(p)), "ek_gemm_plan_make")
    return p.as_dict()


def current_stream_handle(device: torch.device) -> int:
    return _lib.stream_ptr(torch.cuda.current_stream(device))


def gemm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, num_sms: int | None = None,
         b_layout: str = "kn", force_bn: int = 0, force_split: int = 0) -> torch.Tensor:
    """C = A @ B on the tcgen05 kernel.

    a: [M, K]; b: [K, N] (b_layout="kn", the reference's layout) or [N, K]
    (b_layout="nk"); bf16 or fp16; result in the input dtype.
    num_sms=None plans for the partition the current stream belongs to.
    """
    dev = _require_cuda(a, b, out)
    if a.dtype not in _DTYPES or b.dtype != a.dtype:
        raise RuntimeError(f"gemm takes bf16/fp16 operands of one dtype, got {a.dtype}, {b.dtype}")
    if a.dim() != 2 or b.dim() != 2:
        raise RuntimeError("gemm takes 2-D operands")
    _contig("a", a)
    _contig("b", b)
    M, K = a.shape
    if b_layout == "kn":
        K2, N = b.shape
        bl = _lib.EK_B_KN
    elif b_layout == "nk":
        N, K2 = b.shape
        bl = _lib.EK_B_NK
    else:
        raise ValueError(f"b_layout must be 'kn' or 'nk', got {b_layout!r}")
    if K2 != K:
        raise RuntimeError(f"inner dimensions differ: {K} vs {K2}")
    if out is None:
        out = torch.empty((M, N), device=dev, dtype=a.dtype)
    elif out.shape != (M, N) or out.dtype != a.dtype or not out.is_contiguous():
        raise RuntimeError("out must be a contiguous [M, N] tensor of the input dtype")
    if M == 0 or N == 0:
        return out
    if K == 0:
        return out.zero_()
    stream = current_stream_handle(dev)
    ns = int(num_sms) if num_sms else 0
    sms = ns if ns > 0 else _stream_sms(dev, stream)
    p = plan(M, N, K, sms, a.dtype, b_layout, force_bn, force_split)
    ws = _workspace.get(dev, stream, p["workspace_bytes"])
    with torch.cuda.device(dev):
        check(lib().ek_gemm(a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, _DTYPES[a.dtype], bl, sms,
                            int(force_bn), int(force_split), _ptr(ws), 0 if ws is None else ws.numel(), stream),
              "ek_gemm")
    return out


def gemm_fp8(a_q: torch.Tensor, w_q: torch.Tensor, a_scale: torch.Tensor, w_scale: torch.Tensor,
             out: torch.Tensor | None = None, num_sms: int | None = None, force_bn: int = 0,
             force_split: int = 0) -> torch.Tensor:
    """bf16 C[M,N] = (a_q * a_scale[:,None]) @ (w_q * w_scale[:,None])^T with e4m3 a_q [M,K], w_q [N,K]."""
    dev = _require_cuda(a_q, w_q, a_scale, w_scale, out)
    if _FP8 is None or a_q.dtype != _FP8 or w_q.dtype != _FP8:
        raise RuntimeError("gemm_fp8 takes float8_e4m3fn operands")
    for n, t in (("a_q", a_q), ("w_q", w_q), ("a_scale", a_scale), ("w_scale", w_scale)):
        _contig(n, t)
    if a_scale.dtype != torch.float32 or w_scale.dtype != torch.float32:
        raise RuntimeError("scales must be float32")
    M, K = a_q.shape
    N, K2 = w_q.shape
    if K2 != K or a_scale.numel() != M or w_scale.numel() != N:
        raise RuntimeError("shape mismatch in gemm_fp8")
    if out is None:
        out = torch.empty((M, N), device=dev, dtype=torch.bfloat16)
    stream = current_stream_handle(dev)
    ns = int(num_sms) if num_sms else 0
    sms = ns if ns > 0 else _stream_sms(dev, stream)
    p = plan(M, N, K, sms, _FP8, "nk", force_bn, force_split)
    ws = _workspace.get(dev, stream, p["workspace_bytes"])
    with torch.cuda.device(dev):
        check(lib().ek_gemm_fp8(a_q.data_ptr(), w_q.data_ptr(), a_scale.data_ptr(), w_scale.data_ptr(),
                                out.data_ptr(), M, N, K, sms, int(force_bn), int(force_split), _ptr(ws),
                                0 if ws is None else ws.numel(), stream), "ek_gemm_fp8")
    return out


def _stream_sms(dev: torch.device, stream: int) -> int:
    """SM count of the partition `stream` belongs to (registry), else the device's."""
    v = ctypes.c_int(0)
    check(lib().ek_gctx_stream_sm_count(ctypes.c_void_p(stream), ctypes.byref(v)), "ek_gctx_stream_sm_count")
    if v.value > 0:
        return v.value
    return torch.cuda.get_device_properties(dev).multi_processor_count
