"""ctypes binding of the C-ABI library ``_ek.so`` (declared in include/elastikernel.h).

This is the only place Python touches native code. There is no CPU fallback:
if the library is missing, :func:`lib` raises, and every operator that needs
it fails loudly.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

EK_OK = 0
EK_ERR_INVALID = 1
EK_ERR_CUDA = 2
EK_ERR_OVERSUB = 3
EK_ERR_UNSUPPORTED = 4
EK_ERR_DEVICE = 5

EK_DTYPE_BF16 = 0
EK_DTYPE_FP16 = 1
EK_DTYPE_E4M3 = 2

EK_QUANT_POW2_SCALES = 1

EK_B_KN = 0
EK_B_NK = 1

EK_STATUS_WAIT_TIMEOUT = 1
EK_STATUS_BAD_EXPERT = 2
EK_STATUS_BAD_INDEX = 4
EK_STATUS_BAD_SCALE = 8
EK_STATUS_CAPACITY = 16

LIB_PATH = Path(__file__).with_name("_ek.so")

_c_int = ctypes.c_int
_c_vp = ctypes.c_void_p
_c_size = ctypes.c_size_t
_c_ip = ctypes.POINTER(ctypes.c_int)


class GemmPlan(ctypes.Structure):
    """Mirror of ``ek_gemm_plan``."""

    _fields_ = [
        ("bm", _c_int), ("bn", _c_int), ("bk", _c_int), ("cta_pair", _c_int),
        ("tiles_m", _c_int), ("tiles_n", _c_int), ("k_blocks", _c_int),
        ("num_tiles", _c_int), ("num_dp_tiles", _c_int), ("tail_split", _c_int),
        ("num_units", _c_int), ("grid", _c_int), ("num_sms", _c_int), ("waves", _c_int),
        ("wave_efficiency", ctypes.c_double), ("est_us", ctypes.c_double),
        ("workspace_bytes", _c_size), ("cluster_split", _c_int),
    ]

    def as_dict(self) -> dict:
        return {name: getattr(self, name) for name, _ in self._fields_}


# name -> (restype, argtypes)
_SIGNATURES = {
    "ek_abi_version": (_c_int, []),
    "ek_last_error": (ctypes.c_char_p, []),
    "ek_device_status": (_c_int, [_c_int, _c_int, _c_ip]),
    "ek_device_sm_info": (_c_int, [_c_int, _c_ip, _c_ip, _c_ip, _c_ip, _c_ip]),
    "ek_gctx_create": (_c_int, [_c_int, _c_ip, _c_int, _c_int, ctypes.POINTER(_c_vp), _c_ip]),
    "ek_gctx_create_remainder": (_c_int, [_c_int, _c_ip, _c_int, ctypes.POINTER(_c_vp), _c_ip]),
    "ek_gctx_stream_sm_count": (_c_int, [_c_vp, _c_ip]),
    "ek_gctx_destroy_all": (_c_int, []),
    "ek_gctx_fake_driver": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int]),
    "ek_gemm_plan_make": (_c_int, [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                   ctypes.POINTER(GemmPlan)]),
    "ek_gemm_workspace_bytes": (_c_size, [_c_int] * 8),
    "ek_gemm": (_c_int, [_c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                         _c_vp, _c_size, _c_vp]),
    "ek_gemm_fp8": (_c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                             _c_vp, _c_size, _c_vp]),
    "ek_quant_e4m3": (_c_int, [_c_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_vp, _c_vp, _c_vp]),
    "ek_quant_e4m3_kmajor": (_c_int, [_c_vp, _c_int, _c_int, _c_int, _c_vp, _c_vp, _c_vp]),
    "ek_quant_e4m3_ex": (_c_int, [_c_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_vp, _c_vp, _c_vp]),
    "ek_quant_e4m3_kmajor_ex": (_c_int, [_c_vp, _c_int, _c_int, _c_int, _c_int, _c_vp, _c_vp, _c_vp]),
    "ek_gemm_noalloc": (_c_int, [_c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                 _c_int, _c_vp]),
    "ek_gemm_noalloc_max_scratch_bytes": (_c_size, []),
    "ek_moe_route": (_c_int, [_c_vp, _c_int, _c_int, _c_int, _c_vp, _c_vp, _c_vp]),
    "ek_moe_max_padded_rows": (ctypes.c_int64, [_c_int, _c_int, _c_int, _c_int]),
    "ek_moe_permute_scratch_bytes": (_c_size, [_c_int, _c_int, _c_int]),
    "ek_moe_permute": (_c_int, [_c_vp, _c_int, _c_int, _c_int, _c_int, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_int,
                                _c_int, _c_vp, _c_vp, _c_vp]),
    "ek_p2p_mem_base": (_c_int, [_c_vp, ctypes.POINTER(ctypes.c_ulonglong), ctypes.POINTER(_c_size)]),
    "ek_p2p_ipc_handle": (_c_int, [_c_vp, _c_vp]),
    "ek_p2p_ipc_open": (_c_int, [_c_vp, ctypes.POINTER(_c_vp)]),
    "ek_p2p_ipc_close": (_c_int, [_c_vp]),
    "ek_p2p_copy": (_c_int, [_c_vp, _c_vp, _c_size, _c_vp]),
    "ek_p2p_signal": (_c_int, [ctypes.POINTER(_c_vp), _c_int, _c_int, _c_vp]),
    "ek_p2p_wait": (_c_int, [_c_vp, _c_int, _c_int, _c_vp]),
    "ek_p2p_signal_dev": (_c_int, [ctypes.POINTER(_c_vp), _c_int, _c_vp, _c_vp]),
    "ek_p2p_wait_dev": (_c_int, [_c_vp, _c_int, _c_vp, _c_vp]),
    "ek_moe_route_permute": (_c_int, [_c_vp, _c_int, _c_int, _c_int, _c_vp, _c_vp, _c_int, _c_vp, _c_vp, _c_vp, _c_vp,
                                      _c_vp, _c_int, _c_int, _c_vp, _c_vp, _c_vp]),
    "ek_moe_gate_up": (_c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int, _c_int,
                                _c_int, _c_int, _c_int, _c_vp]),
    "ek_moe_down": (_c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int,
                             _c_int, _c_int, _c_int, _c_int, _c_int, _c_vp]),
    "ek_moe_gate_up_packed": (_c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_vp] + [_c_int] * 7 + [_c_vp, _c_size, _c_vp]),
    "ek_moe_down_packed": (_c_int, [_c_vp] * 6 + [_c_int] * 9 + [_c_vp, _c_size, _c_vp]),
    "ek_moe_packed_workspace_bytes": (_c_size, [_c_int, _c_int, _c_int]),
    "ek_moe_combine": (_c_int, [_c_vp, _c_vp, _c_int, _c_int, _c_int, _c_vp]),
    "ek_moe_gate_up_fp8bs": (_c_int, [_c_vp] * 8 + [_c_int] * 7 + [_c_vp]),
    "ek_moe_down_fp8bs": (_c_int, [_c_vp] * 8 + [_c_int] * 9 + [_c_vp]),
    "ek_moe_gate_up_fp8mx": (_c_int, [_c_vp] * 8 + [_c_int] * 7 + [_c_vp]),
    "ek_moe_down_fp8mx": (_c_int, [_c_vp] * 8 + [_c_int] * 9 + [_c_vp]),
    "ek_moe_gather_rows": (_c_int, [_c_vp, _c_vp, _c_int, _c_int, _c_int, _c_vp, _c_int, _c_vp, _c_vp]),
    "ek_moe_gather_cols_f32": (_c_int, [_c_vp, _c_vp, _c_int, _c_int, _c_int, _c_vp, _c_int, _c_vp, _c_vp]),
    "ek_moe_slot_rows": (_c_int, [_c_vp, _c_vp, _c_int, _c_int, _c_vp, _c_vp]),
    "ek_ep_pack_meta": (_c_int, [_c_vp, _c_int, _c_vp, _c_vp, _c_int, _c_int, _c_vp, _c_vp, _c_vp]),
    "ek_ep_capacity_layout": (_c_int, [_c_vp, _c_vp, _c_int, _c_int, _c_int, _c_vp, _c_vp, _c_int, _c_vp, _c_vp, _c_vp,
                                       _c_vp, _c_vp]),
    "ek_moe_combine_rows": (_c_int, [_c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int, _c_vp]),
    "ek_moe_segment_gemm": (_c_int, [_c_vp, _c_vp, _c_vp, _c_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
                                     _c_vp]),
}

_LIB = None
_LOCK = threading.Lock()


class EKError(RuntimeError):
    """A C-ABI call returned an error code."""

    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def lib() -> ctypes.CDLL:
    """Load ``_ek.so`` (once) and declare every exported symbol's signature."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"elastikernel_b200 native library not built ({LIB_PATH}); "
                    "run `python -m elastikernel_b200.csrc.build`")
            L = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(L, name, None)
                if fn is None:
                    continue
                fn.restype = res
                fn.argtypes = args
            _LIB = L
    return _LIB


def exported_symbols() -> list[str]:
    """Names declared in the binding table (the header's entry points)."""
    return list(_SIGNATURES)


def last_error() -> str:
    return lib().ek_last_error().decode(errors="replace")


def check(rc: int, what: str = "") -> None:
    """Raise for a non-zero status: ValueError for over-subscription (as the
    reference's green_ctx.py:151-155), RuntimeError otherwise."""
    if rc == EK_OK:
        return
    msg = last_error() or f"error code {rc}"
    if what:
        msg = f"{what}: {msg}"
    if rc == EK_ERR_OVERSUB:
        raise ValueError(msg)
    raise EKError(rc, msg)


def device_status(dev: int, clear: bool = True) -> int:
    """Synchronise `dev` and return (and by default clear) the kernels' status word.

    A bounded-wait timeout can strike in the middle of a split-K hand-off and
    leave a ticket or a "part written" flag set in the split workspace; a later
    launch over the same workspace would then read a part that was never
    written. So when the word reports EK_STATUS_WAIT_TIMEOUT, every cached
    workspace of the device is zero-filled again before this returns."""
    v = ctypes.c_int(0)
    check(lib().ek_device_status(int(dev), 1 if clear else 0, ctypes.byref(v)), "ek_device_status")
    if v.value & EK_STATUS_WAIT_TIMEOUT:
        import torch

        from . import _workspace

        _workspace.reset(torch.device("cuda", int(dev)))
    return v.value


def stream_ptr(stream) -> int:
    """Raw CUstream of a torch stream (0 for the legacy default stream)."""
    return int(stream.cuda_stream) if stream is not None else 0
