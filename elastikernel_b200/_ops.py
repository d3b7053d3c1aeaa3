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
    # the C-ABI takes 16-byte aligned operands (ragged shapes are padded
    # there); a view that starts mid-line is copied to a fresh device buffer
    if a.data_ptr() % 16:
        a = a.clone()
    if b.data_ptr() % 16:
        b = b.clone()
    if out.data_ptr() % 16:
        tmp = gemm(a, b, None, num_sms, b_layout, force_bn, force_split)
        return out.copy_(tmp)
    L = lib()
    stream = current_stream_handle(dev)
    sms = int(num_sms) if num_sms else _stream_sms(dev, stream)
    dt = _DTYPES[a.dtype]
    need = L.ek_gemm_workspace_bytes(M, N, K, sms, dt, bl, int(force_bn), int(force_split))
    if need == _SIZE_MAX:
        check(_lib.EK_ERR_INVALID, "ek_gemm_workspace_bytes")
    ws = _workspace.get(dev, stream, need)
    with _on_device(dev):
        check(L.ek_gemm(a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, dt, bl, sms, int(force_bn),
                        int(force_split), _ptr(ws), 0 if ws is None else ws.numel(), stream), "ek_gemm")
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
    sms = int(num_sms) if num_sms else _stream_sms(dev, stream)
    need = lib().ek_gemm_workspace_bytes(M, N, K, sms, _lib.EK_DTYPE_E4M3, _lib.EK_B_NK, int(force_bn),
                                         int(force_split))
    if need == _SIZE_MAX:
        check(_lib.EK_ERR_INVALID, "ek_gemm_workspace_bytes")
    ws = _workspace.get(dev, stream, need)
    with _on_device(dev):
        check(lib().ek_gemm_fp8(a_q.data_ptr(), w_q.data_ptr(), a_scale.data_ptr(), w_scale.data_ptr(),
                                out.data_ptr(), M, N, K, sms, int(force_bn), int(force_split), _ptr(ws),
                                0 if ws is None else ws.numel(), stream), "ek_gemm_fp8")
    return out


def quant_e4m3(x: torch.Tensor, block: tuple[int, int] = (1, 0), pow2: bool = False) -> tuple[torch.Tensor,
                                                                                              torch.Tensor]:
    """e4m3 codes and fp32 scales (amax / 448 per block) of a bf16/fp32 [rows, cols] tensor.

    block = (1, 0): one scale per row; (1, 128): per 1 x 128 group;
    (br, bc): per br x bc block. Scales come back shaped [ceil(rows/br), ceil(cols/bc)]
    (or [rows] for row-wise). pow2=True rounds every scale up to a power of
    two (the UE8M0 scale factors of the block-scaled GEMMs)."""
    dev = _require_cuda(x)
    if x.dtype not in (torch.bfloat16, torch.float32) or x.dim() != 2:
        raise RuntimeError("quant_e4m3 takes a 2-D bf16 or fp32 tensor")
    _contig("x", x)
    if _FP8 is None:
        raise RuntimeError("this torch has no float8_e4m3fn")
    rows, cols = x.shape
    br, bc = int(block[0]), int(block[1])
    q = torch.empty((rows, cols), dtype=_FP8, device=dev)
    if br == 1 and bc <= 0:
        scales = torch.empty(rows, dtype=torch.float32, device=dev)
    else:
        scales = torch.empty((-(-rows // br), -(-cols // bc)), dtype=torch.float32, device=dev)
    with _on_device(dev):
        check(lib().ek_quant_e4m3_ex(x.data_ptr(), 0 if x.dtype == torch.bfloat16 else 3, rows, cols, br, bc,
                                     _lib.EK_QUANT_POW2_SCALES if pow2 else 0, q.data_ptr(), scales.data_ptr(),
                                     current_stream_handle(dev)), "ek_quant_e4m3_ex")
    return q, scales


def quant_e4m3_kmajor(x: torch.Tensor, pow2: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """e4m3 codes and 1 x 128 group scales of a bf16/fp32 [rows, cols] tensor, the
    scales K-block-major: [ceil(cols/128), rows] (the transpose of quant_e4m3's
    (1, 128) scales, bit for bit). The FP8 block-scaled MoE GEMMs take this layout.
    pow2=True: power-of-two scales, as quant_e4m3."""
    dev = _require_cuda(x)
    if x.dtype not in (torch.bfloat16, torch.float32) or x.dim() != 2:
        raise RuntimeError("quant_e4m3_kmajor takes a 2-D bf16 or fp32 tensor")
    _contig("x", x)
    if _FP8 is None:
        raise RuntimeError("this torch has no float8_e4m3fn")
    rows, cols = x.shape
    q = torch.empty((rows, cols), dtype=_FP8, device=dev)
    scales = torch.empty((-(-cols // 128), rows), dtype=torch.float32, device=dev)
    with _on_device(dev):
        check(lib().ek_quant_e4m3_kmajor_ex(x.data_ptr(), 0 if x.dtype == torch.bfloat16 else 3, rows, cols,
                                            _lib.EK_QUANT_POW2_SCALES if pow2 else 0, q.data_ptr(),
                                            scales.data_ptr(), current_stream_handle(dev)), "ek_quant_e4m3_kmajor_ex")
    return q, scales


def moe_gather_cols_f32(perm: dict, src: torch.Tensor) -> torch.Tensor:
    """[cols, max_rows] fp32: column c, row r = src[sorted_slots[r] // topk, c] (0 for
    unused rows) - per-row values such as received group scales, gathered in the
    permutation's order and transposed to the K-block-major layout."""
    dev = _require_cuda(src)
    if src.dtype != torch.float32 or src.dim() != 2:
        raise RuntimeError("moe_gather_cols_f32 takes a 2-D fp32 tensor")
    _contig("src", src)
    rows, cols = perm["max_rows"], src.shape[1]
    dst = torch.empty((cols, rows), dtype=torch.float32, device=dev)
    with _on_device(dev):
        check(lib().ek_moe_gather_cols_f32(perm["sorted_slots"].data_ptr(), perm["num_rows_padded"].data_ptr(), rows,
                                           perm["T"] * perm["topk"], perm["topk"], src.data_ptr(), cols,
                                           dst.data_ptr(), current_stream_handle(dev)), "ek_moe_gather_cols_f32")
    return dst


_SIZE_MAX = ctypes.c_size_t(-1).value
_DEV_SMS: dict[int, int] = {}


class _NullCtx:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


_NULL = _NullCtx()


def _on_device(dev: torch.device):
    """Make `dev` current for a launch (a no-op when it already is)."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    return _NULL if torch.cuda.current_device() == idx else torch.cuda.device(dev)


def _stream_sms(dev: torch.device, stream: int) -> int:
    """SM count of the partition `stream` belongs to (registry), else the device's."""
    v = ctypes.c_int(0)
    check(lib().ek_gctx_stream_sm_count(ctypes.c_void_p(stream), ctypes.byref(v)), "ek_gctx_stream_sm_count")
    if v.value > 0:
        return v.value
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    n = _DEV_SMS.get(idx)
    if n is None:
        n = _DEV_SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return n


# ---------------------------------------------------------------------- MoE
BLOCK_M = 128


def moe_route(gate_logits: torch.Tensor, topk: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Softmax top-k routing (definition.py:152-153): int32 ids [T,k] and fp32
    renormalised weights [T,k]. Ties go to the lower expert id."""
    dev = _require_cuda(gate_logits)
    if gate_logits.dtype != torch.float32 or gate_logits.dim() != 2:
        raise RuntimeError("gate_logits must be a 2-D float32 tensor")
    _contig("gate_logits", gate_logits)
    T, E = gate_logits.shape
    ids = torch.empty((T, topk), dtype=torch.int32, device=dev)
    wts = torch.empty((T, topk), dtype=torch.float32, device=dev)
    with _on_device(dev):
        check(lib().ek_moe_route(gate_logits.data_ptr(), T, E, int(topk), ids.data_ptr(), wts.data_ptr(),
                                 current_stream_handle(dev)), "ek_moe_route")
    return ids, wts


def moe_permute(topk_ids: torch.Tensor, num_experts: int, x: torch.Tensor | None = None,
                block_m: int = BLOCK_M) -> dict:
    """Expert-sorted, block-padded layout of the (token, choice) slots, with the
    token rows of `x` gathered into it when given."""
    dev = _require_cuda(topk_ids, x)
    if topk_ids.dtype != torch.int32 or topk_ids.dim() != 2:
        raise RuntimeError("topk_ids must be a 2-D int32 tensor")
    _contig("topk_ids", topk_ids)
    T, k = topk_ids.shape
    E = int(num_experts)
    max_rows = int(lib().ek_moe_max_padded_rows(T, k, E, block_m))
    sorted_slots = torch.empty(max_rows, dtype=torch.int32, device=dev)
    block_expert = torch.empty(max_rows // block_m, dtype=torch.int32, device=dev)
    num_rows = torch.empty(1, dtype=torch.int32, device=dev)
    counts = torch.empty(E, dtype=torch.int32, device=dev)
    x_perm = None
    H = 0
    es = 0
    if x is not None:
        _contig("x", x)
        if x.dim() != 2 or x.shape[0] != T:
            raise RuntimeError("x must be [T, H]")
        H = x.shape[1]
        es = x.element_size()
        x_perm = torch.empty((max_rows, H), dtype=x.dtype, device=dev)
    scratch = torch.empty(int(lib().ek_moe_permute_scratch_bytes(T, k, E)), dtype=torch.uint8, device=dev)
    with _on_device(dev):
        check(lib().ek_moe_permute(topk_ids.data_ptr(), T, k, E, block_m, sorted_slots.data_ptr(),
                                   block_expert.data_ptr(), num_rows.data_ptr(), counts.data_ptr(), _ptr(x), H, es,
                                   _ptr(x_perm), scratch.data_ptr(), current_stream_handle(dev)), "ek_moe_permute")
    return {"sorted_slots": sorted_slots, "block_expert": block_expert, "num_rows_padded": num_rows,
            "expert_counts": counts, "x_perm": x_perm, "max_rows": max_rows, "T": T, "topk": k, "E": E,
            "block_m": block_m}


def moe_route_permute(gate_logits: torch.Tensor, topk: int, num_experts: int, x: torch.Tensor | None = None,
                      block_m: int = BLOCK_M) -> tuple[torch.Tensor, torch.Tensor, dict]:
    """moe_route then moe_permute (same outputs): ids, weights and the
    permutation dict. Up to 128 slots the routing, the permutation and a
    small row gather are one launch."""
    dev = _require_cuda(gate_logits, x)
    if gate_logits.dtype != torch.float32 or gate_logits.dim() != 2:
        raise RuntimeError("gate_logits must be a 2-D float32 tensor")
    _contig("gate_logits", gate_logits)
    T, E_logits = gate_logits.shape
    E = int(num_experts)
    if E_logits != E:
        raise RuntimeError("gate_logits must have one column per expert")
    k = int(topk)
    ids = torch.empty((T, k), dtype=torch.int32, device=dev)
    wts = torch.empty((T, k), dtype=torch.float32, device=dev)
    max_rows = int(lib().ek_moe_max_padded_rows(T, k, E, block_m))
    sorted_slots = torch.empty(max_rows, dtype=torch.int32, device=dev)
    block_expert = torch.empty(max_rows // block_m, dtype=torch.int32, device=dev)
    num_rows = torch.empty(1, dtype=torch.int32, device=dev)
    counts = torch.empty(E, dtype=torch.int32, device=dev)
    x_perm = None
    H = es = 0
    if x is not None:
        _contig("x", x)
        if x.dim() != 2 or x.shape[0] != T:
            raise RuntimeError("x must be [T, H]")
        H, es = x.shape[1], x.element_size()
        x_perm = torch.empty((max_rows, H), dtype=x.dtype, device=dev)
    scratch = torch.empty(int(lib().ek_moe_permute_scratch_bytes(T, k, E)), dtype=torch.uint8, device=dev)
    with _on_device(dev):
        check(lib().ek_moe_route_permute(gate_logits.data_ptr(), T, E, k, ids.data_ptr(), wts.data_ptr(), block_m,
                                         sorted_slots.data_ptr(), block_expert.data_ptr(), num_rows.data_ptr(),
                                         counts.data_ptr(), _ptr(x), H, es, _ptr(x_perm), scratch.data_ptr(),
                                         current_stream_handle(dev)), "ek_moe_route_permute")
    perm = {"sorted_slots": sorted_slots, "block_expert": block_expert, "num_rows_padded": num_rows,
            "expert_counts": counts, "x_perm": x_perm, "max_rows": max_rows, "T": T, "topk": k, "E": E,
            "block_m": block_m}
    return ids, wts, perm


def _check_bf16(name: str, t: torch.Tensor) -> None:
    if t.dtype != torch.bfloat16:
        raise RuntimeError(f"{name} must be bfloat16")
    _contig(name, t)


def moe_gate_up(perm: dict, w1: torch.Tensor, w3: torch.Tensor, num_sms: int | None = None,
                force_bn: int = 0) -> torch.Tensor:
    """act[r] = silu(x_perm[r] . w1[e]) * (x_perm[r] . w3[e]) over the padded rows
    (a layout padded to 256 rows per expert runs on CTA pairs)."""
    x_perm = perm["x_perm"]
    dev = _require_cuda(x_perm, w1, w3)
    for n, t in (("x_perm", x_perm), ("w1", w1), ("w3", w3)):
        _check_bf16(n, t)
    E, I, H = w1.shape
    if w3.shape != w1.shape or x_perm.shape[1] != H or E != perm["E"]:
        raise RuntimeError("gate_up: shape mismatch")
    max_rows = perm["max_rows"]
    act = torch.empty((max_rows, I), dtype=torch.bfloat16, device=dev)
    stream = current_stream_handle(dev)
    with _on_device(dev):
        check(lib().ek_moe_gate_up(x_perm.data_ptr(), w1.data_ptr(), w3.data_ptr(), perm["block_expert"].data_ptr(),
                                   perm["num_rows_padded"].data_ptr(), act.data_ptr(), max_rows, E, H, I,
                                   perm["T"] * perm["topk"], int(num_sms or 0), int(force_bn), int(perm["block_m"]),
                                   stream), "ek_moe_gate_up")
    return act


def moe_down(perm: dict, act: torch.Tensor, w2: torch.Tensor, topk_weights: torch.Tensor,
             num_sms: int | None = None, force_bn: int = 0) -> torch.Tensor:
    """y[s] = topk_weight[s] * (act[r] @ w2[e]^T) for the slot s of each used row r."""
    dev = _require_cuda(act, w2, topk_weights)
    _check_bf16("act", act)
    _check_bf16("w2", w2)
    _contig("topk_weights", topk_weights)
    if topk_weights.dtype != torch.float32:
        raise RuntimeError("topk_weights must be float32")
    E, H, I = w2.shape
    T, k = perm["T"], perm["topk"]
    if act.shape[1] != I or E != perm["E"] or topk_weights.numel() != T * k:
        raise RuntimeError("down: shape mismatch")
    y = torch.empty((T * k, H), dtype=torch.bfloat16, device=dev)
    with _on_device(dev):
        check(lib().ek_moe_down(act.data_ptr(), w2.data_ptr(), perm["block_expert"].data_ptr(),
                                perm["num_rows_padded"].data_ptr(), perm["sorted_slots"].data_ptr(),
                                topk_weights.data_ptr(), y.data_ptr(), perm["max_rows"], E, H, I, T, k,
                                int(num_sms or 0), int(force_bn), int(perm["block_m"]), current_stream_handle(dev)),
              "ek_moe_down")
    return y


def moe_gate_up_packed(perm: dict, w1: torch.Tensor, w3: torch.Tensor, num_sms: int | None = None,
                       tok_tile: int = 0, pair: int = -1, ksplit: bool = True) -> torch.Tensor:
    """Swapped-operand gate/up over the packed layout (permute with block_m=1).
    ksplit=False withholds the workspace, so K is never split."""
    x_perm = perm["x_perm"]
    dev = _require_cuda(x_perm, w1, w3)
    for n, t in (("x_perm", x_perm), ("w1", w1), ("w3", w3)):
        _check_bf16(n, t)
    if perm["block_m"] != 1:
        raise RuntimeError("the packed GEMMs take the packed layout (moe_permute(..., block_m=1))")
    E, I, H = w1.shape
    if w3.shape != w1.shape or x_perm.shape[1] != H or E != perm["E"]:
        raise RuntimeError("gate_up_packed: shape mismatch")
    rows = perm["max_rows"]
    act = torch.empty((rows, I), dtype=torch.bfloat16, device=dev)
    ws, nb = _packed_workspace(rows, H, I, dev) if ksplit else (None, 0)
    with _on_device(dev):
        check(lib().ek_moe_gate_up_packed(x_perm.data_ptr(), w1.data_ptr(), w3.data_ptr(),
                                          perm["expert_counts"].data_ptr(), act.data_ptr(), rows, E, H, I,
                                          int(tok_tile), int(pair), int(num_sms or 0), _ptr(ws), nb,
                                          current_stream_handle(dev)), "ek_moe_gate_up_packed")
    return act


def _packed_workspace(rows: int, H: int, I: int, dev: torch.device) -> tuple[torch.Tensor | None, int]:
    """Workspace of the packed GEMMs' K-split (None where the size never splits)."""
    nb = int(lib().ek_moe_packed_workspace_bytes(int(rows), int(H), int(I)))
    return (torch.empty(nb, dtype=torch.uint8, device=dev) if nb else None), nb


def moe_down_packed(perm: dict, act: torch.Tensor, w2: torch.Tensor, topk_weights: torch.Tensor,
                    num_sms: int | None = None, tok_tile: int = 0, pair: int = -1,
                    ksplit: bool = True) -> torch.Tensor:
    """Swapped-operand down projection with the routing weight, scattered to slots.
    ksplit=False withholds the workspace, so K is never split."""
    dev = _require_cuda(act, w2, topk_weights)
    _check_bf16("act", act)
    _check_bf16("w2", w2)
    _contig("topk_weights", topk_weights)
    E, H, I = w2.shape
    T, k = perm["T"], perm["topk"]
    if act.shape[1] != I or E != perm["E"] or topk_weights.numel() != T * k or perm["block_m"] != 1:
        raise RuntimeError("down_packed: shape mismatch")
    y = torch.empty((T * k, H), dtype=torch.bfloat16, device=dev)
    ws, nb = _packed_workspace(perm["max_rows"], H, I, dev) if ksplit else (None, 0)
    with _on_device(dev):
        check(lib().ek_moe_down_packed(act.data_ptr(), w2.data_ptr(), perm["expert_counts"].data_ptr(),
                                       perm["sorted_slots"].data_ptr(), topk_weights.data_ptr(), y.data_ptr(),
                                       perm["max_rows"], E, H, I, T, k, int(tok_tile), int(pair),
                                       int(num_sms or 0), _ptr(ws), nb, current_stream_handle(dev)),
              "ek_moe_down_packed")
    return y


def quant_moe_weights_fp8(w1: torch.Tensor, w2: torch.Tensor, w3: torch.Tensor, pow2: bool = False) -> dict:
    """e4m3 expert weights with 128 x 128 fp32 block scales (DeepSeek style).
    w1, w3 [E, I, H] and w2 [E, H, I] (bf16 or fp32); I and H multiples of 128.
    pow2=True: power-of-two block scales; the layer then quantises its tokens
    and activations the same way and runs the GEMMs whose tensor cores apply
    the scales (ek_moe_*_fp8mx)."""
    E, I, H = w1.shape
    if I % 128 or H % 128:
        raise RuntimeError("block-scaled FP8 needs I and H multiples of 128")
    out = {"E": E, "I": I, "H": H, "pow2": bool(pow2)}
    for name, w, rows, cols in (("w1", w1, I, H), ("w3", w3, I, H), ("w2", w2, H, I)):
        q, s = quant_e4m3(w.reshape(E * rows, cols).contiguous(), block=(128, 128), pow2=pow2)
        out[name + "q"] = q.view(E, rows, cols)
        out[name + "s"] = s
    return stack_gate_up_planes(out)


def stack_gate_up_planes(qw: dict) -> dict:
    """Store the e4m3 w1 and w3 codes as the two planes of one [2, E, I, H]
    buffer (w1q / w3q become views of it). The gate/up GEMMs then load a
    tile's [w1 rows | w3 rows] with one TMA box instead of two, which lets an
    SM draw about twice the HBM bandwidth (the TMA engine keeps only a few
    boxes in flight). Any layout stays correct; this one is faster. Call it
    again after concatenating the codes of several quantised shards."""
    w1q, w3q = qw["w1q"], qw["w3q"]
    if w1q.shape != w3q.shape:
        raise RuntimeError("w1q and w3q must have one shape")
    planes = torch.stack([w1q, w3q])
    qw = dict(qw)
    qw["w1q"], qw["w3q"] = planes[0], planes[1]
    return qw


def _mx(qw: dict, mx: bool | None) -> bool:
    """Whether the block-scaled GEMMs apply the scales in the tensor cores
    (power-of-two scales) or scale each K block's product in the epilogue."""
    pow2 = bool(qw.get("pow2", False))
    if mx is None:
        return pow2
    if mx and not pow2:
        raise RuntimeError("the tensor-core-scaled FP8 GEMMs need power-of-two scales (quant_moe_weights_fp8(pow2=True))")
    return bool(mx)


def moe_gate_up_fp8bs(perm: dict, xq: torch.Tensor, xs: torch.Tensor, qw: dict, num_sms: int | None = None,
                      tok_tile: int = 0, pair: int = -1, mx: bool | None = None) -> torch.Tensor:
    """Block-scaled FP8 gate/up (SwiGLU) over the packed layout; bf16 act [rows, I].
    xs: K-block-major token scales [H/128, rows] (quant_e4m3_kmajor).
    tok_tile 0 and pair -1 let the library choose (CTA pairs for tiles of 128/256).
    mx (default: the weights' scale form) picks ek_moe_gate_up_fp8mx, whose
    tensor cores apply power-of-two scales, over ek_moe_gate_up_fp8bs."""
    dev = _require_cuda(xq, xs)
    if perm["block_m"] != 1:
        raise RuntimeError("the FP8 block-scaled GEMMs take the packed layout (block_m=1)")
    rows, E, H, I = perm["max_rows"], qw["E"], qw["H"], qw["I"]
    if xq.shape != (rows, H) or xs.shape != (H // 128, rows):
        raise RuntimeError("gate_up_fp8bs: activation shape mismatch")
    act = torch.empty((rows, I), dtype=torch.bfloat16, device=dev)
    fn = lib().ek_moe_gate_up_fp8mx if _mx(qw, mx) else lib().ek_moe_gate_up_fp8bs
    with _on_device(dev):
        check(fn(xq.data_ptr(), xs.data_ptr(), qw["w1q"].data_ptr(), qw["w3q"].data_ptr(), qw["w1s"].data_ptr(),
                 qw["w3s"].data_ptr(), perm["expert_counts"].data_ptr(), act.data_ptr(), rows, E, H, I, int(tok_tile),
                 int(pair), int(num_sms or 0), current_stream_handle(dev)), fn.__name__)
    return act


def moe_down_fp8bs(perm: dict, aq: torch.Tensor, as_: torch.Tensor, qw: dict, topk_weights: torch.Tensor,
                   num_sms: int | None = None, tok_tile: int = 0, pair: int = -1, mx: bool | None = None) -> torch.Tensor:
    """Block-scaled FP8 down projection with the routing weight, scattered to slots (bf16 [T*k, H]).
    as_: K-block-major act scales [I/128, rows]. mx as for moe_gate_up_fp8bs."""
    dev = _require_cuda(aq, as_, topk_weights)
    rows, E, H, I = perm["max_rows"], qw["E"], qw["H"], qw["I"]
    T, k = perm["T"], perm["topk"]
    if aq.shape != (rows, I) or as_.shape != (I // 128, rows) or topk_weights.numel() != T * k:
        raise RuntimeError("down_fp8bs: shape mismatch")
    y = torch.empty((T * k, H), dtype=torch.bfloat16, device=dev)
    fn = lib().ek_moe_down_fp8mx if _mx(qw, mx) else lib().ek_moe_down_fp8bs
    with _on_device(dev):
        check(fn(aq.data_ptr(), as_.data_ptr(), qw["w2q"].data_ptr(), qw["w2s"].data_ptr(),
                 perm["expert_counts"].data_ptr(), perm["sorted_slots"].data_ptr(), topk_weights.data_ptr(),
                 y.data_ptr(), rows, E, H, I, T, k, int(tok_tile), int(pair), int(num_sms or 0),
                 current_stream_handle(dev)), fn.__name__)
    return y


def fused_moe_fp8(hidden_states: torch.Tensor, gate_logits: torch.Tensor, qw: dict, topk: int,
                  out: torch.Tensor | None = None, num_sms: int | None = None) -> torch.Tensor:
    """MoE layer with e4m3 block-scaled experts: route -> quantise the token
    rows (1 x 128 groups; a group lies in one row, so quantising before the
    permutation gives the same codes and scales) -> permute + gather the e4m3
    rows (half the bytes of bf16) and their scales (K-block-major) -> FP8
    gate/up SwiGLU -> quantise act -> FP8 down (+weight) -> combine."""
    _require_cuda(hidden_states, gate_logits, out)
    _check_bf16("hidden_states", hidden_states)
    T = hidden_states.shape[0]
    if T == 0:
        return out if out is not None else torch.empty_like(hidden_states)
    pow2 = bool(qw.get("pow2", False))  # tokens and activations take the weights' scale form
    xq_tok, xs_tok = quant_e4m3(hidden_states, block=(1, 128), pow2=pow2)
    ids, wts, perm = moe_route_permute(gate_logits, topk, qw["E"], x=xq_tok, block_m=1)
    xs = moe_gather_cols_f32(perm, xs_tok)
    act = moe_gate_up_fp8bs(perm, perm["x_perm"], xs, qw, num_sms=num_sms)
    aq, as_ = quant_e4m3_kmajor(act, pow2=pow2)
    y = moe_down_fp8bs(perm, aq, as_, qw, wts, num_sms=num_sms)
    return moe_combine(y, T, topk, out=out)


def moe_combine(y: torch.Tensor, T: int, topk: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """out[t] = sum_j y[t*k + j] (fp32 sum in j order), bf16."""
    dev = _require_cuda(y, out)
    _check_bf16("y", y)
    H = y.shape[1]
    if out is None:
        out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    else:
        _check_bf16("out", out)
    with _on_device(dev):
        check(lib().ek_moe_combine(y.data_ptr(), out.data_ptr(), int(T), int(topk), H, current_stream_handle(dev)),
              "ek_moe_combine")
    return out


PACKED_MIN_SMS = 112
PACKED_MAX_ROWS_PER_EXPERT = 288
# below PACKED_MIN_SMS the packed layout still wins at decode sizes (routed rows)
PACKED_DECODE_MIN_SMS = 64
PACKED_DECODE_ROWS = 2
PACKED_DECODE_WIDE_SMS = 96
PACKED_DECODE_ROWS_WIDE = 4


def moe_layout(num_sms: int, num_experts: int, rows: int | None = None) -> str:
    """Layout the fused MoE uses on a partition of `num_sms` SMs for `rows`
    routed rows (tokens x top-k; None: not known).

    Measured on B200 (Mixtral shapes, T = 1..4096): the packed layout with the
    swapped-operand GEMMs is faster on (nearly) the full device while experts
    get up to a few hundred rows -- T=128: 519 us packed vs 578 us padded,
    T=1024 (256 rows per expert): 861 vs 875 us on 148 SMs -- and the 128-row
    padded layout from 320 rows per expert (T=1280: 1029-1057 vs 1054-1206 us,
    T=1536: 1241 vs 1322 us, T=2048: 1393 vs 1631 us, T=4096: 2402 vs 2572
    us) and on small partitions (T=128 on 72 SMs: 632 us padded
    vs 833 us packed), except at decode sizes, where the packed GEMMs stream
    only the experts hit and split K over the idle SMs (96 SMs: T=1 202 vs
    245 us, T=2 254 vs 284 us, T=4 347 vs 325 us; 72 SMs: T=1 248 vs 254 us,
    T=2 339 vs 314 us)."""
    if num_experts > 256:
        return "padded"
    if num_sms < PACKED_MIN_SMS:
        decode_rows = (PACKED_DECODE_ROWS_WIDE if num_sms >= PACKED_DECODE_WIDE_SMS
                       else PACKED_DECODE_ROWS if num_sms >= PACKED_DECODE_MIN_SMS else 0)
        return "packed" if rows is not None and rows <= decode_rows else "padded"
    if rows is not None and rows > PACKED_MAX_ROWS_PER_EXPERT * num_experts:
        return "padded"
    return "packed"


PAIR_MIN_ROWS_PER_EXPERT = 768        # from PACKED_MIN_SMS SMs up
PAIR_MIN_ROWS_PER_EXPERT_SMALL = 256  # on smaller partitions


def padded_block_m(num_sms: int, num_experts: int, rows: int) -> int:
    """Row padding of the padded layout: 256 (2-SM CTA-pair tiles) from 768
    routed rows per expert on 112+ SMs and from 256 on 2..111 SMs, else 128.
    Measured on B200 (Mixtral shapes): on 148 SMs T=4096 (1024 rows per
    expert) gate/up 1751-1786 vs 1882 us and down 858-887 vs 957-969 us,
    T=2048 (512 rows per expert) no gain, the extra padding eats the pair's
    higher per-row rate; on 72 SMs the layer at T=1024 / 2048 / 4096 takes
    1280 / 1903-1987 / 3598-3731 us with pairs vs 1303-1316 / 2144 /
    4152-4257 us, at T=512 863-976 vs 859-884 us."""
    if num_sms < 2:
        return BLOCK_M
    per_expert = PAIR_MIN_ROWS_PER_EXPERT if num_sms >= PACKED_MIN_SMS else PAIR_MIN_ROWS_PER_EXPERT_SMALL
    return 256 if rows >= per_expert * num_experts else BLOCK_M


def fused_moe(hidden_states: torch.Tensor, gate_logits: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
              w3: torch.Tensor, topk: int, out: torch.Tensor | None = None, num_sms: int | None = None,
              layout: str = "auto") -> torch.Tensor:
    """The whole MoE layer: route -> permute(+gather) -> gate/up SwiGLU -> down(+weight) -> combine.

    layout="packed": expert-major rows without padding and the swapped-operand
    GEMMs; "padded": 128-row padded blocks and the token-major GEMMs; "auto"
    (default): moe_layout() for the partition of the current stream."""
    dev = _require_cuda(hidden_states, gate_logits, w1, w2, w3, out)
    _check_bf16("hidden_states", hidden_states)
    T = hidden_states.shape[0]
    if T == 0:
        return out if out is not None else torch.empty_like(hidden_states)
    sms = int(num_sms) if num_sms else _stream_sms(dev, current_stream_handle(dev))
    if layout == "auto":
        layout = moe_layout(sms, w1.shape[0], T * topk)
    if layout == "packed" and w1.shape[0] <= 256:
        ids, wts, perm = moe_route_permute(gate_logits, topk, w1.shape[0], x=hidden_states, block_m=1)
        act = moe_gate_up_packed(perm, w1, w3, num_sms=num_sms)
        y = moe_down_packed(perm, act, w2, wts, num_sms=num_sms)
    else:
        ids, wts, perm = moe_route_permute(gate_logits, topk, w1.shape[0], x=hidden_states,
                                           block_m=padded_block_m(sms, w1.shape[0], T * topk))
        act = moe_gate_up(perm, w1, w3, num_sms=num_sms)
        y = moe_down(perm, act, w2, wts, num_sms=num_sms)
    return moe_combine(y, T, topk, out=out)


def moe_segment_gemm(hidden_states: torch.Tensor, weights: torch.Tensor, expert_offsets: torch.Tensor,
                     num_experts: int, N: int, K: int, num_sms: int | None = None,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """Reference segment GEMM semantics (sm_aware_benchmark.py:228-290)."""
    dev = _require_cuda(hidden_states, weights, expert_offsets, out)
    if hidden_states.dtype not in _DTYPES or weights.dtype != hidden_states.dtype:
        raise RuntimeError("segment GEMM takes bf16/fp16 operands of one dtype")
    for n, t in (("hidden_states", hidden_states), ("weights", weights), ("expert_offsets", expert_offsets)):
        _contig(n, t)
    if expert_offsets.dtype != torch.int32 or expert_offsets.numel() != num_experts + 1:
        raise RuntimeError("expert_offsets must be int32 [num_experts + 1]")
    M = hidden_states.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=hidden_states.dtype, device=dev)
    with _on_device(dev):
        check(lib().ek_moe_segment_gemm(hidden_states.data_ptr(), weights.data_ptr(), expert_offsets.data_ptr(),
                                        out.data_ptr(), M, int(N), int(K), int(num_experts),
                                        _DTYPES[hidden_states.dtype], int(num_sms or 0),
                                        current_stream_handle(dev)), "ek_moe_segment_gemm")
    return out
