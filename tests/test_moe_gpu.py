"""Fused-MoE parity on the GPU (C-ABI kernels vs the CPU oracle).

* routing indices and the permutation are compared bit-exactly;
* routing weights: |w - w_ref| <= 1e-6 (fp32 softmax, different exp rounding);
* MoE outputs: max|out - ref| / max|ref| <= 1e-2 against the oracle's fp32
  computation on the same bf16 inputs (the spec's bf16 tolerance);
* the segment GEMM (reference kernel semantics) against the oracle and the
  golden output of the reference Triton kernel.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import gemm as og
from oracle import moe as om

pytestmark = pytest.mark.gpu
GOLD = Path(__file__).resolve().parent / "golden"
TOL = 1e-2


@pytest.mark.parametrize("T,E,k", [(4096, 8, 2), (1, 8, 2), (512, 256, 8), (333, 16, 4), (64, 64, 6)])
def test_route_matches_oracle(cuda_dev, T, E, k):
    from elastikernel_b200 import _ops

    g = torch.Generator().manual_seed(T + E + k)
    logits = torch.randn((T, E), generator=g)
    ids, w = _ops.moe_route(logits.to(cuda_dev), k)
    rids, rw = om.route_ref(logits.numpy(), k)
    np.testing.assert_array_equal(ids.cpu().numpy(), rids)
    np.testing.assert_allclose(w.cpu().numpy(), rw, atol=1e-6, rtol=0)


def test_route_golden_and_ties(cuda_dev):
    from elastikernel_b200 import _ops

    z = np.load(GOLD / "routing.npz")
    for name in ("mixtral", "dsv3", "small"):
        ids, w = _ops.moe_route(torch.from_numpy(z[f"{name}_logits"]).to(cuda_dev), int(z[f"{name}_k"]))
        np.testing.assert_array_equal(ids.cpu().numpy(), z[f"{name}_ids"])
        np.testing.assert_allclose(w.cpu().numpy(), z[f"{name}_weights"], atol=1e-6, rtol=0)
    ties = torch.zeros((4, 40))
    ties[1, [3, 35]] = 1.0
    ties[2, :] = -float("inf")
    ties[2, [7, 39]] = 0.0
    ids, w = _ops.moe_route(ties.to(cuda_dev), 2)
    rids, rw = om.route_ref(ties.numpy(), 2)
    np.testing.assert_array_equal(ids.cpu().numpy(), rids)
    np.testing.assert_array_equal(rids, [[0, 1], [3, 35], [7, 39], [0, 1]])


@pytest.mark.parametrize("T,E,k", [(4096, 8, 2), (1, 8, 2), (3000, 256, 8), (17, 4, 4), (2500, 64, 3),
                                   (16384, 256, 8), (2048, 1024, 8), (20000, 8, 2)])
def test_permute_bit_exact(cuda_dev, T, E, k):
    from elastikernel_b200 import _ops

    g = torch.Generator().manual_seed(T * 7 + E)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    H = 64
    x = torch.randn((T, H), generator=g).to(torch.bfloat16)
    perm = _ops.moe_permute(ids.to(cuda_dev), E, x=x.to(cuda_dev))
    ref = om.permute_ref(ids.numpy(), E, 128)
    n = ref["num_rows_padded"]
    assert int(perm["num_rows_padded"].item()) == n
    np.testing.assert_array_equal(perm["sorted_slots"].cpu().numpy(), ref["sorted_slots"])
    np.testing.assert_array_equal(perm["block_expert"].cpu().numpy(), ref["block_expert"])
    np.testing.assert_array_equal(perm["expert_counts"].cpu().numpy(), ref["expert_counts"])
    slots = ref["sorted_slots"][:n]
    used = slots < T * k
    got = perm["x_perm"][:n].cpu()[torch.from_numpy(used)]
    want = x[torch.from_numpy(slots[used] // k).long()]
    assert torch.equal(got, want)


@pytest.mark.parametrize("T,E,k,block_m,H,dtype", [
    (1, 8, 2, 1, 4096, torch.bfloat16),      # one launch, rows gathered in it
    (16, 8, 2, 128, 4096, torch.bfloat16),   # one launch, 256 KB of rows gathered in it
    (64, 8, 2, 1, 4096, torch.bfloat16),     # one launch, rows gathered by the wide gather
    (16, 256, 8, 1, 7168, torch.uint8),      # 128 slots: the largest one-launch batch (e4m3 rows as bytes)
    (3, 64, 6, 256, 0, None),                # no rows
    (17, 256, 8, 1, 512, torch.bfloat16),    # 136 slots: the separate launches
])
def test_route_permute_matches_separate_launches(cuda_dev, T, E, k, block_m, H, dtype):
    """ek_moe_route_permute against ek_moe_route + ek_moe_permute: every
    output bit-identical, and the permutation against the oracle."""
    from elastikernel_b200 import _ops

    g = torch.Generator().manual_seed(T + 3 * E + k)
    logits = torch.randn((T, E), generator=g).to(cuda_dev)
    x = None
    if dtype is not None:
        x = (torch.randint(0, 255, (T, H), generator=g, dtype=torch.uint8) if dtype == torch.uint8
             else torch.randn((T, H), generator=g).to(dtype)).to(cuda_dev)
    ids, wts, perm = _ops.moe_route_permute(logits, k, E, x=x, block_m=block_m)
    ids2, wts2 = _ops.moe_route(logits, k)
    perm2 = _ops.moe_permute(ids2, E, x=x, block_m=block_m)
    torch.cuda.synchronize()
    assert torch.equal(ids, ids2) and torch.equal(wts, wts2)
    for key in ("sorted_slots", "block_expert", "num_rows_padded", "expert_counts"):
        assert torch.equal(perm[key], perm2[key]), key
    ref = om.permute_ref(ids.cpu().numpy(), E, block_m)
    np.testing.assert_array_equal(perm["sorted_slots"].cpu().numpy(), ref["sorted_slots"])
    if x is not None:
        n = int(perm["num_rows_padded"].item())
        used = perm["sorted_slots"][:n] < T * k  # padding rows are not gathered
        assert torch.equal(perm["x_perm"][:n][used], perm2["x_perm"][:n][used])


@pytest.mark.parametrize("T,k,H", [(4096, 8, 7168), (333, 2, 4096), (1, 1, 8), (64, 12, 520)])
def test_combine_bit_exact(cuda_dev, T, k, H):
    """Top-k combine: fp32 sum in choice order, one bf16 rounding (k = 12
    takes the kernel's path for more than eight choices)."""
    from elastikernel_b200 import _ops

    g = torch.Generator().manual_seed(T + k + H)
    y = torch.randn((T * k, H), generator=g).to(torch.bfloat16)
    out = _ops.moe_combine(y.to(cuda_dev), T, k)
    assert torch.equal(out.cpu(), om.combine_ref(y, T, k))


def _moe_inputs(T, H, I, E, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((T, H), generator=g).to(torch.bfloat16)
    logits = torch.randn((T, E), generator=g)
    w1 = (torch.randn((E, I, H), generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn((E, H, I), generator=g) * 0.02).to(torch.bfloat16)
    w3 = (torch.randn((E, I, H), generator=g) * 0.02).to(torch.bfloat16)
    return x, logits, w1, w2, w3


@pytest.mark.parametrize("layout", ["packed", "padded"])
@pytest.mark.parametrize("T,H,I,E,k", [(1, 512, 1024, 8, 2), (16, 512, 1024, 8, 2), (300, 256, 512, 8, 2),
                                       (64, 256, 384, 16, 4), (200, 128, 256, 32, 8), (5, 256, 256, 64, 6)])
def test_fused_moe_small(cuda_dev, T, H, I, E, k, layout):
    from elastikernel_b200 import _ops

    x, logits, w1, w2, w3 = _moe_inputs(T, H, I, E, seed=T + I)
    out = _ops.fused_moe(*(t.to(cuda_dev) for t in (x, logits, w1, w2, w3)), topk=k, layout=layout)
    torch.cuda.synchronize()
    ref = om.moe_ref(x, logits, w1, w2, w3, k)
    err = og.max_rel_err(out, ref)
    assert err <= TOL, f"max rel err {err:.3e}"


@pytest.mark.parametrize("tok", [16, 32, 64, 128, 256])
@pytest.mark.parametrize("pair", [0, 1])
def test_packed_token_tiles(cuda_dev, tok, pair):
    """Swapped-operand GEMMs for every token tile, single CTA and CTA pair,
    with ragged per-expert token counts and an unused expert."""
    from elastikernel_b200 import _ops

    T, H, I, E, k = 700, 256, 384, 8, 2
    x, logits, w1, w2, w3 = _moe_inputs(T, H, I, E, seed=tok + pair)
    logits[:, 5] = -30.0  # expert 5 receives no tokens
    d = [t.to(cuda_dev) for t in (x, logits, w1, w2, w3)]
    ids, wts = _ops.moe_route(d[1], k)
    perm = _ops.moe_permute(ids, E, x=d[0], block_m=1)
    act = _ops.moe_gate_up_packed(perm, d[2], d[4], tok_tile=tok, pair=pair)
    y = _ops.moe_down_packed(perm, act, d[3], wts, tok_tile=tok, pair=pair)
    out = _ops.moe_combine(y, T, k)
    torch.cuda.synchronize()
    assert int(perm["expert_counts"][5].item()) == 0
    assert og.max_rel_err(out, om.moe_ref(x, logits, w1, w2, w3, k)) <= TOL


@pytest.mark.parametrize("tok", [128, 256])
@pytest.mark.parametrize("planes", [False, True])
def test_packed_wide_gate_up(cuda_dev, tok, planes):
    """Wide CTA-pair gate/up tiles (256 weight rows per CTA, two accumulators):
    bit-identical to the 128-row pair tiles (same per-element K order), and
    the layer against the oracle; w1 / w3 as two tensors or as the two planes
    of one (one 3-D box per stage)."""
    from elastikernel_b200 import _ops

    T, H, I, E, k = 700, 256, 512, 8, 2
    x, logits, w1, w2, w3 = _moe_inputs(T, H, I, E, seed=tok + planes)
    d = [t.to(cuda_dev) for t in (x, logits, w1, w2, w3)]
    if planes:
        w13 = torch.stack([d[2], d[4]])
        d[2], d[4] = w13[0], w13[1]
    ids, wts = _ops.moe_route(d[1], k)
    perm = _ops.moe_permute(ids, E, x=d[0], block_m=1)
    act_w = _ops.moe_gate_up_packed(perm, d[2], d[4], tok_tile=tok, pair=2, ksplit=False)
    act_n = _ops.moe_gate_up_packed(perm, d[2], d[4], tok_tile=tok, pair=1, ksplit=False)
    y = _ops.moe_down_packed(perm, act_w, d[3], wts, tok_tile=tok, pair=1)
    out = _ops.moe_combine(y, T, k)
    torch.cuda.synchronize()
    n = int(perm["num_rows_padded"].item())
    assert torch.equal(act_w[:n], act_n[:n])
    assert og.max_rel_err(out, om.moe_ref(x, logits, w1, w2, w3, k)) <= TOL


@pytest.mark.parametrize("T", [1, 16, 128])
def test_fused_moe_mixtral_shapes(cuda_dev, T):
    """Mixtral expert shapes (H=4096, I=14336, E=8, top-2) at small token counts."""
    from elastikernel_b200 import _ops

    x, logits, w1, w2, w3 = _moe_inputs(T, 4096, 14336, 8, seed=42 + T)
    out = _ops.fused_moe(*(t.to(cuda_dev) for t in (x, logits, w1, w2, w3)), topk=2)
    torch.cuda.synchronize()
    ref = om.moe_ref(x, logits, w1, w2, w3, 2)
    err = og.max_rel_err(out, ref)
    assert err <= TOL, f"max rel err {err:.3e}"


@pytest.mark.parametrize("bn", [64, 128, 192, 256])
def test_grouped_tile_widths(cuda_dev, bn):
    from elastikernel_b200 import _ops

    T, H, I, E, k = 400, 256, 640, 8, 2
    x, logits, w1, w2, w3 = _moe_inputs(T, H, I, E, seed=bn)
    d = [t.to(cuda_dev) for t in (x, logits, w1, w2, w3)]
    ids, wts = _ops.moe_route(d[1], k)
    perm = _ops.moe_permute(ids, E, x=d[0])
    act = _ops.moe_gate_up(perm, d[2], d[4], force_bn=bn)
    y = _ops.moe_down(perm, act, d[3], wts, force_bn=bn)
    out = _ops.moe_combine(y, T, k)
    torch.cuda.synchronize()
    assert og.max_rel_err(out, om.moe_ref(x, logits, w1, w2, w3, k)) <= TOL


def test_segment_gemm_golden(cuda_dev):
    from elastikernel_b200 import _ops

    z = np.load(GOLD / "triton_gemm.npz")
    hs = torch.from_numpy(z["seg_hs"])
    w = torch.from_numpy(z["seg_w"])
    offs = torch.from_numpy(z["seg_offsets"])
    N, K, E = z["seg_out"].shape[1], hs.shape[1], offs.numel() - 1
    out = _ops.moe_segment_gemm(hs.to(cuda_dev), w.to(cuda_dev), offs.to(cuda_dev), E, N, K)
    torch.cuda.synchronize()
    ref = z["seg_out"].astype(np.float32)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, rtol=1e-2, atol=5e-2)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_segment_gemm_reference_config(cuda_dev, dtype):
    """The reference MoE benchmark's shapes (sm_aware_benchmark.py:406-444):
    tokens 512, N = K = 4096, 8 experts, top-2 fake contiguous routing."""
    from elastikernel_b200 import _ops

    T, N, K, E, k = 512, 4096, 4096, 8, 2
    g = torch.Generator().manual_seed(42)
    hs = torch.randn((T, K), generator=g).to(dtype)
    w = torch.randn((E * N, K), generator=g).to(dtype)
    tpe = (T * k) // E
    offs = torch.tensor([0] + [min((i + 1) * tpe, T) for i in range(E - 1)] + [T], dtype=torch.int32)
    out = _ops.moe_segment_gemm(hs.to(cuda_dev), w.to(cuda_dev), offs.to(cuda_dev), E, N, K)
    torch.cuda.synchronize()
    ref = og.segment_gemm_ref(hs, w, offs, N, K)
    assert og.max_rel_err(out, ref) <= TOL


@pytest.mark.parametrize("T", [1, 2, 4, 16])
def test_packed_ksplit(cuda_dev, T):
    """Decode-sized packed GEMMs split K on the device (the split shows in
    the workspace header) and agree with the unsplit kernels and the oracle."""
    from elastikernel_b200 import _ops
    from elastikernel_b200._lib import lib

    H, I, E, k = 2048, 1024, 8, 2
    x, logits, w1, w2, w3 = _moe_inputs(T, H, I, E, seed=T + 70)
    x, logits = x.to(cuda_dev), logits.to(cuda_dev)
    w1, w2, w3 = w1.to(cuda_dev), w2.to(cuda_dev), w3.to(cuda_dev)
    ids, wts = _ops.moe_route(logits, k)
    perm = _ops.moe_permute(ids, E, x=x, block_m=1)
    rows = perm["max_rows"]
    nb = int(lib().ek_moe_packed_workspace_bytes(rows, H, I))
    assert nb > 0
    ws = torch.full((nb,), 0, dtype=torch.uint8, device=cuda_dev)
    act = torch.empty((rows, I), dtype=torch.bfloat16, device=cuda_dev)
    assert lib().ek_moe_gate_up_packed(perm["x_perm"].data_ptr(), w1.data_ptr(), w3.data_ptr(),
                                       perm["expert_counts"].data_ptr(), act.data_ptr(), rows, E, H, I, 0, -1, 0,
                                       ws.data_ptr(), nb, _ops.current_stream_handle(cuda_dev)) == 0
    split_gu = int(ws[:4].view(torch.int32).item())
    act_ref = _ops.moe_gate_up_packed(perm, w1, w3, ksplit=False)
    y = _ops.moe_down_packed(perm, act, w2, wts)
    y_ref = _ops.moe_down_packed(perm, act, w2, wts, ksplit=False)
    torch.cuda.synchronize()
    if T == 1:
        assert split_gu > 1, "T=1: the gate/up GEMM did not split K"
    assert og.max_rel_err(act, act_ref.float().cpu().numpy()) <= 1e-2
    assert og.max_rel_err(y, y_ref.float().cpu().numpy()) <= 1e-2
    out = _ops.moe_combine(y, T, k)
    ref = om.moe_ref(x.cpu(), logits.cpu(), w1.cpu(), w2.cpu(), w3.cpu(), k)
    assert og.max_rel_err(out, ref) <= TOL


@pytest.mark.parametrize("T,H,I,E,k", [(300, 256, 512, 8, 2), (1024, 512, 768, 8, 2), (64, 256, 256, 16, 4),
                                       (1, 256, 512, 8, 2)])
def test_padded_pair_tiles(cuda_dev, T, H, I, E, k):
    """The layout padded to 256 rows per expert runs the gate/up and down
    GEMMs on CTA pairs; the layer matches the oracle and the 128-row path."""
    from elastikernel_b200 import _ops

    x, logits, w1, w2, w3 = _moe_inputs(T, H, I, E, seed=T + H + 5)
    x, logits = x.to(cuda_dev), logits.to(cuda_dev)
    w1, w2, w3 = w1.to(cuda_dev), w2.to(cuda_dev), w3.to(cuda_dev)
    ids, wts = _ops.moe_route(logits, k)
    outs = []
    for bm in (256, 128):
        perm = _ops.moe_permute(ids, E, x=x, block_m=bm)
        act = _ops.moe_gate_up(perm, w1, w3)
        y = _ops.moe_down(perm, act, w2, wts)
        outs.append(_ops.moe_combine(y, T, k))
    torch.cuda.synchronize()
    ref = om.moe_ref(x.cpu(), logits.cpu(), w1.cpu(), w2.cpu(), w3.cpu(), k)
    assert og.max_rel_err(outs[0], ref) <= TOL
    assert og.max_rel_err(outs[0], outs[1].float().cpu().numpy()) <= TOL
