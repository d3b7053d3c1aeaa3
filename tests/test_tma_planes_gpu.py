"""The gate/up GEMMs load a tile's [w1 rows | w3 rows] with one 3-D TMA box
when w3 lies a fixed positive distance after w1 (two planes of one buffer),
and with two 2-D boxes otherwise. Both paths put the same bytes in shared
memory, so their results must be bit-identical: checked here for the bf16
packed (swapped) and padded GEMMs and for both FP8 kernels, and the plane
path against the oracle."""
from __future__ import annotations

import pytest
import torch

from oracle import gemm as og
from oracle import moe as om

pytestmark = pytest.mark.gpu


def _two_layouts(w1: torch.Tensor, w3: torch.Tensor):
    """(w1, w3) as planes of one buffer (w3 after w1) and as two halves of a
    buffer with w3 first, which rules the one-box path out."""
    planes = torch.stack([w1, w3])
    buf = torch.empty((2,) + tuple(w1.shape), dtype=w1.dtype, device=w1.device)
    buf[0].copy_(w3)
    buf[1].copy_(w1)
    return (planes[0], planes[1]), (buf[1], buf[0])


@pytest.mark.parametrize("layout,tok,pair", [("packed", 64, 0), ("packed", 128, 1), ("packed", 256, 1),
                                             ("padded", 0, 0)])
def test_bf16_gate_up_one_box_equals_two(cuda_dev, layout, tok, pair):
    from elastikernel_b200 import _ops

    T, H, I, E, k = 400, 512, 384, 8, 2
    g = torch.Generator().manual_seed(tok + pair)
    x = torch.randn((T, H), generator=g).to(torch.bfloat16).to(cuda_dev)
    logits = torch.randn((T, E), generator=g).to(cuda_dev)
    w1 = (torch.randn((E, I, H), generator=g) * 0.02).to(torch.bfloat16).to(cuda_dev)
    w3 = (torch.randn((E, I, H), generator=g) * 0.02).to(torch.bfloat16).to(cuda_dev)
    ids, _ = _ops.moe_route(logits, k)
    outs = []
    for a1, a3 in _two_layouts(w1, w3):
        if layout == "packed":
            perm = _ops.moe_permute(ids, E, x=x, block_m=1)
            outs.append(_ops.moe_gate_up_packed(perm, a1, a3, tok_tile=tok, pair=pair, ksplit=False))
        else:
            perm = _ops.moe_permute(ids, E, x=x, block_m=128)
            outs.append(_ops.moe_gate_up(perm, a1, a3))
    torch.cuda.synchronize()
    # rows that hold a routed slot (the padded layout's padding rows are never
    # gathered, so their products are whatever the buffer held)
    valid = perm["sorted_slots"] < T * k
    assert torch.equal(outs[0][valid], outs[1][valid])


@pytest.mark.parametrize("mx", [False, True])
@pytest.mark.parametrize("tok,pair", [(64, 0), (160, 1)])
def test_fp8_gate_up_one_box_equals_two(cuda_dev, mx, tok, pair):
    from elastikernel_b200 import _ops

    T, H, I, E, k = 300, 512, 256, 4, 4
    g = torch.Generator().manual_seed(7 + tok)
    x = torch.randn((T, H), generator=g).to(torch.bfloat16).to(cuda_dev)
    logits = torch.randn((T, E), generator=g).to(cuda_dev)
    w1 = torch.randn((E, I, H), generator=g).to(cuda_dev) * 0.02
    w2 = torch.randn((E, H, I), generator=g).to(cuda_dev) * 0.02
    w3 = torch.randn((E, I, H), generator=g).to(cuda_dev) * 0.02
    qw = _ops.quant_moe_weights_fp8(w1, w2, w3, pow2=mx)
    ids, _ = _ops.moe_route(logits, k)
    perm = _ops.moe_permute(ids, E, x=x, block_m=1)
    xq, xs = _ops.quant_e4m3_kmajor(perm["x_perm"], pow2=mx)
    outs = []
    for a1, a3 in _two_layouts(qw["w1q"], qw["w3q"]):
        q = dict(qw, w1q=a1, w3q=a3)
        outs.append(_ops.moe_gate_up_fp8bs(perm, xq, xs, q, tok_tile=tok, pair=pair))
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


def test_stacked_planes_fused_layer_matches_oracle(cuda_dev):
    """The fused bf16 layer on stacked [2, E, I, H] gate/up weights (the
    bench's layout) against the oracle."""
    from elastikernel_b200 import _ops

    T, H, I, E, k = 256, 512, 1024, 8, 2
    g = torch.Generator().manual_seed(3)
    x = torch.randn((T, H), generator=g).to(torch.bfloat16)
    logits = torch.randn((T, E), generator=g)
    w13 = (torch.randn((2, E, I, H), generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn((E, H, I), generator=g) * 0.02).to(torch.bfloat16)
    d13 = w13.to(cuda_dev)
    for layout in ("packed", "padded"):
        out = _ops.fused_moe(x.to(cuda_dev), logits.to(cuda_dev), d13[0], w2.to(cuda_dev), d13[1], k, layout=layout)
        torch.cuda.synchronize()
        assert og.max_rel_err(out, om.moe_ref(x, logits, w13[0], w2, w13[1], k)) <= 1e-2
