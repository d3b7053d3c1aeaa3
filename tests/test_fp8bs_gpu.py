"""FP8 e4m3 block-scaled MoE (DeepSeek-V3-shaped experts) on the GPU.

Weights carry 128 x 128 fp32 block scales, activations 1 x 128 group scales.
Tolerance (FP8): max|out - ref| / max|ref| <= 3e-2 against the oracle's fp32
MoE computed from the dequantised weights and the dequantised (gathered)
activations of the same quantisation, as the hot-path spec states for FP8.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import fp8 as of8
from oracle import gemm as og
from oracle import moe as om

pytestmark = pytest.mark.gpu
TOL_FP8 = 3e-2


def _dequant_weights(qw):
    E, I, H = qw["E"], qw["I"], qw["H"]
    w1 = of8.dequant_blocks(qw["w1q"].cpu().view(E * I, H), qw["w1s"].cpu().numpy(), 128, 128).reshape(E, I, H)
    w3 = of8.dequant_blocks(qw["w3q"].cpu().view(E * I, H), qw["w3s"].cpu().numpy(), 128, 128).reshape(E, I, H)
    w2 = of8.dequant_blocks(qw["w2q"].cpu().view(E * H, I), qw["w2s"].cpu().numpy(), 128, 128).reshape(E, H, I)
    return w1, w2, w3


def _setup(T, H, I, E, seed, dev):
    from elastikernel_b200 import _ops

    g = torch.Generator().manual_seed(seed)
    x = torch.randn((T, H), generator=g).to(torch.bfloat16)
    logits = torch.randn((T, E), generator=g)
    w1 = torch.randn((E, I, H), generator=g) * 0.02
    w2 = torch.randn((E, H, I), generator=g) * 0.02
    w3 = torch.randn((E, I, H), generator=g) * 0.02
    qw = _ops.quant_moe_weights_fp8(w1.to(dev), w2.to(dev), w3.to(dev))
    return x, logits, qw


def test_weight_block_quant_matches_oracle(cuda_dev):
    from elastikernel_b200 import _ops

    g = torch.Generator().manual_seed(5)
    w = torch.randn((2, 256, 384), generator=g) * 0.02
    qw = _ops.quant_moe_weights_fp8(w.to(cuda_dev), w.transpose(1, 2).contiguous().to(cuda_dev), w.to(cuda_dev))
    rq, rs = of8.quant_blocks(w.reshape(512, 384), 128, 128)
    np.testing.assert_array_equal(qw["w1s"].cpu().numpy(), rs)
    assert torch.equal(qw["w1q"].cpu().view(torch.uint8).reshape(512, 384), rq.view(torch.uint8))


def test_kmajor_quant_and_scale_gather(cuda_dev):
    """K-block-major group scales are the transpose of the row-major ones, bit
    for bit, and the transposing gather reorders them like the row gather."""
    from elastikernel_b200 import _ops

    g = torch.Generator().manual_seed(11)
    x = (torch.randn((333, 640), generator=g) * 3).to(torch.bfloat16).to(cuda_dev)
    q0, s0 = _ops.quant_e4m3(x, block=(1, 128))
    q1, s1 = _ops.quant_e4m3_kmajor(x)
    assert torch.equal(q0.view(torch.uint8), q1.view(torch.uint8))
    assert torch.equal(s0.t().contiguous(), s1)
    ids, _ = _ops.moe_route(torch.randn((333, 8), generator=g).to(cuda_dev), 2)
    perm = _ops.moe_permute(ids, 8, x=x, block_m=1)
    st = _ops.moe_gather_cols_f32(perm, s0)
    slots = perm["sorted_slots"].cpu()
    ref = torch.zeros_like(st.cpu())
    used = slots >= 0
    ref[:, used] = s0.cpu()[slots[used] // 2].t()
    assert torch.equal(st.cpu(), ref)


@pytest.mark.parametrize("tok,pair,E", [(16, 0, 16), (32, 0, 16), (64, 0, 16), (128, 0, 16), (128, 0, 4),
                                        (128, 1, 16), (128, 1, 4), (160, 1, 16), (160, 1, 4), (192, 1, 16),
                                        (192, 1, 4), (256, 1, 16),
                                        (256, 1, 4)])
def test_fp8bs_gemms_token_tiles(cuda_dev, tok, pair, E):
    """Every token tile on one CTA and on a CTA pair; E=4 puts ~300 tokens on
    each expert so every expert spans several token tiles."""
    from elastikernel_b200 import _ops

    T, H, I, k = 300, 512, 256, 4
    x, logits, qw = _setup(T, H, I, E, seed=tok + pair, dev=cuda_dev)
    ids, wts = _ops.moe_route(logits.to(cuda_dev), k)
    perm = _ops.moe_permute(ids, E, x=x.to(cuda_dev), block_m=1)
    xq, xs = _ops.quant_e4m3_kmajor(perm["x_perm"])
    act = _ops.moe_gate_up_fp8bs(perm, xq, xs, qw, tok_tile=tok, pair=pair)
    aq, as_ = _ops.quant_e4m3_kmajor(act)
    y = _ops.moe_down_fp8bs(perm, aq, as_, qw, wts, tok_tile=tok, pair=pair)
    out = _ops.moe_combine(y, T, k)
    torch.cuda.synchronize()
    w1, w2, w3 = _dequant_weights(qw)
    xd = of8.dequant_blocks(*of8.quant_blocks(x, 1, 128), 1, 128)  # tokens quantised the same way
    ref = om.moe_ref(xd, logits, w1, w2, w3, k)
    err = og.max_rel_err(out, ref)
    assert err <= TOL_FP8, f"tok={tok} pair={pair} E={E}: {err:.3e}"


@pytest.mark.parametrize("T", [64, 512])
def test_fused_moe_fp8_dsv3_expert_shapes(cuda_dev, T):
    """DeepSeek-V3 expert shapes (H=7168, I=2048, top-8) on a 16-expert shard."""
    from elastikernel_b200 import _ops

    H, I, E, k = 7168, 2048, 16, 8
    x, logits, qw = _setup(T, H, I, E, seed=T, dev=cuda_dev)
    out = _ops.fused_moe_fp8(x.to(cuda_dev), logits.to(cuda_dev), qw, k)
    torch.cuda.synchronize()
    w1, w2, w3 = _dequant_weights(qw)
    xd = of8.dequant_blocks(*of8.quant_blocks(x, 1, 128), 1, 128)
    ref = om.moe_ref(xd, logits, w1, w2, w3, k)
    assert og.max_rel_err(out, ref) <= TOL_FP8
