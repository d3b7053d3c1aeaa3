"""FP8 e4m3 MoE GEMMs with the scales applied by the tensor cores
(ek_moe_gate_up_fp8mx / ek_moe_down_fp8mx, tcgen05.mma kind::mxf8f6f4.block_scale).

The scales are powers of two (amax / 448 rounded up), so they are exact UE8M0
scale factors. Checks:
* power-of-two quantisation is bit-exact against the oracle (codes and scales);
* every token tile, on one CTA and on a CTA pair, against the epilogue-scaled
  kernel (ek_moe_*_fp8bs) on the same quantised inputs, which computes the
  same sums in another order (1e-2), and against the oracle's fp32 MoE on the
  dequantised inputs with its SwiGLU activations rounded to e4m3 as the layer
  rounds them (1e-2). At these small shapes (K of 256 and 512) that rounding
  alone moves the output by up to 3 % of its largest value: a power-of-two
  scale leaves a group's largest value to be rounded too, where an fp32 scale
  maps it exactly onto 448;
* the fused layer at DeepSeek-V3 expert shapes against the plain fp32 oracle
  (FP8 tolerance 3e-2);
* a scale that is not a power of two is reported in the device status word.
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
TOL = 1e-2


def _dequant_weights(qw):
    E, I, H = qw["E"], qw["I"], qw["H"]
    w1 = of8.dequant_blocks(qw["w1q"].cpu().view(E * I, H), qw["w1s"].cpu().numpy(), 128, 128).reshape(E, I, H)
    w3 = of8.dequant_blocks(qw["w3q"].cpu().view(E * I, H), qw["w3s"].cpu().numpy(), 128, 128).reshape(E, I, H)
    w2 = of8.dequant_blocks(qw["w2q"].cpu().view(E * H, I), qw["w2s"].cpu().numpy(), 128, 128).reshape(E, H, I)
    return w1, w2, w3


def _block_factors(g, rows, cols, br, bc, lo, hi):
    """A power of two per br x bc block (2^lo .. 2^hi), expanded to [rows, cols]:
    with plain N(0, s) data neighbouring blocks round to the same power-of-two
    scale, so a scale factor read for the wrong row block or token would go
    unnoticed; these factors give every block its own scale."""
    e = torch.randint(lo, hi + 1, (-(-rows // br), -(-cols // bc)), generator=g).to(torch.float32)
    f = torch.pow(2.0, e)
    return f.repeat_interleave(br, 0).repeat_interleave(bc, 1)[:rows, :cols]


def _setup(T, H, I, E, seed, dev):
    from elastikernel_b200 import _ops

    g = torch.Generator().manual_seed(seed)
    x = (torch.randn((T, H), generator=g) * _block_factors(g, T, H, 1, 128, -2, 2)).to(torch.bfloat16)
    logits = torch.randn((T, E), generator=g)
    w1 = torch.randn((E, I, H), generator=g) * 0.02 * _block_factors(g, E * I, H, 128, 128, -3, 3).view(E, I, H)
    w2 = torch.randn((E, H, I), generator=g) * 0.02 * _block_factors(g, E * H, I, 128, 128, -3, 3).view(E, H, I)
    w3 = torch.randn((E, I, H), generator=g) * 0.02 * _block_factors(g, E * I, H, 128, 128, -3, 3).view(E, I, H)
    qw = _ops.quant_moe_weights_fp8(w1.to(dev), w2.to(dev), w3.to(dev), pow2=True)
    return x, logits, qw


def test_pow2_quantisation_matches_oracle(cuda_dev):
    from elastikernel_b200 import _ops

    g = torch.Generator().manual_seed(21)
    x = (torch.randn((300, 640), generator=g) * 5).to(torch.bfloat16)
    x[7] = 0  # an all-zero row / group: scale 1
    dx = x.to(cuda_dev)
    for block, ref in (((1, 0), lambda: of8.quant_rows(x, pow2=True)),
                       ((1, 128), lambda: of8.quant_blocks(x, 1, 128, pow2=True)),
                       ((128, 128), lambda: of8.quant_blocks(x, 128, 128, pow2=True))):
        q, s = _ops.quant_e4m3(dx, block=block, pow2=True)
        rq, rs = ref()
        np.testing.assert_array_equal(s.cpu().numpy().reshape(rs.shape), rs)
        assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8)), block
        sb = s.cpu().numpy().view(np.uint32)
        assert not (sb & 0x007FFFFF).any()  # powers of two
    qk, sk = _ops.quant_e4m3_kmajor(dx, pow2=True)
    q1, s1 = _ops.quant_e4m3(dx, block=(1, 128), pow2=True)
    assert torch.equal(qk.view(torch.uint8), q1.view(torch.uint8)) and torch.equal(sk, s1.t().contiguous())


@pytest.mark.parametrize("tok,pair,E", [(16, 0, 16), (32, 0, 16), (64, 0, 16), (128, 0, 16), (128, 0, 4),
                                        (128, 1, 16), (128, 1, 4), (160, 1, 16), (160, 1, 4), (192, 1, 16),
                                        (192, 1, 4), (128, 2, 16), (160, 2, 4), (192, 2, 16), (192, 2, 4)])
def test_fp8mx_gemms_token_tiles(cuda_dev, tok, pair, E):
    """Every token tile; E=4 puts ~300 tokens on each expert, so every expert
    spans several token tiles. pair=2: the wide pair tiles (256 weight rows
    per CTA, two accumulators), against the epilogue-scaled kernel's pair
    tile and the oracle."""
    from elastikernel_b200 import _ops

    T, H, I, k = 300, 512, 256, 4
    x, logits, qw = _setup(T, H, I, E, seed=tok + pair, dev=cuda_dev)
    ids, wts = _ops.moe_route(logits.to(cuda_dev), k)
    perm = _ops.moe_permute(ids, E, x=x.to(cuda_dev), block_m=1)
    xq, xs = _ops.quant_e4m3_kmajor(perm["x_perm"], pow2=True)
    outs = {}
    for mx in (True, False):
        pr = pair if mx else min(pair, 1)
        act = _ops.moe_gate_up_fp8bs(perm, xq, xs, qw, tok_tile=tok, pair=pr, mx=mx)
        aq, as_ = _ops.quant_e4m3_kmajor(act, pow2=True)
        y = _ops.moe_down_fp8bs(perm, aq, as_, qw, wts, tok_tile=tok, pair=pr, mx=mx)
        outs[mx] = (act, _ops.moe_combine(y, T, k))
    torch.cuda.synchronize()
    # the two kernels on the same quantised inputs: the same math, another summation order
    a_err = og.max_rel_err(outs[True][0], outs[False][0].float().cpu().numpy())
    assert a_err <= TOL, f"act, tensor-core vs epilogue scaling: {a_err:.3e}"
    w1, w2, w3 = _dequant_weights(qw)
    xd = of8.dequant_blocks(*of8.quant_blocks(x, 1, 128, pow2=True), 1, 128)
    ids_r, wts_r = om.route_ref(logits.numpy(), k)

    def act_q(a):  # bf16 activations rounded to e4m3 with power-of-two 1 x 128 scales, as the layer does
        return of8.dequant_blocks(*of8.quant_blocks(torch.from_numpy(a).to(torch.bfloat16), 1, 128, pow2=True),
                                  1, 128)

    _, ref_q = om.moe_ref_by_expert(xd, ids_r, wts_r, E, lambda e: (w1[e], w2[e], w3[e]), act_quant=act_q)
    err = og.max_rel_err(outs[True][1], ref_q)
    assert err <= TOL, f"tok={tok} pair={pair} E={E}: {err:.3e}"


@pytest.mark.parametrize("T", [64, 512])
def test_fused_moe_fp8mx_dsv3_expert_shapes(cuda_dev, T):
    """DeepSeek-V3 expert shapes (H=7168, I=2048, top-8) on a 16-expert shard."""
    from elastikernel_b200 import _ops

    H, I, E, k = 7168, 2048, 16, 8
    x, logits, qw = _setup(T, H, I, E, seed=T, dev=cuda_dev)
    out = _ops.fused_moe_fp8(x.to(cuda_dev), logits.to(cuda_dev), qw, k)
    torch.cuda.synchronize()
    w1, w2, w3 = _dequant_weights(qw)
    xd = of8.dequant_blocks(*of8.quant_blocks(x, 1, 128, pow2=True), 1, 128)
    ref = om.moe_ref(xd, logits, w1, w2, w3, k)
    assert og.max_rel_err(out, ref) <= TOL_FP8


def test_non_power_of_two_scale_is_reported(cuda_dev):
    """fp32 (non power-of-two) scales given to the tensor-core-scaled GEMM:
    the kernel flags EK_STATUS_BAD_SCALE (its result is then invalid)."""
    from elastikernel_b200 import _lib, _ops

    T, H, I, E, k = 64, 256, 256, 4, 2
    x, logits, qw = _setup(T, H, I, E, seed=3, dev=cuda_dev)
    ids, _ = _ops.moe_route(logits.to(cuda_dev), k)
    perm = _ops.moe_permute(ids, E, x=x.to(cuda_dev), block_m=1)
    xq, xs = _ops.quant_e4m3_kmajor(perm["x_perm"])  # fp32 scales: not powers of two
    _ops.moe_gate_up_fp8bs(perm, xq, xs * 1.5, qw, mx=True)
    st = _lib.device_status(0, clear=True)
    assert st & _lib.EK_STATUS_BAD_SCALE
    assert not st & ~_lib.EK_STATUS_BAD_SCALE
