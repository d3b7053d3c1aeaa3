"""FP8 e4m3 path on the GPU: quantisation bit-exact against the oracle, and
the scaled e4m3 GEMM (BASELINE FP8 config: M=4096, N=14336, K=4096, per-row
activation and per-output-channel weight scales, bf16 out) within the FP8
tolerance max|C - ref| / max|ref| <= 3e-2 against the oracle's fp32 GEMM of
the dequantised operands."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import fp8 as of8
from oracle.gemm import gemm_fp8_ref, max_rel_err

pytestmark = pytest.mark.gpu
TOL_FP8 = 3e-2


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (77, 1000), (1, 128)])
def test_quant_rows_bit_exact(cuda_dev, dtype, rows, cols):
    from elastikernel_b200 import _ops

    g = torch.Generator().manual_seed(rows + cols)
    x = torch.randn((rows, cols), generator=g).to(dtype)
    x[0, :] = 0.0  # an all-zero row gets scale 1
    q, s = _ops.quant_e4m3(x.to(cuda_dev))
    rq, rs = of8.quant_rows(x)
    np.testing.assert_array_equal(s.cpu().numpy(), rs)
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))


@pytest.mark.parametrize("block", [(1, 128), (128, 128), (64, 32)])
@pytest.mark.parametrize("dtype,shape", [(torch.float32, (300, 520)), (torch.bfloat16, (300, 520)),
                                         (torch.float32, (130, 517))])
def test_quant_blocks_bit_exact(cuda_dev, block, dtype, shape):
    """Partial edge blocks; rows of a multiple of 8 elements take the vector
    kernels, 517 the element-wise ones."""
    from elastikernel_b200 import _ops

    g = torch.Generator().manual_seed(block[0] * 7 + block[1])
    x = (torch.randn(shape, generator=g) * 3.0).to(dtype)
    q, s = _ops.quant_e4m3(x.to(cuda_dev), block=block)
    rq, rs = of8.quant_blocks(x, *block)
    np.testing.assert_array_equal(s.cpu().numpy(), rs)
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))


@pytest.mark.parametrize("rows,cols", [(512, 7168), (257, 1032), (1, 2048), (3, 8)])
def test_quant_groups_wide_range(cuda_dev, rows, cols):
    """1 x 128 group quantisation over 60 decades of group magnitude, with
    subnormal elements and all-zero groups, row-major and K-block-major
    scales, bit for bit against the oracle."""
    from elastikernel_b200 import _ops

    g = torch.Generator().manual_seed(rows + cols)
    groups = -(-cols // 128)
    mag = torch.pow(10.0, torch.empty((rows, groups)).uniform_(-30, 30, generator=g))
    x = torch.randn((rows, groups * 128), generator=g) * mag.repeat_interleave(128, dim=1)
    x[torch.rand(x.shape, generator=g) < 0.01] = 1e-39  # subnormal elements
    x[:, :128][torch.rand(rows, generator=g) < 0.1] = 0.0  # all-zero first groups
    x = x[:, :cols].contiguous().to(torch.bfloat16)
    rq, rs = of8.quant_blocks(x, 1, 128)
    q, s = _ops.quant_e4m3(x.to(cuda_dev), block=(1, 128))
    np.testing.assert_array_equal(s.cpu().numpy(), rs)
    assert torch.equal(q.cpu().view(torch.uint8), rq.view(torch.uint8))
    qk, sk = _ops.quant_e4m3_kmajor(x.to(cuda_dev))
    np.testing.assert_array_equal(sk.cpu().numpy(), rs.T)
    assert torch.equal(qk.cpu().view(torch.uint8), rq.view(torch.uint8))


def _fp8_operands(M, N, K, dev, seed):
    from elastikernel_b200 import _ops

    g = torch.Generator(device=dev).manual_seed(seed)
    a = torch.randn((M, K), device=dev, generator=g)
    w = torch.randn((N, K), device=dev, generator=g)
    aq, a_s = _ops.quant_e4m3(a)
    wq, w_s = _ops.quant_e4m3(w)
    return aq, a_s, wq, w_s


def test_fp8_gemm_config_shape(cuda_dev):
    from elastikernel_b200 import _ops

    M, N, K = 4096, 14336, 4096
    aq, a_s, wq, w_s = _fp8_operands(M, N, K, cuda_dev, seed=3)
    ref = gemm_fp8_ref(aq.cpu(), wq.cpu(), a_s.cpu(), w_s.cpu())
    for sms in (148, 80):
        c = _ops.gemm_fp8(aq, wq, a_s, w_s, num_sms=sms)
        torch.cuda.synchronize()
        err = max_rel_err(c, ref)
        assert err <= TOL_FP8, f"sms={sms}: {err:.3e}"


@pytest.mark.parametrize("bn,split", [(64, 1), (128, 2), (192, 1), (256, 3), (-128, 2), (-256, 1), (-256, 3)])
def test_fp8_gemm_modes(cuda_dev, bn, split):
    from elastikernel_b200 import _ops

    M, N, K = 1000, 1032, 2048
    aq, a_s, wq, w_s = _fp8_operands(M, N, K, cuda_dev, seed=abs(bn) + split)
    ref = gemm_fp8_ref(aq.cpu(), wq.cpu(), a_s.cpu(), w_s.cpu())
    c = _ops.gemm_fp8(aq, wq, a_s, w_s, num_sms=16, force_bn=bn, force_split=split)
    torch.cuda.synchronize()
    assert max_rel_err(c, ref) <= TOL_FP8
