"""Dense GEMM parity on the GPU: tcgen05 kernel (through the C-ABI) vs the CPU oracle.

Tolerance (bf16/fp16 in, fp32 accumulate, rounded output): max|C - ref| /
max|ref| <= 1e-2 against the oracle's fp32 product of the same inputs, the
bar the hot-path spec sets for bf16. Shapes cover the reference's square and
M-sweep cases (sm_aware_matmul.py:247-250) at sizes the oracle finishes in
seconds, ragged M/N/K tails, every tile width and forced K-splits of the tail
wave.
"""
from __future__ import annotations

import pytest
import torch

from oracle.gemm import gemm_ref, max_rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _inputs(M, N, K, dtype, layout, dev, seed=0):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn((M, K), generator=g).to(dtype)
    b = torch.randn((K, N) if layout == "kn" else (N, K), generator=g).to(dtype)
    return a, b, a.to(dev), b.to(dev)


@pytest.mark.parametrize("M,N,K", [(2048, 2048, 2048), (1, 4096, 4096), (16, 4096, 4096), (128, 4096, 4096),
                                   (1024, 1024, 1024), (300, 520, 784), (129, 136, 48)])
@pytest.mark.parametrize("layout", ["kn", "nk"])
def test_gemm_bf16_shapes(cuda_dev, M, N, K, layout):
    from elastikernel_b200 import _ops

    a, b, da, db = _inputs(M, N, K, torch.bfloat16, layout, cuda_dev)
    c = _ops.gemm(da, db, b_layout=layout)
    torch.cuda.synchronize()
    err = max_rel_err(c, gemm_ref(a, b, layout))
    assert err <= TOL, f"max rel err {err:.3e} for {M}x{N}x{K} {layout}"


@pytest.mark.parametrize("bn", [64, 128, 192, 256])
@pytest.mark.parametrize("split", [1, 2, 3])
def test_gemm_tiles_and_splits(cuda_dev, bn, split):
    from elastikernel_b200 import _ops

    M, N, K = 1000, 1032, 1536
    a, b, da, db = _inputs(M, N, K, torch.bfloat16, "kn", cuda_dev, seed=bn + split)
    ref = gemm_ref(a, b)
    # a small partition size forces a tail wave that the split applies to
    for sms in (16, 148):
        c = _ops.gemm(da, db, num_sms=sms, force_bn=bn, force_split=split)
        torch.cuda.synchronize()
        err = max_rel_err(c, ref)
        assert err <= TOL, f"bn={bn} split={split} sms={sms}: {err:.3e}"


@pytest.mark.parametrize("bn", [-128, -256])
@pytest.mark.parametrize("split", [1, 2, 3])
@pytest.mark.parametrize("layout", ["kn", "nk"])
def test_gemm_cta_pair_mode(cuda_dev, bn, split, layout):
    """2-SM MMA (CTA pair per 256 x |bn| tile), ragged shapes, split tails."""
    from elastikernel_b200 import _ops

    M, N, K = 1000, 1032, 1536
    a, b, da, db = _inputs(M, N, K, torch.bfloat16, layout, cuda_dev, seed=-bn + split)
    ref = gemm_ref(a, b, layout)
    for sms in (16, 148):
        p = _ops.plan(M, N, K, sms, torch.bfloat16, layout, bn, split)
        assert p["cta_pair"] == 1 and p["bm"] == 256
        c = _ops.gemm(da, db, num_sms=sms, b_layout=layout, force_bn=bn, force_split=split)
        torch.cuda.synchronize()
        err = max_rel_err(c, ref)
        assert err <= TOL, f"pair bn={-bn} split={split} sms={sms} {layout}: {err:.3e}"


def test_gemm_pair_vs_single_identical_math(cuda_dev):
    """Both MMA modes accumulate each output in the same K order: results match closely."""
    from elastikernel_b200 import _ops

    a, b, da, db = _inputs(2048, 2048, 2048, torch.bfloat16, "kn", cuda_dev, seed=3)
    c1 = _ops.gemm(da, db, force_bn=256, force_split=1)
    c2 = _ops.gemm(da, db, force_bn=-256, force_split=1)
    torch.cuda.synchronize()
    assert max_rel_err(c1, c2.float().cpu().numpy()) <= 1e-3


def test_gemm_fp16_reference_dtype(cuda_dev):
    """The reference benchmarks fp16 (sm_aware_matmul.py:263-264)."""
    from elastikernel_b200 import _ops

    a, b, da, db = _inputs(1024, 1024, 1024, torch.float16, "kn", cuda_dev)
    c = _ops.gemm(da, db)
    assert c.dtype == torch.float16
    torch.cuda.synchronize()
    assert max_rel_err(c, gemm_ref(a, b)) <= TOL


def test_gemm_split_deterministic_and_reusable(cuda_dev):
    """Split slices reduce in slice order: repeated calls are bit-identical,
    and the workspace tickets are returned to zero between calls."""
    from elastikernel_b200 import _ops

    a, b, da, db = _inputs(512, 4096, 4096, torch.bfloat16, "kn", cuda_dev, seed=7)
    outs = [_ops.gemm(da, db, num_sms=148, force_bn=128, force_split=4) for _ in range(3)]
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    assert max_rel_err(outs[0], gemm_ref(a, b)) <= TOL
