"""Cluster split-K GEMM on the GPU (ek_gemm_csplit.cuh): the K range of each
128 x bn output tile split over the CTAs of one thread-block cluster and the
fp32 partials summed through distributed shared memory.

Against the oracle's fp32 product of the same inputs, with the dense GEMM's
tolerances: max|C - ref| / max|ref| <= 1e-2 for bf16 / fp16 and 3e-2 for the
scaled e4m3 GEMM. The split is offered on the full device only, so every case
runs with num_sms = the device's SM count.
"""
from __future__ import annotations

import pytest
import torch

from oracle.gemm import gemm_fp8_ref, gemm_ref, max_rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-2
TOL_FP8 = 3e-2


def _full_sms(dev) -> int:
    return torch.cuda.get_device_properties(dev).multi_processor_count


def _inputs(M, N, K, dtype, layout, dev, seed=0):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn((M, K), generator=g).to(dtype)
    b = torch.randn((K, N) if layout == "kn" else (N, K), generator=g).to(dtype)
    return a, b, a.to(dev), b.to(dev)


@pytest.mark.parametrize("cs", [2, 4, 8])
@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("layout", ["kn", "nk"])
def test_cluster_split_forced(cuda_dev, cs, bn, layout):
    """Every cluster size and tile width, both B layouts; ragged M, N and K
    (the last K block is partly past K and read as zeros)."""
    from elastikernel_b200 import _ops

    M, N, K = 200, 520, 2000
    S = _full_sms(cuda_dev)
    a, b, da, db = _inputs(M, N, K, torch.bfloat16, layout, cuda_dev, seed=cs * 10 + bn)
    p = _ops.plan(M, N, K, S, torch.bfloat16, layout, bn, -cs)
    assert p["cluster_split"] == cs and p["bn"] == bn and p["workspace_bytes"] == 0
    assert p["grid"] == p["num_tiles"] * cs
    c = _ops.gemm(da, db, num_sms=S, b_layout=layout, force_bn=bn, force_split=-cs)
    torch.cuda.synchronize()
    err = max_rel_err(c, gemm_ref(a, b, layout))
    assert err <= TOL, f"cs={cs} bn={bn} {layout}: {err:.3e}"


@pytest.mark.parametrize("csp", [2, 4])
@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("layout", ["kn", "nk"])
def test_cluster_split_pairs_forced(cuda_dev, csp, bn, layout):
    """CTA-pair tiles (256 x bn, 2-SM MMA) split over csp pairs of one
    cluster; ragged M, N and K."""
    from elastikernel_b200 import _ops

    M, N, K = 500, 520, 2000
    S = _full_sms(cuda_dev)
    a, b, da, db = _inputs(M, N, K, torch.bfloat16, layout, cuda_dev, seed=csp * 7 + bn)
    p = _ops.plan(M, N, K, S, torch.bfloat16, layout, -bn, -csp)
    assert p["cluster_split"] == csp and p["cta_pair"] == 1 and p["bm"] == 256 and p["bn"] == bn
    assert p["grid"] == p["num_tiles"] * csp * 2 and p["workspace_bytes"] == 0
    c = _ops.gemm(da, db, num_sms=S, b_layout=layout, force_bn=-bn, force_split=-csp)
    torch.cuda.synchronize()
    err = max_rel_err(c, gemm_ref(a, b, layout))
    assert err <= TOL, f"pairs csp={csp} bn={bn} {layout}: {err:.3e}"


@pytest.mark.parametrize("M", [1, 77, 128, 256, 512])
def test_small_m_default_plan(cuda_dev, M):
    """The M-sweep shapes N = K = 4096 at small M: the planner's choice (a
    cluster split where the device holds it), against the oracle, and
    bit-identical over two calls (the slice sum order is fixed)."""
    from elastikernel_b200 import _ops

    N = K = 4096
    S = _full_sms(cuda_dev)
    a, b, da, db = _inputs(M, N, K, torch.bfloat16, "kn", cuda_dev, seed=M)
    p = _ops.plan(M, N, K, S, torch.bfloat16, "kn")
    c1 = _ops.gemm(da, db, num_sms=S)
    c2 = _ops.gemm(da, db, num_sms=S)
    torch.cuda.synchronize()
    err = max_rel_err(c1, gemm_ref(a, b))
    assert err <= TOL, f"M={M} plan {p}: {err:.3e}"
    assert torch.equal(c1, c2)


def test_cluster_split_fp16(cuda_dev):
    from elastikernel_b200 import _ops

    M, N, K = 128, 1024, 4096
    S = _full_sms(cuda_dev)
    a, b, da, db = _inputs(M, N, K, torch.float16, "nk", cuda_dev, seed=5)
    c = _ops.gemm(da, db, num_sms=S, b_layout="nk", force_bn=256, force_split=-4)
    torch.cuda.synchronize()
    assert max_rel_err(c, gemm_ref(a, b, "nk")) <= TOL


@pytest.mark.parametrize("cs,bn", [(2, 256), (8, 256), (2, -256)])
def test_cluster_split_fp8_scaled(cuda_dev, cs, bn):
    """e4m3 operands with per-row / per-channel scales applied after the
    cluster's reduction."""
    from elastikernel_b200 import _ops

    M, N, K = 96, 1024, 4096
    S = _full_sms(cuda_dev)
    g = torch.Generator().manual_seed(cs)
    a = torch.randn((M, K), generator=g)
    w = torch.randn((N, K), generator=g)
    aq, a_s = _ops.quant_e4m3(a.to(cuda_dev))
    wq, w_s = _ops.quant_e4m3(w.to(cuda_dev))
    ref = gemm_fp8_ref(aq.cpu(), wq.cpu(), a_s.cpu(), w_s.cpu())
    c = _ops.gemm_fp8(aq, wq, a_s, w_s, num_sms=S, force_bn=bn, force_split=-cs)
    torch.cuda.synchronize()
    assert max_rel_err(c, ref) <= TOL_FP8


def test_cluster_split_not_offered_on_partitions(cuda_dev):
    """A partition smaller than the device gets the persistent schedule."""
    from elastikernel_b200 import _ops

    p = _ops.plan(128, 4096, 4096, 96, torch.bfloat16, "kn")
    assert p["cluster_split"] == 0
    with pytest.raises(RuntimeError):
        _ops.plan(128, 4096, 4096, 96, torch.bfloat16, "kn", 256, -4)
