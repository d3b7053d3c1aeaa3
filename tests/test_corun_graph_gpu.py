"""Partition co-run harness and the graph-captured SM-aware GEMM on the GPU.

* corun: the GEMM and the MoE layer run at once in disjoint partitions (plus
  a copy stressor); every output equals its solo run bit for bit (the kernels
  are deterministic for a given partition size), and the reported slow-downs
  are finite and positive.
* GraphMatmul: a CUDA graph captured on a partition stream replays the same
  product as the eager call (bit-exact) and follows new operand values.
"""
from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_corun_gemm_moe_stressor(cuda_dev):
    from elastikernel_b200 import corun

    r = corun.corun(gemm_sms=64, moe_sms=64, moe_tokens=64, size=2048, iters=3, stressor_sms=16, stressor_mb=256,
                    verbose=False)
    assert r["outputs_equal"]
    assert r["sms"]["gemm"] >= 64 and r["sms"]["moe"] >= 64
    for name in ("gemm", "moe", "stressor"):
        assert math.isfinite(r[name]["slowdown"]) and r[name]["slowdown"] > 0


def test_graph_matmul_matches_eager(cuda_dev):
    from elastikernel_b200 import sm_aware_matmul as smm
    from elastikernel_b200.green_ctx import create_sm_partition

    stream, sms = create_sm_partition(cuda_dev, 32)
    g = torch.Generator(device=cuda_dev).manual_seed(3)
    a = torch.randn((1024, 2048), device=cuda_dev, generator=g).to(torch.bfloat16)
    b = torch.randn((2048, 768), device=cuda_dev, generator=g).to(torch.bfloat16)
    gm = smm.GraphMatmul(a, b, stream=stream)
    with torch.cuda.stream(stream):
        eager = smm.call_sm_aware(a, b)
    out = gm()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    a.copy_(torch.randn((1024, 2048), device=cuda_dev, generator=g).to(torch.bfloat16))
    out2 = gm()
    with torch.cuda.stream(stream):
        eager2 = smm.call_sm_aware(a, b)
    torch.cuda.synchronize()
    assert torch.equal(out2, eager2) and not torch.equal(eager2, eager)


@pytest.mark.parametrize("layout", ["packed", "padded"])
def test_captured_moe_layer_matches_eager(cuda_dev, layout):
    """The whole fused MoE layer captures as one CUDA graph (no host reads of
    device data) and replays bit-exactly; new inputs copied in place are used."""
    from elastikernel_b200 import _ops
    from elastikernel_b200.graph import Captured

    T, H, I, E, k = 16, 512, 256, 8, 2
    g = torch.Generator(device=cuda_dev).manual_seed(5)
    x = torch.randn((T, H), device=cuda_dev, generator=g).to(torch.bfloat16)
    logits = torch.randn((T, E), device=cuda_dev, generator=g)
    w1 = (torch.randn((E, I, H), device=cuda_dev, generator=g) * 0.05).to(torch.bfloat16)
    w3 = (torch.randn((E, I, H), device=cuda_dev, generator=g) * 0.05).to(torch.bfloat16)
    w2 = (torch.randn((E, H, I), device=cuda_dev, generator=g) * 0.05).to(torch.bfloat16)
    y = torch.empty((T, H), device=cuda_dev, dtype=torch.bfloat16)
    cap = Captured(lambda: _ops.fused_moe(x, logits, w1, w2, w3, k, out=y, layout=layout))
    out = cap()
    eager = _ops.fused_moe(x, logits, w1, w2, w3, k, layout=layout)
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    logits.copy_(torch.randn((T, E), device=cuda_dev, generator=g))
    out2 = cap().clone()
    eager2 = _ops.fused_moe(x, logits, w1, w2, w3, k, layout=layout)
    torch.cuda.synchronize()
    assert torch.equal(out2, eager2)
