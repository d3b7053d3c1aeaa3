"""Green-context partitions on the GPU: the shim's real-driver path, grid
sizing from the stream registry, isolation of disjoint partitions
(verify_isolation.py's method on the tcgen05 GEMM), and the reference-shaped
benchmark drivers running end to end on a small subset."""
from __future__ import annotations

import pytest
import torch

from oracle.gemm import gemm_ref, max_rel_err

pytestmark = pytest.mark.gpu


def _ab(M, N, K, dev, seed=0):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn((M, K), generator=g).to(torch.bfloat16)
    b = torch.randn((K, N), generator=g).to(torch.bfloat16)
    return a, b, a.to(dev), b.to(dev)


def test_alignment_and_total(cuda_dev):
    from elastikernel_b200 import green_ctx

    assert green_ctx.get_total_sm_count(cuda_dev) == torch.cuda.get_device_properties(cuda_dev).multi_processor_count
    assert green_ctx.get_sm_alignment(cuda_dev) == (8, 8)  # CC 10.0
    with pytest.raises(ValueError):
        green_ctx.create_sm_partition(cuda_dev, 148)  # rounds to 152 > 148, as the reference


def test_partition_runs_gemm_sized_from_registry(cuda_dev):
    from elastikernel_b200 import green_ctx, sm_aware_matmul as smm

    stream, actual = green_ctx.create_sm_partition(cuda_dev, 16)
    assert actual >= 16 and actual % 8 == 0
    assert green_ctx.stream_sm_count(stream) == actual
    a, b, da, db = _ab(1024, 2048, 1024, cuda_dev)
    with torch.cuda.stream(stream):
        c = smm.call_sm_aware(da, db)  # num_sms taken from the partition
    stream.synchronize()
    assert max_rel_err(c, gemm_ref(a, b)) <= 1e-2


def test_disjoint_partitions(cuda_dev):
    from elastikernel_b200 import green_ctx, sm_aware_matmul as smm

    parts = green_ctx.create_disjoint_partitions(cuda_dev, [32, 112])
    assert [p[1] for p in parts] == [32, 112]
    a, b, da, db = _ab(777, 1032, 512, cuda_dev, seed=1)
    ref = gemm_ref(a, b)
    outs = []
    for s, n in parts:
        with torch.cuda.stream(s):
            outs.append(smm.call_sm_aware(da, db))
    torch.cuda.synchronize()
    for o in outs:
        assert max_rel_err(o, ref) <= 1e-2


def test_verify_isolation(cuda_dev):
    from elastikernel_b200 import verify_isolation

    r = verify_isolation.main(size=4096, iters=10)
    assert max(r["max_rel_err"]) <= 1e-2
    assert r["speedup_disjoint"] > 1.4, r


def test_benchmark_drivers_small(cuda_dev):
    from elastikernel_b200 import sm_aware_benchmark as smb, sm_aware_matmul as smm

    r = smm.run_benchmark(sm_levels=[16, 148], test_cases=[(512, 1024, 1024)], rep_ms=5)
    assert len(r) == 2 and all(x["max_rel_err"] <= 1e-2 for x in r)
    r = smb.run_gemm_benchmark(sm_levels=[32], test_cases=[(256, 1024, 1024)], rep_ms=5)
    assert len(r) == 1
    r = smb.run_moe_benchmark(sm_levels=[32], moe_configs=[{"num_tokens": 128, "hidden_dim": 1024,
                                                            "intermediate_dim": 1024, "num_experts": 8,
                                                            "top_k": 2}], rep_ms=5, full_layer=False)
    assert len(r) == 1


def test_segment_wrappers_match(cuda_dev):
    from elastikernel_b200 import sm_aware_benchmark as smb
    from oracle.gemm import segment_gemm_ref

    T, N, K, E = 300, 512, 512, 4
    g = torch.Generator().manual_seed(9)
    hs = torch.randn((T, K), generator=g).to(torch.float16)
    w = torch.randn((E * N, K), generator=g).to(torch.float16)
    offs = torch.tensor([0, 90, 90, 250, 300], dtype=torch.int32)
    ref = segment_gemm_ref(hs, w, offs, N, K)
    for out in (smb.call_moe_vanilla(hs.to(cuda_dev), w.to(cuda_dev), offs.to(cuda_dev), E, N, K),
                smb.call_moe_sm_aware(hs.to(cuda_dev), w.to(cuda_dev), offs.to(cuda_dev), E, N, K, 32)):
        torch.cuda.synchronize()
        assert out.dtype == torch.float16
        assert max_rel_err(out, ref) <= 1e-2
