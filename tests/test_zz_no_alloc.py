"""GPU test of ek_gemm_noalloc, the GEMM entry point for callers that cannot
allocate device memory (hosts that own the whole device memory pool, or paths
where cudaMalloc/cudaFree would synchronise the device).

It is called through the C-ABI with raw pointers and checked against the
regular entry point ek_gemm (which takes a caller-allocated workspace) within
the GEMM tests' tolerance, for two calls in a row, on shapes whose schedule
uses the built-in scratch (split tail tiles) and on one that does not. This
file is named to be collected last, so a run that stops at the first failure
has already run every other test; it also passes alone in a fresh process.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from oracle.gemm import max_rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _noalloc(a, b, c, M, N, K, layout, sms, force_bn=0, force_split=0):
    from elastikernel_b200 import _lib

    bl = _lib.EK_B_KN if layout == "kn" else _lib.EK_B_NK
    dt = _lib.EK_DTYPE_BF16 if a.dtype == torch.bfloat16 else _lib.EK_DTYPE_FP16
    stream = torch.cuda.current_stream().cuda_stream
    return _lib.lib().ek_gemm_noalloc(a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K, dt, bl, sms, force_bn,
                                      force_split, ctypes.c_void_p(stream))


@pytest.mark.parametrize("M,N,K,layout,sms,bn,split", [
    (4096, 4096, 4096, "kn", 148, 0, 0),     # 68 tail tiles split 2-way (17.8 MB of scratch)
    (1000, 1032, 1536, "kn", 16, 128, 3),    # forced 3-way split of a small partition's tail
    (512, 4096, 4096, "nk", 148, 128, 2),    # every tile split 2-way
    (2048, 2048, 2048, "kn", 148, 0, 0),     # no split: the scratch is not touched
])
def test_noalloc_matches_workspace_entry_point(cuda_dev, M, N, K, layout, sms, bn, split):
    from elastikernel_b200 import _lib, _ops

    g = torch.Generator(device=cuda_dev).manual_seed(M + N + K)
    a = torch.randn((M, K), device=cuda_dev, dtype=torch.bfloat16, generator=g)
    b = torch.randn((K, N) if layout == "kn" else (N, K), device=cuda_dev, dtype=torch.bfloat16, generator=g)
    ref = _ops.gemm(a, b, num_sms=sms, b_layout=layout, force_bn=bn, force_split=split)
    plan = _ops.plan(M, N, K, sms, torch.bfloat16, layout, bn, split)
    assert plan["workspace_bytes"] <= _lib.lib().ek_gemm_noalloc_max_scratch_bytes()
    for _ in range(2):  # two calls in a row share (and reuse) the built-in scratch
        c = torch.full((M, N), float("nan"), device=cuda_dev, dtype=torch.bfloat16)
        rc = _noalloc(a, b, c, M, N, K, layout, sms, bn, split)
        assert rc == 0, _lib.last_error()
        torch.cuda.synchronize()
        assert _lib.device_status(0) == 0
        err = max_rel_err(c, ref.float().cpu().numpy())
        assert err <= TOL, f"no-alloc GEMM differs from ek_gemm: max rel err {err:.3e}"


def test_noalloc_rejects_oversized_schedule(cuda_dev):
    from elastikernel_b200 import _lib

    M, N, K = 4096, 4096, 8192
    a = torch.empty((M, K), device=cuda_dev, dtype=torch.bfloat16)
    b = torch.empty((K, N), device=cuda_dev, dtype=torch.bfloat16)
    c = torch.empty((M, N), device=cuda_dev, dtype=torch.bfloat16)
    rc = _noalloc(a, b, c, M, N, K, "kn", 148, 256, 8)  # 68 tail tiles x 8 slices x 128 KB > 32 MiB
    assert rc == _lib.EK_ERR_UNSUPPORTED
    assert "scratch" in _lib.last_error()


@pytest.mark.parametrize("req_sms", [16, 96])
def test_noalloc_on_green_context_partition(cuda_dev, req_sms):
    """Called on a green-context partition's stream with num_sms = 0, the entry
    point sizes its grid from the partition registry, as ek_gemm does, and
    gives ek_gemm's result there, on two calls in a row."""
    from elastikernel_b200 import _lib, _ops
    from elastikernel_b200.green_ctx import create_sm_partition

    stream, actual = create_sm_partition(cuda_dev, req_sms)
    M, N, K = 4096, 4096, 4096
    g = torch.Generator(device=cuda_dev).manual_seed(req_sms)
    a = torch.randn((M, K), device=cuda_dev, dtype=torch.bfloat16, generator=g)
    b = torch.randn((K, N), device=cuda_dev, dtype=torch.bfloat16, generator=g)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        ref = _ops.gemm(a, b)  # plans for the partition from the registry
        for _ in range(2):
            c = torch.full((M, N), float("nan"), device=cuda_dev, dtype=torch.bfloat16)
            rc = _noalloc(a, b, c, M, N, K, "kn", 0)
            assert rc == 0, _lib.last_error()
            stream.synchronize()
            assert _lib.device_status(0) == 0
            err = max_rel_err(c, ref.float().cpu().numpy())
            assert err <= TOL, f"{actual}-SM partition: max rel err {err:.3e}"
