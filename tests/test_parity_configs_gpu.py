"""Parity on the configurations bench.py measures, through the C-ABI, against
the CPU oracle.

* bf16 GEMM 4096^3 with the schedule of the headline (148 SMs: 256 x 256
  CTA-pair tiles, 2-way K-split of the tail tiles) and inside real
  green-context partitions of the wave sweep (16..132 SMs);
* ragged shapes that the reference's masked Triton kernel accepts
  (sm_aware_matmul.py:164-172): M=77, N=100, K=100 and others, bf16 and fp16,
  through call_sm_aware;
* the GEMM operator run(A, B, C, M, N, K, NUM_SMS) (definition.py:63-65) on
  both of its branches: in place, and through C.copy_;
* the Mixtral-shaped MoE layer (E=8, top-2, H=4096, I=14336) at T=1024 and
  T=4096 in both row layouts (packed rows with swapped-operand GEMMs; padded
  rows, with 256-row CTA-pair tiles where the bench runs them) on the full
  device and on a 72-SM partition;
* the DeepSeek-V3-shaped FP8 layer (E=256, top-8, H=7168, I=2048, 128 x 128
  block scales) at T=4096;
* the benchmark-harness records: workload records -> the solution each names
  -> compared with the oracle and with the record's own CPU reference.

A token's MoE output depends only on that token, so the large layers run on
all their tokens and a seeded sample of tokens is compared with the oracle
(which fetches one expert's weights at a time). Routing ids are compared
bit-exactly on all tokens.

Tolerances (max|out - ref| / max|ref| against the oracle's fp32 result on the
same inputs): bf16 1e-2; FP8 3e-2, the oracle then running on the
dequantised weights and tokens.
"""
from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

from oracle import fp8 as of8
from oracle import gemm as og
from oracle import moe as om

pytestmark = pytest.mark.gpu

TOL = 1e-2
TOL_FP8 = 3e-2


def _total_sms(dev) -> int:
    return torch.cuda.get_device_properties(dev).multi_processor_count


# --------------------------------------------------------------------- GEMM
@pytest.fixture(scope="module")
def square4096(cuda_dev):
    g = torch.Generator().manual_seed(0)
    a = torch.randn((4096, 4096), generator=g).to(torch.bfloat16)
    b = torch.randn((4096, 4096), generator=g).to(torch.bfloat16)
    return a.to(cuda_dev), b.to(cuda_dev), og.gemm_ref(a, b)


def test_gemm_4096_cube_headline_schedule(cuda_dev, square4096):
    from elastikernel_b200 import sm_aware_matmul as smm

    da, db, ref = square4096
    if _total_sms(cuda_dev) == 148:
        p = smm.tcgen05_schedule(4096, 4096, 4096, 148)
        # 256 pair tiles on 74 pairs: 222 whole tiles, the other 34 split 2-way along K
        assert (p["cta_pair"], p["bm"], p["bn"], p["tail_split"]) == (1, 256, 256, 2)
        assert p["num_dp_tiles"] == 222 and p["num_units"] == 222 + 34 * 2
    outs = [smm.call_sm_aware(da, db) for _ in range(2)]  # the default stream plans for the full device
    torch.cuda.synchronize()
    for c in outs:
        err = og.max_rel_err(c, ref)
        assert err <= TOL, f"4096^3 at full device: {err:.3e}"
    assert torch.equal(outs[0], outs[1])  # split tiles sum in slice order: deterministic


@pytest.mark.parametrize("req", [16, 32, 64, 96, 132])
def test_gemm_4096_cube_in_green_context_partition(cuda_dev, square4096, req):
    from elastikernel_b200 import sm_aware_matmul as smm
    from elastikernel_b200.green_ctx import create_sm_partition, stream_sm_count

    da, db, ref = square4096
    stream, actual = create_sm_partition(cuda_dev, req)
    assert stream_sm_count(stream) == actual >= req
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        c = smm.call_sm_aware(da, db)  # num_sms from the partition registry
    stream.synchronize()
    err = og.max_rel_err(c, ref)
    assert err <= TOL, f"4096^3 on a {actual}-SM partition: {err:.3e}"


@pytest.mark.parametrize("M,N,K", [(77, 100, 100), (1, 3, 5), (300, 1000, 1001), (129, 136, 40), (1000, 4100, 4100),
                                   (2048, 2050, 2048)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_ragged_shapes_through_call_sm_aware(cuda_dev, M, N, K, dtype):
    """Shapes the reference's masked kernel accepts; N not a multiple of 8 or K
    not a multiple of 16 run through zero-padded copies on the device."""
    from elastikernel_b200 import sm_aware_matmul as smm

    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randn((M, K), generator=g).to(dtype)
    b = torch.randn((K, N), generator=g).to(dtype)
    ref = og.gemm_ref(a, b)
    for c in (smm.call_sm_aware(a.to(cuda_dev), b.to(cuda_dev)),
              smm.call_sm_aware(a.to(cuda_dev), b.to(cuda_dev), num_sms=16),
              smm.call_vanilla(a.to(cuda_dev), b.to(cuda_dev))):
        torch.cuda.synchronize()
        assert c.shape == (M, N) and c.dtype == dtype
        err = og.max_rel_err(c, ref)
        assert err <= TOL, f"{M}x{N}x{K} {dtype}: {err:.3e}"


@pytest.mark.parametrize("M,N,K", [(77, 100, 100), (500, 4100, 4100)])
def test_ragged_shapes_weight_layout_and_partition(cuda_dev, M, N, K):
    """[N, K] weights with a ragged K, and a ragged shape inside a partition
    (its split tail and the padded copies share one workspace)."""
    from elastikernel_b200 import _ops
    from elastikernel_b200.green_ctx import create_sm_partition

    g = torch.Generator().manual_seed(7)
    a = torch.randn((M, K), generator=g).to(torch.bfloat16)
    w = torch.randn((N, K), generator=g).to(torch.bfloat16)
    ref = og.gemm_ref(a, w, "nk")
    stream, _ = create_sm_partition(cuda_dev, 32)
    da, dw = a.to(cuda_dev), w.to(cuda_dev)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        outs = [_ops.gemm(da, dw, b_layout="nk") for _ in range(2)]
    stream.synchronize()
    for c in outs:
        assert og.max_rel_err(c, ref) <= TOL


def test_unaligned_views(cuda_dev):
    """Operand views that start mid-line are accepted like the reference's
    strided tensors (copied to aligned buffers before the C-ABI call)."""
    from elastikernel_b200 import sm_aware_matmul as smm

    g = torch.Generator().manual_seed(3)
    a = torch.randn((65, 264), generator=g).to(torch.bfloat16)
    b = torch.randn((257, 200), generator=g).to(torch.bfloat16)
    da = a.to(cuda_dev).reshape(-1)[1:1 + 64 * 256].view(64, 256)
    db = b.to(cuda_dev).reshape(-1)[3:3 + 256 * 200].view(256, 200)
    c = smm.call_sm_aware(da, db)
    torch.cuda.synchronize()
    assert og.max_rel_err(c, og.gemm_ref(da.cpu(), db.cpu())) <= TOL


def test_run_gemm_operator_both_branches(cuda_dev):
    """definition.run_gemm writes C in place when it can (contiguous, input
    dtype) and otherwise through C.copy_ (definition.py:63-65)."""
    from elastikernel_b200.definition import run_gemm

    for M, N, K in ((512, 768, 1024), (77, 100, 100)):
        g = torch.Generator().manual_seed(M)
        a = torch.randn((M, K), generator=g).to(torch.bfloat16)
        b = torch.randn((K, N), generator=g).to(torch.bfloat16)
        ref = og.gemm_ref(a, b)
        da, db = a.to(cuda_dev), b.to(cuda_dev)
        c_in = torch.full((M, N), float("nan"), device=cuda_dev, dtype=torch.bfloat16)
        ptr = c_in.data_ptr()
        run_gemm(da, db, c_in, M, N, K, 148)
        c_t = torch.full((N, M), float("nan"), device=cuda_dev, dtype=torch.bfloat16).t()  # not contiguous
        run_gemm(da, db, c_t, M, N, K, 64)
        c_f = torch.full((M, N), float("nan"), device=cuda_dev, dtype=torch.float32)  # another dtype
        run_gemm(da, db, c_f, M, N, K, 16)
        torch.cuda.synchronize()
        assert c_in.data_ptr() == ptr
        for c in (c_in, c_t, c_f):
            err = og.max_rel_err(c, ref)
            assert err <= TOL, f"run_gemm {M}x{N}x{K} into {c.dtype} contiguous={c.is_contiguous()}: {err:.3e}"
    with pytest.raises(RuntimeError):
        run_gemm(da, db, c_in, M + 1, N, K, 148)


# ---------------------------------------------------------------------- MoE
MIX_E, MIX_K, MIX_H, MIX_I = 8, 2, 4096, 14336


@pytest.fixture(scope="module")
def mixtral(cuda_dev):
    g = torch.Generator(device=cuda_dev).manual_seed(42)
    w = {}
    for name, shape in (("w1", (MIX_E, MIX_I, MIX_H)), ("w3", (MIX_E, MIX_I, MIX_H)), ("w2", (MIX_E, MIX_H, MIX_I))):
        w[name] = (torch.randn(shape, device=cuda_dev, generator=g) * 0.02).to(torch.bfloat16)
    yield w
    del w
    torch.cuda.empty_cache()


def _sample(T: int, n: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    if T <= n:
        return np.arange(T)
    idx = rng.choice(T, size=n, replace=False)
    idx[:2] = (0, T - 1)
    return np.unique(idx)


@pytest.mark.parametrize("T", [1024, 4096])
def test_mixtral_layer_bench_shapes(cuda_dev, mixtral, T):
    """Every (layout, partition) combination the bench's Mixtral leg can take
    at T=1024 and T=4096, each compared with the same oracle sample."""
    from elastikernel_b200 import _ops
    from elastikernel_b200.green_ctx import create_sm_partition

    w1, w2, w3 = mixtral["w1"], mixtral["w2"], mixtral["w3"]
    g = torch.Generator(device=cuda_dev).manual_seed(T)
    x = torch.randn((T, MIX_H), device=cuda_dev, generator=g).to(torch.bfloat16)
    logits = torch.randn((T, MIX_E), device=cuda_dev, generator=g)
    rows = T * MIX_K
    half_stream, half_sms = create_sm_partition(cuda_dev, 72)
    full = torch.cuda.current_stream(cuda_dev)
    runs = [("auto", full, 148), ("packed", full, 148), ("padded", full, 148), ("auto", half_stream, half_sms)]
    # what the bench's "auto" calls run at these sizes
    expect_full = "packed" if rows <= _ops.PACKED_MAX_ROWS_PER_EXPERT * MIX_E else "padded"
    assert _ops.moe_layout(148, MIX_E, rows) == expect_full
    assert _ops.moe_layout(half_sms, MIX_E, rows) == "padded"
    assert _ops.padded_block_m(half_sms, MIX_E, rows) == 256          # CTA-pair tiles on the half device
    assert _ops.padded_block_m(148, MIX_E, rows) == (256 if T == 4096 else 128)

    ids, _ = _ops.moe_route(logits, MIX_K)
    outs = {}
    torch.cuda.synchronize()
    for layout, stream, sms in runs:
        with torch.cuda.stream(stream):
            outs[(layout, sms)] = _ops.fused_moe(x, logits, w1, w2, w3, MIX_K, layout=layout)
        stream.synchronize()
    ids_ref, wts_ref = om.route_ref(logits.cpu().numpy(), MIX_K)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_ref)

    s = _sample(T, 256, seed=T)
    ref = om.moe_ref_by_expert(x[s.tolist()].cpu(), ids_ref[s], wts_ref[s], MIX_E,
                               lambda e: (og.to_f32(w1[e]), og.to_f32(w2[e]), og.to_f32(w3[e])))
    for (layout, sms), out in outs.items():
        err = og.max_rel_err(out[s.tolist()], ref)
        assert err <= TOL, f"Mixtral T={T} layout={layout} on {sms} SMs: max rel err {err:.3e}"


@pytest.mark.parametrize("pow2", [False, True])
def test_dsv3_fp8_layer_e256_t4096(cuda_dev, pow2):
    """The DeepSeek-V3-shaped FP8 layer at the bench's 1-GPU load: 256 experts,
    4096 tokens, top-8 (CTA-pair token tiles at ~128 rows per expert), with
    fp32 scales applied in the epilogue and with power-of-two scales applied
    by the tensor cores."""
    from elastikernel_b200 import _ops

    E, k, H, I, T = 256, 8, 7168, 2048, 4096
    g = torch.Generator(device=cuda_dev).manual_seed(1000)
    parts = {"w1q": [], "w1s": [], "w3q": [], "w3s": [], "w2q": [], "w2s": []}
    for _ in range(0, E, 32):  # quantise in chunks to bound the bf16 staging memory, as the bench does
        w1 = (torch.randn((32, I, H), device=cuda_dev, generator=g) * 0.02).to(torch.bfloat16)
        w3 = (torch.randn((32, I, H), device=cuda_dev, generator=g) * 0.02).to(torch.bfloat16)
        w2 = (torch.randn((32, H, I), device=cuda_dev, generator=g) * 0.02).to(torch.bfloat16)
        q = _ops.quant_moe_weights_fp8(w1, w2, w3, pow2=pow2)
        for key in parts:
            parts[key].append(q[key])
        del w1, w2, w3, q
    qw = {"E": E, "I": I, "H": H, "pow2": pow2}
    for key, lst in parts.items():
        qw[key] = torch.cat(lst, dim=0)
    del parts
    qw = _ops.stack_gate_up_planes(qw)
    gx = torch.Generator(device=cuda_dev).manual_seed(42)
    x = torch.randn((T, H), device=cuda_dev, generator=gx).to(torch.bfloat16)
    logits = torch.randn((T, E), device=cuda_dev, generator=gx)
    out = _ops.fused_moe_fp8(x, logits, qw, k)
    ids, _ = _ops.moe_route(logits, k)
    torch.cuda.synchronize()
    ids_ref, wts_ref = om.route_ref(logits.cpu().numpy(), k)
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_ref)

    s = _sample(T, 48, seed=5)
    xs = x[s.tolist()].cpu()
    xd = of8.dequant_blocks(*of8.quant_blocks(xs, 1, 128, pow2=pow2), 1, 128)  # the tokens as the kernels see them
    nI, nH = I // 128, H // 128

    def fetch(e):
        w1e = of8.dequant_block_rows(qw["w1q"][e].cpu(), qw["w1s"][e * nI:(e + 1) * nI].cpu().numpy())
        w3e = of8.dequant_block_rows(qw["w3q"][e].cpu(), qw["w3s"][e * nI:(e + 1) * nI].cpu().numpy())
        w2e = of8.dequant_block_rows(qw["w2q"][e].cpu(), qw["w2s"][e * nH:(e + 1) * nH].cpu().numpy())
        return w1e, w2e, w3e

    def act_q(a):  # the layer rounds its bf16 activations to e4m3 (1 x 128 groups) before the down GEMM
        return of8.dequant_blocks(*of8.quant_blocks(torch.from_numpy(a).to(torch.bfloat16), 1, 128, pow2=pow2), 1, 128)

    ref, ref_q = om.moe_ref_by_expert(xd, ids_ref[s], wts_ref[s], E, fetch, act_quant=act_q)
    err = og.max_rel_err(out[s.tolist()], ref)
    assert err <= TOL_FP8, f"DSv3 FP8 layer T=4096 E=256 pow2={pow2}: max rel err {err:.3e}"
    # against the reference that rounds the activations as the layer does, the
    # remaining difference is fp32 summation order and bf16 output rounding
    err_q = og.max_rel_err(out[s.tolist()], ref_q)
    assert err_q <= TOL, f"DSv3 FP8 layer vs activation-rounded oracle: {err_q:.3e}"
    del qw
    torch.cuda.empty_cache()


# ------------------------------------------------------ harness records
def _solution(definition: str):
    from elastikernel_b200 import bench_schema as bs

    sol = {s["definition"]: s for s in bs.solutions()}[definition]
    mod, fn = sol["entry_point"].split(":")
    return getattr(importlib.import_module(mod), fn)


def _reference(defn: dict):
    ns = {}
    exec(defn["reference"], ns)
    return ns["run"]


def test_workload_records_run_named_solutions(cuda_dev):
    """A harness reading the records: for each workload, build seeded inputs of
    its axes, run the solution the record names on a partition of NUM_SMS SMs,
    and compare with the oracle and with the definition's CPU reference."""
    from elastikernel_b200 import bench_schema as bs
    from elastikernel_b200.green_ctx import create_sm_partition

    total = _total_sms(cuda_dev)
    streams = {}

    def stream_for(sms):
        if sms >= total:
            return torch.cuda.current_stream(cuda_dev)
        if sms not in streams:
            streams[sms] = create_sm_partition(cuda_dev, sms)[0]
        return streams[sms]

    gdef = bs.gemm_definition()
    run, ref_run = _solution(gdef["name"]), _reference(gdef)
    for wl in bs.gemm_workloads(sm_counts=[16, 148], sizes=[(1024, 1024, 1024), (128, 4096, 4096), (1, 4096, 4096),
                                                           (77, 100, 100)]):
        ax = wl["axes_values"]
        M, N, K, S = ax["M"], ax["N"], ax["K"], ax["NUM_SMS"]
        g = torch.Generator().manual_seed(M * 7 + S)
        A = torch.randn((M, K), generator=g).to(torch.bfloat16)
        B = torch.randn((K, N), generator=g).to(torch.bfloat16)
        C = torch.empty((M, N), device=cuda_dev, dtype=torch.bfloat16)
        st = stream_for(S)
        dA, dB = A.to(cuda_dev), B.to(cuda_dev)
        torch.cuda.synchronize()
        with torch.cuda.stream(st):
            run(dA, dB, C, M, N, K, S)
        st.synchronize()
        Cr = torch.empty((M, N), dtype=torch.float32)
        ref_run(A.float(), B.float(), Cr, M, N, K, S)
        oracle = og.gemm_ref(A, B)
        assert og.max_rel_err(C, oracle) <= TOL, wl["description"]
        assert og.max_rel_err(Cr, oracle) <= 1e-5

    E, k, H, I = 8, 2, 1024, 512
    mdef = bs.fused_moe_definition(num_experts=E, top_k=k)
    run, ref_run = _solution(mdef["name"]), _reference(mdef)
    for wl in bs.moe_workloads(hidden=H, inter=I, sm_counts=[32, 148], tokens=[1, 16, 128]):
        ax = wl["axes_values"]
        M, S = ax["M"], ax["NUM_SMS"]
        g = torch.Generator().manual_seed(M * 11 + S)
        x = torch.randn((M, H), generator=g).to(torch.bfloat16)
        logits = torch.randn((M, E), generator=g)
        w1 = (torch.randn((E, I, H), generator=g) * 0.02).to(torch.bfloat16)
        w2 = (torch.randn((E, H, I), generator=g) * 0.02).to(torch.bfloat16)
        w3 = (torch.randn((E, I, H), generator=g) * 0.02).to(torch.bfloat16)
        out = torch.empty((M, H), device=cuda_dev, dtype=torch.bfloat16)
        d = [t.to(cuda_dev) for t in (x, logits, w1, w2, w3)]
        st = stream_for(S)
        torch.cuda.synchronize()
        with torch.cuda.stream(st):
            run(d[0], d[1], d[2], d[3], d[4], out, M, H, I, E, k, S)
        st.synchronize()
        oracle = om.moe_ref(x, logits, w1, w2, w3, k)
        out_r = torch.empty((M, H), dtype=torch.float32)
        ref_run(x.float(), logits, w1.float(), w2.float(), w3.float(), out_r, M, H, I, E, k, S)
        assert og.max_rel_err(out, oracle) <= TOL, wl["description"]
        assert og.max_rel_err(out_r, oracle) <= 1e-4
