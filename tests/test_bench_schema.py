"""Benchmark-harness records (definition / workload / solution): complete,
JSON-serialisable, covering every partition size x shape, and the embedded
CPU reference implementations agree with the oracle."""
from __future__ import annotations

import json

import numpy as np
import torch

from oracle import moe as om


def test_definitions_and_workloads(tmp_path):
    from elastikernel_b200 import bench_schema as bs

    for d in (bs.gemm_definition(), bs.fused_moe_definition()):
        for key in ("name", "op_type", "axes", "inputs", "outputs", "reference", "constraints", "tags"):
            assert key in d
        assert "NUM_SMS" in d["axes"]
        json.dumps(d)
    wl = bs.gemm_workloads()
    assert len(wl) == len(bs.B200_SM_COUNTS) * len(bs.GEMM_SIZES)
    assert {w["axes_values"]["NUM_SMS"] for w in wl} == set(bs.B200_SM_COUNTS)
    assert len({w["uuid"] for w in wl}) == len(wl)
    r = bs.write_all(tmp_path)
    assert r["definitions"] == 2
    lines = (tmp_path / "workloads.jsonl").read_text().splitlines()
    assert len(lines) == r["workloads"] and all(json.loads(x)["definition"] for x in lines)
    sols = json.loads((tmp_path / "solutions.json").read_text())
    assert {s["definition"] for s in sols} == {"gemm_sm_aware", "fused_moe_sm_aware"}


def _exec_reference(src):
    ns = {}
    exec(src, ns)
    return ns["run"]


def test_embedded_references_match_oracle():
    from elastikernel_b200 import bench_schema as bs

    g = torch.Generator().manual_seed(9)
    A = torch.randn((33, 40), generator=g)
    B = torch.randn((40, 24), generator=g)
    C = torch.empty((33, 24))
    _exec_reference(bs.gemm_definition()["reference"])(A, B, C, 33, 24, 40, 148)
    np.testing.assert_allclose(C.numpy(), (A.double() @ B.double()).numpy(), rtol=1e-5, atol=1e-4)

    T, H, I, E, k = 12, 32, 48, 6, 2
    x = torch.randn((T, H), generator=g)
    logits = torch.randn((T, E), generator=g)
    w1 = torch.randn((E, I, H), generator=g) * 0.1
    w2 = torch.randn((E, H, I), generator=g) * 0.1
    w3 = torch.randn((E, I, H), generator=g) * 0.1
    out = torch.empty((T, H))
    _exec_reference(bs.fused_moe_definition(num_experts=E, top_k=k)["reference"])(
        x, logits, w1, w2, w3, out, T, H, I, E, k, 148)
    ref = om.moe_ref(x.numpy(), logits.numpy(), w1, w2, w3, k)
    assert np.abs(out.numpy() - ref).max() / np.abs(ref).max() < 1e-5
