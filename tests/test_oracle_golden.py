"""Pin the CPU oracle to the reference: every golden vector in tests/golden/ was
produced by the reference's own code (see tests/golden/gen_golden.py)."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import gemm as og
from oracle import moe as om
from oracle import wave as ow

GOLD = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def wave():
    return json.loads((GOLD / "wave.json").read_text())


def test_configs_table_matches(wave):
    assert [list(c) for c in ow.CONFIGS] == wave["configs"]


def test_wave_ranking_analytical(wave):
    for rec in wave["analytical"]:
        got = ow.rank_configs(rec["M"], rec["N"], rec["S"])
        assert len(got) == len(rec["ranked"])
        for (c, nw, lwu, eff), (gc, gnw, glwu, geff) in zip(got, rec["ranked"]):
            assert list(c) == gc and nw == gnw and lwu == glwu and eff == geff


def test_wave_sweep_best(wave):
    for rec in wave["sweep"]:
        c, nw, lwu, eff = ow.rank_configs(rec["M"], 4096, rec["S"])[0]
        gc, gnw, glwu, geff = rec["best"]
        assert (list(c), nw, lwu, eff) == (gc, gnw, glwu, geff)
        assert ow.ceil_div(rec["M"], 128) == rec["ceil_div"]


def test_workload_suggest(wave):
    for rec in wave["workload"]:
        assert ow.compute_wave_efficiency(rec["M"], rec["N"], 128, 256, rec["S"]) == rec["metrics_128x256"]
        bm, bn, m = ow.suggest_optimal_block_size(rec["M"], rec["N"], rec["S"])
        assert [bm, bn, m] == rec["suggest"]


def test_routing_matches_reference():
    z = np.load(GOLD / "routing.npz")
    for name in ("mixtral", "dsv3", "small"):
        ids, w = om.route_ref(z[f"{name}_logits"], int(z[f"{name}_k"]))
        np.testing.assert_array_equal(ids, z[f"{name}_ids"])
        np.testing.assert_allclose(w, z[f"{name}_weights"], rtol=2e-6, atol=1e-7)


def test_moe_operator_matches_reference():
    z = np.load(GOLD / "moe_def.npz")
    for name in ("a", "b"):
        out = om.moe_ref(z[f"{name}_x"], z[f"{name}_logits"], z[f"{name}_w1"], z[f"{name}_w2"], z[f"{name}_w3"],
                         int(z[f"{name}_k"]))
        ref = z[f"{name}_out"]
        assert og.max_rel_err(out, ref) < 1e-5


def test_moe_loop_and_vec_restatements():
    z = np.load(GOLD / "moe_def.npz")
    args = [torch.from_numpy(z[f"a_{k}"]) for k in ("x", "logits", "w1", "w2", "w3")]
    ref = z["a_out"]
    assert og.max_rel_err(om.moe_loop_ref(*args, int(z["a_k"])), ref) < 1e-5
    assert og.max_rel_err(om.moe_vec_ref(*args, int(z["a_k"])), ref) < 1e-5


def test_gemm_matches_reference_triton_kernel():
    z = np.load(GOLD / "triton_gemm.npz")
    for name in ("g1", "g2"):
        ref = og.gemm_ref(z[f"{name}_a"], z[f"{name}_b"])
        # the kernel rounds its fp32 accumulator to fp16 once
        np.testing.assert_allclose(z[f"{name}_c"].astype(np.float32), ref.astype(np.float16).astype(np.float32),
                                   rtol=2e-3, atol=2e-2)


def test_segment_gemm_matches_reference_triton_kernel():
    z = np.load(GOLD / "triton_gemm.npz")
    hs, w, offs, out = z["seg_hs"], z["seg_w"], z["seg_offsets"], z["seg_out"]
    N = out.shape[1]
    K = hs.shape[1]
    ref = og.segment_gemm_ref(hs, w, offs, N, K)
    covered = np.isfinite(ref[:, 0])
    assert covered.sum() == offs[-1]
    np.testing.assert_allclose(out[covered].astype(np.float32), ref[covered].astype(np.float16).astype(np.float32),
                               rtol=2e-3, atol=2e-2)


def test_route_tie_break_lower_id_first():
    logits = np.zeros((3, 6), dtype=np.float32)
    logits[1, [2, 4]] = 1.0
    logits[2] = [0.5, 2.0, 2.0, -1, 2.0, 0.0]
    ids, w = om.route_ref(logits, 2)
    np.testing.assert_array_equal(ids, [[0, 1], [2, 4], [1, 2]])
    np.testing.assert_allclose(w, 0.5, rtol=1e-6)


def test_permute_ref_layout():
    ids = np.array([[1, 0], [1, 3], [0, 1], [3, 1]], dtype=np.int32)  # T=4, k=2
    r = om.permute_ref(ids, E=4, block_m=4)
    # expert 0: slots 1,4 ; expert 1: 0,2,5,7 ; expert 2: none ; expert 3: 3,6
    s = 8
    assert r["expert_counts"].tolist() == [2, 4, 0, 2]
    assert r["num_rows_padded"] == 12
    assert r["sorted_slots"][:12].tolist() == [1, 4, s, s, 0, 2, 5, 7, 3, 6, s, s]
    assert r["block_expert"][:3].tolist() == [0, 1, 3]
    assert (r["block_expert"][3:] == -1).all()
    assert len(r["sorted_slots"]) == om.max_padded_rows(4, 2, 4, 4)


def test_combine_ref_sums_weighted_slots_to_reference():
    """Per-slot weighted expert rows summed by combine_ref give the
    reference operator's output (bf16 rounding of the sum only)."""
    z = np.load(GOLD / "moe_def.npz")
    x, logits = z["a_x"].astype(np.float32), z["a_logits"]
    w1, w2, w3, k = z["a_w1"], z["a_w2"], z["a_w3"], int(z["a_k"])
    ids, wts = om.route_ref(logits, k)
    T = x.shape[0]
    y = np.zeros((T * k, x.shape[1]), dtype=np.float32)
    for t in range(T):
        for j in range(k):
            e = ids[t, j]
            h = x[t]
            a = (h @ w1[e].T) / (1 + np.exp(-(h @ w1[e].T))) * (h @ w3[e].T)
            y[t * k + j] = wts[t, j] * (a @ w2[e].T)
    out = om.combine_ref(torch.from_numpy(y), T, k)
    assert og.max_rel_err(out.float().numpy(), z["a_out"]) < 1e-2
