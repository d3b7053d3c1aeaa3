"""The reference arm of bench.py runs on the host and prints the one JSON line
the benchmark driver parses (CPU only: torch.matmul on the host cores, the
reference's GEMM operator body)."""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def test_reference_arm_json_line():
    proc = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                          cwd=REPO, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "dtype", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["steps"] == 1 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["unit"] == "TFLOP/s" and d["e2e"]["unit"] == d["unit"]
    assert d["e2e"]["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["value"] == d["value"] and d["cpu_baseline"]["cores"] >= 1
    assert d["config"]["M"] == d["config"]["N"] == d["config"]["K"] == 4096


def test_summary_is_compact_and_complete():
    """The line's last key condenses every leg; it must stay short enough for a
    driver that keeps only the tail of stdout (a few KB)."""
    sys.path.insert(0, str(REPO))
    import bench

    parts = {"square_4096": [{"sm": s, "actual_sm": s, "us": 600.5, "tflops": 228.9, "pct_sm_peak_at_clock": 88.8,
                              "sm_mhz": 1965.0, "pct_cublas_8192": 97.1, "speedup_vs_cublas": 1.05}
                             for s in (16, 32, 64, 96, 132, 148)] + [{"sm": 200, "error": "x"}],
             "m_sweep_148": [{"M": m, "us": 22.9, "pct_roofline_time": 50.1, "cublas_us": 25.0}
                             for m in (128, 256, 512, 1024, 2048, 4096, 8192)]}
    fp8 = {"results": [{"actual_sm": 148, "tflops": 2700.0, "pct_scaled_fp8_peak": 81.0,
                        "speedup_vs_torch_scaled_mm": 1.1}, {"actual_sm": 80, "tflops": 1770.0,
                                                              "pct_scaled_fp8_peak": 98.0}]}
    moe = {"results": [{"T": t, "actual_sm": s, "us": 181.2, "pct_roofline_time": 59.9, "graph_us": 164.0,
                        "graph_pct_roofline_time": 65.1} for t in (1, 16, 128, 1024, 4096) for s in (148, 72)],
           "cpu": {"cores": 16, "results": [{"T": t, "vectorised_tokens_per_s": 1000.5, "loop_tokens_per_s": 10.5}
                                            for t in (1, 16, 128, 1024, 4096)]}}
    ep = {"n_gpus": 8, "ms_per_layer": 5.9, "tokens_per_s": 5.5e6, "pct_fp8_peak_scaled": 19.4,
          "gemm_partition_sms": 116, "ep_max_rel_err": 0.011, "ep_max_rel_err_act_e4m3": 0.004,
          "expert_groups": 4,
          "phases_ms_ungrouped": {k: 0.123 for k in ("route_permute", "count_exchange", "dispatch", "experts",
                                                    "combine_exchange", "final_combine")},
          "all_to_all": {"dispatch_gbs_per_rank": 300.1, "combine_gbs_per_rank": 310.2}}
    line = {"value": 1331.57, "roofline": {"frac": 0.798}, "e2e": {"value": 101.0}, "clocks": {"sm_mhz": 1965.0},
            "partitions": parts, "fp8": fp8, "moe": moe, "moe_ep": ep,
            "cpu_baseline": {"value": 5.1, "cores": 16}}
    s = bench.summarize(line)
    text = json.dumps(s)
    assert len(text) < 2600, len(text)
    assert set(s["partitions"]) == {"16", "32", "64", "96", "132", "148"}
    assert s["moe_ep"]["ep_max_rel_err"] == [0.011, 0.004] and "moe_cpu" in s and "fp8" in s and "m_sweep" in s


def test_summary_reports_an_ep_leg_error():
    """An expert-parallel leg that raised leaves an error field; the summary
    carries it instead of failing on the missing measurements."""
    sys.path.insert(0, str(REPO))
    import bench

    line = {"value": 1400.0, "roofline": {"frac": 0.85}, "e2e": {"value": 99.0}, "clocks": {"sm_mhz": 1965.0},
            "moe_ep": {"n_gpus": 8, "error": "RuntimeError: " + "x" * 400}}
    s = bench.summarize(line)
    assert s["moe_ep"]["n_gpus"] == 8 and s["moe_ep"]["error"].startswith("RuntimeError")
    assert len(s["moe_ep"]["error"]) <= 160
