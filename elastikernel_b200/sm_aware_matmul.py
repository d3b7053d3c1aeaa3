"""SM-aware matrix multiplication (drop-in for elastikernel/sm_aware_matmul.py).

Usage:
    python -m elastikernel_b200.sm_aware_matmul --analytical
    python -m elastikernel_b200.sm_aware_matmul --benchmark

Part 1, the wave analysis, keeps the reference's functions and candidate list
(sm_aware_matmul.py:17-86) and adds the same table for the tcgen05 kernel's
own schedule, read from the C planner (ek_gemm_plan_make), which splits the
tail wave instead of only choosing among whole tiles.

Part 2, the kernels: call_vanilla / call_sm_aware have the reference
wrappers' signatures (sm_aware_matmul.py:219-234) but run the persistent
tcgen05 GEMM. call_sm_aware plans for `num_sms` (default: the partition of
the current stream); call_vanilla always plans for the full device, which is
what a kernel tuned without the partition size does inside a partition.
"""
from __future__ import annotations

import argparse
from typing import Dict, List, Tuple


# =============================================================================
# Part 1: wave analysis (pure Python / host planner, no GPU)
# =============================================================================

def ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


def wave_efficiency(M, N, block_m, block_n, num_sms):
    """Returns (num_waves, last_wave_util, overall_efficiency) of a grid with
    one tile per CTA (sm_aware_matmul.py:21-28)."""
    num_blocks = ceil_div(M, block_m) * ceil_div(N, block_n)
    num_waves = ceil_div(num_blocks, num_sms)
    last_wave_blocks = num_blocks % num_sms
    if last_wave_blocks == 0:
        last_wave_blocks = num_sms
    return num_waves, last_wave_blocks / num_sms, num_blocks / (num_waves * num_sms)


def _cfg(bm, bn, bk):
    return {"BLOCK_SIZE_M": bm, "BLOCK_SIZE_N": bn, "BLOCK_SIZE_K": bk, "GROUP_SIZE_M": 8}


# The reference's analytical candidate list (sm_aware_matmul.py:31-48), same order.
CONFIGS: List[Dict[str, int]] = [
    _cfg(128, 256, 64), _cfg(64, 256, 32), _cfg(128, 128, 32), _cfg(128, 64, 32), _cfg(64, 128, 32),
    _cfg(128, 32, 32), _cfg(64, 32, 32), _cfg(32, 64, 32), _cfg(128, 256, 128), _cfg(256, 128, 128),
    _cfg(256, 64, 128), _cfg(64, 256, 128), _cfg(128, 128, 128), _cfg(128, 64, 64), _cfg(64, 128, 64),
    _cfg(128, 32, 64),
]

SM_LEVELS = [16, 32, 48, 64, 80, 96, 112, 132]
B200_LEVELS = [16, 32, 64, 96, 132, 148]


def rank_configs(M: int, N: int, num_sms: int) -> List[Tuple[dict, int, float, float]]:
    """CONFIGS ranked by (waves, -last_wave_util) (sm_aware_matmul.py:62-67)."""
    ranked = []
    for c in CONFIGS:
        nw, lwu, eff = wave_efficiency(M, N, c["BLOCK_SIZE_M"], c["BLOCK_SIZE_N"], num_sms)
        ranked.append((c, nw, lwu, eff))
    ranked.sort(key=lambda x: (x[1], -x[2]))
    return ranked


def tcgen05_schedule(M: int, N: int, K: int, num_sms: int, dtype: str = "bf16") -> dict:
    """The tcgen05 kernel's schedule for this shape and partition (C planner)."""
    import torch

    from . import _ops

    dt = {"bf16": torch.bfloat16, "fp16": torch.float16}[dtype]
    return _ops.plan(M, N, K, num_sms, dt)


def plan_table(M: int, N: int, K: int, sm_levels=None, dtype: str = "bf16") -> Dict[int, dict]:
    """The kernel-family dispatch table for one shape: the tcgen05 schedule
    (tile, CTA pair, tail split, waves, model time) precomputed for every
    partition size in `sm_levels`. A caller that knows its partition sizes
    builds it once and dispatches by SM count with a dict lookup; the C
    planner also caches recent plans per thread, so repeated calls of a shape
    never re-run the model."""
    levels = sm_levels or SM_LEVELS + [148]
    return {int(s): tcgen05_schedule(M, N, K, int(s), dtype) for s in levels}


class GraphMatmul:
    """C = A @ B for fixed operand buffers, captured once into a CUDA graph on
    a partition stream and replayed there: the per-call host cost (planning,
    tensor-map encoding, the ctypes launch) is paid once at capture.

    `stream` is the partition's stream (default: the current stream) and
    `num_sms` its SM count (default: from the partition registry). Refill
    `a` and `b` in place between replays; `__call__` returns the same output
    tensor each time."""

    def __init__(self, a, b, num_sms=None, stream=None):
        from .graph import Captured

        self.a, self.b = a, b
        self._cap = Captured(lambda: call_sm_aware(a, b, num_sms), stream, a.device)
        self.stream = self._cap.stream
        self.c = self._cap.out

    def __call__(self):
        return self._cap()


def compute_wave_efficiency(M: int, N: int, block_m: int, block_n: int, num_sms: int) -> Dict[str, float]:
    """Tile count, waves, last-wave utilisation and overall efficiency of a
    one-tile-per-CTA grid, as a dict (sm_aware_agent/workload.py:86-107)."""
    nw, lwu, eff = wave_efficiency(M, N, block_m, block_n, num_sms)
    return {"num_blocks": ceil_div(M, block_m) * ceil_div(N, block_n), "num_waves": nw,
            "last_wave_util": lwu, "overall_efficiency": eff if nw > 0 else 0}


# Default (BLOCK_M, BLOCK_N) candidates of suggest_optimal_block_size
# (sm_aware_agent/workload.py:126-131), in order: the first of equally
# efficient candidates wins.
SUGGEST_BLOCKS: List[Tuple[int, int]] = [(16, 64), (32, 64), (32, 128), (64, 64), (64, 128), (128, 64), (128, 128),
                                         (128, 256), (256, 128), (64, 256), (256, 64)]


def suggest_optimal_block_size(M: int, N: int, num_sms: int, block_sizes=None):
    """(block_m, block_n, metrics) of the candidate with the strictly highest
    overall wave efficiency (sm_aware_agent/workload.py:110-143)."""
    best, best_eff = None, 0
    for bm, bn in block_sizes or SUGGEST_BLOCKS:
        m = compute_wave_efficiency(M, N, bm, bn, num_sms)
        if m["overall_efficiency"] > best_eff:
            best_eff, best = m["overall_efficiency"], (bm, bn, m)
    return best


# tcgen05 tile modes of the persistent kernel: (cta_pair, tile_m, tile_n),
# passed to the planner as force_bn (> 0 one CTA, < 0 a CTA pair)
TCGEN05_MODES = [(1, 256, 256), (1, 256, 128), (0, 128, 256), (0, 128, 192), (0, 128, 128), (0, 128, 64)]


def get_configs_for_sm(num_sms: int, M: int = 4096, N: int = 4096, K: int = 4096, dtype: str = "bf16") -> List[dict]:
    """The candidate tiles for a partition of `num_sms` SMs, best first.

    The reference preselects Triton configs by SM regime -- small tiles up to
    24 SMs, medium up to 64, large above (sm_aware_agent/generator.py:41-79) --
    and lets autotuning pick among them. The tcgen05 kernel has six tile
    modes; its planner prices every mode for the partition and shape (MMA vs
    operand-feed rate per K step, the busiest CTA's K steps, a split of the
    tail wave, the HBM floor), so the "regime" becomes this ranking: each
    mode's schedule at its best tail split, sorted by the model's time. The
    first entry is the schedule call_sm_aware runs."""
    import torch

    from . import _ops

    dt = {"bf16": torch.bfloat16, "fp16": torch.float16}[dtype]
    out = []
    for pair, tm, tn in TCGEN05_MODES:
        if pair and num_sms < 2:
            continue
        p = _ops.plan(M, N, K, num_sms, dt, force_bn=-tn if pair else tn)
        out.append({"cta_pair": pair, "tile_m": tm, "tile_n": tn, "tail_split": p["tail_split"],
                    "tiles": p["num_tiles"], "units": p["num_units"], "waves": p["waves"],
                    "wave_efficiency": p["wave_efficiency"], "est_us": p["est_us"]})
    out.sort(key=lambda c: c["est_us"])
    return out


def run_analytical(sm_levels=None, test_cases=None) -> list:
    """Wave table per shape and partition size: the best whole-tile grid among
    the reference's candidate list (ranked by waves, then last-wave fill) next
    to the tcgen05 kernel's own schedule, which can also split the tail wave
    along K. Returns the rows it prints."""
    sm_levels = sm_levels or SM_LEVELS
    test_cases = test_cases or [(1024, 1024, 1024), (2048, 2048, 2048), (4096, 4096, 4096)]
    rows = []
    hdr = (f"{'SMs':>4} | {'grid tile':>9} {'tiles':>6} {'waves':>5} {'fill':>6} {'eff':>6} | "
           f"{'tcgen05':>9} {'split':>5} {'units':>6} {'waves':>5} {'eff':>6} {'model us':>8}")
    for M, N, K in test_cases:
        print(f"\n[{M} x {N} x {K}]  whole-tile grid (candidate list)  vs  persistent tcgen05 schedule")
        print(hdr)
        print("-" * len(hdr))
        prev = None
        for S in sm_levels:
            c, nw, lwu, eff = rank_configs(M, N, S)[0]
            tile = f"{c['BLOCK_SIZE_M']}x{c['BLOCK_SIZE_N']}"
            p = tcgen05_schedule(M, N, K, S)
            mode = f"{p['bm']}x{p['bn']}" + ("p" if p["cta_pair"] else "")
            mark = "" if prev is None or tile == prev else "  (grid tile changes)"
            prev = tile
            print(f"{S:>4} | {tile:>9} {ceil_div(M, c['BLOCK_SIZE_M']) * ceil_div(N, c['BLOCK_SIZE_N']):>6} "
                  f"{nw:>5} {lwu * 100:>5.1f}% {eff * 100:>5.1f}% | {mode:>9} {p['tail_split']:>5} "
                  f"{p['num_units']:>6} {p['waves']:>5} {p['wave_efficiency'] * 100:>5.1f}% {p['est_us']:>8.1f}{mark}")
            rows.append({"M": M, "N": N, "K": K, "sms": S, "grid_tile": tile, "grid_waves": nw,
                         "grid_last_util": lwu, "grid_eff": eff, "tcgen05": p})
    print("\n(p = 2-SM CTA pair; fill = share of SMs busy in the last wave)")
    return rows


# =============================================================================
# Part 2: kernels
# =============================================================================

def call_vanilla(a, b):
    """C = a @ b planned for the full device (no partition awareness)."""
    import torch

    from . import _ops

    total = torch.cuda.get_device_properties(a.device).multi_processor_count
    return _ops.gemm(a, b, num_sms=total)


def call_sm_aware(a, b, num_sms=None):
    """C = a @ b planned for `num_sms` SMs (None: the current stream's partition)."""
    from . import _ops

    return _ops.gemm(a, b, num_sms=num_sms)


def run_benchmark(sm_levels=None, test_cases=None, rep_ms: float = 50.0) -> list:
    """Vanilla vs SM-aware tcgen05 GEMM under green-context partitions
    (the reference's benchmark, sm_aware_matmul.py:237-295), timed with CUDA
    events on the partition stream with the L2 flushed before each rep."""
    import torch

    from .green_ctx import create_sm_partition, full_device_partition, get_sm_alignment, get_total_sm_count
    from .timing import time_on_stream

    dev = torch.device("cuda:0")
    total_sms = get_total_sm_count(dev)
    min_sm, align = get_sm_alignment(dev)
    print(f"Device: {torch.cuda.get_device_name(dev)}")
    print(f"Total SMs: {total_sms}, SM alignment: min={min_sm}, align={align}")
    sm_levels = [s for s in (sm_levels or SM_LEVELS + [total_sms]) if s <= total_sms]
    square_cases = [(1024, 1024, 1024), (2048, 2048, 2048), (4096, 4096, 4096)]
    m_sweep_cases = [(M, 4096, 4096) for M in [1, 16, 32, 64, 128, 256, 512, 1024, 2048]]
    results = []
    for M, N, K in test_cases or (square_cases + m_sweep_cases):
        print(f"\n{'=' * 80}\nM={M}, N={N}, K={K}\n{'=' * 80}")
        print(f"  {'SM':>4} {'Actual':>6}  {'Vanilla(us)':>11} {'Aware(us)':>11} {'Speedup':>8}  Schedule")
        torch.manual_seed(0)
        a = torch.randn((M, K), device=dev, dtype=torch.bfloat16)
        b = torch.randn((K, N), device=dev, dtype=torch.bfloat16)
        ref = torch.matmul(a.float(), b.float())
        for sm_count in sm_levels:
            try:
                if sm_count >= total_sms:
                    stream, actual = full_device_partition(dev)
                else:
                    stream, actual = create_sm_partition(dev, sm_count)
                with torch.cuda.stream(stream):
                    for _ in range(3):
                        call_vanilla(a, b)
                        call_sm_aware(a, b, actual)
                    van = time_on_stream(lambda: call_vanilla(a, b), stream, rep_ms=rep_ms)
                    aw = time_on_stream(lambda: call_sm_aware(a, b, actual), stream, rep_ms=rep_ms)
                    out = call_sm_aware(a, b, actual)
                stream.synchronize()
                p = tcgen05_schedule(M, N, K, actual)
                err = ((out.float() - ref).abs().max() / ref.abs().max()).item()
                sp = van["mean_ms"] / aw["mean_ms"] if aw["mean_ms"] > 0 else 0.0
                print(f"  {sm_count:>4} {actual:>6}  {van['mean_ms'] * 1e3:>11.1f} {aw['mean_ms'] * 1e3:>11.1f} "
                      f"{sp:>7.2f}x  BN={p['bn']} split={p['tail_split']} eff={p['wave_efficiency'] * 100:.1f}%"
                      + ("" if err < 1e-2 else f"  WARNING: max rel err {err:.2e}"))
                results.append({"M": M, "N": N, "K": K, "sm": sm_count, "actual": actual,
                                "vanilla_us": van["mean_ms"] * 1e3, "aware_us": aw["mean_ms"] * 1e3,
                                "tflops": 2.0 * M * N * K / (aw["mean_ms"] * 1e-3) / 1e12, "max_rel_err": err,
                                "plan": p})
            except Exception as e:  # per-level failures are reported, as the reference does
                print(f"  {sm_count:>4}  Error: {e}")
    return results


def main():
    parser = argparse.ArgumentParser(description="SM-Aware Matmul Benchmark")
    parser.add_argument("--analytical", action="store_true", help="Wave analysis (no GPU)")
    parser.add_argument("--benchmark", action="store_true", help="GPU benchmark with Green Context")
    args = parser.parse_args()
    if args.analytical:
        run_analytical()
    elif args.benchmark:
        run_benchmark()
    else:
        parser.print_help()


if __name__ == "__main__":
    main()
