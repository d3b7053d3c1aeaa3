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


def run_analytical(sm_levels=None, test_cases=None) -> None:
    sm_levels = sm_levels or SM_LEVELS
    test_cases = test_cases or [(1024, 1024, 1024), (2048, 2048, 2048), (4096, 4096, 4096)]
    for M, N, K in test_cases:
        print(f"\n{'=' * 90}")
        print(f"Wave Analysis: M={M}, N={N}, K={K}")
        print(f"{'=' * 90}")
        best_per_sm = {}
        for num_sms in sm_levels:
            ranked = rank_configs(M, N, num_sms)
            best_per_sm[num_sms] = ranked[0]
            print(f"\n--- {num_sms} SMs ---")
            print(f"  {'Rank':<5} {'Config':<45} {'Waves':<7} {'LastUtil':<10} {'Eff':<10}")
            for i, (c, nw, lwu, eff) in enumerate(ranked[:5], 1):
                s = f"M={c['BLOCK_SIZE_M']},N={c['BLOCK_SIZE_N']},K={c['BLOCK_SIZE_K']}"
                print(f"  {i:<5} {s:<45} {nw:<7} {lwu * 100:>5.1f}%    {eff * 100:>5.1f}%")
        print(f"\n{'=' * 90}")
        print(f"Best Config per SM (M={M}, N={N}, K={K})")
        print(f"{'=' * 90}")
        print(f"  {'SM':<6} {'Best Config':<45} {'Waves':<7} {'Eff':<10} {'Changed?'}")
        prev = None
        for num_sms in sm_levels:
            c, nw, lwu, eff = best_per_sm[num_sms]
            s = f"M={c['BLOCK_SIZE_M']},N={c['BLOCK_SIZE_N']},K={c['BLOCK_SIZE_K']}"
            changed = " <-- CHANGED" if prev is not None and c != prev else ""
            print(f"  {num_sms:<6} {s:<45} {nw:<7} {eff * 100:>5.1f}%{changed}")
            prev = c
        print(f"\n  tcgen05 schedule (128 x BN tiles, split tail wave):")
        print(f"  {'SM':<6} {'BN':<5} {'tiles':<7} {'split':<6} {'units':<7} {'waves':<6} {'Eff':<8} {'est us':<8}")
        for num_sms in sm_levels:
            p = tcgen05_schedule(M, N, K, num_sms)
            print(f"  {num_sms:<6} {p['bn']:<5} {p['num_tiles']:<7} {p['tail_split']:<6} {p['num_units']:<7} "
                  f"{p['waves']:<6} {p['wave_efficiency'] * 100:>5.1f}%  {p['est_us']:>7.1f}")


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
