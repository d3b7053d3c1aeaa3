"""Partition co-run harness: the dense GEMM and the fused MoE in disjoint
green-context partitions at the same time, optionally beside a memory
stressor in a third partition.

This applies the method of the reference's isolation check
(verify_isolation.py:87-204: time each load alone, then all at once from a
common start event) to the two hot-path operators, and reports how much each
slows down when the others run: SM isolation removes contention for SMs, not
for HBM and L2, which the stressor exercises on purpose.

Usage:
    python -m elastikernel_b200.corun --gemm-sms 72 --moe-sms 72 --moe-tokens 128
    python -m elastikernel_b200.corun --gemm-sms 64 --moe-sms 64 --stressor-sms 16
"""
from __future__ import annotations

import argparse

import torch

from . import _ops
from .green_ctx import create_disjoint_partitions, get_total_sm_count


class _Load:
    """A repeatable piece of work on one partition stream."""

    def __init__(self, name: str, stream, fn, flop_per_call: float = 0.0, tokens_per_call: int = 0):
        self.name, self.stream, self.fn = name, stream, fn
        self.flop, self.tokens = flop_per_call, tokens_per_call

    def run(self, iters: int):
        with torch.cuda.stream(self.stream):
            for _ in range(iters):
                self.fn()


def _time_alone(load: _Load, iters: int) -> float:
    load.run(2)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(load.stream)
    load.run(iters)
    e.record(load.stream)
    torch.cuda.synchronize()
    return s.elapsed_time(e)


def _time_together(loads: list[_Load], iters: list[int]) -> list[float]:
    """All loads start on a common event; per-load time to its own last event (ms)."""
    for ld in loads:
        ld.run(1)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    start.record()
    ends = []
    for ld, n in zip(loads, iters):
        ld.stream.wait_event(start)
        ld.run(n)
        e = torch.cuda.Event(enable_timing=True)
        e.record(ld.stream)
        ends.append(e)
    torch.cuda.synchronize()
    return [start.elapsed_time(e) for e in ends]


def corun(gemm_sms: int = 72, moe_sms: int = 72, moe_tokens: int = 128, size: int = 4096, iters: int = 20,
          stressor_sms: int = 0, stressor_mb: int = 1024, verbose: bool = True) -> dict:
    """Run the GEMM (size^3 bf16) and the Mixtral-shaped MoE layer (moe_tokens
    tokens) alone and together in disjoint partitions; with stressor_sms > 0 a
    third partition copies a stressor_mb buffer back and forth meanwhile.
    Returns per-load solo / co-run times, slow-downs and rates, and whether the
    co-run outputs equal the solo outputs bit for bit."""
    dev = torch.device("cuda:0")
    total = get_total_sm_count(dev)
    counts = [gemm_sms, moe_sms] + ([stressor_sms] if stressor_sms > 0 else [])
    parts = create_disjoint_partitions(dev, counts)
    (s_gemm, n_gemm), (s_moe, n_moe) = parts[0], parts[1]

    g = torch.Generator(device=dev).manual_seed(0)
    a = torch.randn((size, size), device=dev, generator=g).to(torch.bfloat16)
    b = torch.randn((size, size), device=dev, generator=g).to(torch.bfloat16)
    c = torch.empty((size, size), device=dev, dtype=torch.bfloat16)
    E, k, H, I = 8, 2, 4096, 14336
    gm = torch.Generator(device=dev).manual_seed(42)
    w1 = (torch.randn((E, I, H), device=dev, generator=gm) * 0.02).to(torch.bfloat16)
    w3 = (torch.randn((E, I, H), device=dev, generator=gm) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn((E, H, I), device=dev, generator=gm) * 0.02).to(torch.bfloat16)
    x = torch.randn((moe_tokens, H), device=dev, generator=gm).to(torch.bfloat16)
    logits = torch.randn((moe_tokens, E), device=dev, generator=gm)
    y = torch.empty((moe_tokens, H), device=dev, dtype=torch.bfloat16)

    loads = [
        _Load("gemm", s_gemm, lambda: _ops.gemm(a, b, out=c, num_sms=n_gemm), flop_per_call=2.0 * size ** 3),
        _Load("moe", s_moe, lambda: _ops.fused_moe(x, logits, w1, w2, w3, k, out=y, num_sms=n_moe),
              tokens_per_call=moe_tokens),
    ]
    if stressor_sms > 0:
        s_str, n_str = parts[2]
        src = torch.empty(stressor_mb << 20, dtype=torch.uint8, device=dev)
        dst = torch.empty_like(src)
        loads.append(_Load("stressor", s_str, lambda: dst.copy_(src)))

    # solo references (and their outputs)
    solo = [_time_alone(ld, iters) for ld in loads]
    c_solo, y_solo = c.clone(), y.clone()
    # co-run: every load gets the iteration count that keeps it busy about as
    # long as the longest solo run, so the loads overlap for the whole window
    longest = max(solo)
    co_iters = [max(1, int(round(iters * longest / max(t, 1e-3)))) for t in solo]
    together = _time_together(loads, co_iters)
    same = bool(torch.equal(c, c_solo) and torch.equal(y, y_solo))

    res = {"total_sms": total, "sms": {"gemm": n_gemm, "moe": n_moe}, "iters": iters, "outputs_equal": same}
    for ld, t1, t2, n in zip(loads, solo, together, co_iters):
        per_solo, per_co = t1 / iters, t2 / n
        r = {"solo_ms_per_call": per_solo, "corun_ms_per_call": per_co, "slowdown": per_co / per_solo}
        if ld.flop:
            r["solo_tflops"] = ld.flop / (per_solo * 1e9)
            r["corun_tflops"] = ld.flop / (per_co * 1e9)
        if ld.tokens:
            r["solo_tokens_per_s"] = ld.tokens / (per_solo * 1e-3)
            r["corun_tokens_per_s"] = ld.tokens / (per_co * 1e-3)
        if ld.name == "stressor":
            r["sms"] = parts[2][1]
            r["solo_gbs"] = 2.0 * stressor_mb * (1 << 20) / (per_solo * 1e6)
            r["corun_gbs"] = 2.0 * stressor_mb * (1 << 20) / (per_co * 1e6)
        res[ld.name] = r
    if verbose:
        print(f"Device SMs: {total}; partitions: GEMM {n_gemm}, MoE {n_moe}"
              + (f", stressor {parts[2][1]}" if stressor_sms > 0 else ""))
        for ld in loads:
            r = res[ld.name]
            extra = ""
            if "solo_tflops" in r:
                extra = f"  {r['solo_tflops']:.0f} -> {r['corun_tflops']:.0f} TFLOP/s"
            elif "solo_tokens_per_s" in r:
                extra = f"  {r['solo_tokens_per_s']:.0f} -> {r['corun_tokens_per_s']:.0f} tokens/s"
            elif "solo_gbs" in r:
                extra = f"  {r['solo_gbs']:.0f} -> {r['corun_gbs']:.0f} GB/s"
            print(f"  {ld.name:9s} solo {r['solo_ms_per_call'] * 1e3:9.1f} us  co-run "
                  f"{r['corun_ms_per_call'] * 1e3:9.1f} us  slow-down {r['slowdown']:.2f}x{extra}")
        print(f"  outputs equal to the solo runs: {same}")
    return res


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gemm-sms", type=int, default=72)
    ap.add_argument("--moe-sms", type=int, default=72)
    ap.add_argument("--moe-tokens", type=int, default=128)
    ap.add_argument("--size", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--stressor-sms", type=int, default=0)
    ap.add_argument("--stressor-mb", type=int, default=1024)
    a = ap.parse_args()
    corun(a.gemm_sms, a.moe_sms, a.moe_tokens, a.size, a.iters, a.stressor_sms, a.stressor_mb)


if __name__ == "__main__":
    main()
