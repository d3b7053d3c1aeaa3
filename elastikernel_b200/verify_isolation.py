"""SM-isolation check of green-context partitions, with the partition-planned
tcgen05 GEMM as the load (drop-in for elastikernel/verify_isolation.py: the
module name, `main()` and the three pass thresholds are the reference's,
verify_isolation.py:128,160,200).

Two pairs of half-device partitions are compared: a disjoint pair from
create_disjoint_partitions and an overlapping pair, two splits of the full
device from create_sm_partition. Each partition repeats one GEMM; the timing
reuses the co-run harness (corun._time_alone, corun._time_together): each
load alone, then both from one start event. If the SM sets are disjoint the
pair runs about twice as fast together as back to back; if they overlap, about
as fast. Every partition's product is also checked against an fp32 product.

Usage:
    python -m elastikernel_b200.verify_isolation [--size 4096] [--iters 20]
"""
from __future__ import annotations

import argparse
from dataclasses import asdict, dataclass

import torch

from . import _ops, corun
from .green_ctx import create_disjoint_partitions, create_sm_partition, get_sm_alignment, get_total_sm_count

# Pass thresholds of the reference's check.
DISJOINT_MIN_GAIN = 1.5   # disjoint pair: together vs back to back
OVERLAP_MAX_GAIN = 1.3    # overlapping pair: expected to stay below
ISOLATION_MIN_RATIO = 1.5  # disjoint gain / overlapping gain


@dataclass
class PairResult:
    kind: str                # "disjoint" or "overlapping"
    sms: tuple               # actual SM counts of the two partitions
    solo_ms: tuple           # each load alone (iters GEMMs)
    together_ms: float       # both from a common start, until the later one ends
    gain: float              # sum(solo_ms) / together_ms
    max_rel_err: tuple       # per partition, vs an fp32 product


def _run_pair(kind: str, parts, a, b, ref, iters: int) -> PairResult:
    outs = [torch.empty((a.shape[0], b.shape[1]), device=a.device, dtype=a.dtype) for _ in parts]
    loads = [corun._Load(f"{kind}-{i}", stream, (lambda o=outs[i], n=sms: _ops.gemm(a, b, out=o, num_sms=n)),
                         flop_per_call=2.0 * a.shape[0] * a.shape[1] * b.shape[1])
             for i, (stream, sms) in enumerate(parts)]
    solo = tuple(corun._time_alone(ld, iters) for ld in loads)
    together = max(corun._time_together(loads, [iters] * len(loads)))
    denom = ref.abs().max()
    errs = tuple(float(((o.float() - ref).abs().max() / denom).item()) for o in outs)
    return PairResult(kind, tuple(n for _, n in parts), solo, together, sum(solo) / together, errs)


def check_isolation(size: int = 4096, iters: int = 20, device: str = "cuda:0") -> dict:
    """Time both pairs and return the structured result (no printing)."""
    dev = torch.device(device)
    total = get_total_sm_count(dev)
    _, align = get_sm_alignment(dev)
    half = (total // 2 // align) * align
    g = torch.Generator(device=dev).manual_seed(0)
    a = torch.randn((size, size), device=dev, generator=g).to(torch.bfloat16)
    b = torch.randn((size, size), device=dev, generator=g).to(torch.bfloat16)
    ref = a.float() @ b.float()
    disjoint = _run_pair("disjoint", create_disjoint_partitions(dev, [half, half]), a, b, ref, iters)
    overlapping = _run_pair("overlapping", [create_sm_partition(dev, half), create_sm_partition(dev, half)],
                            a, b, ref, iters)
    ratio = disjoint.gain / overlapping.gain
    correct = max(disjoint.max_rel_err + overlapping.max_rel_err) <= 1e-2
    return {
        "device": torch.cuda.get_device_name(dev), "total_sms": total, "half_sms": half, "size": size, "iters": iters,
        "disjoint": asdict(disjoint), "overlapping": asdict(overlapping), "isolation_ratio": ratio,
        "disjoint_pass": disjoint.gain > DISJOINT_MIN_GAIN, "overlap_as_expected": overlapping.gain < OVERLAP_MAX_GAIN,
        "correct": correct, "isolated": ratio > ISOLATION_MIN_RATIO and correct,
        # flat keys kept for callers of the earlier result layout
        "speedup_disjoint": disjoint.gain, "speedup_overlap": overlapping.gain,
        "max_rel_err": list(disjoint.max_rel_err + overlapping.max_rel_err),
    }


def report(r: dict) -> str:
    lines = [f"SM isolation on {r['device']} ({r['total_sms']} SMs): {r['size']}^3 bf16 tcgen05 GEMM x{r['iters']} "
             f"per partition, partitions of {r['half_sms']} SMs requested"]
    for key, bound in (("disjoint", f"> {DISJOINT_MIN_GAIN}x to pass"),
                       ("overlapping", f"< {OVERLAP_MAX_GAIN}x expected")):
        p = r[key]
        lines.append(f"  {key:<11} SMs {p['sms'][0]}+{p['sms'][1]}: alone {p['solo_ms'][0]:.2f} / "
                     f"{p['solo_ms'][1]:.2f} ms, together {p['together_ms']:.2f} ms -> gain {p['gain']:.2f}x "
                     f"({bound}); max rel err {max(p['max_rel_err']):.1e}")
    lines.append(f"  gain ratio disjoint / overlapping: {r['isolation_ratio']:.2f}x "
                 f"(> {ISOLATION_MIN_RATIO}x means the disjoint SM sets do not share SMs)")
    lines.append("  result: " + ("isolated" if r["isolated"] else
                                 "not shown (" + ("products wrong" if not r["correct"] else
                                                  "loads limited by shared HBM/L2, or SMs shared") + ")"))
    return "\n".join(lines)


def main(size: int = 4096, iters: int = 20) -> dict:
    """Run the check, print the report and return the structured result.
    The default product is 4096^3: a 2048^3 GEMM on half the device takes
    ~40 us, close to the per-call launch cost, which would then be measured."""
    r = check_isolation(size, iters)
    print(report(r))
    return r


if __name__ == "__main__":
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--size", type=int, default=4096)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    main(args.size, args.iters)
