"""Verify that disjoint green-context partitions isolate SMs, with the tcgen05
GEMM as the load (drop-in for elastikernel/verify_isolation.py).

Method (verify_isolation.py:87-204): two disjoint partitions of half the
device each; time 20 GEMMs on A alone, B alone and both at once. Disjoint SM
sets give parallel ~ solo (speed-up ~2x over running them back to back);
two partitions split from the full device overlap and give ~1x. The
reference used cuBLAS; here the load is the partition-planned tcgen05 GEMM,
and correctness is checked against an fp32 product (max rel err <= 1e-2).

Usage:
    python -m elastikernel_b200.verify_isolation
"""
from __future__ import annotations

import torch

from . import sm_aware_matmul as smm
from .green_ctx import create_disjoint_partitions, create_sm_partition, get_sm_alignment, get_total_sm_count


def make_workload(dev, size=4096):
    a = torch.randn(size, size, device=dev, dtype=torch.bfloat16)
    b = torch.randn(size, size, device=dev, dtype=torch.bfloat16)
    return a, b


def bench_single_stream(stream, a, b, num_sms, iters=20):
    """Device time of `iters` GEMMs on one partition stream (ms)."""
    with torch.cuda.stream(stream):
        for _ in range(3):
            smm.call_sm_aware(a, b, num_sms)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(iters):
            smm.call_sm_aware(a, b, num_sms)
        end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end)


def bench_parallel_streams(stream_a, stream_b, sms_a, sms_b, a1, b1, a2, b2, iters=20):
    """Both partitions at once; returns the later finish time (ms) from a common start."""
    with torch.cuda.stream(stream_a):
        for _ in range(3):
            smm.call_sm_aware(a1, b1, sms_a)
    with torch.cuda.stream(stream_b):
        for _ in range(3):
            smm.call_sm_aware(a2, b2, sms_b)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end_a = torch.cuda.Event(enable_timing=True)
    end_b = torch.cuda.Event(enable_timing=True)
    start.record()
    # both partition streams wait on the common start
    stream_a.wait_event(start)
    stream_b.wait_event(start)
    with torch.cuda.stream(stream_a):
        for _ in range(iters):
            smm.call_sm_aware(a1, b1, sms_a)
        end_a.record(stream_a)
    with torch.cuda.stream(stream_b):
        for _ in range(iters):
            smm.call_sm_aware(a2, b2, sms_b)
        end_b.record(stream_b)
    torch.cuda.synchronize()
    return max(start.elapsed_time(end_a), start.elapsed_time(end_b))


def main(size: int = 4096, iters: int = 20) -> dict:
    """Run the three checks. The reference used 2048^2 cuBLAS GEMMs; the
    tcgen05 GEMM finishes a 2048^2 product on half the device in ~40 us, close
    to the host's per-call launch cost, so the default here is 4096^2 to keep
    the comparison about the GPU rather than the launching thread."""
    dev = torch.device("cuda:0")
    total_sms = get_total_sm_count(dev)
    min_sm, align = get_sm_alignment(dev)
    print(f"Device: {torch.cuda.get_device_name(dev)}")
    print(f"Total SMs: {total_sms}, alignment: min={min_sm}, align={align}")
    half_sms = (total_sms // 2 // align) * align
    print(f"\nPartition size: {half_sms} SMs each (total used: {half_sms * 2}/{total_sms})")
    a1, b1 = make_workload(dev, size)
    a2, b2 = make_workload(dev, size)

    print(f"\n{'=' * 70}\nTEST 1: DISJOINT partitions (create_disjoint_partitions)\n{'=' * 70}")
    (stream_a, actual_a), (stream_b, actual_b) = create_disjoint_partitions(dev, [half_sms, half_sms])
    print(f"  Partition A: {actual_a} SMs\n  Partition B: {actual_b} SMs")
    t_a = bench_single_stream(stream_a, a1, b1, actual_a, iters)
    t_b = bench_single_stream(stream_b, a2, b2, actual_b, iters)
    t_par = bench_parallel_streams(stream_a, stream_b, actual_a, actual_b, a1, b1, a2, b2, iters)
    speedup = (t_a + t_b) / t_par
    print(f"\n  A solo:     {t_a:8.2f} ms\n  B solo:     {t_b:8.2f} ms\n  Parallel:   {t_par:8.2f} ms")
    print(f"  Sequential: {t_a + t_b:8.2f} ms\n  Speedup (seq/parallel): {speedup:.2f}x")
    print(f"  Parallel/AvgSolo ratio: {t_par / ((t_a + t_b) / 2):.2f}x")
    if speedup > 1.5:
        print(f"\n  >> PASS: Speedup {speedup:.2f}x indicates true SM isolation")
    else:
        print(f"\n  >> WARN: Speedup only {speedup:.2f}x -- possible SM overlap or memory bandwidth bottleneck")

    print(f"\n{'=' * 70}\nTEST 2: OVERLAPPING partitions (create_sm_partition x2)\n{'=' * 70}")
    stream_c, actual_c = create_sm_partition(dev, half_sms)
    stream_d, actual_d = create_sm_partition(dev, half_sms)
    print(f"  Partition C: {actual_c} SMs (from full device)\n  Partition D: {actual_d} SMs (from full device)")
    t_c = bench_single_stream(stream_c, a1, b1, actual_c, iters)
    t_d = bench_single_stream(stream_d, a2, b2, actual_d, iters)
    t_ov = bench_parallel_streams(stream_c, stream_d, actual_c, actual_d, a1, b1, a2, b2, iters)
    speedup_2 = (t_c + t_d) / t_ov
    print(f"\n  C solo:     {t_c:8.2f} ms\n  D solo:     {t_d:8.2f} ms\n  Parallel:   {t_ov:8.2f} ms")
    print(f"  Sequential: {t_c + t_d:8.2f} ms\n  Speedup (seq/parallel): {speedup_2:.2f}x")
    if speedup_2 < 1.3:
        print(f"\n  >> EXPECTED: Speedup only {speedup_2:.2f}x -- SMs overlap, kernels contend")
    else:
        print(f"\n  >> UNEXPECTED: Speedup {speedup_2:.2f}x -- overlapping partitions show parallelism")

    print(f"\n{'=' * 70}\nTEST 3: Correctness check\n{'=' * 70}")
    ref = a1.float() @ b1.float()
    with torch.cuda.stream(stream_a):
        out_a = smm.call_sm_aware(a1, b1, actual_a)
    with torch.cuda.stream(stream_b):
        out_b = smm.call_sm_aware(a1, b1, actual_b)
    torch.cuda.synchronize()
    denom = ref.abs().max()
    err_a = ((out_a.float() - ref).abs().max() / denom).item()
    err_b = ((out_b.float() - ref).abs().max() / denom).item()
    ok = err_a <= 1e-2 and err_b <= 1e-2
    print(f"  Partition A max rel err: {err_a:.2e}\n  Partition B max rel err: {err_b:.2e}")
    print("  >> PASS: Both partitions produce correct results" if ok else "  >> FAIL: Result mismatch!")

    print(f"\n{'=' * 70}\nSUMMARY\n{'=' * 70}")
    print(f"  Disjoint partitions parallel speedup:    {speedup:.2f}x (expect ~2.0x)")
    print(f"  Overlapping partitions parallel speedup:  {speedup_2:.2f}x (expect ~1.0x)")
    print(f"  Isolation ratio (disjoint/overlapping):   {speedup / speedup_2:.2f}x")
    verdict = speedup > 1.5 * speedup_2
    print("\n  VERDICT: Green Context disjoint partitions provide real SM isolation." if verdict else
          "\n  VERDICT: Results inconclusive -- may be memory-bandwidth bound.")
    return {"half_sms": half_sms, "actual": [actual_a, actual_b, actual_c, actual_d], "solo_ms": [t_a, t_b, t_c, t_d],
            "parallel_disjoint_ms": t_par, "parallel_overlap_ms": t_ov, "speedup_disjoint": speedup,
            "speedup_overlap": speedup_2, "max_rel_err": [err_a, err_b], "isolated": verdict and ok}


if __name__ == "__main__":
    main()
