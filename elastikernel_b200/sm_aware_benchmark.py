"""SM-aware kernel benchmark suite (drop-in for elastikernel/sm_aware_benchmark.py).

Usage:
    python -m elastikernel_b200.sm_aware_benchmark --gemm
    python -m elastikernel_b200.sm_aware_benchmark --moe
    python -m elastikernel_b200.sm_aware_benchmark --all

GEMM: vanilla (planned for the full device) vs SM-aware (planned for the
partition) tcgen05 GEMM under green-context partitions, with the wave
analysis of the schedule actually run (sm_aware_benchmark.py:17-181).

MoE: the reference's segment "fused MoE" (grouped GEMM over CSR expert
segments with its fake contiguous routing, sm_aware_benchmark.py:184-468),
vanilla vs SM-aware, plus the full fused-MoE layer (routing, permutation,
SwiGLU gate/up, weighted down-projection, combine) at Mixtral shapes.
"""
from __future__ import annotations

import argparse


def call_moe_vanilla(hidden_states, weights, expert_offsets, num_experts, N, K):
    """Segment GEMM with the reference kernel's semantics (sm_aware_benchmark.py:351-370),
    planned for the full device."""
    import torch

    from . import _ops

    total = torch.cuda.get_device_properties(hidden_states.device).multi_processor_count
    return _ops.moe_segment_gemm(hidden_states, weights, expert_offsets, num_experts, N, K, num_sms=total)


def call_moe_sm_aware(hidden_states, weights, expert_offsets, num_experts, N, K, num_sms=None):
    """Segment GEMM planned for `num_sms` SMs (None: the current stream's partition)
    (sm_aware_benchmark.py:372-391)."""
    from . import _ops

    return _ops.moe_segment_gemm(hidden_states, weights, expert_offsets, num_experts, N, K, num_sms=num_sms)


def _partition(dev, sm_count, total):
    from .green_ctx import create_sm_partition, full_device_partition

    if sm_count >= total:
        return full_device_partition(dev)
    return create_sm_partition(dev, sm_count)


def run_gemm_benchmark(sm_levels=None, test_cases=None, rep_ms: float = 30.0) -> list:
    """Vanilla vs SM-aware GEMM per partition size (sm_aware_benchmark.py:17-181)."""
    import torch

    from . import sm_aware_matmul as smm
    from .green_ctx import get_sm_alignment, get_total_sm_count
    from .timing import time_on_stream

    dev = torch.device("cuda:0")
    total_sms = get_total_sm_count(dev)
    min_sm, align = get_sm_alignment(dev)
    print(f"GEMM Benchmark on {torch.cuda.get_device_name(dev)}")
    print(f"Total SMs: {total_sms}, alignment: min={min_sm}, align={align}")
    sm_levels = [s for s in (sm_levels or [16, 32, 48, 64, 96, 132, total_sms]) if s <= total_sms]
    square_cases = [(1024, 1024, 1024), (2048, 2048, 2048), (4096, 4096, 4096)]
    m_sweep_cases = [(M, 4096, 4096) for M in [1, 16, 32, 64, 128, 256, 512, 1024, 2048]]
    results = []
    for M, N, K in test_cases or (square_cases + m_sweep_cases):
        print(f"\n{'=' * 80}\nGEMM: M={M}, N={N}, K={K}\n{'=' * 80}")
        print(f"  {'SM':>4} {'Vanilla(us)':>11} {'Aware(us)':>11} {'Speedup':>8}  {'TFLOP/s':>8}  schedule")
        torch.manual_seed(0)
        a = torch.randn((M, K), device=dev, dtype=torch.bfloat16)
        b = torch.randn((K, N), device=dev, dtype=torch.bfloat16)
        for sm_count in sm_levels:
            try:
                stream, actual = _partition(dev, sm_count, total_sms)
                with torch.cuda.stream(stream):
                    for _ in range(3):
                        smm.call_vanilla(a, b)
                        smm.call_sm_aware(a, b, actual)
                    van = time_on_stream(lambda: smm.call_vanilla(a, b), stream, rep_ms=rep_ms)
                    aw = time_on_stream(lambda: smm.call_sm_aware(a, b, actual), stream, rep_ms=rep_ms)
                p = smm.tcgen05_schedule(M, N, K, actual)
                sp = van["mean_ms"] / aw["mean_ms"] if aw["mean_ms"] > 0 else 0.0
                tf = 2.0 * M * N * K / (aw["mean_ms"] * 1e-3) / 1e12
                mode = f"{p['bm']}x{p['bn']}{' pair' if p['cta_pair'] else ''} split={p['tail_split']}"
                print(f"  {sm_count:>4} {van['mean_ms'] * 1e3:>11.1f} {aw['mean_ms'] * 1e3:>11.1f} {sp:>7.2f}x  "
                      f"{tf:>8.1f}  {mode} eff={p['wave_efficiency'] * 100:.1f}%")
                results.append({"M": M, "N": N, "K": K, "sm": sm_count, "actual": actual,
                                "vanilla_us": van["mean_ms"] * 1e3, "aware_us": aw["mean_ms"] * 1e3,
                                "tflops": tf, "plan": p})
            except Exception as e:
                print(f"  {sm_count:>4}  Error: {e}")
    return results


def _fake_offsets(num_tokens, num_experts, top_k, dev):
    """The reference's uniform fake routing (sm_aware_benchmark.py:438-444)."""
    import torch

    tpe = (num_tokens * top_k) // num_experts
    offs = [0] + [min((i + 1) * tpe, num_tokens) for i in range(num_experts)]
    offs[-1] = num_tokens
    return torch.tensor(offs, dtype=torch.int32, device=dev)


def run_moe_benchmark(sm_levels=None, moe_configs=None, rep_ms: float = 30.0, full_layer: bool = True) -> list:
    """Segment-GEMM MoE of the reference, vanilla vs SM-aware, per partition
    size; then the full fused-MoE layer at Mixtral shapes."""
    import torch

    from . import _ops
    from .green_ctx import get_sm_alignment, get_total_sm_count
    from .timing import time_on_stream

    dev = torch.device("cuda:0")
    total_sms = get_total_sm_count(dev)
    min_sm, align = get_sm_alignment(dev)
    print(f"\n{'=' * 80}\nFused MoE Benchmark on {torch.cuda.get_device_name(dev)}")
    print(f"Total SMs: {total_sms}, alignment: min={min_sm}, align={align}\n{'=' * 80}")
    sm_levels = [s for s in (sm_levels or [16, 32, 48, 64, total_sms]) if s <= total_sms]
    moe_configs = moe_configs or [
        {"num_tokens": 128, "hidden_dim": 4096, "intermediate_dim": 4096, "num_experts": 8, "top_k": 2},
        {"num_tokens": 512, "hidden_dim": 4096, "intermediate_dim": 4096, "num_experts": 8, "top_k": 2},
        {"num_tokens": 1024, "hidden_dim": 4096, "intermediate_dim": 4096, "num_experts": 8, "top_k": 2},
        {"num_tokens": 512, "hidden_dim": 4096, "intermediate_dim": 4096, "num_experts": 16, "top_k": 4},
    ]
    results = []
    for cfg in moe_configs:
        T, K, N = cfg["num_tokens"], cfg["hidden_dim"], cfg["intermediate_dim"]
        E, k = cfg["num_experts"], cfg["top_k"]
        print(f"\n{'=' * 80}\nMoE segment GEMM: tokens={T}, hidden={K}, intermediate={N}, experts={E}, top_k={k}")
        print(f"  {'SM':>4} {'Vanilla(us)':>11} {'Aware(us)':>11} {'Speedup':>8}")
        torch.manual_seed(42)
        hs = torch.randn((T, K), device=dev, dtype=torch.bfloat16)
        w = torch.randn((E * N, K), device=dev, dtype=torch.bfloat16)
        offs = _fake_offsets(T, E, k, dev)
        for sm_count in sm_levels:
            try:
                stream, actual = _partition(dev, sm_count, total_sms)
                with torch.cuda.stream(stream):
                    for _ in range(3):
                        call_moe_vanilla(hs, w, offs, E, N, K)
                        call_moe_sm_aware(hs, w, offs, E, N, K, actual)
                    van = time_on_stream(lambda: call_moe_vanilla(hs, w, offs, E, N, K), stream, rep_ms=rep_ms)
                    aw = time_on_stream(lambda: call_moe_sm_aware(hs, w, offs, E, N, K, actual), stream,
                                        rep_ms=rep_ms)
                sp = van["mean_ms"] / aw["mean_ms"] if aw["mean_ms"] > 0 else 0.0
                print(f"  {sm_count:>4} {van['mean_ms'] * 1e3:>11.1f} {aw['mean_ms'] * 1e3:>11.1f} {sp:>7.2f}x")
                results.append({"kind": "segment", **cfg, "sm": sm_count, "actual": actual,
                                "vanilla_us": van["mean_ms"] * 1e3, "aware_us": aw["mean_ms"] * 1e3})
            except Exception as e:
                print(f"  {sm_count:>4}  Error: {e}")
    if full_layer:
        E, k, H, I = 8, 2, 4096, 14336
        print(f"\n{'=' * 80}\nFused MoE layer (Mixtral: E={E}, top-{k}, H={H}, I={I}, bf16)")
        print(f"  {'T':>5} {'SM':>4} {'us':>9} {'tokens/s':>12} {'TFLOP/s':>8}")
        g = torch.Generator(device=dev).manual_seed(42)
        w1 = (torch.randn((E, I, H), device=dev, generator=g) * 0.02).to(torch.bfloat16)
        w3 = (torch.randn((E, I, H), device=dev, generator=g) * 0.02).to(torch.bfloat16)
        w2 = (torch.randn((E, H, I), device=dev, generator=g) * 0.02).to(torch.bfloat16)
        for T in [1, 16, 128, 1024, 4096]:
            x = torch.randn((T, H), device=dev, generator=g).to(torch.bfloat16)
            logits = torch.randn((T, E), device=dev, generator=g)
            for sm_count in (total_sms, total_sms // 2):
                try:
                    stream, actual = _partition(dev, sm_count, total_sms)
                    with torch.cuda.stream(stream):
                        for _ in range(2):
                            _ops.fused_moe(x, logits, w1, w2, w3, k)
                        r = time_on_stream(lambda: _ops.fused_moe(x, logits, w1, w2, w3, k), stream, rep_ms=rep_ms)
                    t = r["mean_ms"] * 1e-3
                    tf = T * k * 6.0 * H * I / t / 1e12
                    print(f"  {T:>5} {actual:>4} {r['mean_ms'] * 1e3:>9.1f} {T / t:>12.1f} {tf:>8.1f}")
                    results.append({"kind": "layer", "T": T, "sm": sm_count, "actual": actual,
                                    "us": r["mean_ms"] * 1e3, "tokens_per_s": T / t, "tflops": tf})
                except Exception as e:
                    print(f"  {T:>5} {sm_count:>4}  Error: {e}")
    return results


def run_layer(tokens: int, reps: int = 5, num_sms: int | None = None, layout: str = "packed") -> None:
    """Run the Mixtral-shaped fused-MoE layer at `tokens` tokens a few times
    (no timing; a fixed launch sequence for profilers)."""
    import torch

    from . import _ops

    dev = torch.device("cuda:0")
    E, k, H, I = 8, 2, 4096, 14336
    g = torch.Generator(device=dev).manual_seed(42)
    w1 = (torch.randn((E, I, H), device=dev, generator=g) * 0.02).to(torch.bfloat16)
    w3 = (torch.randn((E, I, H), device=dev, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn((E, H, I), device=dev, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn((tokens, H), device=dev, generator=g).to(torch.bfloat16)
    logits = torch.randn((tokens, E), device=dev, generator=g)
    for _ in range(reps):
        _ops.fused_moe(x, logits, w1, w2, w3, k, num_sms=num_sms, layout=layout)
    torch.cuda.synchronize()


def run_layer_fp8(tokens: int, reps: int = 3, experts: int = 256, pow2: bool = False, timed: bool = False) -> None:
    """Run the DeepSeek-V3-shaped e4m3 block-scaled MoE layer (top-8, H=7168,
    I=2048) with all `experts` on this GPU a few times (for profilers).
    pow2: power-of-two scales and the GEMMs whose tensor cores apply them.
    timed: also print the layer's device time (CUDA events, L2 flushed)."""
    import torch

    from . import _ops
    from .timing import time_on_stream

    dev = torch.device("cuda:0")
    E, k, H, I = experts, 8, 7168, 2048
    g = torch.Generator(device=dev).manual_seed(1000)
    qs = []
    for c0 in range(0, E, 32):
        n = min(32, E - c0)
        w1 = (torch.randn((n, I, H), device=dev, generator=g) * 0.02).to(torch.bfloat16)
        w3 = (torch.randn((n, I, H), device=dev, generator=g) * 0.02).to(torch.bfloat16)
        w2 = (torch.randn((n, H, I), device=dev, generator=g) * 0.02).to(torch.bfloat16)
        qs.append(_ops.quant_moe_weights_fp8(w1, w2, w3, pow2=pow2))
        del w1, w2, w3
    qw = {"E": E, "I": I, "H": H, "pow2": pow2}
    for key in ("w1q", "w1s", "w3q", "w3s", "w2q", "w2s"):
        qw[key] = torch.cat([q[key] for q in qs], dim=0)
    del qs
    qw = _ops.stack_gate_up_planes(qw)
    x = torch.randn((tokens, H), device=dev, generator=g).to(torch.bfloat16)
    logits = torch.randn((tokens, E), device=dev, generator=g)
    for _ in range(reps):
        _ops.fused_moe_fp8(x, logits, qw, k)
    torch.cuda.synchronize()
    if timed:
        r = time_on_stream(lambda: _ops.fused_moe_fp8(x, logits, qw, k), reps=max(reps, 5))
        flop = tokens * k * 6.0 * H * I
        print(f"DSv3 FP8 layer T={tokens} E={E} scales={'pow2/tensor-core' if pow2 else 'fp32/epilogue'}: "
              f"{r['mean_ms'] * 1e3:.1f} us mean, {r['median_ms'] * 1e3:.1f} us median, "
              f"{flop / (r['mean_ms'] * 1e-3) / 1e12:.0f} TFLOP/s")


HBM_SPEC_GBS = 8000.0  # B200 HBM3e spec-sheet bandwidth


def run_stages(tokens: int, experts: int, topk: int, hidden: int, inter: int = 2048, reps: int = 20) -> list:
    """Time the memory-bound MoE stages one by one -- routing, permutation
    (count + stable scatter), row gather, e4m3 quantisation of the token rows
    and of the activations (1 x 128 groups) and top-k combine -- at `tokens`
    tokens, with their algorithmic bytes and GB/s (L2 flushed before each
    repetition)."""
    import torch

    from . import _ops
    from .timing import time_on_stream

    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(42)
    T, E, k, H = tokens, experts, topk, hidden
    logits = torch.randn((T, E), device=dev, generator=g)
    x = torch.randn((T, H), device=dev, generator=g).to(torch.bfloat16)
    y = torch.randn((T * k, H), device=dev, generator=g).to(torch.bfloat16)
    act = torch.randn((T * k, inter), device=dev, generator=g).to(torch.bfloat16)
    ids, _ = _ops.moe_route(logits, k)
    perm = _ops.moe_permute(ids, E, x)
    used = int(perm["num_rows_padded"].item())
    slots = T * k
    stages = [
        ("route", lambda: _ops.moe_route(logits, k), T * E * 4 + slots * 8),
        ("permute", lambda: _ops.moe_permute(ids, E), slots * 4 + perm["max_rows"] * 4),
        ("permute+gather", lambda: _ops.moe_permute(ids, E, x), slots * 4 + perm["max_rows"] * 4 + 2 * slots * H * 2),
        ("quant tokens", lambda: _ops.quant_e4m3(x, block=(1, 128)), T * H * 3 + T * (H // 128) * 4),
        ("quant act", lambda: _ops.quant_e4m3_kmajor(act), slots * inter * 3 + slots * (inter // 128) * 4),
        ("combine", lambda: _ops.moe_combine(y, T, k), slots * H * 2 + T * H * 2),
    ]
    print(f"MoE stages: T={T}, E={E}, top-{k}, H={H}, I={inter} (bf16 rows; {used} padded rows)")
    print(f"  {'stage':<16} {'us':>9} {'MB':>9} {'GB/s':>8} {'% 8TB/s':>8}")
    out = []
    for name, fn, nbytes in stages:
        for _ in range(3):
            fn()
        r = time_on_stream(fn, reps=reps)
        us = r["median_ms"] * 1e3
        gbs = nbytes / (us * 1e-6) / 1e9
        print(f"  {name:<16} {us:>9.1f} {nbytes / 1e6:>9.1f} {gbs:>8.0f} {100 * gbs / HBM_SPEC_GBS:>7.1f}%")
        out.append({"stage": name, "us": us, "bytes": nbytes, "gbs": gbs})
    return out


def run_gemm_shape(M: int, N: int, K: int, dtype: str = "bf16", sm_count: int = 0, reps: int = 3) -> None:
    """Run one GEMM shape a few times in a partition of `sm_count` SMs (0: the
    whole device); bf16 is A[M,K] @ B[K,N], fp8 is e4m3 A[M,K] x W[N,K]^T with
    per-row / per-channel scales (a fixed launch sequence for profilers)."""
    import torch

    from . import _ops
    from . import sm_aware_matmul as smm
    from .green_ctx import get_total_sm_count

    dev = torch.device("cuda:0")
    total = get_total_sm_count(dev)
    stream, actual = _partition(dev, sm_count or total, total)
    g = torch.Generator(device=dev).manual_seed(0)
    with torch.cuda.stream(stream):
        if dtype == "fp8":
            aq, a_s = _ops.quant_e4m3(torch.randn((M, K), device=dev, generator=g))
            wq, w_s = _ops.quant_e4m3(torch.randn((N, K), device=dev, generator=g))
            fn = lambda: _ops.gemm_fp8(aq, wq, a_s, w_s)  # noqa: E731
        else:
            a = torch.randn((M, K), device=dev, generator=g).to(torch.bfloat16)
            b = torch.randn((K, N), device=dev, generator=g).to(torch.bfloat16)
            fn = lambda: smm.call_sm_aware(a, b, actual)  # noqa: E731
        for _ in range(reps):
            fn()
    torch.cuda.synchronize()
    print(f"GEMM {dtype} {M}x{N}x{K} on {actual} SMs: {reps} launches")


def main():
    parser = argparse.ArgumentParser(description="SM-Aware Kernel Benchmark")
    parser.add_argument("--gemm", action="store_true", help="Benchmark GEMM")
    parser.add_argument("--moe", action="store_true", help="Benchmark Fused MoE")
    parser.add_argument("--all", action="store_true", help="Benchmark all operators")
    parser.add_argument("--layer-tokens", type=int, default=0,
                        help="only run the Mixtral fused-MoE layer at this token count (for profiling)")
    parser.add_argument("--reps", type=int, default=5)
    parser.add_argument("--layout", choices=["packed", "padded"], default="packed")
    parser.add_argument("--fp8-layer-tokens", type=int, default=0,
                        help="only run the DeepSeek-V3-shaped e4m3 MoE layer at this token count (for profiling)")
    parser.add_argument("--pow2", action="store_true",
                        help="--fp8-layer-tokens: power-of-two scales applied by the tensor cores")
    parser.add_argument("--timed", action="store_true", help="--fp8-layer-tokens: print the layer's device time")
    parser.add_argument("--experts", type=int, default=256,
                        help="experts on this GPU for --fp8-layer-tokens / --stages-tokens")
    parser.add_argument("--stages-tokens", type=int, default=0,
                        help="time routing, permutation, gather and combine at this token count")
    parser.add_argument("--topk", type=int, default=8, help="top-k for --stages-tokens")
    parser.add_argument("--hidden", type=int, default=7168, help="hidden size for --stages-tokens")
    parser.add_argument("--inter", type=int, default=2048, help="expert intermediate size for --stages-tokens")
    parser.add_argument("--gemm-shape", type=int, nargs=3, metavar=("M", "N", "K"),
                        help="only run this GEMM shape --reps times (for profiling)")
    parser.add_argument("--dtype", choices=["bf16", "fp8"], default="bf16", help="dtype for --gemm-shape")
    parser.add_argument("--sms", type=int, default=0, help="partition size for --gemm-shape (0: whole device)")
    args = parser.parse_args()
    if args.stages_tokens > 0:
        run_stages(args.stages_tokens, args.experts, args.topk, args.hidden, args.inter, args.reps)
    elif args.gemm_shape:
        run_gemm_shape(*args.gemm_shape, dtype=args.dtype, sm_count=args.sms, reps=args.reps)
    elif args.fp8_layer_tokens > 0:
        run_layer_fp8(args.fp8_layer_tokens, args.reps, args.experts, pow2=args.pow2, timed=args.timed)
    elif args.layer_tokens > 0:
        run_layer(args.layer_tokens, args.reps, layout=args.layout)
    elif args.all:
        run_gemm_benchmark()
        run_moe_benchmark()
    elif args.gemm:
        run_gemm_benchmark()
    elif args.moe:
        run_moe_benchmark()
    else:
        parser.print_help()


if __name__ == "__main__":
    main()
