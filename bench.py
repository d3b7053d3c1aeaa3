#!/usr/bin/env python
"""Benchmark of the SM-aware GEMM + fused-MoE hot path on B200.

Headline (`value`): bf16 GEMM M = N = K = 4096 (the N=K=4096 wave-sweep's
square point) on the full 148-SM device, TFLOP/s, whole job (sum over ranks;
ranks are independent replicas, "weak" scaling). One step = one GEMM of
synthetic N(0,1) inputs (seed 0) resident in HBM; the L2 is flushed (256 MB
write) before every timed step, outside the timed events. After the W
warm-up steps and the clock sampler's start, about 30 ms of untimed steps
bring the SM clock back up from idle before the K timed steps.

Also on the same line:
* e2e       the same metric through the public API (sm_aware_matmul.call_sm_aware)
            with pinned host buffers: H2D of A and B, the GEMM, D2H of C per step
* roofline  achieved TFLOP/s of the GEMM kernel vs the measured bf16 peak
* partitions  4096^3 on green-context partitions of {16,32,64,96,132,148} SMs:
            % of the partition's own peak (SMs x 8192 FLOP/clk x the median SM
            clock sampled while it ran) and of cuBLAS 8192^3 in the same
            partition, cuBLAS 4096^3 beside it; the M sweep at 148 SMs
* fp8       e4m3 GEMM 4096 x 14336 x 4096 (per-row / per-channel scales)
* moe       Mixtral-shaped fused MoE tokens/s at T in {1,16,128,1024,4096}
* moe_cpu   the reference's CPU MoE operator on the box's host cores
* moe_ep    DeepSeek-V3-shaped FP8 expert-parallel layer: phases, NVLink
            bytes, and its output checked against the oracle on a token sample
* triton_reference  the reference's own Triton GEMM (4096^3 fp16, autotuned as
            the reference does) and MoE segment kernel on this GPU beside the
            tcgen05 kernels (baseline/triton_comparator.py; N=1 only)
* cpu_baseline  the reference's CPU GEMM (torch.matmul on CPU) on a bounded sample
* summary   (the line's last key) the figures above in compact form

`--impl reference` times the reference's own CPU implementation of the path
(the oracle restatement of the GEMM operator, torch.matmul on CPU bf16) on the
host cores, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import datetime, timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

M = N = K = 4096
FLOP = 2.0 * M * N * K
METRIC = "bf16 GEMM TFLOP/s per green-ctx partition (4096^3, 148-SM full device)"
UNIT = "TFLOP/s"
FALLBACK_PEAKS = {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0}
# FP8 expert weights of the DeepSeek-V3-shaped layer: power-of-two scales
# applied by the tensor cores (True) or fp32 scales applied per K block (False)
FP8_POW2 = True
# dense bf16 / fp16 MMA rate of one B200 SM per clock (tcgen05); e4m3 is twice it
MMA_FLOP_PER_CLK_SM = 8192


def load_peaks() -> tuple[dict, str]:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def dist_env() -> tuple[int, int, int]:
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region;
    summary(window) restricts the statistics to samples taken inside a
    (start, end) wall-clock window (time.time())."""

    FIELDS = ("timestamp,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        self.uuid = None
        try:
            self.uuid = str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            pass
        self.proc = None
        self.path = Path(tempfile.mkstemp(prefix="ek_clocks_", suffix=".csv")[1])

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.fh, stderr=subprocess.DEVNULL)
            # let nvidia-smi finish its start-up (NVML init) before the timed region
            t0 = time.time()
            while time.time() - t0 < 5.0 and self.path.stat().st_size == 0:
                time.sleep(0.05)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.fh.close()

    def _rows(self) -> list:
        rows = []
        try:
            for line in self.path.read_text().splitlines():
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 10:
                    continue
                if self.uuid and self.uuid.replace("GPU-", "") not in parts[1]:
                    continue
                try:
                    ts = datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                except ValueError:
                    ts = None
                rows.append([ts] + parts[2:])
        except Exception:
            pass
        return rows

    def summary(self, window: tuple | None = None) -> dict:
        rows = self._rows()
        if window is not None:
            rows = [r for r in rows if r[0] is not None and window[0] <= r[0] <= window[1]]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows),
                "power_w_max": max((num(r[3]) or 0.0) for r in rows)}


def max_over_ranks(x: float, world: int) -> float:
    if world <= 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=torch.device("cuda", torch.cuda.current_device()))
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def settle(step_fn, flush, ms: float = 30.0) -> None:
    """Untimed steps for about `ms` of GPU time right before a timed region.
    The clock sampler's start-up leaves the GPU idle for a few tenths of a
    second, and an idle B200 needs a few milliseconds under load to bring its
    SM clock back up: without this the first timed steps of a short region
    run at the lower clock."""
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    if flush is not None:
        flush()
    step_fn()
    e.record()
    torch.cuda.synchronize()
    n = max(1, min(2000, int(ms / max(s.elapsed_time(e), 1e-3))))
    for _ in range(n):
        if flush is not None:
            flush()
        step_fn()
    torch.cuda.synchronize()


def timed_steps(step_fn, steps: int, flush) -> tuple[float, list]:
    """Run `steps` steps; each is bracketed by events on the current stream
    (flush outside them). Returns (mean ms per step, per-step ms)."""
    evs = []
    for _ in range(steps):
        if flush is not None:
            flush()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        step_fn()
        e.record()
        evs.append((s, e))
    torch.cuda.synchronize()
    ms = [s.elapsed_time(e) for s, e in evs]
    return sum(ms) / len(ms), ms


def e2e_pipelined(smm, a_h, b_h, a_like, b_like, steps: int) -> float:
    """Mean ms per step of `steps` end-to-end GEMM steps through the public
    call: every step copies its inputs from pinned host memory, multiplies
    with sm_aware_matmul.call_sm_aware and reads the product back to pinned
    host memory. Host->device copies run on a copy stream into two device
    buffers, so step i+1's inputs cross PCIe while step i computes and reads
    back; every copy of every step is inside the timed region."""
    cmp = torch.cuda.current_stream()
    cin = torch.cuda.Stream()
    bufs = [(torch.empty_like(a_like), torch.empty_like(b_like)) for _ in range(2)]
    c_hs = [torch.empty((a_like.shape[0], b_like.shape[1]), dtype=a_like.dtype).pin_memory() for _ in range(2)]
    loaded = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(cmp)
    cin.wait_event(start)
    for i in range(steps):
        j = i % 2
        with torch.cuda.stream(cin):
            if i >= 2:
                cin.wait_event(free[j])  # the product of step i-2 no longer reads buffer j
            bufs[j][0].copy_(a_h, non_blocking=True)
            bufs[j][1].copy_(b_h, non_blocking=True)
            loaded[j].record(cin)
        cmp.wait_event(loaded[j])
        c = smm.call_sm_aware(bufs[j][0], bufs[j][1])
        free[j].record(cmp)
        c_hs[j].copy_(c, non_blocking=True)
    end.record(cmp)
    torch.cuda.synchronize()
    return start.elapsed_time(end) / steps


def _timed_window(fn, stream, min_s: float, max_reps: int = 20000) -> tuple[dict, tuple]:
    """time_on_stream of fn with enough repetitions to last about min_s (so the
    clock sampler sees several samples), and the wall-clock window it ran in."""
    from elastikernel_b200.timing import time_on_stream

    probe = time_on_stream(fn, stream, reps=3)
    per_ms = probe["mean_ms"] + 0.05  # + the L2 flush between repetitions
    reps = int(min(max_reps, max(3, math.ceil(min_s * 1e3 / per_ms))))
    torch.cuda.synchronize()
    t0 = time.time()
    r = time_on_stream(fn, stream, reps=reps)
    return r, (t0, time.time())


def partition_sweep(dev, peak_tflops: float, steps: int, hbm_gbs: float = FALLBACK_PEAKS["hbm_gbs"]) -> dict:
    """4096^3 bf16 on each partition size, with the partition's own peak as
    denominator: SMs x 8192 FLOP/clk x the median SM clock sampled while the
    GEMM ran (`pct_sm_peak_at_clock`), and cuBLAS 8192^3 launched in the same
    partition (`pct_cublas_8192`). cuBLAS 4096^3 in the same partition is the
    vendor comparator. Then the M sweep at 148 SMs, CUDA-graph timed, with the
    max(tensor, HBM) floor and cuBLAS beside it."""
    from elastikernel_b200 import sm_aware_matmul as smm
    from elastikernel_b200.green_ctx import create_sm_partition, full_device_partition, get_total_sm_count
    from elastikernel_b200.timing import time_on_stream

    total = get_total_sm_count(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    out = {"square_4096": [], "m_sweep_148": []}
    a = torch.randn((M, K), device=dev, dtype=torch.bfloat16, generator=g)
    b = torch.randn((K, N), device=dev, dtype=torch.bfloat16, generator=g)
    a8 = torch.randn((8192, 8192), device=dev, dtype=torch.bfloat16, generator=g)
    b8 = torch.randn((8192, 8192), device=dev, dtype=torch.bfloat16, generator=g)
    sampler = ClockSampler(dev)
    with sampler:
        for S in [16, 32, 64, 96, 132, 148]:
            try:
                stream, actual = full_device_partition(dev) if S >= total else create_sm_partition(dev, S)
                with torch.cuda.stream(stream):
                    for _ in range(2):
                        smm.call_sm_aware(a, b)
                    r, win = _timed_window(lambda: smm.call_sm_aware(a, b), stream, min_s=1.0)
                    torch.matmul(a, b)
                    rc = time_on_stream(lambda: torch.matmul(a, b), stream, reps=max(3, steps // 2))
                    torch.matmul(a8, b8)
                    rc8 = time_on_stream(lambda: torch.matmul(a8, b8), stream, reps=3)
                clk = sampler.summary(win)
                p = smm.tcgen05_schedule(M, N, K, actual)
                tf = FLOP / (r["mean_ms"] * 1e-3) / 1e12
                tf_cub = FLOP / (rc["mean_ms"] * 1e-3) / 1e12
                tf_cub8 = 2.0 * 8192 ** 3 / (rc8["min_ms"] * 1e-3) / 1e12
                rec = {"sm": S, "actual_sm": actual, "us": round(r["mean_ms"] * 1e3, 1),
                       "us_median": round(r["median_ms"] * 1e3, 1), "reps": r["reps"], "tflops": round(tf, 1),
                       "sm_mhz": clk["sm_mhz"], "clock_samples": clk["samples"],
                       "cublas_us": round(rc["mean_ms"] * 1e3, 1), "cublas_tflops": round(tf_cub, 1),
                       "speedup_vs_cublas": round(rc["mean_ms"] / r["mean_ms"], 3),
                       "cublas_8192_tflops": round(tf_cub8, 1), "pct_cublas_8192": round(100 * tf / tf_cub8, 1),
                       "bm": p["bm"], "bn": p["bn"], "split": p["tail_split"],
                       "wave_eff": round(p["wave_efficiency"], 3)}
                if clk["sm_mhz"]:
                    peak_clk = actual * MMA_FLOP_PER_CLK_SM * clk["sm_mhz"] * 1e6 / 1e12
                    rec["peak_at_clock_tflops"] = round(peak_clk, 1)
                    rec["pct_sm_peak_at_clock"] = round(100 * tf / peak_clk, 1)
                out["square_4096"].append(rec)
            except Exception as e:  # report and continue, as the reference benchmark does
                out["square_4096"].append({"sm": S, "error": str(e)[:200]})
    del a8, b8
    # M sweep: the GEMM replayed from a CUDA graph (device time of the kernel;
    # an eager call's host work -- planning, tensor maps, the ctypes launch --
    # outlasts the L2 flush for the small M and would be timed too), with the
    # eager call's time beside it, cuBLAS, and the max(tensor, HBM) floor.
    for Mi in [128, 256, 512, 1024, 2048, 4096, 8192]:
        a2 = torch.randn((Mi, K), device=dev, dtype=torch.bfloat16, generator=g)
        for _ in range(2):
            smm.call_sm_aware(a2, b)
        r_eager = time_on_stream(lambda: smm.call_sm_aware(a2, b), reps=max(3, steps // 2))
        gm = smm.GraphMatmul(a2, b, num_sms=total)
        r = time_on_stream(gm, reps=max(3, steps // 2))
        torch.matmul(a2, b)
        rc = time_on_stream(lambda: torch.matmul(a2, b), reps=max(3, steps // 2))
        flop = 2.0 * Mi * N * K
        nbytes = 2.0 * (Mi * K + K * N + Mi * N)
        floor_us = max(flop / (peak_tflops * 1e12), nbytes / (hbm_gbs * 1e9)) * 1e6
        tf = flop / (r["mean_ms"] * 1e-3) / 1e12
        p = smm.tcgen05_schedule(Mi, N, K, total)
        out["m_sweep_148"].append({"M": Mi, "us": round(r["mean_ms"] * 1e3, 1),
                                   "us_eager": round(r_eager["mean_ms"] * 1e3, 1), "tflops": round(tf, 1),
                                   "cublas_us": round(rc["mean_ms"] * 1e3, 1),
                                   "pct_peak": round(100 * tf / peak_tflops, 1),
                                   "pct_roofline_time": round(100 * floor_us / (r["mean_ms"] * 1e3), 1),
                                   "bound": "tensor" if flop / (peak_tflops * 1e12) >= nbytes / (hbm_gbs * 1e9)
                                   else "hbm", "bn": p["bn"], "split": p["tail_split"], "tiles": p["num_tiles"]})
        del gm
    return out


def fp8_bench(dev, peak_bf16_tflops: float, steps: int) -> dict:
    """FP8 e4m3 GEMM 4096 x 14336 x 4096 with per-row / per-channel scales on
    the full device and a 74-SM request (rounded up to the alignment)."""
    from elastikernel_b200 import _ops
    from elastikernel_b200.green_ctx import create_sm_partition, get_total_sm_count
    from elastikernel_b200.timing import time_on_stream

    Mf, Nf, Kf = 4096, 14336, 4096
    flop = 2.0 * Mf * Nf * Kf
    peak_fp8 = 2.0 * peak_bf16_tflops  # dense e4m3 rate is twice bf16 on B200
    g = torch.Generator(device=dev).manual_seed(0)
    aq, a_s = _ops.quant_e4m3(torch.randn((Mf, Kf), device=dev, generator=g))
    wq, w_s = _ops.quant_e4m3(torch.randn((Nf, Kf), device=dev, generator=g))
    total = get_total_sm_count(dev)
    res = []
    for req in (total, 74):
        stream, actual = (torch.cuda.current_stream(dev), total) if req >= total else create_sm_partition(dev, req)
        with torch.cuda.stream(stream):
            for _ in range(2):
                _ops.gemm_fp8(aq, wq, a_s, w_s)
            r = time_on_stream(lambda: _ops.gemm_fp8(aq, wq, a_s, w_s), stream, reps=max(3, steps // 2))
            cub = None
            try:  # the vendor path for the same math: torch._scaled_mm with row-wise scales
                def scaled():
                    return torch._scaled_mm(aq, wq.t(), scale_a=a_s.view(-1, 1), scale_b=w_s.view(1, -1),
                                            out_dtype=torch.bfloat16)
                scaled()
                cub = time_on_stream(scaled, stream, reps=max(3, steps // 2))["mean_ms"]
            except Exception as e:  # not every torch build has row-wise scaled FP8 on this GPU
                cub = str(e)[:120]
        tf = flop / (r["mean_ms"] * 1e-3) / 1e12
        p = _ops.plan(Mf, Nf, Kf, actual, _ops._FP8, "nk")
        rec = {"sm_request": req, "actual_sm": actual, "us": round(r["mean_ms"] * 1e3, 1),
               "tflops": round(tf, 1), "pct_scaled_fp8_peak": round(100 * tf / (peak_fp8 * actual / 148), 1),
               "bm": p["bm"], "bn": p["bn"], "split": p["tail_split"]}
        if isinstance(cub, float):
            rec["torch_scaled_mm_us"] = round(cub * 1e3, 1)
            rec["speedup_vs_torch_scaled_mm"] = round(cub / r["mean_ms"], 3)
        else:
            rec["torch_scaled_mm"] = cub
        res.append(rec)
    return {"config": "e4m3 4096x14336x4096, per-row A / per-channel W fp32 scales, bf16 out",
            "fp8_peak_tflops": peak_fp8, "peak_note": "2 x measured bf16 burst", "results": res}


def moe_ep_bench(dev, world: int, steps: int, peak_bf16_tflops: float, groups: int = 0) -> dict:
    """DeepSeek-V3-shaped expert-parallel MoE: 256 experts, top-8 softmax
    routing, H=7168, I=2048, e4m3 experts with 128 x 128 block scales, 4096
    tokens per rank, 256/world experts per rank, e4m3 dispatch over NCCL
    all-to-all. The expert GEMMs run in a 116-SM green-context partition, the
    remainder of a 32-SM one split off for the collectives."""
    from elastikernel_b200 import _ops
    from elastikernel_b200.ep_moe import CudaEPOps, ExpertParallelMoE
    from elastikernel_b200.green_ctx import create_disjoint_partitions, get_total_sm_count

    E, k, H, I, T = 256, 8, 7168, 2048, 4096
    eg = E // world
    rank = int(os.environ.get("RANK", 0))
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    parts = {"w1q": [], "w1s": [], "w3q": [], "w3s": [], "w2q": [], "w2s": []}
    for c0 in range(0, eg, 32):  # quantise in chunks to bound the bf16 staging memory
        n = min(32, eg - c0)
        w1 = (torch.randn((n, I, H), device=dev, generator=g) * 0.02).to(torch.bfloat16)
        w3 = (torch.randn((n, I, H), device=dev, generator=g) * 0.02).to(torch.bfloat16)
        w2 = (torch.randn((n, H, I), device=dev, generator=g) * 0.02).to(torch.bfloat16)
        q = _ops.quant_moe_weights_fp8(w1, w2, w3, pow2=FP8_POW2)
        for key in parts:
            parts[key].append(q[key])
        del w1, w2, w3, q
    qw = {"E": eg, "I": I, "H": H, "pow2": FP8_POW2}
    for key, lst in parts.items():
        qw[key] = torch.cat(lst, dim=0)
    del parts
    qw = _ops.stack_gate_up_planes(qw)  # w1 / w3 codes as two planes of one buffer
    gx = torch.Generator(device=dev).manual_seed(42 + rank)
    x = torch.randn((T, H), device=dev, generator=gx).to(torch.bfloat16)
    logits = torch.randn((T, E), device=dev, generator=gx)
    total = get_total_sm_count(dev)
    if total >= 148:
        (comm_stream, comm_sms), (gemm_stream, gemm_sms) = create_disjoint_partitions(dev, [32], with_remainder=True)
    else:
        gemm_stream, gemm_sms = torch.cuda.current_stream(dev), total
        comm_stream, comm_sms = torch.cuda.Stream(dev), 0
    # fixed-capacity exchanges: equal all-to-all splits known to the host, so
    # nothing is read back between the routing and the combine
    # the equal-split exchanges go through an NCCL communicator driven on the
    # communication partition's stream, so their kernels stay on its 32 SMs
    # The grouped layer's exchanges go by copy engines straight into the
    # peers' IPC-mapped receive buffers (no NCCL, no SM); the ungrouped
    # layer's through an NCCL communicator driven on the communication
    # partition's stream.
    stream_a2a = p2p = None
    if world > 1:
        from elastikernel_b200.nccl_stream import StreamAllToAll
        from elastikernel_b200.p2p_exchange import P2PAllToAll

        stream_a2a = StreamAllToAll()
        p2p = P2PAllToAll(device_epochs=True)  # device-side epochs: the layer can be graph-replayed
    moe = ExpertParallelMoE(E, k, qw=qw, ops=CudaEPOps(num_sms=gemm_sms), capacity="auto", stream_a2a=stream_a2a,
                            p2p=p2p)
    # Expert groups (N > 1): each rank's experts in 2 groups; a group's
    # exchanges run on the 32-SM partition (NCCL driven on its stream) while
    # another group's GEMMs run in the 116-SM partition, and every expert
    # still streams its weights once. The ungrouped layer (routing, exchanges
    # and the experts' 116-CTA GEMMs one after another on a full-device
    # stream) is timed beside it.
    if groups <= 0:
        groups = 2 if world > 1 else 1
    main = torch.cuda.Stream(dev)

    def time_layer(gr):
        def layer():
            return moe(x, logits, groups=gr, compute_stream=gemm_stream, comm_stream=comm_stream)

        with torch.cuda.stream(main):
            for _ in range(2):
                layer()
            torch.cuda.synchronize()
            barrier(world)
            reps = max(3, steps // 10)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(main)
            for _ in range(reps):
                y = layer()
            e.record(main)
            torch.cuda.synchronize()
        return max_over_ranks(s.elapsed_time(e) / reps, world), y

    exchange = "copy engines into IPC-mapped buffers" if (p2p is not None and groups > 1) else "NCCL"
    try:
        ms, out = time_layer(groups)
    except RuntimeError as err:  # the copy-engine path could not map the peers' buffers: NCCL instead
        if p2p is None:
            raise
        moe.p2p = None
        exchange = f"NCCL (copy-engine exchange unavailable: {str(err)[:160]})"
        ms, out = time_layer(groups)
    ms_ungrouped = time_layer(1)[0] if groups > 1 else ms
    # The same layer captured once in a CUDA graph and replayed (no host work
    # between its launches; the copy-engine exchanges keep their epochs on the
    # device). This is the layer time reported; the eager time stays beside it.
    # At N > 1 only the grouped copy-engine layer is captured (no NCCL call in
    # a graph).
    ms_graph, graph_match, graph_note = None, None, None
    if world == 1 or (groups > 1 and moe.p2p is not None):
        from elastikernel_b200.graph import Captured

        cap = None
        try:
            with torch.cuda.stream(main):
                cap = Captured(lambda: moe(x, logits, groups=groups, compute_stream=gemm_stream,
                                           comm_stream=comm_stream), main)
        except RuntimeError as err:  # the eager time stands
            graph_note = f"capture failed: {str(err)[:160]}"
            torch.cuda.synchronize()
        ok = max_over_ranks(float(cap is None), world) == 0.0  # every rank captured
        if ok:
            with torch.cuda.stream(main):
                for _ in range(2):
                    cap()
                torch.cuda.synchronize()
                barrier(world)
                reps = max(3, steps // 10)
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(main)
                for _ in range(reps):
                    yg = cap()
                e.record(main)
                torch.cuda.synchronize()
            ms_graph = max_over_ranks(s.elapsed_time(e) / reps, world)
            graph_match = bool(max_over_ranks(float(not torch.equal(yg, out)), world) == 0.0)
            del yg
        del cap
        torch.cuda.synchronize()
        barrier(world)
    ms_eager = ms
    if ms_graph is not None:
        ms = ms_graph
    # phase split of one ungrouped layer (device time between phase events on
    # the experts' partition stream; NCCL inside the same timeline)
    barrier(world)
    with torch.cuda.stream(gemm_stream):
        moe.profile_phases(x, logits)  # warm-up: the allocator's blocks for this stream
        barrier(world)
        prof = moe.profile_phases(x, logits)
    phases = {kk: round(max_over_ranks(v, world), 3) for kk, v in prof["ms"].items()}
    a2a = {"dispatch_bytes_per_rank": prof["dispatch_bytes"], "combine_bytes_per_rank": prof["combine_bytes"]}
    if world > 1:
        for key, ph in (("dispatch", "dispatch"), ("combine", "combine_exchange")):
            t = phases.get(ph, 0.0)
            a2a[f"{key}_gbs_per_rank"] = round(prof[f"{key}_bytes"] / (t * 1e-3) / 1e9, 1) if t > 0 else None
    from elastikernel_b200 import _lib

    # overflow of a rank's capacity shows in the device status word (read, not cleared)
    overflow = bool(_lib.device_status(dev.index if dev.index is not None else 0, clear=False)
                    & _lib.EK_STATUS_CAPACITY)
    overflow = bool(max_over_ranks(float(overflow), world))
    err, err_q = ep_parity(dev, x, logits, out, qw, E, k, world, rank)
    if stream_a2a is not None:
        barrier(world)
        stream_a2a.close()
    if moe.p2p is not None:
        moe.p2p.close()
    flop = T * k * 6.0 * H * I
    tf = flop / (ms * 1e-3) / 1e12
    peak_fp8 = 2.0 * peak_bf16_tflops
    return {"config": "DeepSeek-V3-shaped: E=256 top-8 H=7168 I=2048, e4m3 128x128 block scales, 4096 tokens/rank, "
                      f"{eg} experts/rank, e4m3 dispatch and bf16 combine by all-to-all (path in 'exchange')",
            "n_gpus": world, "ms_per_layer": round(ms, 3), "tokens_per_s": round(world * T / (ms * 1e-3), 1),
            "tflops_per_gpu": round(tf, 1), "gemm_partition_sms": gemm_sms, "comm_partition_sms": comm_sms,
            "pct_fp8_peak_scaled": round(100 * tf / (peak_fp8 * gemm_sms / 148), 1),
            "expert_groups": groups, "exchange": exchange, "ms_per_layer_ungrouped": round(ms_ungrouped, 3),
            "ms_per_layer_eager": round(ms_eager, 3), "timing": ("the layer replayed from a CUDA graph"
                                                                if ms_graph is not None else "eager launches"),
            "graph_equals_eager": graph_match, **({"graph_note": graph_note} if graph_note else {}),
            "placement": ("experts in the 116-SM green context, exchanges on the 32-SM one, overlapped group by "
                          "group" if groups > 1 else "routing, exchanges and the experts' 116-CTA GEMMs in turn on "
                          "a full-device stream"),
            "phases_ms_ungrouped": phases, "all_to_all": a2a,
            "ep_max_rel_err": err, "ep_parity_tol": 3e-2, "ep_max_rel_err_act_e4m3": err_q,
            "fp8_scales": "power-of-two, applied by the tensor cores (kind::mxf8f6f4.block_scale)" if FP8_POW2
            else "fp32, applied per 128-wide K block in the epilogue",
            "host_sync": "none: fixed-capacity exchanges (equal all-to-all splits, padding rows on a dummy expert)",
            "capacity_rows_per_rank": prof["capacity"], "rows_routed_per_rank": T * k,
            "capacity_overflow": overflow}


def ep_parity(dev, x, logits, out, qw, E: int, k: int, world: int, rank: int, per_rank: int = 32) -> float:
    """The checker of the expert-parallel layer (outside every timed region):
    `per_rank` seeded tokens of each rank are compared with the CPU oracle on
    the dequantised inputs. Experts live on different ranks, so the oracle is
    distributed the same way: the sampled tokens are gathered on every rank,
    each rank computes with the oracle the contribution of ITS experts to
    every sampled token, and a sum over ranks gives each token's reference.
    Returns the max over ranks of max|out - ref| / max|ref| against the fp32
    oracle, and against the oracle that also rounds the SwiGLU activations
    to e4m3 with 1 x 128 scales as the layer does (a tighter check)."""
    import numpy as np

    from oracle import fp8 as of8
    from oracle import gemm as og
    from oracle import moe as om

    T, H = x.shape
    torch.set_num_threads(max(1, (os.cpu_count() or 1) // max(1, world)))
    rng = np.random.default_rng(7 + rank)
    idx = sorted(rng.choice(T, size=per_rank, replace=False).tolist())
    xs, ls = x[idx].contiguous(), logits[idx].contiguous()
    if world > 1:
        import torch.distributed as dist

        xs_all = torch.empty((world * per_rank, H), dtype=xs.dtype, device=dev)
        ls_all = torch.empty((world * per_rank, logits.shape[1]), dtype=ls.dtype, device=dev)
        dist.all_gather_into_tensor(xs_all, xs)
        dist.all_gather_into_tensor(ls_all, ls)
    else:
        xs_all, ls_all = xs, ls
    ids, wts = om.route_ref(ls_all.cpu().numpy(), k)
    eg = E // world
    lo = rank * eg
    ids_local = np.where((ids >= lo) & (ids < lo + eg), ids - lo, -1)
    xd = of8.dequant_blocks(*of8.quant_blocks(xs_all.cpu(), 1, 128, pow2=bool(qw.get("pow2", False))), 1,
                            128)  # e4m3 rows, as dispatched
    nI, nH = qw["I"] // 128, qw["H"] // 128

    def fetch(e):
        w1e = of8.dequant_block_rows(qw["w1q"][e].cpu(), qw["w1s"][e * nI:(e + 1) * nI].cpu().numpy())
        w3e = of8.dequant_block_rows(qw["w3q"][e].cpu(), qw["w3s"][e * nI:(e + 1) * nI].cpu().numpy())
        w2e = of8.dequant_block_rows(qw["w2q"][e].cpu(), qw["w2s"][e * nH:(e + 1) * nH].cpu().numpy())
        return w1e, w2e, w3e

    pow2 = bool(qw.get("pow2", False))

    def act_q(a):  # the layer's e4m3 activations: bf16 act, 1 x 128 groups
        ab = torch.from_numpy(a).to(torch.bfloat16)
        return of8.dequant_blocks(*of8.quant_blocks(ab, 1, 128, pow2=pow2), 1, 128)

    plain, actq = om.moe_ref_by_expert(xd, ids_local, wts, eg, fetch, act_quant=act_q)
    part = torch.from_numpy(np.stack([plain, actq])).to(dev)
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(part)
    sl = slice(rank * per_rank, (rank + 1) * per_rank)
    err = og.max_rel_err(out[idx], part[0, sl].cpu().numpy())
    err_q = og.max_rel_err(out[idx], part[1, sl].cpu().numpy())
    return round(max_over_ranks(err, world), 6), round(max_over_ranks(err_q, world), 6)


def moe_bench(dev, steps: int, hbm_gbs: float, peak_bf16_tflops: float, cpu: bool = False) -> dict:
    """Mixtral-shaped fused MoE (E=8, top-2, H=4096, I=14336, bf16) tokens/s;
    with cpu=True also the reference's CPU operator on the same weights."""
    from elastikernel_b200 import _ops
    from elastikernel_b200.graph import Captured
    from elastikernel_b200.green_ctx import create_sm_partition
    from elastikernel_b200.timing import time_on_stream

    E, k, H, I = 8, 2, 4096, 14336
    g = torch.Generator(device=dev).manual_seed(42)
    w1 = (torch.randn((E, I, H), device=dev, generator=g) * 0.02).to(torch.bfloat16)
    w3 = (torch.randn((E, I, H), device=dev, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn((E, H, I), device=dev, generator=g) * 0.02).to(torch.bfloat16)
    # w1 and w3 as the two planes of one [2, E, I, H] tensor (a fused gate/up
    # weight): the gate/up GEMMs then read a tile's [w1 | w3] rows in one TMA box
    w13 = torch.stack([w1, w3])
    del w1, w3
    w1, w3 = w13[0], w13[1]
    res = []
    half_stream, half_sms = create_sm_partition(dev, 72)
    for T in [1, 16, 128, 1024, 4096]:
        x = torch.randn((T, H), device=dev, generator=g).to(torch.bfloat16)
        logits = torch.randn((T, E), device=dev, generator=g)
        for label, stream, sms in (("full", torch.cuda.current_stream(dev), 148), ("half", half_stream, half_sms)):
            with torch.cuda.stream(stream):
                for _ in range(2):
                    _ops.fused_moe(x, logits, w1, w2, w3, k)
                r = time_on_stream(lambda: _ops.fused_moe(x, logits, w1, w2, w3, k), stream,
                                   reps=max(3, steps // 2), warmup=2)
                # the same layer replayed from a CUDA graph (no host work between its launches)
                y = torch.empty((T, H), device=dev, dtype=torch.bfloat16)
                cap = Captured(lambda: _ops.fused_moe(x, logits, w1, w2, w3, k, out=y), stream)
                rg = time_on_stream(cap, stream, reps=max(3, steps // 2), warmup=2)
                del cap
                ids, _ = _ops.moe_route(logits, k)
            hit = int(torch.unique(ids).numel())
            t_s = r["mean_ms"] * 1e-3
            tg_s = rg["mean_ms"] * 1e-3
            flop = T * k * 6.0 * H * I
            wbytes = hit * 3.0 * H * I * 2
            t_floor = max(flop / (peak_bf16_tflops * 1e12 * sms / 148), wbytes / (hbm_gbs * 1e9))
            res.append({"T": T, "sms": label, "actual_sm": sms, "us": round(r["mean_ms"] * 1e3, 1),
                        "tokens_per_s": round(T / t_s, 1), "tflops": round(flop / t_s / 1e12, 1),
                        "experts_hit": hit, "pct_roofline_time": round(100 * t_floor / t_s, 1),
                        "graph_us": round(rg["mean_ms"] * 1e3, 1), "graph_tokens_per_s": round(T / tg_s, 1),
                        "graph_pct_roofline_time": round(100 * t_floor / tg_s, 1),
                        "eager_reps_us": [round(v * 1e3) for v in r["all_ms"]],
                        "graph_reps_us": [round(v * 1e3) for v in rg["all_ms"]]})
    out = {"config": "Mixtral E=8 k=2 H=4096 I=14336 bf16, weights N(0,0.02); us = eager launches from "
                     "Python, graph_us = the layer replayed from a CUDA graph; roofline = max(tensor at the "
                     "measured bf16 burst x SMs/148, expert weights at the measured HBM rate)",
           "results": res}
    if cpu:
        out["cpu"] = moe_cpu_baseline(w1, w2, w3, E, k, H)
    return out


def moe_cpu_baseline(w1, w2, w3, E: int, k: int, H: int) -> dict:
    """The reference's CPU implementation of the MoE operator on the host
    cores, same weights (bf16) and shapes: the definition's per-token loop
    (definition.py:152-168) at T <= 16 and the vectorised per-expert
    restatement at every T, each a bounded sample (one or two layers)."""
    from oracle import cpu_baseline

    threads = cpu_baseline.set_threads()
    cw1, cw2, cw3 = w1.cpu(), w2.cpu(), w3.cpu()
    g = torch.Generator().manual_seed(42)
    res = []
    for T in [1, 16, 128, 1024, 4096]:
        x = torch.randn((T, H), generator=g).to(torch.bfloat16)
        logits = torch.randn((T, E), generator=g)
        rec = {"T": T}
        for label, loop in (("loop", True), ("vectorised", False)):
            if loop and T > 16:
                continue
            r = cpu_baseline.time_moe(x, logits, cw1, cw2, cw3, k, loop=loop, reps=2 if T <= 128 else 1,
                                      budget_s=15.0)
            mean_s = statistics.fmean(r["seconds"])
            rec[f"{label}_ms"] = round(mean_s * 1e3, 2)
            rec[f"{label}_tokens_per_s"] = round(T / mean_s, 1)
        res.append(rec)
    return {"cores": threads, "kind": "port", "dtype": "bf16",
            "sample": "one or two Mixtral layers per T on CPU tensors (definition loop at T<=16, vectorised "
                      "per-expert torch at every T)", "results": res}


def cpu_baseline_sample() -> dict:
    from oracle import cpu_baseline

    threads = cpu_baseline.set_threads()
    r = cpu_baseline.time_gemm(M, N, K, reps=3, budget_s=20.0)
    mean_s = statistics.fmean(r["seconds"])
    return {"value": round(r["flop"] / mean_s / 1e12, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{len(r['seconds'])} x bf16 torch.matmul {M}x{N}x{K} on CPU (the reference GEMM operator "
                      f"body), mean {mean_s * 1e3:.0f} ms"}


def run_reference(args, rank: int, world: int) -> None:
    """The reference's own CPU implementation of the path: torch.matmul on CPU
    bf16 tensors (oracle restatement of definition.py:63-65), all host threads."""
    if rank != 0:
        return
    from oracle import cpu_baseline

    threads = cpu_baseline.set_threads()
    g = torch.Generator().manual_seed(0)
    a = torch.randn((M, K), generator=g).to(torch.bfloat16)
    b = torch.randn((K, N), generator=g).to(torch.bfloat16)
    for _ in range(args.warmup):
        cpu_baseline.gemm_cpu(a, b)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_baseline.gemm_cpu(a, b)
    dt = (time.perf_counter() - t0) / args.steps
    value = FLOP / dt / 1e12
    line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1), seed 0",
            "config": {"workload": "bf16 GEMM 4096x4096x4096, torch.matmul on host CPU", "M": M, "N": N, "K": K},
            "impl": "reference",
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{args.steps} x bf16 torch.matmul {M}x{N}x{K} on CPU"},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-extras", action="store_true", help="skip the partition sweep, MoE and CPU legs")
    ap.add_argument("--legs", default="partitions,fp8,moe,moe_ep,triton,cpu",
                    help="comma list of the extra legs to run (default: all)")
    ap.add_argument("--triton-sms", default="16,32,64,96,132,148",
                    help="partition sizes (comma list, '' for none) at which the reference's own Triton GEMM is "
                         "timed beside the tcgen05 one; its MoE segment kernel runs at 64 SMs")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    rank, world, local_rank = dist_env()

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import torch.distributed as dist

        # NCCL's kernels for the expert all-to-all get at most 32 CTAs, the
        # size of the communication partition beside the 112-SM GEMM partition
        os.environ.setdefault("NCCL_MAX_CTAS", "32")
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    from elastikernel_b200 import _lib, sm_aware_matmul as smm
    from elastikernel_b200.timing import flush_l2

    peaks, peak_kind = load_peaks()
    peak_tf = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))

    g = torch.Generator(device=dev).manual_seed(0)
    a = torch.randn((M, K), device=dev, dtype=torch.bfloat16, generator=g)
    b = torch.randn((K, N), device=dev, dtype=torch.bfloat16, generator=g)
    plan = smm.tcgen05_schedule(M, N, K, torch.cuda.get_device_properties(dev).multi_processor_count)
    for _ in range(args.warmup):
        smm.call_sm_aware(a, b)
    flush_l2(dev)
    torch.cuda.synchronize()

    # ---------------------------------------------------------------- device-resident timed region
    sampler = ClockSampler(dev)
    with sampler:
        settle(lambda: smm.call_sm_aware(a, b), lambda: flush_l2(dev))
        barrier(world)
        torch.cuda.synchronize()
        ms, per = timed_steps(lambda: smm.call_sm_aware(a, b), args.steps, lambda: flush_l2(dev))
        torch.cuda.synchronize()
        barrier(world)
        # ------------------------------------------------------------ end-to-end (host buffers)
        a_h = a.cpu().pin_memory()
        b_h = b.cpu().pin_memory()
        e2e_ms = e2e_pipelined(smm, a_h, b_h, a, b, 2)  # warm-up
        barrier(world)
        e2e_ms = e2e_pipelined(smm, a_h, b_h, a, b, args.steps)
        barrier(world)
    clocks = sampler.summary()
    status = _lib.device_status(local_rank)

    ms_max = max_over_ranks(ms, world)
    e2e_max = max_over_ranks(e2e_ms, world)
    value = world * FLOP / (ms_max * 1e-3) / 1e12
    e2e_value = world * FLOP / (e2e_max * 1e-3) / 1e12
    achieved = FLOP / (ms * 1e-3) / 1e12

    traffic = None
    tfile = REPO / "profiles" / "gemm_bf16_4096_traffic.json"
    if tfile.exists():
        try:
            traffic = json.loads(tfile.read_text()).get("dram_bytes_per_launch")
        except Exception:
            traffic = None

    extras = {}
    legs = set() if args.no_extras else {v.strip() for v in args.legs.split(",")}
    if "partitions" in legs:
        extras["partitions"] = partition_sweep(dev, peak_tf, args.steps, hbm)
    if "fp8" in legs:
        extras["fp8"] = fp8_bench(dev, peak_tf, args.steps)
    if "moe" in legs:
        extras["moe"] = moe_bench(dev, args.steps, hbm, peak_tf, cpu=(rank == 0 and world == 1 and "cpu" in legs))
    if "moe_ep" in legs:
        # An error in this leg is reported in its field; the GEMM line above
        # it still prints (every rank takes the same collective steps unless
        # the error is one rank's alone, which the process group's timeout ends).
        try:
            extras["moe_ep"] = moe_ep_bench(dev, world, args.steps, peak_tf)
        except Exception as err:  # noqa: BLE001
            extras["moe_ep"] = {"n_gpus": world, "error": f"{type(err).__name__}: {str(err)[:300]}"}
    if "triton" in legs and rank == 0 and world == 1 and args.triton_sms.strip():
        extras["triton_reference"] = triton_reference(dev, [int(x) for x in args.triton_sms.split(",")])
    if "cpu" in legs and rank == 0 and world == 1:
        extras["cpu_baseline"] = cpu_baseline_sample()
    if world > 1:
        import torch.distributed as dist

        barrier(world)
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max, 4),
        "ms_per_step_median": round(statistics.median(per), 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1), seed 0",
        "config": {"workload": "bf16 GEMM 4096x4096x4096 on the full 148-SM device (N=K=4096 wave sweep, "
                               "square point); replicas per GPU", "M": M, "N": N, "K": K,
                   "parallelism": f"replicas x{world}", "l2": "flushed (256 MB write) before every timed step",
                   "clock_settle": "~30 ms of untimed steps between the clock sampler's start and the timed steps",
                   "schedule": {k: plan[k] for k in ("bn", "tail_split", "num_units", "grid",
                                                      "wave_efficiency")}},
        "e2e": {"value": round(e2e_value, 2), "unit": UNIT, "h2d_bytes_per_step": 2 * M * K * 2,
                "d2h_bytes_per_step": M * N * 2,
                "path": "sm_aware_matmul.call_sm_aware with pinned host A, B -> device -> host C; the next step's "
                    "host-to-device copies overlap this step (copy stream, two device buffers)"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak_tf, "unit": UNIT,
                     "frac": round(achieved / peak_tf, 4), "traffic": traffic,
                     "peak_source": f"{peak_kind} bf16_tflops (burst)"},
        "gpu_launches": args.steps,
        "clocks": clocks,
        "device_status": status,
    }
    if "cpu_baseline" in extras:
        line["cpu_baseline"] = extras.pop("cpu_baseline")
    line.update(extras)
    line["summary"] = summarize(line)  # last key: a driver that keeps the line's tail keeps this
    print(json.dumps(line), flush=True)


def triton_reference(dev, sm_levels) -> dict:
    """The reference's own Triton kernels on this GPU (GEMM 4096^3 fp16 per
    partition, the MoE segment case at 64 SMs) beside the tcgen05 kernels;
    unavailable when the reference package is not installed under
    baseline/_ref."""
    sys.path.insert(0, str(REPO / "baseline"))
    try:
        import triton_comparator as tc
    finally:
        sys.path.pop(0)
    why = tc.available()
    if why:
        return {"unavailable": why}
    try:
        return tc.compare(dev, sm_levels=tuple(sm_levels), moe_levels=(64,))
    except Exception as e:
        return {"unavailable": f"{type(e).__name__}: {str(e)[:300]}"}


def summarize(line: dict) -> dict:
    """The line's figures in compact form (lists in a fixed, stated order)."""
    sm = {}
    sm["headline"] = [line["value"], line["roofline"]["frac"], line["e2e"]["value"], line["clocks"].get("sm_mhz")]
    sm["headline_order"] = "TFLOP/s, frac of measured burst, e2e TFLOP/s, median SM MHz"
    parts = line.get("partitions")
    if parts:
        sm["partitions_order"] = ("SMs: us, TFLOP/s, % SMs x 8192 x sampled clock, MHz, % cuBLAS 8192^3 there, "
                                  "x vs cuBLAS 4096^3 there")
        sm["partitions"] = {str(r["actual_sm"]): [r["us"], r["tflops"], r.get("pct_sm_peak_at_clock"), r["sm_mhz"],
                                                  r["pct_cublas_8192"], r["speedup_vs_cublas"]]
                            for r in parts["square_4096"] if "error" not in r}
        sm["m_sweep_order"] = "M: graph us, % max(tensor, HBM) roofline time, cuBLAS us"
        sm["m_sweep"] = {str(r["M"]): [r["us"], r["pct_roofline_time"], r["cublas_us"]] for r in parts["m_sweep_148"]}
    fp8 = line.get("fp8")
    if fp8:
        sm["fp8_order"] = "SMs: TFLOP/s, % 2 x burst x SMs/148, x vs torch._scaled_mm"
        sm["fp8"] = {str(r["actual_sm"]): [r["tflops"], r["pct_scaled_fp8_peak"], r.get("speedup_vs_torch_scaled_mm")]
                     for r in fp8["results"]}
    moe = line.get("moe")
    if moe:
        sm["moe_order"] = "T/partition: eager us, % roofline time, graph us, % roofline time"
        sm["moe"] = {f"{r['T']}/{r['actual_sm']}": [r["us"], r["pct_roofline_time"], r["graph_us"],
                                                     r["graph_pct_roofline_time"]] for r in moe["results"]}
        if "cpu" in moe:
            sm["moe_cpu_order"] = f"T: vectorised tokens/s, loop tokens/s ({moe['cpu']['cores']} cores)"
            sm["moe_cpu"] = {str(r["T"]): [r.get("vectorised_tokens_per_s"), r.get("loop_tokens_per_s")]
                             for r in moe["cpu"]["results"]}
    ep = line.get("moe_ep")
    if ep and "error" in ep:
        sm["moe_ep"] = {"n_gpus": ep["n_gpus"], "error": ep["error"][:160]}
    elif ep:
        sm["moe_ep"] = {"n_gpus": ep["n_gpus"], "ms": ep["ms_per_layer"], "tokens_per_s": ep["tokens_per_s"],
                        "pct_fp8_peak_scaled": ep["pct_fp8_peak_scaled"], "gemm_sms": ep["gemm_partition_sms"],
                        "ep_max_rel_err": [ep["ep_max_rel_err"], ep.get("ep_max_rel_err_act_e4m3")],
                        "expert_groups": ep["expert_groups"], "exchange": ep.get("exchange", "")[:40],
                        "ms_ungrouped": ep.get("ms_per_layer_ungrouped"), "ms_eager": ep.get("ms_per_layer_eager"),
                        "phases_ms_ungrouped": ep["phases_ms_ungrouped"],
                        "a2a_gbs": [ep["all_to_all"].get("dispatch_gbs_per_rank"),
                                    ep["all_to_all"].get("combine_gbs_per_rank")]}
    tr = line.get("triton_reference")
    if tr:
        if "unavailable" in tr:
            sm["triton_reference"] = tr["unavailable"]
        else:
            sm["triton_order"] = "SMs: reference Triton us, tcgen05 us, x speed-up (fp16 4096^3; moe: segment case)"
            sm["triton_gemm"] = {str(r["actual_sm"]): [r["triton_us"], r["ek_us"], r["speedup_vs_triton"]]
                                 for r in tr["gemm_4096_fp16"] if "error" not in r}
            sm["triton_moe"] = {str(r["actual_sm"]): [r["triton_us"], r["ek_us"], r["speedup_vs_triton"]]
                                for r in tr["moe_segment"] if "error" not in r}
    if "cpu_baseline" in line:
        sm["cpu_gemm_tflops"] = [line["cpu_baseline"]["value"], line["cpu_baseline"]["cores"]]
    return sm


if __name__ == "__main__":
    main()
