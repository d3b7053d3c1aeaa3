"""GPU comparator: the reference's own Triton kernels, timed on this B200
beside the tcgen05 kernels on the same inputs, partitions and timing method.

The reference's GEMM (`matmul_sm_aware`, elastikernel/sm_aware_matmul.py:183-216)
and segment MoE (`fused_moe_sm_aware`, elastikernel/sm_aware_benchmark.py:292-349)
kernels are defined inside its benchmark functions (`run_benchmark`,
`run_moe_benchmark`), so they cannot be imported. Their definitions -- the
`@triton.autotune` / `@triton.jit` decorators, the autotune config lists and
the `call_*` wrappers, unmodified -- are lifted out of the reference package
installed under baseline/_ref (baseline/install_ref.sh) with `ast` and
executed as a module of their own in a temporary directory. Triton autotunes
them exactly as the reference does (key M, N, K, NUM_SMS), so the first call
per partition compiles and times every config.

Comparators only: the product path never imports this file.
"""
from __future__ import annotations

import ast
import importlib.util
import tempfile
import textwrap
from pathlib import Path

REF_PKG = Path(__file__).resolve().parent / "_ref" / "elastikernel"

GEMM_NAMES = ("make_sm_aware_configs", "matmul_sm_aware", "call_sm_aware")
MOE_NAMES = ("make_moe_sm_aware_configs", "fused_moe_sm_aware", "call_moe_sm_aware")
# the reference's own MoE benchmark case (sm_aware_benchmark.py:434-443)
MOE_CASE = {"num_tokens": 512, "hidden_dim": 4096, "intermediate_dim": 4096, "num_experts": 8, "top_k": 2}


def available() -> str | None:
    """None when the reference package is installed, else why not."""
    for f in ("sm_aware_matmul.py", "sm_aware_benchmark.py"):
        if not (REF_PKG / f).exists():
            return ("reference package not installed under baseline/_ref "
                    "(run baseline/install_ref.sh with the reference checkout)")
    return None


def _lift(path: Path, outer: str, names: tuple) -> str:
    """Source of the functions `names` defined directly in `outer`, with their
    decorators, dedented to module level, in the order given."""
    text = path.read_text()
    lines = text.splitlines()
    for node in ast.walk(ast.parse(text)):
        if isinstance(node, ast.FunctionDef) and node.name == outer:
            found = {}
            for sub in node.body:
                if isinstance(sub, ast.FunctionDef) and sub.name in names:
                    start = min([d.lineno for d in sub.decorator_list] + [sub.lineno])
                    found[sub.name] = textwrap.dedent("\n".join(lines[start - 1:sub.end_lineno]))
            missing = [n for n in names if n not in found]
            if missing:
                raise LookupError(f"{path.name}:{outer} defines no {missing}")
            return "\n\n\n".join(found[n] for n in names)
    raise LookupError(f"{path.name} defines no {outer}")


def load():
    """The reference's Triton kernels and wrappers as one module."""
    why = available()
    if why:
        raise RuntimeError(why)
    src = "\n\n\n".join([
        "import torch\nimport triton\nimport triton.language as tl",
        _lift(REF_PKG / "sm_aware_matmul.py", "run_benchmark", GEMM_NAMES),
        _lift(REF_PKG / "sm_aware_benchmark.py", "run_moe_benchmark", MOE_NAMES),
    ]) + "\n"
    # Triton reads a kernel's source back from its file, so the module is a real file
    path = Path(tempfile.mkdtemp(prefix="ek_ref_triton_")) / "ek_ref_triton.py"
    path.write_text(src)
    spec = importlib.util.spec_from_file_location("ek_ref_triton", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _best(kernel) -> str | None:
    cfg = getattr(kernel, "best_config", None)
    if cfg is None:
        return None
    kw = cfg.kwargs
    return (f"{kw.get('BLOCK_SIZE_M')}x{kw.get('BLOCK_SIZE_N')}x{kw.get('BLOCK_SIZE_K')} "
            f"g{kw.get('GROUP_SIZE_M')} s{cfg.num_stages} w{cfg.num_warps}")


def _rel_diff(x, ref) -> float:
    x, ref = x.float(), ref.float()
    return float((x - ref).abs().max() / ref.abs().max().clamp_min(1e-30))


def compare(dev, sm_levels=(148,), reps: int = 10, moe_levels=(64,)) -> dict:
    """4096^3 fp16 GEMM (the reference's inputs: N(0,1) fp16, fp16 out) and the
    reference's MoE segment case, reference Triton vs tcgen05, per partition.
    Both sides are timed with CUDA events on the partition stream, L2 flushed
    before every repetition, after the reference's own 3 warm-up calls (the
    first of which autotunes)."""
    import torch

    from elastikernel_b200 import sm_aware_benchmark as smb
    from elastikernel_b200 import sm_aware_matmul as smm
    from elastikernel_b200.green_ctx import get_total_sm_count
    from elastikernel_b200.timing import time_on_stream

    ref = load()
    total = get_total_sm_count(dev)
    out = {"gemm_4096_fp16": [], "moe_segment": []}
    torch.manual_seed(0)
    M = N = K = 4096
    a = torch.randn((M, K), device=dev, dtype=torch.float16)
    b = torch.randn((K, N), device=dev, dtype=torch.float16)
    flop = 2.0 * M * N * K
    for S in sm_levels:
        try:
            stream, actual = smb._partition(dev, S, total)
            with torch.cuda.stream(stream):
                for _ in range(3):
                    c_ref = ref.call_sm_aware(a, b, actual)
                    c_ek = smm.call_sm_aware(a, b)
                torch.cuda.synchronize()
                rt = time_on_stream(lambda: ref.call_sm_aware(a, b, actual), stream, reps=reps)
                re = time_on_stream(lambda: smm.call_sm_aware(a, b), stream, reps=reps)
            out["gemm_4096_fp16"].append({
                "sm": S, "actual_sm": actual,
                "triton_us": round(rt["mean_ms"] * 1e3, 1), "triton_tflops": round(flop / rt["mean_ms"] / 1e9, 1),
                "triton_config": _best(ref.matmul_sm_aware),
                "ek_us": round(re["mean_ms"] * 1e3, 1), "ek_tflops": round(flop / re["mean_ms"] / 1e9, 1),
                "speedup_vs_triton": round(rt["mean_ms"] / re["mean_ms"], 2),
                "max_rel_diff": round(_rel_diff(c_ek, c_ref), 5)})
        except Exception as e:  # report and continue, as the reference benchmark does
            out["gemm_4096_fp16"].append({"sm": S, "error": str(e)[:200]})
    del a, b
    c = MOE_CASE
    T, H, I, E, k = c["num_tokens"], c["hidden_dim"], c["intermediate_dim"], c["num_experts"], c["top_k"]
    torch.manual_seed(42)
    hs = torch.randn((T, H), device=dev, dtype=torch.float16)
    w = torch.randn((E * I, H), device=dev, dtype=torch.float16)
    offs = smb._fake_offsets(T, E, k, dev)
    flop = 2.0 * T * I * H  # every token row multiplies one expert's [I, H] (the reference's offsets cover T rows)
    for S in moe_levels:
        try:
            stream, actual = smb._partition(dev, S, total)
            with torch.cuda.stream(stream):
                for _ in range(3):
                    o_ref = ref.call_moe_sm_aware(hs, w, offs, E, I, H, actual)
                    o_ek = smb.call_moe_sm_aware(hs, w, offs, E, I, H)
                torch.cuda.synchronize()
                rt = time_on_stream(lambda: ref.call_moe_sm_aware(hs, w, offs, E, I, H, actual), stream, reps=reps)
                re = time_on_stream(lambda: smb.call_moe_sm_aware(hs, w, offs, E, I, H), stream, reps=reps)
            out["moe_segment"].append({
                "case": dict(c), "sm": S, "actual_sm": actual,
                "triton_us": round(rt["mean_ms"] * 1e3, 1), "triton_config": _best(ref.fused_moe_sm_aware),
                "ek_us": round(re["mean_ms"] * 1e3, 1), "ek_tflops": round(flop / re["mean_ms"] / 1e9, 1),
                "speedup_vs_triton": round(rt["mean_ms"] / re["mean_ms"], 2),
                "max_rel_diff": round(_rel_diff(o_ek, o_ref), 5)})
        except Exception as e:
            out["moe_segment"].append({"sm": S, "error": str(e)[:200]})
    return out
