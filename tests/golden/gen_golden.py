"""Generate the golden vectors in tests/golden/ by running the reference's own code.

Run in a container that has the reference checked out (read-only) and
Triton installed, naming the checkout's root (the directory that holds the
`elastikernel/` package):

    python tests/golden/gen_golden.py --reference-root <path>

What it records (all small; the files are committed and the tests read only
them, never the reference):

* wave.json         sm_aware_matmul.wave_efficiency + its (waves, -last_util)
                    ranking over CONFIGS, for the analytical grid
                    (sm_aware_matmul.py:51-67) and for the N=K=4096 M-sweep at
                    {16,32,64,96,132,148} SMs; workload.compute_wave_efficiency
                    and suggest_optimal_block_size (workload.py:86-143) over
                    GEMM_SIZES x SM_COUNTS.
* routing.npz       the routing lines of the fused-MoE definition's reference
                    operator (definition.py:152-153), executed verbatim from
                    the definition string on seeded N(0,1) logits.
* moe_def.npz       outputs of that operator's run(...) (definition.py:149-170)
                    on small seeded fp32 problems.
* triton_gemm.npz   the reference Triton kernels matmul_sm_aware
                    (sm_aware_matmul.py:183-216) and fused_moe_sm_aware
                    (sm_aware_benchmark.py:292-349), extracted from the source
                    with `ast`, autotune removed, run with one explicit config
                    under the Triton CPU interpreter (TRITON_INTERPRET=1).
"""
from __future__ import annotations

import ast
import json
import os
import sys
import textwrap
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

REF: Path = None  # the reference checkout's root, set from --reference-root
OUT = Path(__file__).resolve().parent


def _import_reference():
    sys.path.insert(0, str(REF))
    import elastikernel.sm_aware_matmul as smm  # noqa: F401

    # sm_aware_agent/__init__.py imports a module that does not exist; load the
    # submodules through a stub package instead.
    pkg = types.ModuleType("elastikernel.sm_aware_agent")
    pkg.__path__ = [str(REF / "elastikernel" / "sm_aware_agent")]
    sys.modules["elastikernel.sm_aware_agent"] = pkg
    import elastikernel.sm_aware_agent.definition as definition
    import elastikernel.sm_aware_agent.workload as workload

    return smm, workload, definition


def gen_wave(smm, workload) -> None:
    rec = {"analytical": [], "sweep": [], "workload": []}
    for (M, N, K) in [(1024, 1024, 1024), (2048, 2048, 2048), (4096, 4096, 4096)]:
        for S in [16, 32, 48, 64, 80, 96, 112, 132]:
            ranked = []
            for c in smm.CONFIGS:
                nw, lwu, eff = smm.wave_efficiency(M, N, c["BLOCK_SIZE_M"], c["BLOCK_SIZE_N"], S)
                ranked.append(([c["BLOCK_SIZE_M"], c["BLOCK_SIZE_N"], c["BLOCK_SIZE_K"]], nw, lwu, eff))
            ranked.sort(key=lambda x: (x[1], -x[2]))
            rec["analytical"].append({"M": M, "N": N, "K": K, "S": S, "ranked": ranked})
    for M in [128, 256, 512, 1024, 2048, 4096, 8192]:
        for S in [16, 32, 64, 96, 132, 148]:
            ranked = []
            for c in smm.CONFIGS:
                nw, lwu, eff = smm.wave_efficiency(M, 4096, c["BLOCK_SIZE_M"], c["BLOCK_SIZE_N"], S)
                ranked.append(([c["BLOCK_SIZE_M"], c["BLOCK_SIZE_N"], c["BLOCK_SIZE_K"]], nw, lwu, eff))
            ranked.sort(key=lambda x: (x[1], -x[2]))
            rec["sweep"].append({"M": M, "S": S, "best": ranked[0], "ceil_div": smm.ceil_div(M, 128)})
    for (M, N, K) in workload.GEMM_SIZES:
        for S in workload.SM_COUNTS:
            best = workload.suggest_optimal_block_size(M, N, S)
            rec["workload"].append({
                "M": M, "N": N, "S": S,
                "metrics_128x256": workload.compute_wave_efficiency(M, N, 128, 256, S),
                "suggest": [best[0], best[1], best[2]],
            })
    rec["configs"] = [[c["BLOCK_SIZE_M"], c["BLOCK_SIZE_N"], c["BLOCK_SIZE_K"]] for c in smm.CONFIGS]
    (OUT / "wave.json").write_text(json.dumps(rec))


def _moe_reference_run(definition):
    src = definition.create_fused_moe_definition()["reference"]
    ns: dict = {}
    exec(src, ns)
    return src, ns["run"]


def gen_routing(definition) -> None:
    src, _ = _moe_reference_run(definition)
    # The two routing statements of the operator, executed as written.
    lines = [ln.strip() for ln in src.splitlines() if "topk" in ln and "=" in ln and "for" not in ln]
    lines = [ln for ln in lines if ln.startswith("topk_weights")]
    assert len(lines) == 2, lines
    out = {}
    for name, (T, E, k, seed) in {"mixtral": (512, 8, 2, 42), "dsv3": (256, 256, 8, 43),
                                   "small": (33, 16, 4, 44)}.items():
        g = torch.Generator().manual_seed(seed)
        logits = torch.randn((T, E), generator=g, dtype=torch.float32)
        ns = {"torch": torch, "gate_logits": logits, "TOP_K": k}
        for ln in lines:
            exec(ln, ns)
        out[f"{name}_logits"] = logits.numpy()
        out[f"{name}_ids"] = ns["topk_ids"].numpy().astype(np.int32)
        out[f"{name}_weights"] = ns["topk_weights"].numpy()
        out[f"{name}_k"] = np.array(k)
    np.savez_compressed(OUT / "routing.npz", **out)


def gen_moe_def(definition) -> None:
    _, run = _moe_reference_run(definition)
    out = {}
    for name, (T, H, I, E, k, seed) in {"a": (8, 32, 48, 8, 2, 1), "b": (12, 64, 32, 16, 4, 2)}.items():
        g = torch.Generator().manual_seed(seed)
        x = torch.randn((T, H), generator=g)
        logits = torch.randn((T, E), generator=g)
        w1 = torch.randn((E, I, H), generator=g) * 0.1
        w2 = torch.randn((E, H, I), generator=g) * 0.1
        w3 = torch.randn((E, I, H), generator=g) * 0.1
        res = torch.empty_like(x)
        run(x, logits, w1, w2, w3, res, T, H, I, E, k, 148)
        for key, v in dict(x=x, logits=logits, w1=w1, w2=w2, w3=w3, out=res).items():
            out[f"{name}_{key}"] = v.numpy()
        out[f"{name}_k"] = np.array(k)
    np.savez_compressed(OUT / "moe_def.npz", **out)


def _extract_kernel(path: Path, outer: str, name: str):
    """Return the source of the nested @triton.jit function `name` without decorators."""
    text = path.read_text()
    tree = ast.parse(text)
    for node in ast.walk(tree):
        if isinstance(node, ast.FunctionDef) and node.name == outer:
            for sub in ast.walk(node):
                if isinstance(sub, ast.FunctionDef) and sub.name == name:
                    seg_lines = text.splitlines()[sub.lineno - 1:sub.end_lineno]
                    return textwrap.dedent("\n".join(seg_lines))
    raise LookupError(name)


def _jit(src: str, name: str):
    import triton
    import triton.language as tl

    path = OUT / f"_tmp_{name}.py"
    path.write_text("import triton\nimport triton.language as tl\n\n@triton.jit\n" + src + "\n")
    try:
        import importlib.util

        spec = importlib.util.spec_from_file_location(f"_tmp_{name}", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return getattr(mod, name), triton, tl
    finally:
        pass


def gen_triton() -> None:
    out = {}
    src = _extract_kernel(REF / "elastikernel" / "sm_aware_matmul.py", "run_benchmark", "matmul_sm_aware")
    kern, triton, _ = _jit(src, "matmul_sm_aware")
    for name, (M, N, K, cfg, seed) in {"g1": (64, 80, 96, (32, 32, 32, 2), 3),
                                        "g2": (50, 64, 72, (16, 64, 32, 1), 4)}.items():
        g = torch.Generator().manual_seed(seed)
        a = torch.randn((M, K), generator=g).half()
        b = torch.randn((K, N), generator=g).half()
        c = torch.empty((M, N), dtype=torch.float16)
        bm, bn, bk, gm = cfg
        grid = (triton.cdiv(M, bm) * triton.cdiv(N, bn),)
        kern[grid](a, b, c, M, N, K, a.stride(0), a.stride(1), b.stride(0), b.stride(1), c.stride(0), c.stride(1),
                   BLOCK_SIZE_M=bm, BLOCK_SIZE_N=bn, BLOCK_SIZE_K=bk, GROUP_SIZE_M=gm, NUM_SMS=16)
        out.update({f"{name}_a": a.numpy(), f"{name}_b": b.numpy(), f"{name}_c": c.numpy()})

    src = _extract_kernel(REF / "elastikernel" / "sm_aware_benchmark.py", "run_moe_benchmark", "fused_moe_sm_aware")
    kern, triton, _ = _jit(src, "fused_moe_sm_aware")
    T, N, K, E = 40, 64, 64, 4
    g = torch.Generator().manual_seed(5)
    hs = torch.randn((T, K), generator=g).half()
    w = torch.randn((E * N, K), generator=g).half()
    offs = torch.tensor([0, 10, 10, 25, 40], dtype=torch.int32)
    o = torch.full((T, N), float("nan"), dtype=torch.float16)
    grid = (triton.cdiv(T, 16) * triton.cdiv(N, 64), E)
    kern[grid](hs, w, o, offs, T, N, K, E, hs.stride(0), hs.stride(1), w.stride(0), w.stride(1), o.stride(0),
               o.stride(1), BLOCK_SIZE_M=16, BLOCK_SIZE_N=64, BLOCK_SIZE_K=32, GROUP_SIZE_M=1, NUM_SMS=16)
    out.update({"seg_hs": hs.numpy(), "seg_w": w.numpy(), "seg_offsets": offs.numpy(), "seg_out": o.numpy()})
    np.savez_compressed(OUT / "triton_gemm.npz", **out)
    for p in OUT.glob("_tmp_*.py"):
        p.unlink()


def main() -> None:
    smm, workload, definition = _import_reference()
    gen_wave(smm, workload)
    gen_routing(definition)
    gen_moe_def(definition)
    gen_triton()
    print("golden vectors written to", OUT)


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser(description="regenerate tests/golden/ from the reference's own code")
    ap.add_argument("--reference-root", required=True, type=Path,
                    help="root of the reference checkout (holds the elastikernel/ package)")
    REF = ap.parse_args().reference_root.resolve()
    if not (REF / "elastikernel" / "sm_aware_matmul.py").exists():
        raise SystemExit(f"{REF} does not hold the reference's elastikernel/ package")
    main()
