"""Definition / workload / solution records for kernel benchmark harnesses
that use the FlashInfer-Bench schema, with the partition size NUM_SMS as an
axis (the reference emits the same kind of records in
sm_aware_agent/definition.py:14-175 and workload.py:13-83). Here the records
point at this package's operators (`definition.run_gemm`,
`definition.run_fused_moe`) and cover B200 partition sizes.

* definition: name, op_type, axes (var / const), inputs and outputs with
  symbolic shapes and dtypes, a `reference` CPU implementation of run(...),
  constraints, description, tags;
* workload: uuid, definition, axes_values, description;
* solution: which callable implements a definition, for which target.

Usage: python -m elastikernel_b200.bench_schema --out DIR
(writes definitions.json, workloads.jsonl, solutions.json).
"""
from __future__ import annotations

import argparse
import json
import uuid
from pathlib import Path

# B200 partition sizes: multiples of the 8-SM alignment up to the whole device
B200_SM_COUNTS = [16, 32, 48, 64, 80, 96, 112, 128, 136, 148]

GEMM_SIZES = [
    (1024, 1024, 1024), (2048, 2048, 2048), (4096, 4096, 4096), (8192, 8192, 8192),
    (4096, 14336, 4096), (14336, 4096, 4096), (1, 4096, 4096), (128, 4096, 4096),
]
MOE_TOKENS = [1, 16, 128, 1024, 4096]

_GEMM_REFERENCE = '''
import torch

def run(A, B, C, M, N, K, NUM_SMS):
    """C = A @ B, accumulated in fp32 (NUM_SMS does not change the result)."""
    C.copy_((A.float() @ B.float()).to(C.dtype))
'''

_MOE_REFERENCE = '''
import torch
import torch.nn.functional as F

def run(hidden_states, gate_logits, w1, w2, w3, out, M, K, N, NUM_EXPERTS, TOP_K, NUM_SMS):
    """Softmax top-k routing (weights renormalised over the k choices), per
    choice silu(w1[e] h) * (w3[e] h) through w2[e], summed with the weights."""
    probs = gate_logits.float().softmax(dim=-1)
    w, ids = torch.topk(probs, TOP_K, dim=-1)
    w = w / w.sum(dim=-1, keepdim=True)
    h = hidden_states.float()
    acc = torch.zeros((M, K), dtype=torch.float32)
    for e in range(NUM_EXPERTS):
        tok, choice = (ids == e).nonzero(as_tuple=True)
        if tok.numel() == 0:
            continue
        x = h[tok]
        a = F.silu(x @ w1[e].float().t()) * (x @ w3[e].float().t())
        acc.index_add_(0, tok, (a @ w2[e].float().t()) * w[tok, choice].unsqueeze(1))
    out.copy_(acc.to(out.dtype))
'''


def gemm_definition(name: str = "gemm_sm_aware", dtype: str = "bfloat16") -> dict:
    return {
        "name": name,
        "op_type": "gemm",
        "axes": {
            "M": {"type": "var", "description": "rows of A and C"},
            "N": {"type": "var", "description": "columns of B and C"},
            "K": {"type": "var", "description": "reduction dimension"},
            "NUM_SMS": {"type": "var", "description": "SMs of the green-context partition the kernel runs in"},
        },
        "inputs": {
            "A": {"shape": ["M", "K"], "dtype": dtype, "description": "left operand, row-major"},
            "B": {"shape": ["K", "N"], "dtype": dtype, "description": "right operand, row-major"},
        },
        "outputs": {"C": {"shape": ["M", "N"], "dtype": dtype, "description": "product, written in place"}},
        "reference": _GEMM_REFERENCE,
        "constraints": ["M > 0", "N > 0", "K > 0", "NUM_SMS > 0"],
        "description": "GEMM planned for the SM count of the partition it runs in",
        "tags": ["gemm", "sm-aware", "sm_100a", "tcgen05"],
    }


def fused_moe_definition(name: str = "fused_moe_sm_aware", num_experts: int = 8, top_k: int = 2,
                         dtype: str = "bfloat16") -> dict:
    return {
        "name": name,
        "op_type": "moe",
        "axes": {
            "M": {"type": "var", "description": "tokens"},
            "K": {"type": "var", "description": "model hidden size"},
            "N": {"type": "var", "description": "expert intermediate size"},
            "NUM_EXPERTS": {"type": "const", "value": num_experts},
            "TOP_K": {"type": "const", "value": top_k},
            "NUM_SMS": {"type": "var", "description": "SMs of the green-context partition"},
        },
        "inputs": {
            "hidden_states": {"shape": ["M", "K"], "dtype": dtype, "description": "token activations"},
            "gate_logits": {"shape": ["M", "NUM_EXPERTS"], "dtype": "float32", "description": "router logits"},
            "w1": {"shape": ["NUM_EXPERTS", "N", "K"], "dtype": dtype, "description": "gate projections (SiLU side)"},
            "w2": {"shape": ["NUM_EXPERTS", "K", "N"], "dtype": dtype, "description": "down projections"},
            "w3": {"shape": ["NUM_EXPERTS", "N", "K"], "dtype": dtype, "description": "up projections"},
        },
        "outputs": {"out": {"shape": ["M", "K"], "dtype": dtype, "description": "layer output, written in place"}},
        "reference": _MOE_REFERENCE,
        "constraints": ["M > 0", "TOP_K <= NUM_EXPERTS", "NUM_SMS > 0", "K % 16 == 0", "N % 16 == 0"],
        "description": "Fused MoE layer (routing, SwiGLU experts, weighted combine) planned per partition size",
        "tags": ["moe", "sm-aware", "sm_100a", "tcgen05"],
    }


def gemm_workloads(definition: str = "gemm_sm_aware", sm_counts=None, sizes=None) -> list[dict]:
    out = []
    for sm in sm_counts or B200_SM_COUNTS:
        for M, N, K in sizes or GEMM_SIZES:
            out.append({"uuid": str(uuid.uuid4()), "definition": definition,
                        "axes_values": {"M": M, "N": N, "K": K, "NUM_SMS": sm},
                        "description": f"GEMM {M}x{N}x{K} on {sm} SMs"})
    return out


def moe_workloads(definition: str = "fused_moe_sm_aware", hidden: int = 4096, inter: int = 14336,
                  sm_counts=None, tokens=None) -> list[dict]:
    out = []
    for sm in sm_counts or B200_SM_COUNTS:
        for M in tokens or MOE_TOKENS:
            out.append({"uuid": str(uuid.uuid4()), "definition": definition,
                        "axes_values": {"M": M, "K": hidden, "N": inter, "NUM_SMS": sm},
                        "description": f"fused MoE, {M} tokens, K={hidden} N={inter}, on {sm} SMs"})
    return out


def solutions() -> list[dict]:
    """The callables of this package that implement the definitions."""
    return [
        {"definition": "gemm_sm_aware", "entry_point": "elastikernel_b200.definition:run_gemm",
         "target": "sm_100a", "language": "cuda", "library": "elastikernel_b200/_ek.so"},
        {"definition": "fused_moe_sm_aware", "entry_point": "elastikernel_b200.definition:run_fused_moe",
         "target": "sm_100a", "language": "cuda", "library": "elastikernel_b200/_ek.so"},
    ]


def write_all(out_dir) -> dict:
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    defs = [gemm_definition(), fused_moe_definition()]
    wls = gemm_workloads() + moe_workloads()
    (out / "definitions.json").write_text(json.dumps(defs, indent=2))
    (out / "workloads.jsonl").write_text("".join(json.dumps(w) + "\n" for w in wls))
    (out / "solutions.json").write_text(json.dumps(solutions(), indent=2))
    return {"definitions": len(defs), "workloads": len(wls), "dir": str(out)}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--out", required=True)
    print(write_all(ap.parse_args().out))


if __name__ == "__main__":
    main()
