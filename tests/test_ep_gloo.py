"""Expert-parallel MoE orchestration on CPU ranks (gloo, world_size 2 and 4).

The same ExpertParallelMoE dispatch / all-to-all / combine logic the GPU
path runs, driven by an oracle-backed CPU implementation of the kernel steps,
is checked against the single-process oracle with all experts: the
bookkeeping (destination sort, split sizes, per-row metadata, return order,
choice-order combine) must reproduce the MoE exactly. A second test makes one
rank leave before the exchange and checks that the other rank gets an error
instead of hanging (failure made on the host, no GPU involved).
"""
from __future__ import annotations

import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe as om

E, K_TOP, H, I = 8, 2, 32, 48


class CpuEPOps:
    """Oracle-backed CPU implementation of the kernel steps (test only)."""

    def route(self, logits, topk):
        ids, w = om.route_ref(logits.numpy(), topk)
        return torch.from_numpy(ids), torch.from_numpy(w)

    def dest_of(self, ids, experts_per_rank):
        return torch.div(ids, experts_per_rank, rounding_mode="floor").to(torch.int32)

    def permute_by_dest(self, dest, world, x):
        T, k = dest.shape
        r = om.permute_ref(dest.numpy(), world, 1)
        slots = torch.from_numpy(r["sorted_slots"][: T * k].astype(np.int64))
        return {"sorted_slots": slots, "expert_counts": torch.from_numpy(r["expert_counts"]),
                "x_perm": x[slots // k], "max_rows": T * k, "T": T, "topk": k}

    def pack_meta(self, perm, ids, wts, experts_per_rank):
        s = perm["sorted_slots"]
        return (ids.reshape(-1)[s] % experts_per_rank).to(torch.int32), wts.reshape(-1)[s].float()

    def slot_rows(self, perm):
        s = perm["sorted_slots"]
        out = torch.empty(s.numel(), dtype=torch.int64)
        out[s] = torch.arange(s.numel())
        return out

    def experts(self, x_recv, local_ids, w_recv, w1, w2, w3):
        y = torch.zeros((x_recv.shape[0], w2.shape[1]))
        for r in range(x_recv.shape[0]):
            e = int(local_ids[r])
            h = x_recv[r].float()
            a = torch.nn.functional.silu(w1[e].float() @ h) * (w3[e].float() @ h)
            y[r] = float(w_recv[r]) * (w2[e].float() @ a)
        return y

    def combine_rows(self, y_back, slot_row, T, topk):
        return y_back[slot_row.view(T, topk)].sum(dim=1)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights():
    g = torch.Generator().manual_seed(1234)
    w1 = torch.randn((E, I, H), generator=g) * 0.1
    w2 = torch.randn((E, H, I), generator=g) * 0.1
    w3 = torch.randn((E, I, H), generator=g) * 0.1
    return w1, w2, w3


def _worker(rank, world, port, q, mode):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        import datetime

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
        from elastikernel_b200.ep_moe import ExpertParallelMoE

        w1, w2, w3 = _weights()
        eg = E // world
        sl = slice(rank * eg, (rank + 1) * eg)
        moe = ExpertParallelMoE(E, K_TOP, w1[sl], w2[sl], w3[sl], ops=CpuEPOps())
        g = torch.Generator().manual_seed(100 + rank)
        T = 17 + 5 * rank  # ragged token counts per rank
        x = torch.randn((T, H), generator=g)
        logits = torch.randn((T, E), generator=g)
        if mode == "leave":
            moe(x, logits)  # one full step on both ranks
            if rank == 1:
                q.put((rank, "left"))
                q.close()
                q.join_thread()  # the message must reach the parent before the hard exit
                os._exit(0)  # leaves between steps, without cleanup
        # "chunked": the tokens go through in 3 chunks (ragged: T is not a multiple of 3)
        out = moe(x, logits, chunks=3) if mode == "chunked" else moe(x, logits)
        ref = om.moe_ref(x.numpy(), logits.numpy(), w1, w2, w3, K_TOP)
        err = float(np.abs(out.numpy() - ref).max() / np.abs(ref).max())
        q.put((rank, err))
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put((rank, "error: " + repr(e)[:200] + traceback.format_exc()[-300:]))


def _run(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, val = q.get(timeout=90)
        results[rank] = val
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("world,mode", [(2, "normal"), (4, "normal"), (2, "chunked")])
def test_ep_matches_single_process_oracle(world, mode):
    res = _run(world, mode)
    for rank, err in res.items():
        assert not isinstance(err, str), f"rank {rank}: {err}"
        assert err < 1e-5, f"rank {rank}: max rel err {err:.3e}"


def test_ep_rank_leaving_is_an_error_not_a_hang():
    res = _run(2, "leave")
    assert res[1] == "left"
    assert isinstance(res[0], str) and res[0].startswith("error"), res[0]
