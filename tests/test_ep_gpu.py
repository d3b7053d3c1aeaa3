"""Expert-parallel MoE on GPUs.

* world size 1 (any single-GPU box): the EP data flow (destination sort,
  metadata packing, slot rows, indexed combine) around the local experts must
  reproduce the fused single-GPU layer, for bf16 and for e4m3 block-scaled
  experts with e4m3 dispatch;
* fixed-capacity exchanges (equal splits, padding rows on a dummy expert)
  give the exact exchange's result; a capacity too small for the routing
  drops the slots past it, raises EK_STATUS_CAPACITY, and leaves every token
  that kept its slots unchanged;
* world size 2 (skipped with fewer GPUs): NCCL all-to-all over NVLink, each
  rank's EP output against the fused layer run with all experts on that rank.
Tolerance: max|out - ref| / max|ref| <= 1e-2 (same kernels, same math).
"""
from __future__ import annotations

import os
import socket
import traceback

import pytest
import torch

from oracle.gemm import max_rel_err

pytestmark = pytest.mark.gpu

E, K_TOP, H, I = 16, 4, 512, 256


def _weights(dev):
    g = torch.Generator(device=dev).manual_seed(77)
    w1 = (torch.randn((E, I, H), device=dev, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn((E, H, I), device=dev, generator=g) * 0.02).to(torch.bfloat16)
    w3 = (torch.randn((E, I, H), device=dev, generator=g) * 0.02).to(torch.bfloat16)
    return w1, w2, w3


def _tokens(dev, rank, T):
    g = torch.Generator(device=dev).manual_seed(500 + rank)
    x = torch.randn((T, H), device=dev, generator=g).to(torch.bfloat16)
    logits = torch.randn((T, E), device=dev, generator=g)
    return x, logits


def test_ep_world1_bf16(cuda_dev):
    from elastikernel_b200 import _ops
    from elastikernel_b200.ep_moe import ExpertParallelMoE

    w1, w2, w3 = _weights(cuda_dev)
    x, logits = _tokens(cuda_dev, 0, 333)
    out = ExpertParallelMoE(E, K_TOP, w1, w2, w3)(x, logits)
    ref = _ops.fused_moe(x, logits, w1, w2, w3, K_TOP)
    torch.cuda.synchronize()
    assert max_rel_err(out, ref.float().cpu().numpy()) <= 1e-2


def test_ep_world1_fp8(cuda_dev):
    from elastikernel_b200 import _ops
    from elastikernel_b200.ep_moe import ExpertParallelMoE

    w1, w2, w3 = _weights(cuda_dev)
    qw = _ops.quant_moe_weights_fp8(w1, w2, w3)
    x, logits = _tokens(cuda_dev, 0, 333)
    out = ExpertParallelMoE(E, K_TOP, qw=qw)(x, logits)
    ref = _ops.fused_moe_fp8(x, logits, qw, K_TOP)
    torch.cuda.synchronize()
    # e4m3 dispatch quantises per token row before the gather; the fused layer
    # quantises the gathered rows: the same values, so the results agree closely
    assert max_rel_err(out, ref.float().cpu().numpy()) <= 1e-2


@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("capacity", ["auto", 333 * K_TOP + 37])
def test_ep_world1_capacity(cuda_dev, fp8, capacity):
    """Fixed-capacity exchanges ("auto": exactly the routed rows on one rank;
    an explicit capacity above them: padding rows on the dummy expert)
    against the exact exchanges."""
    from elastikernel_b200 import _lib, _ops
    from elastikernel_b200.ep_moe import ExpertParallelMoE

    w1, w2, w3 = _weights(cuda_dev)
    kw = {"qw": _ops.quant_moe_weights_fp8(w1, w2, w3, pow2=True)} if fp8 else {"w1": w1, "w2": w2, "w3": w3}
    x, logits = _tokens(cuda_dev, 0, 333)
    ref = ExpertParallelMoE(E, K_TOP, **kw)(x, logits)
    _lib.device_status(0, clear=True)
    out = ExpertParallelMoE(E, K_TOP, capacity=capacity, **kw)(x, logits)
    st = _lib.device_status(0, clear=True)
    assert st == 0, f"status {st:#x}"
    assert max_rel_err(out, ref.float().cpu().numpy()) <= 1e-3


def test_ep_world1_capacity_overflow_flags(cuda_dev):
    """One rank, capacity 50 rows short of the T*k routed slots: the slots
    are dropped in destination-sorted (slot index) order, so the tokens whose
    k slots all lie below the capacity are unchanged; the status word says
    slots were dropped."""
    from elastikernel_b200 import _lib
    from elastikernel_b200.ep_moe import ExpertParallelMoE

    w1, w2, w3 = _weights(cuda_dev)
    T = 333
    C = T * K_TOP - 50
    x, logits = _tokens(cuda_dev, 0, T)
    ref = ExpertParallelMoE(E, K_TOP, w1, w2, w3)(x, logits)
    _lib.device_status(0, clear=True)
    out = ExpertParallelMoE(E, K_TOP, w1, w2, w3, capacity=C)(x, logits)
    st = _lib.device_status(0, clear=True)
    assert st & _lib.EK_STATUS_CAPACITY and not st & ~_lib.EK_STATUS_CAPACITY, f"status {st:#x}"
    keep = C // K_TOP
    assert max_rel_err(out[:keep], ref[:keep].float().cpu().numpy()) <= 1e-3


@pytest.mark.parametrize("fp8", [False, True])
def test_ep_world1_chunked_streams(cuda_dev, fp8):
    """Chunks pipelined over two green-context partitions (experts on the
    large one, routing / dispatch / combine on the small one) give the same
    layer as the unchunked forward."""
    from elastikernel_b200 import _ops
    from elastikernel_b200.ep_moe import CudaEPOps, ExpertParallelMoE
    from elastikernel_b200.green_ctx import create_disjoint_partitions

    w1, w2, w3 = _weights(cuda_dev)
    (comm, _), (comp, comp_sms) = create_disjoint_partitions(cuda_dev, [32, 112])
    kw = {"qw": _ops.quant_moe_weights_fp8(w1, w2, w3)} if fp8 else {"w1": w1, "w2": w2, "w3": w3}
    moe = ExpertParallelMoE(E, K_TOP, ops=CudaEPOps(num_sms=comp_sms), **kw)
    x, logits = _tokens(cuda_dev, 0, 333)
    ref = moe(x, logits)
    out = moe(x, logits, chunks=3, compute_stream=comp, comm_stream=comm)
    torch.cuda.synchronize()
    assert out.shape == ref.shape
    assert max_rel_err(out, ref.float().cpu().numpy()) <= 1e-3


@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("groups", [2, 4])
def test_ep_world1_expert_groups_streams(cuda_dev, fp8, groups):
    """Expert groups pipelined over two green-context partitions (each group's
    exchange on the small one, its GEMMs on the large one) give the layer of
    the ungrouped forward, to fp32-sum-order tolerance (the groups run the same
    per-row math on the same rows)."""
    from elastikernel_b200 import _ops
    from elastikernel_b200.ep_moe import CudaEPOps, ExpertParallelMoE
    from elastikernel_b200.green_ctx import create_disjoint_partitions

    w1, w2, w3 = _weights(cuda_dev)
    (comm, _), (comp, comp_sms) = create_disjoint_partitions(cuda_dev, [32, 112])
    kw = ({"qw": _ops.quant_moe_weights_fp8(w1, w2, w3, pow2=True)} if fp8
          else {"w1": w1, "w2": w2, "w3": w3})
    moe = ExpertParallelMoE(E, K_TOP, ops=CudaEPOps(num_sms=comp_sms), capacity="auto", **kw)
    x, logits = _tokens(cuda_dev, 0, 333)
    ref = moe(x, logits)
    out = moe(x, logits, groups=groups, compute_stream=comp, comm_stream=comm)
    out_seq = moe(x, logits, groups=groups)  # the same steps on one stream
    torch.cuda.synchronize()
    assert out.shape == ref.shape
    assert max_rel_err(out, ref.float().cpu().numpy()) <= 1e-3
    assert torch.equal(out, out_seq)


def _lib_status(dev) -> int:
    from elastikernel_b200 import _lib

    return _lib.device_status(dev.index if dev.index is not None else 0, clear=True)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    try:
        import datetime

        import torch.distributed as dist

        from elastikernel_b200 import _ops
        from elastikernel_b200.ep_moe import ExpertParallelMoE

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        w1, w2, w3 = _weights(dev)
        eg = E // world
        sl = slice(rank * eg, (rank + 1) * eg)
        x, logits = _tokens(dev, rank, 200 + 37 * rank)
        out = ExpertParallelMoE(E, K_TOP, w1[sl].contiguous(), w2[sl].contiguous(), w3[sl].contiguous())(x, logits)
        ref = _ops.fused_moe(x, logits, w1, w2, w3, K_TOP)
        err_bf16 = max_rel_err(out, ref.float().cpu().numpy())
        qw_all = _ops.quant_moe_weights_fp8(w1, w2, w3)
        qw = _ops.quant_moe_weights_fp8(w1[sl].contiguous(), w2[sl].contiguous(), w3[sl].contiguous())
        out8 = ExpertParallelMoE(E, K_TOP, qw=qw)(x, logits)
        ref8 = _ops.fused_moe_fp8(x, logits, qw_all, K_TOP)
        err_fp8 = max_rel_err(out8, ref8.float().cpu().numpy())
        # the same layer pipelined in 2 chunks over two streams (dispatch of one
        # chunk and combine of the other overlap the experts)
        comp, comm = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        out8c = ExpertParallelMoE(E, K_TOP, qw=qw)(x, logits, chunks=2, compute_stream=comp, comm_stream=comm)
        err_fp8 = max(err_fp8, max_rel_err(out8c, ref8.float().cpu().numpy()))
        # fixed-capacity exchanges (both ranks route the same number of tokens)
        xc, lc = _tokens(dev, rank, 256)
        outc = ExpertParallelMoE(E, K_TOP, qw=qw, capacity="auto")(xc, lc, chunks=2, compute_stream=comp,
                                                                     comm_stream=comm)
        refc = _ops.fused_moe_fp8(xc, lc, qw_all, K_TOP)
        err_fp8 = max(err_fp8, max_rel_err(outc, refc.float().cpu().numpy()))
        # expert groups: each group's rows and results cross NVLink while another group computes
        outg = ExpertParallelMoE(E, K_TOP, qw=qw, capacity="auto")(xc, lc, groups=2, compute_stream=comp,
                                                                     comm_stream=comm)
        err_fp8 = max(err_fp8, max_rel_err(outg, refc.float().cpu().numpy()))
        # the equal-split exchanges on a communication partition's own stream
        # (an NCCL communicator driven directly): the same bytes as
        # all_to_all_single, and the same grouped layer
        from elastikernel_b200.green_ctx import create_disjoint_partitions
        from elastikernel_b200.nccl_stream import StreamAllToAll

        (p_comm, _), (p_comp, p_sms) = create_disjoint_partitions(dev, [32], with_remainder=True)
        sa = StreamAllToAll()
        inp = torch.randn(world * 4099, device=dev)
        want = torch.empty_like(inp)
        dist.all_to_all_single(want, inp)
        got = torch.empty_like(inp)
        with torch.cuda.stream(p_comm):
            sa.all_to_all(got, inp)
        p_comm.synchronize()
        if not torch.equal(got, want):
            raise AssertionError("StreamAllToAll differs from all_to_all_single")
        from elastikernel_b200.ep_moe import CudaEPOps

        outs = ExpertParallelMoE(E, K_TOP, qw=qw, capacity="auto", ops=CudaEPOps(num_sms=p_sms), stream_a2a=sa)(
            xc, lc, groups=2, compute_stream=p_comp, comm_stream=p_comm)
        err_fp8 = max(err_fp8, max_rel_err(outs, refc.float().cpu().numpy()))
        torch.cuda.synchronize()
        dist.barrier()
        sa.close()
        # the copy-engine exchange: the same bytes as all_to_all_single (three
        # calls of one key: both buffers and a reuse), a multi-part key, and
        # the grouped layer over it
        from elastikernel_b200.p2p_exchange import P2PAllToAll

        px = P2PAllToAll()
        for rep in range(3):
            inp = torch.randn(world * 4096, device=dev) + rep
            want = torch.empty_like(inp)
            dist.all_to_all_single(want, inp)
            p_comm.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(p_comm):
                got = px.all_to_all(inp, "probe").clone()
            p_comm.synchronize()
            if not torch.equal(got, want):
                raise AssertionError(f"P2PAllToAll differs from all_to_all_single (call {rep})")
        parts = [torch.randn(world * 512, device=dev) for _ in range(3)]
        for i, t in enumerate(parts):
            px.all_to_all(t, "multi", part=i, parts=3)
        torch.cuda.synchronize()
        whole = px.buffer_view("multi", torch.float32, (3, world * 512))
        for i, t in enumerate(parts):
            want = torch.empty_like(t)
            dist.all_to_all_single(want, t)
            if not torch.equal(whole[i], want):
                raise AssertionError(f"P2PAllToAll part {i} differs")
        moe_p = ExpertParallelMoE(E, K_TOP, qw=qw, capacity="auto", ops=CudaEPOps(num_sms=p_sms), p2p=px)
        for _ in range(3):  # the arenas' two buffers, then the first again
            outp = moe_p(xc, lc, groups=2, compute_stream=p_comp, comm_stream=p_comm)
            err_fp8 = max(err_fp8, max_rel_err(outp, refc.float().cpu().numpy()))
        torch.cuda.synchronize()
        st = _lib_status(dev)
        if st:
            raise AssertionError(f"device status {st} after the copy-engine exchanges")
        px.close()
        # device-side epochs: the grouped layer captured in a CUDA graph and
        # replayed gives the eager layer's output, replay after replay
        from elastikernel_b200.graph import Captured

        pxd = P2PAllToAll(device_epochs=True)
        moe_d = ExpertParallelMoE(E, K_TOP, qw=qw, capacity="auto", ops=CudaEPOps(num_sms=p_sms), p2p=pxd)
        side = torch.cuda.Stream(dev)
        with torch.cuda.stream(side):
            eager = moe_d(xc, lc, groups=2, compute_stream=p_comp, comm_stream=p_comm)
            cap = Captured(lambda: moe_d(xc, lc, groups=2, compute_stream=p_comp, comm_stream=p_comm), side)
            for _ in range(3):
                yg = cap()
                side.synchronize()
                if not torch.equal(yg, eager):
                    raise AssertionError("graph-replayed EP layer differs from the eager one")
        err_fp8 = max(err_fp8, max_rel_err(yg, refc.float().cpu().numpy()))
        del cap
        torch.cuda.synchronize()
        st = _lib_status(dev)
        if st:
            raise AssertionError(f"device status {st} after the graph-replayed exchanges")
        pxd.close()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, (err_bf16, err_fp8)))
    except Exception as e:
        q.put((rank, "error: " + repr(e)[:300] + traceback.format_exc()[-600:]))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_two_gpus_nccl():
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, v = q.get(timeout=300)
        res[r] = v
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    for r, v in res.items():
        assert not isinstance(v, str), f"rank {r}: {v}"
        assert v[0] <= 1e-2 and v[1] <= 1e-2, f"rank {r}: errors {v}"
