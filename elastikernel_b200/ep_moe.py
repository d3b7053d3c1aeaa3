"""Expert-parallel fused MoE across the GPUs of one node (one process per GPU).

Experts are split contiguously: rank g owns experts [g*Eg, (g+1)*Eg),
Eg = num_experts / world_size. One forward pass:

1. route locally (softmax top-k, renormalised);
2. sort the (token, choice) slots by destination rank and gather their rows
   (ek_moe_permute with the ranks as "experts", block_m = 1), with each row's
   expert id local to its destination and its routing weight (ek_ep_pack_meta);
3. exchange the per-rank counts, then the rows and their metadata
   (all-to-all over NCCL / NVLink);
4. run the received rows through the local experts (packed expert-major
   GEMMs), each output row already multiplied by its routing weight;
5. send the rows back (all-to-all with the splits reversed);
6. sum every token's k returned rows in choice order (ek_moe_combine_rows).

Two ways to size the exchanges. By default the per-rank counts are
exchanged and read on the host, which sizes both all-to-alls exactly. With
``capacity`` set, every rank sends every other rank exactly ``capacity`` rows
(padding rows carry a dummy expert id and are never computed), so the
exchanges have equal splits the host knows in advance: nothing is read back
and the layer can be captured in a CUDA graph. "auto" sizes the capacity for
a uniform routing (mean + 6 standard deviations of a destination's count);
slots past it are dropped and flagged in the device status word
(EK_STATUS_CAPACITY).

The reference has no multi-GPU path (its only parallelism is SM partitioning
inside one GPU); this follows the expert-parallel MoE layout of the hot-path
spec. The kernel steps go through an ``ops`` object: ``CudaEPOps`` (the
product, C-ABI kernels) or any object with the same methods (the tests drive
the same orchestration with a CPU implementation on gloo ranks).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass
class Dispatched:
    """Per-forward bookkeeping kept between dispatch and combine."""

    T: int
    topk: int
    send_counts: list | None  # exact exchanges: rows to / from every rank
    recv_counts: list | None
    slot_row: torch.Tensor  # [T*k] row of every slot in send order (-1: dropped)
    capacity: int = 0  # fixed-capacity exchanges: rows per rank (0: exact)


class CudaEPOps:
    """Kernel steps of the expert-parallel MoE on the C-ABI kernels."""

    def __init__(self, num_sms: int | None = None):
        self.num_sms = num_sms

    def route(self, logits, topk):
        from . import _ops

        return _ops.moe_route(logits, topk)

    def dest_of(self, ids, experts_per_rank):
        return torch.div(ids, experts_per_rank, rounding_mode="floor").to(torch.int32)

    def permute_by_dest(self, dest, world, x):
        from . import _ops

        return _ops.moe_permute(dest.contiguous(), world, x=x, block_m=1)

    def pack_meta(self, perm, ids, wts, experts_per_rank):
        from . import _lib, _ops

        rows = perm["max_rows"]
        dev = ids.device
        local_ids = torch.empty(rows, dtype=torch.int32, device=dev)
        wout = torch.empty(rows, dtype=torch.float32, device=dev)
        with _ops._on_device(dev):
            _lib.check(_lib.lib().ek_ep_pack_meta(perm["sorted_slots"].data_ptr(), rows, ids.data_ptr(),
                                                  wts.data_ptr(), ids.numel(), experts_per_rank,
                                                  local_ids.data_ptr(), wout.data_ptr(),
                                                  _ops.current_stream_handle(dev)), "ek_ep_pack_meta")
        return local_ids, wout

    def slot_rows(self, perm):
        from . import _lib, _ops

        dev = perm["sorted_slots"].device
        n = perm["T"] * perm["topk"]
        slot_row = torch.full((n,), -1, dtype=torch.int32, device=dev)
        with _ops._on_device(dev):
            _lib.check(_lib.lib().ek_moe_slot_rows(perm["sorted_slots"].data_ptr(), perm["num_rows_padded"].data_ptr(),
                                                   perm["max_rows"], n, slot_row.data_ptr(),
                                                   _ops.current_stream_handle(dev)), "ek_moe_slot_rows")
        return slot_row

    def capacity_layout(self, perm, ids, wts, experts_per_rank, world, capacity):
        """Fixed-capacity send layout (ek_ep_capacity_layout): per capacity
        row its slot, local expert id (experts_per_rank for padding) and
        weight, and every slot's capacity row (-1 when dropped)."""
        from . import _lib, _ops

        dev = ids.device
        n = ids.numel()
        rows = world * capacity
        out = {"slots": torch.empty(rows, dtype=torch.int32, device=dev),
               "local_ids": torch.empty(rows, dtype=torch.int32, device=dev),
               "weights": torch.empty(rows, dtype=torch.float32, device=dev),
               "slot_row": torch.empty(n, dtype=torch.int32, device=dev),
               "rows": torch.full((1,), rows, dtype=torch.int32, device=dev), "n": n, "topk": ids.shape[1]}
        with _ops._on_device(dev):
            _lib.check(_lib.lib().ek_ep_capacity_layout(
                perm["sorted_slots"].data_ptr(), perm["expert_counts"].data_ptr(), world, capacity, n, ids.data_ptr(),
                wts.data_ptr(), experts_per_rank, out["slots"].data_ptr(), out["local_ids"].data_ptr(),
                out["weights"].data_ptr(), out["slot_row"].data_ptr(), _ops.current_stream_handle(dev)),
                "ek_ep_capacity_layout")
        return out

    def gather_capacity(self, cap, src):
        """Rows of `src` (one per token) in the capacity layout; padding rows are left unwritten."""
        from . import _lib, _ops

        dev = src.device
        rows = cap["slots"].numel()
        dst = torch.empty((rows,) + tuple(src.shape[1:]), dtype=src.dtype, device=dev)
        row_bytes = src[0].numel() * src.element_size()
        with _ops._on_device(dev):
            _lib.check(_lib.lib().ek_moe_gather_rows(cap["slots"].data_ptr(), cap["rows"].data_ptr(), rows, cap["n"],
                                                     cap["topk"], src.data_ptr(), row_bytes, dst.data_ptr(),
                                                     _ops.current_stream_handle(dev)), "ek_moe_gather_rows")
        return dst

    @staticmethod
    def _local_permute(local_ids, E, x, block_m, dummy):
        """Expert-major layout of the received rows. With `dummy`, ids equal to
        E mark padding rows: they form an extra expert after the real ones,
        which the GEMMs (given E experts) never reach."""
        from . import _ops

        R = local_ids.numel()
        perm = _ops.moe_permute(local_ids.view(R, 1), E + 1 if dummy else E, x=x, block_m=block_m)
        if dummy:
            perm = dict(perm, E=E, expert_counts=perm["expert_counts"][:E])
        return perm

    def experts(self, x_recv, local_ids, w_recv, w1, w2, w3, dummy: bool = False):
        """Local experts on the received rows; row r of the result is
        w_recv[r] * expert(local_ids[r])(x_recv[r]) (rows of the dummy
        expert, with `dummy`, are not computed)."""
        from . import _ops

        R = x_recv.shape[0]
        H = w2.shape[1]
        if R == 0:
            return torch.empty((0, H), dtype=torch.bfloat16, device=x_recv.device)
        E = w1.shape[0]
        layout = _ops.moe_layout(int(self.num_sms or _ops._stream_sms(x_recv.device, _ops.current_stream_handle(
            x_recv.device))), E, R)
        if layout == "packed" or dummy:
            perm = self._local_permute(local_ids, E, x_recv, 1, dummy)
            act = _ops.moe_gate_up_packed(perm, w1, w3, num_sms=self.num_sms)
            return _ops.moe_down_packed(perm, act, w2, w_recv, num_sms=self.num_sms)
        perm = _ops.moe_permute(local_ids.view(R, 1), E, x=x_recv)
        act = _ops.moe_gate_up(perm, w1, w3, num_sms=self.num_sms)
        return _ops.moe_down(perm, act, w2, w_recv, num_sms=self.num_sms)

    # ---------------------------------------------------------------- FP8 dispatch
    def quant_rows(self, x, pow2: bool = False):
        from . import _ops

        return _ops.quant_e4m3(x, block=(1, 128), pow2=pow2)

    def gather_rows(self, perm, src):
        """Rows of `src` in the permutation's order (e.g. the scales of gathered FP8 rows)."""
        from . import _lib, _ops

        dev = src.device
        rows = perm["max_rows"]
        dst = torch.empty((rows,) + tuple(src.shape[1:]), dtype=src.dtype, device=dev)
        row_bytes = src[0].numel() * src.element_size()
        with _ops._on_device(dev):
            _lib.check(_lib.lib().ek_moe_gather_rows(perm["sorted_slots"].data_ptr(), perm["num_rows_padded"].data_ptr(),
                                                     rows, perm["T"] * perm["topk"], perm["topk"], src.data_ptr(),
                                                     row_bytes, dst.data_ptr(), _ops.current_stream_handle(dev)),
                       "ek_moe_gather_rows")
        return dst

    def experts_fp8(self, xq_recv, xs_recv, local_ids, w_recv, qw, dummy: bool = False):
        """Local block-scaled FP8 experts on received e4m3 rows and their 1 x 128 scales."""
        from . import _ops

        R = xq_recv.shape[0]
        if R == 0:
            return torch.empty((0, qw["H"]), dtype=torch.bfloat16, device=xq_recv.device)
        perm = self._local_permute(local_ids, qw["E"], xq_recv, 1, dummy)
        xs = _ops.moe_gather_cols_f32(perm, xs_recv)  # K-block-major scales of the gathered rows
        act = _ops.moe_gate_up_fp8bs(perm, perm["x_perm"], xs, qw, num_sms=self.num_sms)
        aq, as_ = _ops.quant_e4m3_kmajor(act, pow2=bool(qw.get("pow2", False)))
        return _ops.moe_down_fp8bs(perm, aq, as_, qw, w_recv, num_sms=self.num_sms)

    def combine_rows(self, y_back, slot_row, T, topk):
        from . import _lib, _ops

        dev = y_back.device
        H = y_back.shape[1]
        out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        with _ops._on_device(dev):
            _lib.check(_lib.lib().ek_moe_combine_rows(y_back.data_ptr(), slot_row.data_ptr(), out.data_ptr(), T, topk,
                                                      H, y_back.shape[0], _ops.current_stream_handle(dev)),
                       "ek_moe_combine_rows")
        return out


class ExpertParallelMoE:
    """Expert-parallel MoE layer. Each rank holds the weights of its own experts:
    w1, w3 [Eg, I, H] and w2 [Eg, H, I] (bf16), or ``qw`` = their e4m3
    block-scaled form (_ops.quant_moe_weights_fp8), in which case the rows
    are dispatched as e4m3 with 1 x 128 scales (half the bytes of bf16)."""

    def __init__(self, num_experts: int, topk: int, w1=None, w2=None, w3=None, group=None, ops=None, qw=None,
                 capacity=None, stream_a2a=None, p2p=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if num_experts % self.world != 0:
            raise ValueError(f"{num_experts} experts do not split over {self.world} ranks")
        self.num_experts = num_experts
        self.experts_per_rank = num_experts // self.world
        self.fp8 = qw is not None
        held = qw["E"] if self.fp8 else w1.shape[0]
        if held != self.experts_per_rank:
            raise ValueError(f"rank holds {held} experts, expected {self.experts_per_rank}")
        self.topk = topk
        self.w1, self.w2, self.w3, self.qw = w1, w2, w3, qw
        self.ops = ops or CudaEPOps()
        self._marks = None  # (phase, CUDA event) pairs while profile_phases runs
        if capacity is not None and capacity != "auto" and int(capacity) < 0:
            raise ValueError("capacity must be None, 'auto' or a row count >= 0")
        self.capacity = capacity  # None: exact exchanges (host read of the counts)
        # nccl_stream.StreamAllToAll: equal-split exchanges launched on the
        # current stream (e.g. a communication partition's) instead of the
        # process group's internal one
        self.stream_a2a = stream_a2a
        # p2p_exchange.P2PAllToAll: the grouped layer's equal-split exchanges
        # by copy engines into IPC-mapped receive buffers (no NCCL, no SM)
        self.p2p = p2p

    def capacity_rows(self, n_slots: int, groups: int = 1) -> int:
        """Rows per destination of a fixed-capacity exchange of n_slots slots,
        the destinations being the ranks (groups = 1) or the (expert group,
        rank) pairs of a grouped layer: the given count (split evenly over the
        groups), or for "auto" the mean of a uniform routing plus 6 standard
        deviations of a destination's (binomial) count, plus 16, rounded up
        to 16 (a single destination: exactly n_slots). Every rank must use the
        same value, so with "auto" every rank passes the same number of
        tokens."""
        if self.capacity != "auto":
            return -(-int(self.capacity) // groups)
        G = self.world * groups
        if G == 1:
            return n_slots
        m = n_slots / G
        c = math.ceil(m + 6.0 * math.sqrt(m * (1.0 - 1.0 / G)) + 16)
        return min(n_slots, -(-c // 16) * 16)

    def _mark(self, name: str) -> None:
        if self._marks is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._marks.append((name, ev))

    # ---------------------------------------------------------------- phases
    def _a2a(self, out, inp, out_splits, in_splits):
        if self.world == 1:
            out.copy_(inp)
            return out
        if self.stream_a2a is not None and out_splits is None and in_splits is None and out.is_cuda:
            return self.stream_a2a.all_to_all(out, inp)
        dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits,
                               group=self.group)
        return out

    def dispatch(self, x, gate_logits):
        """Route, sort by destination and exchange rows + metadata.
        Returns (x_recv, local_ids_recv, w_recv, Dispatched)."""
        if self.capacity is not None:
            return self._dispatch_capacity(x, gate_logits)
        ops = self.ops
        T, H = x.shape
        self._mark("start")
        ids, wts = ops.route(gate_logits, self.topk)
        dest = ops.dest_of(ids, self.experts_per_rank)
        xs = None
        if self.fp8:
            # e4m3 rows + 1 x 128 scales travel instead of bf16 (power-of-two
            # scales when the experts' GEMMs apply them in the tensor cores)
            x, xs = (ops.quant_rows(x, pow2=True) if self.qw.get("pow2") else ops.quant_rows(x))
        perm = ops.permute_by_dest(dest, self.world, x)
        local_ids, row_w = ops.pack_meta(perm, ids, wts, self.experts_per_rank)
        counts = perm["expert_counts"].to(torch.int64)
        self._mark("route_permute")
        recv = torch.empty_like(counts)
        self._a2a(recv, counts, None, None)
        send_counts = counts.cpu().tolist()
        recv_counts = recv.cpu().tolist()
        self._mark("count_exchange")
        R = int(sum(recv_counts))
        n = T * self.topk
        x_send = perm["x_perm"][:n]
        x_recv = torch.empty((R, H), dtype=x.dtype, device=x.device)
        if self.fp8:  # byte view: the exchange does not need to know the float8 type
            self._a2a(x_recv.view(torch.uint8), x_send.view(torch.uint8), recv_counts, send_counts)
            xs_send = ops.gather_rows(perm, xs)[:n]
            xs_recv = torch.empty((R, xs.shape[1]), dtype=torch.float32, device=x.device)
            self._a2a(xs_recv, xs_send, recv_counts, send_counts)
            x_recv = (x_recv, xs_recv)
        else:
            self._a2a(x_recv, x_send, recv_counts, send_counts)
        ids_recv = torch.empty(R, dtype=torch.int32, device=ids.device)
        self._a2a(ids_recv, local_ids[:n], recv_counts, send_counts)
        w_recv = torch.empty(R, dtype=torch.float32, device=ids.device)
        self._a2a(w_recv, row_w[:n], recv_counts, send_counts)
        slot_row = ops.slot_rows(perm)
        self._mark("dispatch")
        return x_recv, ids_recv, w_recv, Dispatched(T, self.topk, send_counts, recv_counts, slot_row)

    def _dispatch_capacity(self, x, gate_logits):
        """dispatch() with fixed-capacity exchanges: equal splits of
        capacity rows per rank, no host read."""
        ops = self.ops
        T, H = x.shape
        n = T * self.topk
        C = self.capacity_rows(n)
        self._mark("start")
        ids, wts = ops.route(gate_logits, self.topk)
        dest = ops.dest_of(ids, self.experts_per_rank)
        xs = None
        if self.fp8:
            x, xs = (ops.quant_rows(x, pow2=True) if self.qw.get("pow2") else ops.quant_rows(x))
        perm = ops.permute_by_dest(dest, self.world, None)  # the slot order only
        cap = ops.capacity_layout(perm, ids, wts, self.experts_per_rank, self.world, C)
        x_send = ops.gather_capacity(cap, x)
        xs_send = ops.gather_capacity(cap, xs) if self.fp8 else None
        self._mark("route_permute")
        self._mark("count_exchange")  # nothing to exchange: the splits are fixed
        x_recv = torch.empty_like(x_send)
        if self.fp8:  # byte view: the exchange does not need to know the float8 type
            self._a2a(x_recv.view(torch.uint8), x_send.view(torch.uint8), None, None)
            xs_recv = torch.empty_like(xs_send)
            self._a2a(xs_recv, xs_send, None, None)
            x_recv = (x_recv, xs_recv)
        else:
            self._a2a(x_recv, x_send, None, None)
        ids_recv = torch.empty_like(cap["local_ids"])
        self._a2a(ids_recv, cap["local_ids"], None, None)
        w_recv = torch.empty_like(cap["weights"])
        self._a2a(w_recv, cap["weights"], None, None)
        self._mark("dispatch")
        return x_recv, ids_recv, w_recv, Dispatched(T, self.topk, None, None, cap["slot_row"], capacity=C)

    # ---------------------------------------------------------------- expert groups
    def _dispatch_groups(self, x, gate_logits, groups: int):
        """Routing and the fixed-capacity send layout of a grouped layer. The
        local experts of every rank are split into `groups` contiguous groups;
        the slots are laid out by (group, destination rank), group-major, so
        group g's rows for all ranks are one block of world * Cg rows that one
        equal-split all-to-all moves. Done by renaming expert l of rank r to
        g * (world * eg) + r * eg + l % eg (g = l // eg, eg experts per
        group) and laying out by "rank" = id // eg over world * groups
        destinations: the local ids that arrive are l % eg, the expert's index
        inside its group. Returns the send tensors (rows, scales or None,
        local ids, weights), the slots' layout rows and Cg."""
        ops = self.ops
        T = x.shape[0]
        n = T * self.topk
        W, epr = self.world, self.experts_per_rank
        eg = epr // groups
        Cg = self.capacity_rows(n, groups)
        ids, wts = ops.route(gate_logits, self.topk)
        r = torch.div(ids, epr, rounding_mode="floor")
        loc = ids - r * epr
        g = torch.div(loc, eg, rounding_mode="floor")
        vids = (g * (W * eg) + r * eg + (loc - g * eg)).to(ids.dtype).contiguous()
        xs = None
        if self.fp8:
            x, xs = (ops.quant_rows(x, pow2=True) if self.qw.get("pow2") else ops.quant_rows(x))
        perm = ops.permute_by_dest(ops.dest_of(vids, eg), W * groups, None)
        cap = ops.capacity_layout(perm, vids, wts, eg, W * groups, Cg)
        x_send = ops.gather_capacity(cap, x)
        xs_send = ops.gather_capacity(cap, xs) if self.fp8 else None
        return (x_send, xs_send, cap["local_ids"], cap["weights"]), cap["slot_row"], Cg

    def _xchg(self, inp, key):
        """Equal-split all-to-all of `inp`: through the copy-engine exchange
        when one is configured, else into a new tensor over NCCL."""
        if self.p2p is not None and self.world > 1 and inp.is_cuda:
            return self.p2p.all_to_all(inp, key)
        out = torch.empty_like(inp)
        self._a2a(out, inp, None, None)
        return out

    def _exchange_group(self, send, g: int, rows_g: int, groups: int):
        """All-to-all of group g's block of the send layout (equal splits).
        The exchange keys name the group count and the block's rows, so
        layers of other shapes on the same exchanger get buffers of their own."""
        sl = slice(g * rows_g, (g + 1) * rows_g)
        x_send, xs_send, ids_send, w_send = send
        xb = x_send[sl]
        tag = (groups, rows_g, g)
        if self.fp8:  # byte view: the exchange does not need to know the float8 type
            x_recv = (self._xchg(xb.view(torch.uint8), ("x",) + tag).view(xb.dtype),
                      self._xchg(xs_send[sl], ("xs",) + tag))
        else:
            x_recv = self._xchg(xb, ("x",) + tag)
        return x_recv, self._xchg(ids_send[sl], ("ids",) + tag), self._xchg(w_send[sl], ("w",) + tag)

    def _group_weights(self, a: int, b: int):
        """The weights of local experts [a, b): views, e4m3 codes with their
        128 x 128 block scales (rows of the scale grids), or bf16 tensors."""
        if not self.fp8:
            return self.w1[a:b], self.w2[a:b], self.w3[a:b]
        q = dict(self.qw)
        for name, rows in (("w1", q["I"]), ("w3", q["I"]), ("w2", q["H"])):
            q[name + "q"] = self.qw[name + "q"][a:b]
            q[name + "s"] = self.qw[name + "s"][a * (rows // 128):b * (rows // 128)]
        q["E"] = b - a
        return q

    def _group_experts(self, recv, a: int, b: int):
        x_recv, ids_recv, w_recv = recv
        if self.fp8:
            return self.ops.experts_fp8(x_recv[0], x_recv[1], ids_recv, w_recv, self._group_weights(a, b),
                                        dummy=True)
        return self.ops.experts(x_recv, ids_recv, w_recv, *self._group_weights(a, b), dummy=True)

    def _forward_groups(self, x, gate_logits, groups: int, compute=None, comm=None):
        """The layer with the local experts in `groups` groups. With CUDA
        streams the routing and every exchange run on `comm`, the expert
        GEMMs on `compute`: group g+1's rows travel while group g computes,
        and group g's results travel back while group g+1 computes. Each
        expert still sees all its rows in one GEMM, so no weight is streamed
        twice (token chunks would stream every expert's weights once per
        chunk). Without streams the same steps run in order."""
        import contextlib

        piped = x.is_cuda and compute is not None and comm is not None
        on = (lambda st: torch.cuda.stream(st)) if piped else (lambda st: contextlib.nullcontext())
        T = x.shape[0]
        eg = self.experts_per_rank // groups
        # routing and the send layout on the caller's stream (nothing else runs
        # yet, so they get every SM the caller's stream has)
        send, slot_row, Cg = self._dispatch_groups(x, gate_logits, groups)
        rows_g = self.world * Cg
        # Cross-stream uses are recorded on the allocator (record_stream) in
        # eager mode. Under CUDA-graph capture they are not needed: every
        # tensor outlives its last use inside the captured layer, which ends
        # joined back on the caller's stream.
        track = piped and not torch.cuda.is_current_stream_capturing()
        if piped:
            cur = torch.cuda.current_stream(x.device)
            comm.wait_stream(cur)
            compute.wait_stream(cur)
            for t in send:
                if t is not None and track:
                    t.record_stream(comm)  # made on the caller's stream, sent from the comm stream
        with on(comm):
            recvs = []
            for g in range(groups):
                recv = self._exchange_group(send, g, rows_g, groups)
                ev = None
                if piped:
                    ev = torch.cuda.Event()
                    ev.record(comm)
                recvs.append((recv, ev))
        ys = []
        for g, (recv, ev) in enumerate(recvs):
            with on(compute):
                if piped:
                    compute.wait_event(ev)
                    xr, ids_r, w_r = recv
                    for t in (xr if isinstance(xr, tuple) else (xr,)) + (ids_r, w_r):
                        if track:
                            t.record_stream(compute)  # made on the comm stream, read here
                y = self._group_experts(recv, g * eg, (g + 1) * eg)
                ev_y = None
                if piped:
                    ev_y = torch.cuda.Event()
                    ev_y.record(compute)
                ys.append((y, ev_y))
        use_p2p = self.p2p is not None and self.world > 1 and x.is_cuda
        with on(comm):
            y0 = ys[0][0]
            shape = (groups * rows_g, y0.shape[1])
            y_back = None if use_p2p else torch.empty(shape, dtype=y0.dtype, device=y0.device)
            for g, (y, ev_y) in enumerate(ys):
                if piped:
                    comm.wait_event(ev_y)
                    if track:
                        y.record_stream(comm)  # made on the compute stream, sent from here
                if use_p2p:  # every group's results land in one buffer, group after group
                    self.p2p.all_to_all(y, ("y", groups, rows_g), part=g, parts=groups)
                else:
                    self._a2a(y_back[g * rows_g:(g + 1) * rows_g], y, None, None)
            if use_p2p:
                y_back = self.p2p.buffer_view(("y", groups, rows_g), y0.dtype, shape)
        if piped:
            cur.wait_stream(comm)
            if track:
                y_back.record_stream(cur)  # made on the comm stream, read here
        # each token's k rows summed on the caller's stream, every SM again
        return self.ops.combine_rows(y_back, slot_row, T, self.topk)

    def combine(self, y_local, d: Dispatched):
        n = d.T * d.topk
        self._mark("experts")
        rows = self.world * d.capacity if d.capacity else n
        y_back = torch.empty((rows, y_local.shape[1]), dtype=y_local.dtype, device=y_local.device)
        self._a2a(y_back, y_local, d.send_counts, d.recv_counts)
        self._mark("combine_exchange")
        out = self.ops.combine_rows(y_back, d.slot_row, d.T, d.topk)
        self._mark("final_combine")
        return out

    def profile_phases(self, x, gate_logits) -> dict:
        """One unchunked forward on the current stream with CUDA events at the
        phase boundaries. Returns the output, each phase's device time (ms) and
        the bytes this rank sent to other ranks in the two row exchanges. The
        phases: route_permute (routing, FP8 quantisation of the rows, sort by
        destination, metadata), count_exchange (the per-rank counts and their
        host read), dispatch (rows, scales, expert ids and weights), experts
        (the local grouped GEMMs), combine_exchange (weighted rows back),
        final_combine (each token's k rows summed)."""
        self._marks = []
        try:
            x_recv, ids_recv, w_recv, d = self.dispatch(x, gate_logits)
            out = self.combine(self._experts(x_recv, ids_recv, w_recv), d)
            torch.cuda.synchronize()
            marks = self._marks
        finally:
            self._marks = None
        ms = {name: marks[i - 1][1].elapsed_time(ev) for i, (name, ev) in enumerate(marks) if i > 0}
        H = x.shape[1]
        if d.capacity:  # every rank sends and receives `capacity` rows per peer, padding included
            remote_send = remote_back = (self.world - 1) * d.capacity
            sent = received = self.world * d.capacity
        else:
            remote_send = sum(c for r, c in enumerate(d.send_counts) if r != self.rank)
            remote_back = sum(c for r, c in enumerate(d.recv_counts) if r != self.rank)
            sent, received = int(sum(d.send_counts)), int(sum(d.recv_counts))
        row_bytes = (H + (H // 128) * 4 if self.fp8 else 2 * H) + 8  # row (+ scales) + expert id + weight
        return {"out": out, "ms": ms, "dispatch_bytes": remote_send * row_bytes, "combine_bytes": remote_back * 2 * H,
                "rows_sent": sent, "rows_received": received, "capacity": d.capacity}

    def _experts(self, x_recv, ids_recv, w_recv):
        kw = {"dummy": True} if self.capacity is not None else {}
        if self.fp8:
            return self.ops.experts_fp8(x_recv[0], x_recv[1], ids_recv, w_recv, self.qw, **kw)
        return self.ops.experts(x_recv, ids_recv, w_recv, self.w1, self.w2, self.w3, **kw)

    def forward(self, x, gate_logits, chunks: int = 1, compute_stream=None, comm_stream=None, groups: int = 1):
        """The layer for this rank's tokens x [T, H] (router logits [T, E]).

        groups > 1 (fixed-capacity exchanges only; a divisor of the experts
        per rank) splits each rank's experts into that many groups and
        pipelines the exchanges of one group with the expert GEMMs of another
        (_forward_groups); every rank must use the same value.

        chunks > 1 splits the tokens into that many contiguous chunks and
        pipelines them: with CUDA streams given (the expert GEMMs on
        `compute_stream`, e.g. the large green-context partition; routing,
        dispatch and combine on `comm_stream`, e.g. the small one), the
        dispatch of chunk i+1 and the combine of chunk i-1 run while chunk i's
        experts compute. Every rank must use the same number of chunks (the
        collectives of a chunk pair up across ranks). Results equal the
        unchunked layer: every token's rows are computed and summed the same
        way whichever chunk carries them."""
        T = x.shape[0]
        groups = int(groups)
        if groups > 1:
            if self.capacity is None:
                raise ValueError("expert groups need fixed-capacity exchanges (capacity='auto' or a row count)")
            if self.experts_per_rank % groups != 0:
                raise ValueError(f"{groups} groups do not split {self.experts_per_rank} experts per rank")
            return self._forward_groups(x, gate_logits, groups, compute_stream, comm_stream)
        chunks = max(1, min(int(chunks), T))
        if chunks == 1:
            x_recv, ids_recv, w_recv, d = self.dispatch(x, gate_logits)
            return self.combine(self._experts(x_recv, ids_recv, w_recv), d)
        bounds = [(c * T // chunks, (c + 1) * T // chunks) for c in range(chunks)]
        if not x.is_cuda or compute_stream is None or comm_stream is None:
            # one stream: the chunks run one after another (same collectives, same results)
            return torch.cat([self.forward(x[a:b], gate_logits[a:b]) for a, b in bounds], dim=0)
        return self._forward_pipelined(x, gate_logits, bounds, compute_stream, comm_stream)

    def _forward_pipelined(self, x, gate_logits, bounds, compute, comm):
        cur = torch.cuda.current_stream(x.device)
        out = torch.empty_like(x)
        comm.wait_stream(cur)
        compute.wait_stream(cur)

        def dispatch(c):
            a, b = bounds[c]
            with torch.cuda.stream(comm):
                r = self.dispatch(x[a:b], gate_logits[a:b])
                ev = torch.cuda.Event()
                ev.record(comm)
            return r, ev

        pending = dispatch(0)
        for c, (a, b) in enumerate(bounds):
            (x_recv, ids_recv, w_recv, d), ev_d = pending
            with torch.cuda.stream(compute):
                compute.wait_event(ev_d)
                for t in (x_recv if isinstance(x_recv, tuple) else (x_recv,)) + (ids_recv, w_recv):
                    t.record_stream(compute)  # made on the comm stream, read here
                y_local = self._experts(x_recv, ids_recv, w_recv)
                ev_e = torch.cuda.Event()
                ev_e.record(compute)
            if c + 1 < len(bounds):
                # The next chunk's routing and dispatch (and its host read of
                # the split sizes) go ahead of this chunk's combine on the comm
                # stream, so they overlap the experts just queued.
                pending = dispatch(c + 1)
            with torch.cuda.stream(comm):
                comm.wait_event(ev_e)
                y_local.record_stream(comm)  # made on the compute stream, sent from here
                out[a:b].copy_(self.combine(y_local, d))
        out.record_stream(comm)
        cur.wait_stream(comm)
        return out

    __call__ = forward
