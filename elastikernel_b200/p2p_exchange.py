"""Equal-split all-to-all over NVLink with the copy engines, without NCCL.

Every rank keeps, per exchange key (one per all-to-all call site of a layer:
each expert group's rows, scales, ids and weights, and the groups' results),
a receive arena of two buffers plus a flag per (buffer, part, peer). The arenas are
mapped into every other rank with CUDA IPC once, on a key's first use (a
collective: every rank must make the same calls in the same order). A call:

1. copies this rank's block for peer p into buffer e % 2 of p's arena, at
   this rank's slot, with cudaMemcpyAsync on the IPC mapping (copy engines
   over NVLink; no SM is used, so the expert GEMMs keep every SM of their
   partition while the rows travel);
2. stores the call's epoch e into the flag (e % 2, this rank) of every rank's
   arena, in a one-thread kernel ordered after those copies (system scope);
3. waits, in a one-thread kernel, until this rank's flags (e % 2, every peer)
   hold e (bounded: EK_STATUS_WAIT_TIMEOUT after 2 s);
4. returns buffer e % 2 of this rank's arena as a tensor shaped like the
   input: block p holds what peer p sent.

All of it is queued on the current stream; nothing waits on the host. A
buffer is rewritten two calls of its key later. In the expert-parallel layer
a rank reaches a key's next call only after every peer has sent it its
combine results of the previous layer, which those peers send after their
experts have read what this key delivered, so the rewrite never meets a
reader.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib

_ALIGN = 256


class P2PAllToAll:
    """Copy-engine all-to-all among the ranks of `group` (one GPU each, with
    peer access over NVLink). Construction is cheap; every method that maps
    memory is collective.

    device_epochs=True: the epochs live in device counters (one per key and
    part) that the signal kernel increments, and every key has one buffer,
    so a layer built on these exchanges can be captured in a CUDA graph and
    replayed (a host-side epoch would be frozen into the graph). One buffer
    is enough for the expert-parallel layer: a rank copies into a peer's
    buffer for the next layer only after that peer has signalled the next
    layer's dispatch, which it does after it has finished the previous one.
    Every rank must use the same mode."""

    def __init__(self, group=None, device_epochs: bool = False):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device_epochs = bool(device_epochs)
        self._nbuf = 1 if self.device_epochs else 2
        self._keys = {}
        self._opened = {}  # (peer, handle bytes) -> mapped base address
        self._closed = False

    def _map_key(self, key, nbytes: int, parts: int, device):
        """Allocate this rank's arena for `key` (two buffers of `parts` parts of
        nbytes) and map every peer's."""
        lib = _lib.lib()
        nb = self._nbuf
        # header: flags [buffer][part][peer], then (device epochs) a counter per part
        flag_bytes = nb * parts * self.world * 4 + (parts * 4 if self.device_epochs else 0)
        data_off = -(-flag_bytes // _ALIGN) * _ALIGN
        buf_bytes = -(-nbytes // _ALIGN) * _ALIGN
        arena = torch.zeros(data_off + nb * parts * buf_bytes, dtype=torch.uint8, device=device)
        base = ctypes.c_ulonglong()
        size = ctypes.c_size_t()
        _lib.check(lib.ek_p2p_mem_base(ctypes.c_void_p(arena.data_ptr()), ctypes.byref(base), ctypes.byref(size)),
                   "ek_p2p_mem_base")
        handle = (ctypes.c_byte * 64)()
        _lib.check(lib.ek_p2p_ipc_handle(ctypes.c_void_p(base.value), handle), "ek_p2p_ipc_handle")
        mine = (bytes(bytearray(handle)), arena.data_ptr() - base.value, nbytes)
        torch.cuda.synchronize(device)  # the zeroed flags are in place before any peer can signal them
        got = [None] * self.world
        dist.all_gather_object(got, mine, group=self.group)
        peers = []
        for p, (h, off, nb) in enumerate(got):
            if nb != nbytes:
                raise RuntimeError(f"p2p all-to-all key {key!r}: rank {p} exchanges {nb} bytes, this rank {nbytes}")
            if p == self.rank:
                peers.append(arena.data_ptr())
                continue
            if (p, h) not in self._opened:
                ptr = ctypes.c_void_p()
                hb = (ctypes.c_byte * 64).from_buffer_copy(h)
                _lib.check(lib.ek_p2p_ipc_open(hb, ctypes.byref(ptr)), "ek_p2p_ipc_open")
                self._opened[(p, h)] = ptr.value
            peers.append(self._opened[(p, h)] + off)
        dist.barrier(group=self.group)  # every mapping exists before the first copy into it
        slot = {"arena": arena, "peers": peers, "data_off": data_off, "buf_bytes": buf_bytes, "nbytes": nbytes,
                "parts": parts, "epoch": 0}
        self._keys[key] = slot
        return slot

    def all_to_all(self, inp: torch.Tensor, key, part: int = 0, parts: int = 1) -> torch.Tensor:
        """Block p of the result (a view of this rank's arena, shaped and
        typed like `inp`) is block `rank` of peer p's `inp`. inp: a contiguous
        CUDA tensor whose bytes split into world equal blocks. Queued on the
        current stream. With parts > 1 the key's buffer holds `parts`
        consecutive results (calls part = 0 .. parts-1, in that order, every
        time): buffer_view() then returns them as one tensor."""
        if self._closed:
            raise RuntimeError("P2PAllToAll is closed")
        if not (inp.is_cuda and inp.is_contiguous()):
            raise RuntimeError("p2p all_to_all takes a contiguous CUDA tensor")
        nbytes = inp.numel() * inp.element_size()
        if nbytes % self.world:
            raise RuntimeError("p2p all_to_all: the bytes must split into equal blocks per rank")
        slot = self._keys.get(key)
        if slot is None:
            slot = self._map_key(key, nbytes, parts, inp.device)
        elif slot["nbytes"] != nbytes or slot["parts"] != parts:
            raise RuntimeError(f"p2p all_to_all key {key!r} was mapped for {slot['parts']} x {slot['nbytes']} "
                               f"bytes, got {parts} x {nbytes}")
        if not 0 <= part < parts:
            raise RuntimeError("p2p all_to_all: part out of range")
        if not self.device_epochs and torch.cuda.is_current_stream_capturing():
            raise RuntimeError("capturing p2p exchanges in a CUDA graph needs P2PAllToAll(device_epochs=True)")
        lib = _lib.lib()
        stream = ctypes.c_void_p(torch.cuda.current_stream(inp.device).cuda_stream)
        if part == 0:
            slot["epoch"] += 1
        e = slot["epoch"]
        b = e % self._nbuf
        blk = nbytes // self.world
        dbuf = slot["data_off"] + (b * parts + part) * slot["buf_bytes"]
        fbase = (b * parts + part) * self.world
        src = inp.data_ptr()
        for i in range(self.world):
            p = (self.rank + i) % self.world  # start with the local block, then the peers in ring order
            _lib.check(lib.ek_p2p_copy(ctypes.c_void_p(slot["peers"][p] + dbuf + self.rank * blk),
                                       ctypes.c_void_p(src + p * blk), blk, stream), "ek_p2p_copy")
        flags = (ctypes.c_void_p * self.world)(*[slot["peers"][p] + (fbase + self.rank) * 4
                                                 for p in range(self.world)])
        arena = slot["arena"]
        my_flags = ctypes.c_void_p(arena.data_ptr() + fbase * 4)
        if self.device_epochs:
            counter = ctypes.c_void_p(arena.data_ptr() + (parts * self.world + part) * 4)
            _lib.check(lib.ek_p2p_signal_dev(flags, self.world, counter, stream), "ek_p2p_signal_dev")
            _lib.check(lib.ek_p2p_wait_dev(my_flags, self.world, counter, stream), "ek_p2p_wait_dev")
        else:
            _lib.check(lib.ek_p2p_signal(flags, self.world, e, stream), "ek_p2p_signal")
            _lib.check(lib.ek_p2p_wait(my_flags, self.world, e, stream), "ek_p2p_wait")
        return arena[dbuf:dbuf + nbytes].view(inp.dtype).view(inp.shape)

    def buffer_view(self, key, dtype, shape) -> torch.Tensor:
        """The current buffer of a parts > 1 key (its parts back to back, each
        padded to 256 bytes; the view requires nbytes to be a multiple of 256
        when parts > 1) as one tensor."""
        slot = self._keys[key]
        if slot["parts"] > 1 and slot["nbytes"] % _ALIGN:
            raise RuntimeError("buffer_view: parts are not contiguous (nbytes not a multiple of 256)")
        b = slot["epoch"] % self._nbuf
        dbuf = slot["data_off"] + b * slot["parts"] * slot["buf_bytes"]
        n = slot["parts"] * slot["nbytes"]
        return slot["arena"][dbuf:dbuf + n].view(dtype).view(shape)

    def close(self) -> None:
        """Unmap the peers' arenas (collective: after every rank's last call
        has completed)."""
        if self._closed:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        lib = _lib.lib()
        for ptr in self._opened.values():
            _lib.check(lib.ek_p2p_ipc_close(ctypes.c_void_p(ptr)), "ek_p2p_ipc_close")
        self._opened.clear()
        dist.barrier(group=self.group)  # no rank frees its arena while a peer still maps it
        self._keys.clear()
        self._closed = True
