"""Equal-split all-to-all launched on a caller-chosen CUDA stream.

torch.distributed's NCCL backend launches its kernels on the process group's
own internal stream, which belongs to the device's primary context, so those
kernels may be placed on any SM -- including the SMs of a green-context
partition that is running a persistent expert GEMM. A GEMM CTA that finds its
SM taken waits for the collective to finish, and with it the whole GEMM: an
exchange overlapped with the experts then costs about as much as one that is
not. This module drives a separate NCCL communicator through NCCL's C API
(the library torch already loaded) and passes it the stream of the
communication partition, so the collective's kernels run on that partition's
SMs only and the expert partition keeps all of its SMs.

Only the calls the expert-parallel layer needs: communicator set-up (the
unique id travels over the existing torch.distributed group), a grouped
send/receive all-to-all with equal per-peer byte counts, and tear-down.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

_NCCL_UINT8 = 1


class _UniqueId(ctypes.Structure):
    _fields_ = [("internal", ctypes.c_byte * 128)]


_LIB = None


def _lib():
    global _LIB
    if _LIB is None:
        lib = None
        for name in ("libnccl.so.2", "libnccl.so"):
            try:
                lib = ctypes.CDLL(name)  # after `import torch`: the NCCL torch links against
                break
            except OSError:
                continue
        if lib is None:
            import os

            import nvidia.nccl as pkg  # torch's NCCL wheel

            lib = ctypes.CDLL(os.path.join(list(pkg.__path__)[0], "lib", "libnccl.so.2"))
        lib.ncclGetErrorString.restype = ctypes.c_char_p
        lib.ncclGetUniqueId.argtypes = [ctypes.POINTER(_UniqueId)]
        lib.ncclCommInitRank.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, _UniqueId, ctypes.c_int]
        for fn in (lib.ncclSend, lib.ncclRecv):
            fn.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                           ctypes.c_void_p]
        lib.ncclCommDestroy.argtypes = [ctypes.c_void_p]
        lib.ncclCommAbort.argtypes = [ctypes.c_void_p]
        _LIB = lib
    return _LIB


def _check(rc: int, what: str) -> None:
    if rc != 0:
        msg = _lib().ncclGetErrorString(rc)
        raise RuntimeError(f"{what}: NCCL error {rc}: {msg.decode() if msg else '?'}")


class StreamAllToAll:
    """An NCCL communicator over the ranks of `group` whose all-to-all runs on
    the stream given to each call. Construction is collective (every rank of
    the group, with its CUDA device current); so is close()."""

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        lib = _lib()
        uid = _UniqueId()
        if self.rank == 0:
            _check(lib.ncclGetUniqueId(ctypes.byref(uid)), "ncclGetUniqueId")
        payload = [bytes(bytearray(uid.internal)) if self.rank == 0 else None]
        src = dist.get_global_rank(group, 0) if group is not None else 0
        dist.broadcast_object_list(payload, src=src, group=group)
        ctypes.memmove(ctypes.addressof(uid), payload[0], 128)
        self._comm = ctypes.c_void_p()
        _check(lib.ncclCommInitRank(ctypes.byref(self._comm), self.world, uid, self.rank), "ncclCommInitRank")

    def all_to_all(self, out: torch.Tensor, inp: torch.Tensor, stream=None) -> torch.Tensor:
        """out[p-th block] = the rank-p block that peer p sent this rank: inp
        and out are contiguous CUDA tensors of one byte size, a multiple of
        the world size, split into equal per-peer blocks (as
        all_to_all_single without split sizes). Runs on `stream` (default:
        the current stream) and returns at once."""
        if self._comm is None:
            raise RuntimeError("StreamAllToAll is closed")
        if not (out.is_cuda and inp.is_contiguous() and out.is_contiguous()):
            raise RuntimeError("all_to_all takes contiguous CUDA tensors")
        nbytes = inp.numel() * inp.element_size()
        if out.numel() * out.element_size() != nbytes or nbytes % self.world:
            raise RuntimeError("all_to_all: out and inp must hold the same bytes, a multiple of the world size")
        per = nbytes // self.world
        st = stream if stream is not None else torch.cuda.current_stream(out.device)
        handle = ctypes.c_void_p(st.cuda_stream)
        lib = _lib()
        src, dst = inp.data_ptr(), out.data_ptr()
        _check(lib.ncclGroupStart(), "ncclGroupStart")
        try:
            for p in range(self.world):
                _check(lib.ncclSend(ctypes.c_void_p(src + p * per), per, _NCCL_UINT8, p, self._comm, handle),
                       "ncclSend")
                _check(lib.ncclRecv(ctypes.c_void_p(dst + p * per), per, _NCCL_UINT8, p, self._comm, handle),
                       "ncclRecv")
        finally:
            _check(lib.ncclGroupEnd(), "ncclGroupEnd")
        return out

    def close(self) -> None:
        """Destroy the communicator (collective; after the last call's work
        has completed)."""
        if self._comm is not None:
            torch.cuda.synchronize()
            _check(_lib().ncclCommDestroy(self._comm), "ncclCommDestroy")
            self._comm = None
