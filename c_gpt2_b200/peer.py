"""Peer memory between the GPUs of one node (one process per GPU).

Thin Python side of the library's peer-memory C ABI (include/gpt2_w8a8.h:
w8a8_peer_alloc / _open / _close / _free / _signal / _wait): a rank allocates
a zero-filled exchange buffer, the 64-byte CUDA IPC handles go round through
torch.distributed, and every rank maps the others' buffers, which its kernels
then read and write directly over NVLink. Tensors over these buffers are made
with the CUDA array interface (no copy).
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from ._lib import check, core

_TYPESTR = {torch.int8: "|i1", torch.int32: "<i4", torch.float32: "<f4", torch.uint8: "|u1"}


class _DeviceArray:
    def __init__(self, ptr: int, shape: tuple[int, ...], dtype: torch.dtype):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": _TYPESTR[dtype],
                                         "data": (int(ptr), False), "version": 3,
                                         "strides": None}


def view(ptr: int, shape: tuple[int, ...], dtype: torch.dtype) -> torch.Tensor:
    """A tensor over this GPU's own device memory at `ptr`. (Never for a mapped
    peer buffer: torch would place such a tensor on the peer's device; only the
    library's kernels and copies touch peer memory.)"""
    return torch.as_tensor(_DeviceArray(ptr, shape, dtype), device="cuda")


class PeerBuffer:
    """One exchange buffer per rank, mapped by every rank of `group`."""

    def __init__(self, nbytes: int, group=None):
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.nbytes = nbytes
        ptr = C.c_void_p()
        handle = (C.c_ubyte * 64)()
        check(core().w8a8_peer_alloc(nbytes, C.byref(ptr), handle), "w8a8_peer_alloc")
        self.local = ptr.value
        handles = [bytes(handle)]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
        self.base: list[int] = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.base.append(self.local)
                continue
            p = C.c_void_p()
            hb = (C.c_ubyte * 64).from_buffer_copy(h)
            check(core().w8a8_peer_open(hb, C.byref(p)), "w8a8_peer_open")
            self.base.append(p.value)

    def close(self) -> None:
        """Collective: every rank's device work is finished before any rank
        unmaps a peer's buffer, and every mapping is gone before any rank
        frees its own."""
        if not self.base:
            return
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)
        for r, p in enumerate(self.base):
            if r != self.rank:
                core().w8a8_peer_close(C.c_void_p(p))
        if self.world > 1:
            dist.barrier(group=self.group)
        core().w8a8_peer_free(C.c_void_p(self.local))
        self.base = []


def _ptrs(ps) -> C.Array:
    arr = (C.c_void_p * len(ps))()
    for i, p in enumerate(ps):
        arr[i] = p
    return arr


def signal(flag_ptrs: list[int], value: int) -> None:
    """After the work before it on the current stream, flags := value."""
    check(core().w8a8_peer_signal(_ptrs(flag_ptrs), len(flag_ptrs), value & 0xffffffff,
                                  torch.cuda.current_stream().cuda_stream), "w8a8_peer_signal")


def wait(flags_ptr: int, n: int, value: int) -> None:
    """The work after it on the current stream waits for n flags >= value."""
    check(core().w8a8_peer_wait(C.c_void_p(flags_ptr), n, value & 0xffffffff,
                                torch.cuda.current_stream().cuda_stream), "w8a8_peer_wait")


def copy(dst_ptr: int, src_ptr: int, nbytes: int) -> None:
    """Device-to-device copy on the current stream (into or out of a peer's buffer)."""
    check(core().w8a8_peer_copy(C.c_void_p(dst_ptr), C.c_void_p(src_ptr), nbytes,
                                torch.cuda.current_stream().cuda_stream), "w8a8_peer_copy")


def ptr_array(ps) -> C.Array:
    return _ptrs(ps)
