"""Symmetric device memory over the GPUs of one box.

Each rank ``cudaMalloc``'s one region of the same size, exports it as a CUDA
IPC handle, and maps every peer's region (``csrc/comm.cu``).  Buffers are
carved out with the same bump sequence on every rank, so a buffer has the same
offset everywhere and a kernel addresses rank ``r``'s copy as
``peers[r] + offset``: stores through that address cross NVLink / NVSwitch.

No counterpart in the reference (single device, no communication at all).
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch
import torch.distributed as dist

from ops._ext import native

ALIGN = 256


def _align(n: int, a: int = ALIGN) -> int:
    return (n + a - 1) // a * a


class SymmetricHeap:
    """``nbytes`` of zeroed device memory on every rank of ``group``, each
    rank's region mapped into every other rank.

    With no process group (or a group of one) the heap is a plain local region
    whose only "peer" is itself, which lets the peer-memory kernels run on a
    single GPU unchanged.
    """

    def __init__(self, nbytes: int, group=None, device: Optional[torch.device] = None):
        self.C = native()
        self.group = group
        self.distributed = dist.is_available() and dist.is_initialized()
        self.rank = dist.get_rank(group) if self.distributed else 0
        self.world = dist.get_world_size(group) if self.distributed else 1
        if device is not None and device.index is not None:
            torch.cuda.set_device(device)
        self.device_index = torch.cuda.current_device()
        self.nbytes = _align(max(nbytes, ALIGN))
        self.ptr, handle = self.C.symm_alloc(self.nbytes)
        handles: List[bytes] = [handle]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle, group=group)
        self.peers: List[int] = [self.ptr if r == self.rank else self.C.symm_open(h) for r, h in enumerate(handles)]
        self._bytes = self.C.symm_view(self.ptr, self.nbytes, self.device_index)
        self._top = 0
        self._closed = False
        if self.world > 1:
            dist.barrier(group=group)  # every region zeroed and mapped before anyone stores into it

    def alloc(self, nbytes: int) -> int:
        """Reserve ``nbytes`` (256-byte aligned); returns the symmetric offset."""
        off = self._top
        self._top = _align(off + nbytes)
        if self._top > self.nbytes:
            raise RuntimeError(f"symmetric heap exhausted: need {self._top} of {self.nbytes} bytes")
        return off

    def tensor(self, offset: int, shape: Sequence[int], dtype: torch.dtype) -> torch.Tensor:
        """This rank's copy of the buffer at ``offset`` as a tensor (aliases the heap)."""
        n = 1
        for s in shape:
            n *= int(s)
        nbytes = n * torch.empty((), dtype=dtype).element_size()
        return self._bytes[offset:offset + nbytes].view(dtype).view(*shape)

    def close(self) -> None:
        if self._closed:
            return
        self._closed = True
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)  # no peer still stores into a region about to go away
        for r, p in enumerate(self.peers):
            if r != self.rank:
                self.C.symm_close(p)
        if self.world > 1:
            dist.barrier(group=self.group)
        self._bytes = None
        self.C.symm_free(self.ptr)


def heap_layout(sizes: Sequence[int]) -> List[int]:
    """Offsets of consecutive 256-byte aligned buffers of the given sizes."""
    offs, top = [], 0
    for s in sizes:
        offs.append(top)
        top = _align(top + int(s))
    offs.append(top)
    return offs
