"""Symmetric device heap: one allocation per rank, same size and layout on
every rank, mapped into every peer with CUDA IPC.

A tensor allocated from the heap sits at the same offset on every rank, so a
kernel can address "the same tensor on rank r" as ``base[r] + offset``: the
tensor-parallel GEMMs load peer tiles with TMA (no multicast), the
reduce-scatter epilogues and the flag signals store into peers.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import _ext


class SymmetricHeap:
    def __init__(self, nbytes: int, group=None):
        assert dist.is_initialized(), "init the process group first"
        self.mod = _ext.comm()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.cuda.current_device()
        self.nbytes = (int(nbytes) + 255) // 256 * 256
        self.id, handle = self.mod.sym_create(self.device, self.rank, self.world, self.nbytes)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.mod.sym_open(self.id, handles)
        self.buf = self.mod.sym_tensor(self.id)
        self.base = self.buf.data_ptr()
        self.ptrs = list(self.mod.sym_ptrs(self.id))
        self.off = 0
        dist.barrier(group=group)

    def alloc(self, shape, dtype=torch.bfloat16, align: int = 1024) -> torch.Tensor:
        """Carve a tensor out of the heap. Every rank must make the same
        sequence of calls (same offsets everywhere)."""
        n = 1
        for s in shape:
            n *= int(s)
        esz = torch.empty((), dtype=dtype).element_size()
        self.off = (self.off + align - 1) // align * align
        end = self.off + n * esz
        if end > self.nbytes:
            raise RuntimeError(f"symmetric heap exhausted: need {end} bytes of {self.nbytes}")
        t = self.buf[self.off : end].view(dtype).view(*shape)
        self.off = end
        return t

    def peer_addrs(self, t: torch.Tensor) -> list[int]:
        """Address of tensor `t` (allocated from this heap) on every rank."""
        off = t.data_ptr() - self.base
        assert 0 <= off < self.nbytes, "tensor is not in the symmetric heap"
        return [p + off for p in self.ptrs]

    def close(self):
        if self.id is not None:
            torch.cuda.synchronize()
            self.buf = None
            self.mod.sym_destroy(self.id)
            self.id = None
