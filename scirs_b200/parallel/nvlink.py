"""Symmetric peer buffers and the in-kernel NVLink collectives.

`NVLinkComm` allocates one device buffer per rank (4 x `area_bytes`: two
alternating sets of two data areas, plus flags), exchanges CUDA IPC handles
over the process group and maps every peer's buffer, after which the kernels
in scirs_b200/csrc/comm.cu move data with P2P stores over NVLink 5 / NVSwitch
(no NCCL on the data path). Every wait inside
those kernels is bounded; a timed-out wait is reported through the status
word (see :func:`scirs_b200._ext.check_status`).

All ranks must issue the same collectives with the same sizes in the same
order, and all collectives of one NVLinkComm must run on one CUDA stream.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import _ext


class NVLinkComm:
    def __init__(self, area_bytes: int = 256 << 20, timeout_s: float | None = None, group=None):
        assert dist.is_initialized(), "init the process group first"
        self.mod = _ext.comm()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.cuda.current_device()
        import os

        self.timeout_s = float(timeout_s if timeout_s is not None else os.environ.get("SCIRS_WAIT_TIMEOUT_S", 5.0))
        self.area_bytes = (int(area_bytes) + 255) // 256 * 256
        self.id, handle = self.mod.create(self.device, self.rank, self.world, self.area_bytes)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.mod.open_peers(self.id, handles)
        dist.barrier(group=group)
        self._nvls = []

    @property
    def max_elems(self) -> int:
        """Largest payload (elements) of any collective on this buffer."""
        return self.area_bytes // 2 - 8 * self.world

    def allreduce_(self, t: torch.Tensor, scale: float = 1.0, blocks: int = 0, algo: int = 0) -> torch.Tensor:
        """In place: t <- scale * sum over ranks (fp32 tensor, bf16 on the wire).
        algo: 0 automatic, 1 one-shot, 2 two-shot."""
        self.mod.allreduce(self.id, t, t, float(scale), int(blocks), self.timeout_s, int(algo))
        return t

    def allreduce(self, src: torch.Tensor, dst: torch.Tensor, scale: float = 1.0, blocks: int = 0, algo: int = 0):
        self.mod.allreduce(self.id, src, dst, float(scale), int(blocks), self.timeout_s, int(algo))
        return dst

    # ------------------------------------------------------------- NVLS
    def nvls_supported(self) -> bool:
        """True when this GPU can bind memory to an NVLink multicast object
        (NVSwitch with multicast enabled)."""
        try:
            from torch._C._distributed_c10d import _SymmetricMemory

            return bool(_SymmetricMemory.has_multicast_support(torch._C._autograd.DeviceType.CUDA, self.device))
        except Exception:
            return False

    def nvls_buffer(self, numel: int, dtype=torch.float32) -> torch.Tensor:
        """A tensor in symmetric memory bound to an NVLink multicast object
        (same size and dtype on every rank; collective). In-place NVLS
        all-reduces run on it and on any 16-byte aligned slice of it."""
        import torch.distributed._symmetric_memory as symm

        t = symm.empty(int(numel), dtype=dtype, device=torch.device("cuda", self.device))
        h = symm.rendezvous(t, self.group if self.group is not None else dist.group.WORLD)
        mc = int(h.multicast_ptr)
        if mc == 0:
            raise RuntimeError("symmetric memory has no NVLink multicast mapping on this system")
        base = int(h.buffer_ptrs[self.rank])
        self._nvls.append((t.data_ptr(), t.numel() * t.element_size(), mc + (t.data_ptr() - base), h, t))
        return t

    def _mc_addr(self, t: torch.Tensor) -> int:
        p = t.data_ptr()
        for start, size, mc, _h, _t in self._nvls:
            if start <= p and p + t.numel() * t.element_size() <= start + size:
                return mc + (p - start)
        raise ValueError("tensor is not inside an NVLS buffer of this communicator")

    def allreduce_nvls_(self, t: torch.Tensor, scale: float = 1.0, blocks: int = 0) -> torch.Tensor:
        """In place: t <- scale * sum over ranks, reduced inside the NVSwitch
        (fp32, or bf16 with fp32 accumulation). `t` must lie in a buffer from
        :meth:`nvls_buffer`, at the same offset on every rank."""
        self.mod.allreduce_nvls(self.id, t, self._mc_addr(t), float(scale), int(blocks), self.timeout_s)
        return t

    def reduce_scatter_nvls(self, full: torch.Tensor, shard: torch.Tensor, scale: float = 1.0, blocks: int = 0):
        """shard (fp32, local) = scale * sum over ranks of this rank's part of
        `full` (fp32, inside an NVLS buffer), reduced inside the NVSwitch."""
        self.mod.reduce_scatter_nvls(self.id, full, self._mc_addr(full), shard, float(scale), int(blocks),
                                     self.timeout_s)
        return shard

    def all_gather_nvls(self, shard: torch.Tensor, full: torch.Tensor, blocks: int = 0):
        """full (bf16, inside an NVLS buffer) = concat over ranks of shard
        (bf16, local); each rank's shard is written to every GPU with one
        multicast store."""
        self.mod.allgather_nvls(self.id, shard, full, self._mc_addr(full), int(blocks), self.timeout_s)
        return full

    def reduce_scatter(self, src: torch.Tensor, dst: torch.Tensor, scale: float = 1.0, blocks: int = 0):
        """dst (this rank's shard, fp32) = scale * sum over ranks of src's shard."""
        self.mod.reduce_scatter(self.id, src, dst, float(scale), int(blocks), self.timeout_s)
        return dst

    def all_gather(self, shard: torch.Tensor, full: torch.Tensor, blocks: int = 0):
        """full (bf16) = concat over ranks of shard (bf16)."""
        self.mod.allgather(self.id, shard, full, int(blocks), self.timeout_s)
        return full

    def close(self):
        if self.id is not None:
            torch.cuda.synchronize()
            self._nvls = []
            self.mod.destroy(self.id)
            self.id = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass
