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
    def __init__(self, area_bytes: int = 256 << 20, timeout_s: float = 5.0, group=None):
        assert dist.is_initialized(), "init the process group first"
        self.mod = _ext.comm()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = torch.cuda.current_device()
        self.timeout_s = float(timeout_s)
        self.area_bytes = (int(area_bytes) + 255) // 256 * 256
        self.id, handle = self.mod.create(self.device, self.rank, self.world, self.area_bytes)
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.mod.open_peers(self.id, handles)
        dist.barrier(group=group)

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
            self.mod.destroy(self.id)
            self.id = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass
