"""Data parallelism for the flat-buffer engine: bucketed gradient all-reduce
overlapped with the backward pass.

Each gradient bucket is a contiguous slice of the model's flat fp32
gradient buffer (for the GPT engine: one transformer block, plus the
embeddings at the end). When the backward pass has finished a bucket, the
engine calls :meth:`GradSync.bucket_ready`; the all-reduce of that slice is
launched on a high-priority communication stream that waits only on an
event for that point of the backward stream, so it overlaps the remaining
backward kernels. :meth:`GradSync.finish` joins the streams before the
optimizer step.

Modes:
  "nvls" : the gradient buffer itself lives in symmetric memory bound to an
           NVLink multicast object; each bucket is all-reduced IN PLACE by
           the NVLS kernel (fp32 multimem.ld_reduce inside the NVSwitch +
           multimem.st of the 1/world-scaled sum): no staging copy, no cast,
           about one payload per GPU per direction over NVLink.
  "push" : the in-kernel NVLink push all-reduce (scale by 1/world and the
           fp32->bf16 cast fused into the publish phase, bf16 on the wire,
           fp32 accumulation, identical result on every rank).
  "fused": "nvls" where the GPUs support NVLink multicast, else "push".
  "nccl" : torch.distributed.all_reduce (fp32, AVG) on the same stream
           schedule; the baseline.

Reference parity: scirs2-autograd/src/distributed/mod.rs:13-84
(DistributedGradient::allreduce, a local divide) and the bucketing of
scirs2-autograd/src/distributed_grad.rs:229-330 (GradientBucketer,
simulated), here as real collectives.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class GradSync:
    def __init__(self, grad: torch.Tensor, bounds: list[tuple[int, int]], mode: str = "fused", comm=None):
        self.grad = grad
        self.bounds = bounds
        self.mode = mode
        self.world = dist.get_world_size()
        self.comm = comm
        if mode == "push":
            assert comm is not None
            biggest = max(e - s for s, e in bounds)
            assert biggest <= comm.max_elems, f"bucket of {biggest} elements exceeds the symmetric buffer"
        self.stream = torch.cuda.Stream(priority=-1)
        self.events = [torch.cuda.Event() for _ in bounds]
        self.launches = 0

    def bucket_ready(self, i: int):
        s, e = self.bounds[i]
        ev = self.events[i]
        ev.record(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(ev)
            sl = self.grad[s:e]
            if self.mode == "nvls":
                self.comm.allreduce_nvls_(sl, 1.0 / self.world)
            elif self.mode == "push":
                self.comm.allreduce_(sl, 1.0 / self.world)
            else:
                dist.all_reduce(sl, op=dist.ReduceOp.AVG)
            self.launches += 1

    def finish(self):
        torch.cuda.current_stream().wait_stream(self.stream)


def data_parallel(model, mode: str = "fused", comm=None, area_bytes: int | None = None):
    """Attach a GradSync to a flat-buffer model (e.g. GPTModel).

    Also broadcasts rank 0's parameters so all replicas start equal.
    """
    import os

    from .nvlink import NVLinkComm

    if not dist.is_initialized() or dist.get_world_size() == 1:
        return model
    if mode == "fused" and os.environ.get("SCIRS_COMM") == "nccl":
        mode = "nccl"
    fp = model.fp
    dist.broadcast(fp.master, src=0)
    fp.sync_bf16()
    if mode in ("fused", "push", "nvls") and comm is None:
        biggest = max(e - s for s, e in model.bucket_bounds)
        comm = NVLinkComm(area_bytes=area_bytes or (biggest * 2 + (1 << 20)))
    if mode == "fused":
        mode = "nvls" if comm.nvls_supported() else "push"
    if mode == "nvls":
        # move the flat gradient buffer into multicast-bound symmetric memory
        # (kernels take their gradient views from fp.grad at every call)
        g = comm.nvls_buffer(fp.total, torch.float32)
        g.copy_(fp.grad)
        fp.grad = g
    model.grad_sync = GradSync(fp.grad, model.bucket_bounds, mode=mode, comm=comm)
    return model
