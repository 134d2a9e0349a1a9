"""Pipeline parallelism: GPipe and 1F1B schedules over point-to-point
send/recv (NCCL on GPUs, gloo on the host).

A model is cut into consecutive stages, one per rank of the pipeline group.
Each step splits the batch into micro-batches; stage s receives the
activations of micro-batch i from stage s-1, runs its forward, sends the
result on, and later receives the gradient of its output from stage s+1,
runs its backward and sends the gradient of its input back. Receives are
posted early (irecv) so transfers overlap the neighbouring compute.

  GPipe: all forwards, then all backwards (activation stash = all micro-batches).
  1F1B : warm-up of (stages - stage - 1) forwards, then alternate one forward
         / one backward, then drain the remaining backwards (stash bounded by
         the number of stages).

Reference parity: scirs2-neural/src/training/pipeline_parallel.rs:48-380
(PipelineSchedule GPipe / 1F1B, MicroBatch, activation stash, run_schedule)
and scirs2-autograd/src/distributed_grad.rs:603-735 (generate_1f1b_schedule);
there single-process simulations.
"""
from __future__ import annotations

import enum
from dataclasses import dataclass

import torch
import torch.distributed as dist


class PipelineSchedule(enum.Enum):
    GPIPE = "gpipe"
    ONE_F_ONE_B = "1f1b"


def generate_gpipe_schedule(num_stages: int, num_micro: int, stage: int):
    return [("F", i) for i in range(num_micro)] + [("B", i) for i in range(num_micro)]


def generate_1f1b_schedule(num_stages: int, num_micro: int, stage: int):
    warm = min(num_micro, num_stages - stage - 1)
    acts = [("F", i) for i in range(warm)]
    f, b = warm, 0
    while f < num_micro:
        acts.append(("F", f))
        f += 1
        acts.append(("B", b))
        b += 1
    while b < num_micro:
        acts.append(("B", b))
        b += 1
    return acts


@dataclass
class MicroBatch:
    index: int
    inputs: torch.Tensor
    targets: torch.Tensor | None = None


class PipelineStage:
    """One stage: a module run on this rank; `loss_fn(out, targets)` on the
    last stage. Activation shapes must be known (static) for the receives."""

    def __init__(self, module, stage: int, num_stages: int, act_shape, act_dtype=torch.float32, group=None,
                 ranks=None):
        self.module = module
        self.stage = stage
        self.num_stages = num_stages
        self.act_shape = tuple(act_shape)
        self.act_dtype = act_dtype
        self.group = group
        self.ranks = ranks or list(range(num_stages))
        self.is_first = stage == 0
        self.is_last = stage == num_stages - 1

    @property
    def device(self):
        try:
            return next(self.module.parameters()).device
        except StopIteration:
            return torch.device("cpu")

    def _recv(self, src_stage: int, shape):
        buf = torch.empty(shape, dtype=self.act_dtype, device=self.device)
        return buf, dist.irecv(buf, src=self.ranks[src_stage], group=self.group)

    def _send(self, t: torch.Tensor, dst_stage: int):
        return dist.isend(t.contiguous(), dst=self.ranks[dst_stage], group=self.group)


class PipelineParallel:
    def __init__(self, stage: PipelineStage, schedule: PipelineSchedule = PipelineSchedule.ONE_F_ONE_B):
        self.stage = stage
        self.schedule = schedule
        self.max_stash = 0

    def run_schedule(self, micro_batches: list[MicroBatch], loss_fn=None):
        """Forward + backward of all micro-batches (gradients accumulate in
        the stage module's parameters). Returns the summed loss on the last
        stage, None elsewhere."""
        st = self.stage
        n = len(micro_batches)
        gen = generate_gpipe_schedule if self.schedule == PipelineSchedule.GPIPE else generate_1f1b_schedule
        actions = gen(st.num_stages, n, st.stage)
        stash: dict[int, tuple] = {}
        pending_sends = []
        total = None
        act_shape = st.act_shape
        for kind, i in actions:
            mb = micro_batches[i]
            if kind == "F":
                if st.is_first:
                    x = mb.inputs.to(st.device)
                else:
                    x, req = st._recv(st.stage - 1, act_shape)
                    req.wait()
                    x.requires_grad_(True)
                out = st.module(x)
                if st.is_last:
                    loss = loss_fn(out, mb.targets.to(out.device)) / n
                    total = loss.detach() if total is None else total + loss.detach()
                    stash[i] = (x, loss)
                else:
                    pending_sends.append(st._send(out.detach(), st.stage + 1))
                    stash[i] = (x, out)
                self.max_stash = max(self.max_stash, len(stash))
            else:
                x, out = stash.pop(i)
                if st.is_last:
                    out.backward()
                else:
                    g, req = st._recv(st.stage + 1, out.shape)
                    req.wait()
                    out.backward(g)
                if not st.is_first:
                    pending_sends.append(st._send(x.grad, st.stage - 1))
        for r in pending_sends:
            r.wait()
        return total


def split_micro_batches(inputs: torch.Tensor, targets: torch.Tensor, num_micro: int) -> list[MicroBatch]:
    xs, ys = inputs.chunk(num_micro), targets.chunk(num_micro)
    return [MicroBatch(i, x, y) for i, (x, y) in enumerate(zip(xs, ys))]
