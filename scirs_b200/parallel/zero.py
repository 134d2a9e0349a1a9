"""ZeRO-style sharded data parallelism for the flat-buffer engines.

Every gradient bucket [s, e) of the model's flat buffer is split evenly into
`world` shards; rank r owns [s + r*len/world, s + (r+1)*len/world) of every
bucket. The shards of all buckets are stored back to back in this rank's
shard buffers, so the optimizer over them is still ONE fused launch:

  backward:  bucket i done -> reduce-scatter of its fp32 gradient (scaled by
             1/world, bf16 on the wire, fp32 accumulation) into this rank's
             gradient shard, on the communication stream (overlaps backward)
  step:      sum of squares of the gradient shard -> summed over ranks
             (global-norm clipping sees the full gradient) -> fused AdamW on
             the fp32 master / moment SHARDS, writing the bf16 parameter shard
  forward:   all-gather of bucket i's bf16 parameter shards into the full
             bf16 parameter buffer, issued for all buckets at the start of
             the forward on the communication stream; block i waits only for
             its own bucket (prefetch overlapped with compute)

Tied vocabulary tables (the GPT engine's wte, used by the input embedding and
the LM head) get an early reduce-scatter: the engine hands over the wte
bucket right after the LM-head weight-gradient GEMM, so its reduce-scatter
overlaps the whole backward pass, and the input-embedding part of the
gradient (only the rows of this step's tokens) is sent to the rank that owns
each row (`VocabGradRoute`: one peer-store kernel on the sender, one local
accumulation kernel on the owner) instead of waiting for a dense reduction.

The fp32 master weights and both Adam moments exist only as shards (1/world
of the model each); the bf16 parameters and the fp32 gradient accumulator
stay full size (the kernels read full weights; the gradient is produced
block by block and reduce-scattered as soon as a bucket is final).

Modes: "nvls" keeps the full fp32 gradient and the full bf16 parameters in
symmetric memory bound to an NVLink multicast object: the reduce-scatter is
one multimem.ld_reduce per 16 bytes of this rank's shard (summed inside the
NVSwitch, written to the local shard) and the all-gather one multimem.st of
this rank's bf16 shard into every GPU's copy. "push" uses the in-kernel
NVLink push collectives (scirs_b200/csrc/comm.cu); "fused" picks "nvls" where
the GPUs support multicast, else "push"; "nccl" uses torch.distributed
reduce_scatter_tensor / all_gather_into_tensor on the same schedule (the
baseline).

Reference parity: the reference's data-parallel primitives are local
simulations (scirs2-autograd/src/distributed/mod.rs:13-84,
scirs2-core/src/gpu/kernels/multi_gpu_sync.cu:381-440 reduce-scatter /
all-gather kernels that a single process launches on one device); ZeRO is
named in its parallelism planner (scirs2-neural/src/distributed/) without an
implementation.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from ..ops import kernels as K


@dataclass
class ShardView:
    """The flat-buffer attributes the fused optimizer reads, for one shard."""

    master: torch.Tensor
    grad: torch.Tensor
    p16: torch.Tensor
    decay_mask: torch.Tensor

    @property
    def total(self) -> int:
        return self.master.numel()


class VocabGradRoute:
    """Sends the embedding-lookup part of a row-sharded vocabulary gradient to
    the rows' owners over NVLink.

    The fp32 gradient of a [V_padded, D] table is owned by rows: rank o holds
    rows [o * R, (o + 1) * R), R = V_padded / world, as its shard of the
    table's gradient bucket. `route(tok, dout)` (compute stream) stores each
    of this rank's token rows dout[m] (bf16) and its row id into the owner's
    receive buffers and signals every peer; `accumulate(shard, scale)`
    (any stream ordered after it) waits (bounded) for every peer's signal and
    adds scale * the received rows into the owner's shard. Receive buffers
    live in a symmetric heap: [world, M, D] bf16 rows and [world, M] int32
    ids (-1 where a source row belongs to another owner). A buffer is rewritten
    one step later only after a collective that every owner joins after its
    accumulation (the optimizer's norm all-reduce), so no read-done signal is
    needed.
    """

    SIG = 1

    def __init__(self, rows_per_rank: int, dim: int, vocab: int, timeout_s: float = 5.0, group=None):
        self.R, self.D, self.V = int(rows_per_rank), int(dim), int(vocab)
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.timeout_s = float(timeout_s)
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.M = 0
        self.heap = None
        self.launches = 0

    def _ensure(self, M: int):
        """(Re)allocate the receive buffers for M tokens per rank. Collective:
        every rank reaches it with the same M (same step shapes)."""
        if M == self.M:
            return
        from .symmetric import SymmetricHeap

        W, D = self.world, self.D
        if self.heap is not None:
            self.heap.close()
        self.heap = SymmetricHeap(W * M * D * 2 + W * M * 4 + 8192, group=self.group)
        self.rows = self.heap.alloc((W, M, D), torch.bfloat16)
        self.ids = self.heap.alloc((W, M), torch.int32)
        self.flags = self.heap.alloc((W,), torch.int32)
        self.flags.zero_()
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        self.rows_at = self.heap.peer_addrs(self.rows)
        self.ids_at = self.heap.peer_addrs(self.ids)
        self.sig = [a + 4 * self.rank for a in self.heap.peer_addrs(self.flags)]
        self.M = M

    def route(self, tok: torch.Tensor, dout: torch.Tensor):
        from .. import _ext

        self._ensure(tok.numel())
        k = _ext.kernels()
        k.tp_step_begin(self.epoch, None)
        k.vocab_route(tok, dout, self.R, self.V, self.rows_at, self.ids_at, self.rank, self.sig, self.epoch,
                      self.SIG)
        self.launches += 2

    def accumulate(self, shard: torch.Tensor, scale: float):
        from .. import _ext

        _ext.kernels().vocab_accum(self.rows, self.ids, shard, float(scale), self.rank, self.flags, self.epoch,
                                   self.SIG, self.timeout_s)
        self.launches += 1

    def close(self):
        if self.heap is not None:
            self.heap.close()
            self.heap = None
            self.M = 0


class ZeroSharding:
    """Owns the shard buffers and the two collectives of a ZeRO step.

    Attach with :func:`zero_data_parallel`. The model must have been built
    with buckets padded to a multiple of 64 * world elements.
    """

    def __init__(self, model, mode: str = "fused", comm=None, group=None):
        fp = model.fp
        self.model = model
        self.fp = fp
        if mode == "fused":
            mode = "nvls" if (comm is not None and comm.nvls_supported()) else "push"
        self.mode = mode
        self.comm = comm
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        N, r = self.world, self.rank
        self.bounds = list(model.bucket_bounds)
        for s, e in self.bounds:
            assert (e - s) % (64 * N) == 0 and s % (64 * N) == 0, (
                "buckets must be padded to a multiple of 64*world elements (bucket_align)"
            )
        self.shard_bounds = [(s // N, e // N) for s, e in self.bounds]
        n = fp.total // N
        dev = fp.master.device
        self.master = torch.empty(n, dtype=torch.float32, device=dev)
        self.p16 = torch.empty(n, dtype=torch.bfloat16, device=dev)
        self.grad = torch.zeros(n, dtype=torch.float32, device=dev)
        mask = torch.empty((n + 63) // 64, dtype=torch.uint8, device=dev)
        for (s, e), (ss, se) in zip(self.bounds, self.shard_bounds):
            ln = (e - s) // N
            self.master[ss:se].copy_(fp.master[s + r * ln : s + (r + 1) * ln])
            mask[ss // 64 : se // 64].copy_(fp.decay_mask[(s + r * ln) // 64 : (s + (r + 1) * ln) // 64])
        self.p16.copy_(self.master)
        self.view = ShardView(self.master, self.grad, self.p16, mask)
        self.cuda = dev.type == "cuda"
        if self.cuda:
            self.stream = torch.cuda.Stream(priority=-1)
            self.rs_events = [torch.cuda.Event() for _ in self.bounds]
            self.ag_events = [torch.cuda.Event() for _ in self.bounds]
        self.launches = 0
        self._gathered = False
        self.vocab_route: VocabGradRoute | None = None  # set by zero_data_parallel for tied vocab tables

    # Host-only ranks (gloo, CPU tensors) run the same schedule synchronously
    # with collectives that gloo provides; used to test the sharding logic.
    def _rs_host(self, full: torch.Tensor, shard: torch.Tensor):
        t = full.clone()
        dist.all_reduce(t, group=self.group)
        ln = shard.numel()
        shard.copy_(t[self.rank * ln : (self.rank + 1) * ln] / self.world)

    def _ag_host(self, shard: torch.Tensor, full: torch.Tensor):
        parts = [torch.empty_like(shard) for _ in range(self.world)]
        dist.all_gather(parts, shard.contiguous(), group=self.group)
        full.copy_(torch.cat(parts))

    # ------------------------------------------------------------- gradients
    def bucket_ready(self, i: int):
        s, e = self.bounds[i]
        ss, se = self.shard_bounds[i]
        if not self.cuda:
            self._rs_host(self.fp.grad[s:e], self.grad[ss:se])
            return
        ev = self.rs_events[i]
        ev.record(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(ev)
            if self.mode == "nvls":
                self.comm.reduce_scatter_nvls(self.fp.grad[s:e], self.grad[ss:se], 1.0 / self.world)
            elif self.mode == "push":
                self.comm.reduce_scatter(self.fp.grad[s:e], self.grad[ss:se], 1.0 / self.world)
            else:
                dist.reduce_scatter_tensor(self.grad[ss:se], self.fp.grad[s:e], op=dist.ReduceOp.AVG,
                                           group=self.group)
            self.launches += 1

    def finish(self):
        if self.cuda:
            torch.cuda.current_stream().wait_stream(self.stream)

    @property
    def early_vocab(self) -> bool:
        """True when the engine may hand over the vocabulary bucket (0) right
        after the LM-head weight gradient and route the lookup part of the
        gradient with :meth:`route_vocab` / :meth:`vocab_ready`."""
        return self.vocab_route is not None

    def route_vocab(self, tok: torch.Tensor, dout: torch.Tensor):
        """Compute stream: send this rank's lookup-gradient rows to their owners."""
        self.vocab_route.route(tok, dout)
        self.launches += 2
        self._route_ev = torch.cuda.Event()
        self._route_ev.record(torch.cuda.current_stream())

    def vocab_ready(self):
        """Communication stream, after bucket 0's reduce-scatter: add the rows
        routed to this rank (scaled by 1/world) into its shard of bucket 0."""
        ss, se = self.shard_bounds[0]
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(self._route_ev)
            vr = self.vocab_route
            self.vocab_route.accumulate(self.grad[ss:se].view(vr.R, vr.D), 1.0 / self.world)
            self.launches += 1

    # ------------------------------------------------------------ parameters
    def begin_forward(self):
        """Issue the all-gather of every bucket's bf16 parameter shards."""
        if not self.cuda:
            for (s, e), (ss, se) in zip(self.bounds, self.shard_bounds):
                self._ag_host(self.p16[ss:se], self.fp.p16[s:e])
            return
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(ev)
            for i, ((s, e), (ss, se)) in enumerate(zip(self.bounds, self.shard_bounds)):
                if self.mode == "nvls":
                    self.comm.all_gather_nvls(self.p16[ss:se], self.fp.p16[s:e])
                elif self.mode == "push":
                    self.comm.all_gather(self.p16[ss:se], self.fp.p16[s:e])
                else:
                    dist.all_gather_into_tensor(self.fp.p16[s:e], self.p16[ss:se], group=self.group)
                self.ag_events[i].record(self.stream)
                self.launches += 1
        self._gathered = True

    def wait_bucket(self, i: int):
        if self._gathered and self.cuda:
            torch.cuda.current_stream().wait_event(self.ag_events[i])

    def end_forward(self):
        self._gathered = False

    # ------------------------------------------------------------- optimizer
    def norm_allreduce(self, part: torch.Tensor, n: int):
        """Sum the per-rank partial sums of squares (tiny; fp32 NCCL)."""
        dist.all_reduce(part[:n], group=self.group)

    @torch.no_grad()
    def consolidate(self, shard: torch.Tensor) -> torch.Tensor:
        """All-gather an fp32 shard-layout buffer into the full flat layout."""
        full = torch.zeros(self.fp.total, dtype=torch.float32, device=shard.device)
        for (s, e), (ss, se) in zip(self.bounds, self.shard_bounds):
            if self.cuda:
                dist.all_gather_into_tensor(full[s:e], shard[ss:se].contiguous(), group=self.group)
            else:
                self._ag_host(shard[ss:se], full[s:e])
        return full

    @torch.no_grad()
    def take_shard(self, full: torch.Tensor, shard: torch.Tensor):
        """Copy this rank's part of a full flat buffer into a shard buffer."""
        N, r = self.world, self.rank
        for (s, e), (ss, se) in zip(self.bounds, self.shard_bounds):
            ln = (e - s) // N
            shard[ss:se].copy_(full[s + r * ln : s + (r + 1) * ln])

    def consolidated_master(self) -> torch.Tensor:
        return self.consolidate(self.master)

    @torch.no_grad()
    def sync_full_master(self):
        """Refresh the model's full fp32 master copy (for checkpoints and
        state_dict) from the shards; the shards are authoritative."""
        self.fp.master.copy_(self.consolidated_master())


class ZeroAdamW:
    """Fused AdamW over the ZeRO shards with the global-norm clip summed over
    ranks. Same hyperparameter interface as FusedFlatOptimizer."""

    def __init__(self, zero: ZeroSharding, **kw):
        from ..optim.fused import FusedFlatOptimizer

        self.zero = zero
        self.inner = FusedFlatOptimizer(zero.view, "adamw", **kw)
        self.launches_per_step = 2

    def __getattr__(self, k):  # hyperparameters and the step counter live on the inner optimizer
        if k in ("zero", "inner", "launches_per_step"):
            raise AttributeError(k)
        return getattr(self.inner, k)

    def __setattr__(self, k, v):
        if k in ("zero", "inner", "launches_per_step"):
            object.__setattr__(self, k, v)
        else:
            setattr(self.inner, k, v)

    def set_lr(self, lr: float):
        self.inner.set_lr(lr)

    def step(self):
        o, z = self.inner, self.zero
        o._hyper()
        n = K.grad_sumsq(z.grad, o.part, o.hp)
        z.norm_allreduce(o.part, n)
        K.optim_step(o.mode, z.master, o.state1, o.state2, z.grad, z.p16, z.master.numel(), o.hp, part=o.part,
                     norm_out=o.grad_norm, decay_mask=z.view.decay_mask, parts_ready=n)


def zero_state_dict(model) -> dict:
    """World-size independent optimizer + parameter state of a ZeRO model:
    per-parameter fp32 tensors (master weights and both Adam moments) keyed
    by parameter name, plus the step counter. Collective: every rank calls
    it; every rank gets the full dict."""
    z, o = model.param_sync, model.optimizer.inner
    fp = z.fp
    out = {"step": int(o.t), "params": {}, "exp_avg": {}, "exp_avg_sq": {}}
    for key, shard in (("params", z.master), ("exp_avg", o.state1), ("exp_avg_sq", o.state2)):
        full = z.consolidate(shard)
        for name in fp.order:
            out[key][name] = fp.view(full, name).detach().clone().cpu()
    return out


@torch.no_grad()
def load_zero_state_dict(model, sd: dict):
    """Inverse of :func:`zero_state_dict` for any world size: lays the named
    tensors out in this run's flat layout (bucket padding depends on the
    world size) and keeps this rank's shards; also refreshes the full master
    and bf16 buffers."""
    z, o = model.param_sync, model.optimizer.inner
    fp = z.fp
    for key, shard in (("params", z.master), ("exp_avg", o.state1), ("exp_avg_sq", o.state2)):
        full = torch.zeros(fp.total, dtype=torch.float32, device=shard.device)
        for name in fp.order:
            fp.view(full, name).copy_(sd[key][name].reshape(fp.slots[name].shape))
        z.take_shard(full, shard)
        if key == "params":
            fp.master.copy_(full)
            fp.sync_bf16()
    z.p16.copy_(z.master)
    o.t = int(sd["step"])
    o.hp[9] = float(o.t)
    o._uploaded = None


def zero_data_parallel(model, mode: str = "fused", comm=None, lr=1e-3, betas=(0.9, 0.999), eps=1e-8,
                       weight_decay=0.0, max_grad_norm=0.0):
    """Shard a flat-buffer model's optimizer state over the data-parallel
    group and attach the reduce-scatter / all-gather schedule.

    Broadcasts rank 0's parameters first so all replicas start equal.
    Returns the model; its `optimizer` is the sharded AdamW.
    """
    import os

    from .nvlink import NVLinkComm

    assert dist.is_initialized()
    if mode == "fused" and os.environ.get("SCIRS_COMM") == "nccl":
        mode = "nccl"
    fp = model.fp
    dist.broadcast(fp.master, src=0)
    fp.sync_bf16()
    if mode in ("fused", "push", "nvls") and comm is None and fp.master.is_cuda:
        biggest = max(e - s for s, e in model.bucket_bounds)
        comm = NVLinkComm(area_bytes=biggest * 2 + (1 << 20))
    if mode in ("fused", "nvls") and comm is not None and comm.nvls_supported():
        # full gradient and bf16 weights in multicast-bound symmetric memory
        # (the kernels take their views from fp.grad / fp.p16 at every call)
        g = comm.nvls_buffer(fp.total, torch.float32)
        g.copy_(fp.grad)
        fp.grad = g
        w = comm.nvls_buffer(fp.total, torch.bfloat16)
        w.copy_(fp.p16)
        fp.p16 = w
        mode = "nvls"
    elif mode == "nvls":
        raise RuntimeError("NVLS requested but this GPU has no NVLink multicast support")
    z = ZeroSharding(model, mode=mode, comm=comm)
    spec = getattr(model, "vocab_grad_spec", None)
    if spec is not None and mode in ("nvls", "push") and fp.master.is_cuda:
        rows, dim, valid = spec["rows"], spec["dim"], spec["valid"]
        s0, e0 = model.bucket_bounds[0]
        N = z.world
        if rows % N == 0 and e0 - s0 == rows * dim and N <= 8:
            z.vocab_route = VocabGradRoute(rows // N, dim, valid)
    model.grad_sync = z
    model.param_sync = z
    model.optimizer = ZeroAdamW(z, lr=lr, betas=betas, eps=eps, weight_decay=weight_decay,
                                max_grad_norm=max_grad_norm)
    return model
