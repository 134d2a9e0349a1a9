"""Mixture of experts: top-k softmax routing with per-expert capacity and the
load-balancing auxiliary loss, on one device or expert-parallel over a
process group.

Routing semantics (scirs2-neural/src/layers/moe.rs:120-440): gate logits =
x @ Wg + bg (+ Gaussian noise during training if `gating_noise` > 0);
probabilities = softmax; each token keeps its k most probable experts with
the k weights renormalised to sum to 1; expert e accepts at most
capacity = ceil(tokens * capacity_factor / num_experts) assignments, taken
in token order (token-major, then rank within the token's top k); an
assignment past capacity is dropped (its weight is not redistributed).
aux = coeff * E * sum_e f_e * P_e, f_e = assignments to e / tokens (before
the capacity cut), P_e = mean probability of e. Experts are
Linear(d, d_ff) -> ReLU -> Linear(d_ff, d).

Execution: assignments are scattered into a dense [E, capacity, d] buffer
(one slot per accepted assignment) so every expert's FFN is one batched
GEMM over all experts (tensor cores, no per-expert launches), then gathered
back and combined with the routing weights.

Expert parallel (ExpertParallelMoE): rank r owns experts
[r*E/W, (r+1)*E/W). Two transports:

  "peer" (GPUs, NCCL group, up to 8 ranks): the permutation and the
      all-to-all are one kernel: each rank gathers its routed token rows and
      stores them over NVLink straight into the owners' receive buffers
      ([E/W, W, capacity, d], in a symmetric heap mapped into every peer),
      then signals. The owners run their experts on the received rows and
      publish the outputs; the return all-to-all and the weighted
      combination are again one kernel, which reads each token's k expert
      outputs from the owners' buffers and sums them in fp32. The backward
      pass runs the same two kernels the other way round (the routing-weight
      gradient <dout, y_j> is read against the owners' outputs).
      Every buffer is reused only after the chain of signals proves its
      readers are done, so a layer may run forward / backward repeatedly;
      two forward passes whose backward passes are both still pending are
      not supported (the second overwrites the first's buffers).
  "nccl": each rank routes its tokens into a [W, E/W, capacity, d] send
      buffer; one all-to-all delivers every rank the slots of its experts
      from all sources, the local batched GEMMs run, and a second all-to-all
      returns the results to the token owners.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from .. import _ext


@dataclass
class MoEConfig:
    num_experts: int = 8
    expert_dim: int = 2048
    top_k: int = 2
    capacity_factor: float = 1.25
    load_balance_coeff: float = 0.01
    gating_type: str = "topk"  # "topk" | "switch" (top-1)
    gating_noise: float = 0.0

    def __post_init__(self):
        if self.gating_type == "switch":
            self.top_k = 1
        if not 1 <= self.top_k <= self.num_experts:
            raise ValueError(f"top_k ({self.top_k}) must be in [1, num_experts ({self.num_experts})]")
        if self.capacity_factor <= 0:
            raise ValueError("capacity_factor must be > 0")


@dataclass
class Routing:
    expert: torch.Tensor  # [T, k] expert index
    weight: torch.Tensor  # [T, k] renormalised routing weight
    slot: torch.Tensor  # [T, k] position within the expert's capacity (-1: dropped)
    capacity: int
    aux_loss: torch.Tensor
    probs: torch.Tensor


def route(logits: torch.Tensor, cfg: MoEConfig, capacity: int | None = None) -> Routing:
    T, E = logits.shape
    k = cfg.top_k
    probs = torch.softmax(logits.float(), dim=-1)
    w, idx = probs.topk(k, dim=-1)
    w = w / w.sum(-1, keepdim=True).clamp_min(1e-30)
    if capacity is None:
        capacity = max(1, math.ceil(T * cfg.capacity_factor / E))
    onehot = F.one_hot(idx.reshape(-1), E)  # token-major order of assignments
    pos = (onehot.cumsum(0) - 1).gather(1, idx.reshape(-1, 1)).reshape(T, k)
    slot = torch.where(pos < capacity, pos, torch.full_like(pos, -1))
    f = onehot.sum(0).float() / T
    P = probs.mean(0)
    aux = cfg.load_balance_coeff * E * (f * P).sum()
    return Routing(idx, w.to(logits.dtype), slot, capacity, aux, probs)


def _dispatch(x: torch.Tensor, r: Routing, E: int) -> torch.Tensor:
    """[T, d] tokens -> [E * capacity, d] expert slots (zeros where empty)."""
    T, k = r.expert.shape
    keep = r.slot >= 0
    dest = (r.expert * r.capacity + r.slot)[keep]
    src = torch.arange(T, device=x.device)[:, None].expand(T, k)[keep]
    buf = x.new_zeros(E * r.capacity, x.shape[1])
    return buf.index_copy(0, dest, x[src])


def _combine(y: torch.Tensor, r: Routing, T: int) -> torch.Tensor:
    """[E * capacity, d] expert outputs -> [T, d] weighted sum per token."""
    keep = r.slot >= 0
    dest = (r.expert * r.capacity + r.slot)[keep]
    tok = torch.arange(T, device=y.device)[:, None].expand_as(r.expert)[keep]
    contrib = y[dest] * r.weight[keep][:, None]
    return y.new_zeros(T, y.shape[1]).index_add(0, tok, contrib)


class _Experts(nn.Module):
    """E feed-forward experts as stacked weights (one batched GEMM each)."""

    def __init__(self, n: int, d: int, d_ff: int, generator=None):
        super().__init__()
        s = math.sqrt(2.0 / (d + d_ff))  # uniform(-s, s), the reference's init scale
        self.w1 = nn.Parameter((torch.rand(n, d, d_ff, generator=generator) * 2 - 1) * s)
        self.b1 = nn.Parameter(torch.zeros(n, d_ff))
        self.w2 = nn.Parameter((torch.rand(n, d_ff, d, generator=generator) * 2 - 1) * s)
        self.b2 = nn.Parameter(torch.zeros(n, d))

    def forward(self, slots: torch.Tensor) -> torch.Tensor:  # [n, C, d]
        h = torch.relu(torch.baddbmm(self.b1[:, None, :], slots, self.w1))
        return torch.baddbmm(self.b2[:, None, :], h, self.w2)


class MixtureOfExperts(nn.Module):
    def __init__(self, d_model: int, config: MoEConfig, seed: int = 0):
        super().__init__()
        self.d_model, self.config = d_model, config
        g = torch.Generator().manual_seed(seed)
        E = config.num_experts
        self.gate = nn.Linear(d_model, E)
        with torch.no_grad():
            self.gate.weight.copy_((torch.rand(E, d_model, generator=g) * 2 - 1) / math.sqrt(d_model))
            self.gate.bias.zero_()
        self.experts = _Experts(E, d_model, config.expert_dim, g)
        self.aux_loss = torch.zeros(())
        self.last_routing: Routing | None = None

    def last_aux_loss(self) -> torch.Tensor:
        return self.aux_loss

    def gate_logits(self, x2: torch.Tensor) -> torch.Tensor:
        logits = self.gate(x2)
        if self.training and self.config.gating_noise > 0:
            logits = logits + torch.randn_like(logits) * self.config.gating_noise
        return logits

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, self.d_model)
        T, E = x2.shape[0], self.config.num_experts
        r = route(self.gate_logits(x2), self.config)
        slots = _dispatch(x2, r, E).view(E, r.capacity, self.d_model)
        y = self.experts(slots).reshape(E * r.capacity, self.d_model)
        self.aux_loss, self.last_routing = r.aux_loss, r
        return _combine(y, r, T).reshape(shape)

    def parameter_count(self) -> int:
        return sum(p.numel() for p in self.parameters())


class _AllToAll(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        out = torch.empty_like(x)
        dist.all_to_all_single(out, x.contiguous(), group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        out = torch.empty_like(g)
        dist.all_to_all_single(out, g.contiguous(), group=ctx.group)
        return out, None


def _send_rows(r: Routing, E: int, T: int):
    """Destination-major send rows q = expert * capacity + slot of the kept
    assignments: (q, token of each kept assignment, keep mask)."""
    keep = r.slot >= 0
    q = (r.expert * r.capacity + r.slot)[keep]
    tok = torch.arange(T, device=r.expert.device)[:, None].expand_as(r.expert)[keep]
    return q, tok, keep


class _PeerBuffers:
    """Symmetric buffers and the signal counter of one expert-parallel layer
    on the peer-memory kernels: receive rows, expert outputs and their two
    gradients, each [L, W * C, d] bf16, plus one flag word per source rank.
    Signal values count up by one per signal, identically on every rank."""

    def __init__(self, group, L: int, C: int, d: int, device, timeout_s: float):
        from ..parallel.symmetric import SymmetricHeap

        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.L, self.C, self.d, self.timeout_s = L, C, d, float(timeout_s)
        W = self.world
        n = L * W * C * d * 2
        self.heap = SymmetricHeap(4 * (n + 1024) + 2048, group=group)
        self.flags = self.heap.alloc((8,), torch.int32, align=256)
        self.sig = [a + 4 * self.rank for a in self.heap.peer_addrs(self.flags)]
        self.bufs = {name: self.heap.alloc((L, W * C, d)) for name in ("recv", "y", "dy", "drecv")}
        self.addr = {name: self.heap.peer_addrs(t) for name, t in self.bufs.items()}
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self.count = 0

    def next(self) -> int:
        self.count += 1
        return self.count

    def push(self, src, idx, scale, dst: str) -> None:
        """Gather rows of `src` by `idx` (x scale), store them into every
        owner's `dst` buffer and wait until every source has done so."""
        K = _ext.kernels()
        i = self.next()
        K.ep_dispatch(src, idx, scale, self.addr[dst], self.L, self.C, self.world * self.C, self.C, self.rank,
                      self.sig, self.epoch, i)
        K.tp_wait(self.flags, self.epoch, i, self.rank, self.world, self.timeout_s)

    def publish(self, name: str, t: torch.Tensor) -> int:
        self.bufs[name].copy_(t)
        i = self.next()
        _ext.kernels().tp_signal(self.sig, self.epoch, i)
        return i

    def pull(self, name: str, expert, slot, wt, T: int, wait: int) -> torch.Tensor:
        out = torch.empty(T, self.d, dtype=torch.bfloat16, device=expert.device)
        _ext.kernels().ep_combine(self.addr[name], expert, slot, wt, out, self.L, self.C, self.rank, self.flags,
                                  self.epoch, wait, self.timeout_s)
        return out

    def close(self):
        self.heap.close()


class _PeerDispatch(torch.autograd.Function):
    """x [T, d] bf16 -> this rank's expert inputs [L, W * C, d] from every source."""

    @staticmethod
    def forward(ctx, x, idx, expert, slot, bufs):
        bufs.push(x.contiguous(), idx, None, "recv")
        ctx.bufs, ctx.T = bufs, x.shape[0]
        ctx.save_for_backward(expert, slot)
        # a copy: the heap buffers are views of one allocation that later
        # transfers overwrite in place, so autograd must not save the view
        return bufs.bufs["recv"].view(bufs.L, bufs.world * bufs.C, bufs.d).clone()

    @staticmethod
    def backward(ctx, g):
        expert, slot = ctx.saved_tensors
        bufs = ctx.bufs
        i = bufs.publish("drecv", g)
        return bufs.pull("drecv", expert, slot, None, ctx.T, i), None, None, None, None


class _PeerCombine(torch.autograd.Function):
    """Expert outputs y [L, W * C, d] bf16 -> out[t] = sum_j w[t, j] y_j [T, d]."""

    @staticmethod
    def forward(ctx, y, wt, expert, slot, idx, bufs):
        i = bufs.publish("y", y)
        w32 = wt.float().contiguous()
        out = bufs.pull("y", expert, slot, w32, expert.shape[0], i)
        ctx.bufs, ctx.wdtype = bufs, wt.dtype
        ctx.save_for_backward(w32, expert, slot, idx)
        return out

    @staticmethod
    def backward(ctx, dout):
        w32, expert, slot, idx = ctx.saved_tensors
        bufs = ctx.bufs
        dout = dout.to(torch.bfloat16).contiguous()
        gw = torch.empty_like(w32)
        _ext.kernels().ep_grad_w(bufs.addr["y"], expert, slot, dout, gw, bufs.L, bufs.C, bufs.rank)
        keep = slot >= 0
        scale = torch.zeros(idx.numel(), dtype=torch.float32, device=dout.device)
        scale[(expert * bufs.C + slot)[keep].long()] = w32[keep]
        bufs.push(dout, idx, scale, "dy")
        dy = bufs.bufs["dy"].view(bufs.L, bufs.world * bufs.C, bufs.d)
        return dy, gw.to(ctx.wdtype), None, None, None, None


class ExpertParallelMoE(nn.Module):
    """Experts sharded over `group`; the gate is replicated (its gradient
    must be all-reduced with the data-parallel gradients like any other
    replicated parameter). Build every rank with the same `seed`: each rank
    keeps its slice of the same expert initialisation, so the layer equals
    :class:`MixtureOfExperts` with the same seed."""

    def __init__(self, d_model: int, config: MoEConfig, group=None, seed: int = 0, transport: str = "auto",
                 timeout_s: float = 30.0):
        super().__init__()
        if transport not in ("auto", "peer", "nccl"):
            raise ValueError(f"unknown transport {transport!r}")
        self.transport, self.timeout_s, self._bufs = transport, timeout_s, None
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        E = config.num_experts
        if E % self.world:
            raise ValueError("num_experts must be a multiple of the expert-parallel group size")
        self.local = E // self.world
        full = MixtureOfExperts(d_model, config, seed)
        self.d_model, self.config = d_model, config
        self.gate = full.gate
        lo, hi = self.rank * self.local, (self.rank + 1) * self.local
        self.experts = _Experts(self.local, d_model, config.expert_dim)
        with torch.no_grad():
            for n in ("w1", "b1", "w2", "b2"):
                getattr(self.experts, n).copy_(getattr(full.experts, n)[lo:hi])
        self.aux_loss = torch.zeros(())

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, self.d_model)
        T, E, W, L, d = x2.shape[0], self.config.num_experts, self.world, self.local, self.d_model
        logits = self.gate(x2)
        if self.training and self.config.gating_noise > 0:
            logits = logits + torch.randn_like(logits) * self.config.gating_noise
        r = route(logits, self.config)
        C = r.capacity
        if self._use_peer(x2):
            return self._forward_peer(x, x2, r).reshape(shape)
        send = _dispatch(x2, r, E)  # [E*C, d] = [W, L, C, d]: destination-rank major
        recv = _AllToAll.apply(send, self.group)  # [W (source), L, C, d]
        y = self.experts(recv.view(W, L, C, d).transpose(0, 1).reshape(L, W * C, d))
        y = y.view(L, W, C, d).transpose(0, 1).reshape(E * C, d)
        back = _AllToAll.apply(y, self.group)  # [W (owner of expert), L, C, d] for this rank's tokens
        self.aux_loss = r.aux_loss
        return _combine(back, r, T).reshape(shape)

    def _use_peer(self, x2: torch.Tensor) -> bool:
        if self.transport == "nccl":
            return False
        ok = (x2.is_cuda and dist.get_backend(self.group) == "nccl" and self.world <= 8 and self.config.top_k <= 8
              and self.d_model % 8 == 0)
        if self.transport == "peer" and not ok:
            raise RuntimeError("the peer transport needs CUDA tensors, an NCCL group of at most 8 ranks, "
                               "top_k <= 8 and d_model a multiple of 8")
        return ok

    def _peer_buffers(self, C: int, device) -> _PeerBuffers:
        b = self._bufs
        if b is None or b.C != C:
            if b is not None:
                b.close()
            b = self._bufs = _PeerBuffers(self.group, self.local, C, self.d_model, device, self.timeout_s)
        return b

    def _forward_peer(self, x, x2, r: Routing) -> torch.Tensor:
        T, E = x2.shape[0], self.config.num_experts
        bufs = self._peer_buffers(r.capacity, x2.device)
        q, tok, _ = _send_rows(r, E, T)
        idx = torch.full((E * r.capacity,), -1, dtype=torch.int32, device=x2.device)
        idx[q] = tok.int()
        expert, slot = r.expert.int().contiguous(), r.slot.int().contiguous()
        recv = _PeerDispatch.apply(x2.to(torch.bfloat16), idx, expert, slot, bufs)
        y = self.experts(recv.to(self.experts.w1.dtype))
        out = _PeerCombine.apply(y.to(torch.bfloat16), r.weight, expert, slot, idx, bufs)
        self.aux_loss = r.aux_loss
        return out.to(x.dtype)

    def close(self):
        """Release the symmetric buffers (collective: every rank calls it)."""
        if self._bufs is not None:
            self._bufs.close()
            self._bufs = None
