"""Context parallelism: ring attention over a sequence split across ranks.

Rank r holds tokens [r*Sc, (r+1)*Sc) of every sequence (q, k, v all
[B, Sc, H, D]). The key/value chunks travel around the ring (point-to-point
send/recv to rank r+1, receive from r-1, posted before each step's compute
so the transfer overlaps it); after W steps every rank has attended to every
chunk it may see:

  forward   per visited chunk j: (o_j, lse_j) = attention(q, k_j, v_j), causal
            inside the diagonal chunk (j == r), skipped for j > r when causal;
            partial results merged with the log-sum-exp rule
            lse = logaddexp(lse, lse_j), o = o e^(lse_old - lse) + o_j e^(lse_j - lse)
  backward  the chunks travel again together with their dK / dV accumulators;
            each visit adds this rank's contribution computed against the
            GLOBAL output and log-sum-exp (P = exp(S - lse)); after W sends the
            accumulators are back at their owners. dQ stays local.

On GPUs each chunk uses the framework's flash-attention forward / backward
kernels (the backward kernel takes the global out / lse as inputs); on CPU
an fp32 restatement of the same math.

Reference parity: none (the reference has no sequence / context
parallelism); it builds on the online-softmax merge of
scirs2-neural/src/attention/flash_v2.rs:213 (tile_attention_block).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import kernels as K


def _chunk_fwd(q, k, v, causal, scale):
    if q.is_cuda:
        B, S, H, D = q.shape
        out = torch.empty_like(q)
        lse = torch.empty(B, H, S, device=q.device, dtype=torch.float32)
        K.flash_attn_fwd(q, k, v, out, lse, causal, scale)
        return out.float(), lse
    o, lse = K.attention_reference(q, k, v, causal, scale)
    return o, lse


def _chunk_bwd(dout, q, k, v, out, lse, causal, scale):
    """Gradients of this rank's queries against one key/value chunk, with the
    probabilities normalised by the global log-sum-exp."""
    if q.is_cuda:
        B, S, H, D = q.shape
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        dq_acc = torch.empty(B * S * H * D, device=q.device, dtype=torch.float32)
        delta = torch.empty(B * H * S, device=q.device, dtype=torch.float32)
        K.flash_attn_bwd(dout.contiguous(), q, k, v, out.to(q.dtype).contiguous(), lse.contiguous(), dq, dk, dv,
                         dq_acc, delta, causal, scale)
        return dq.float(), dk.float(), dv.float()
    qf, kf, vf, dof, of = (t.float().transpose(1, 2) for t in (q, k, v, dout, out))  # [B, H, S, D]
    s = (qf @ kf.transpose(-1, -2)) * scale
    if causal:
        Sq = s.shape[-1]
        s = s.masked_fill(torch.ones(Sq, Sq, dtype=torch.bool, device=s.device).triu(1), float("-inf"))
    p = torch.exp(s - lse.unsqueeze(-1))
    dv = p.transpose(-1, -2) @ dof
    dp = dof @ vf.transpose(-1, -2)
    delta = (dof * of).sum(-1, keepdim=True)
    ds = p * (dp - delta)
    dq = (ds @ kf) * scale
    dk = (ds.transpose(-1, -2) @ qf) * scale
    return dq.transpose(1, 2), dk.transpose(1, 2), dv.transpose(1, 2)


def _ring_exchange(tensors, group, rank, world):
    """Send `tensors` to rank+1 and receive the same shapes from rank-1."""
    nxt = (rank + 1) % world
    prv = (rank - 1) % world
    gn = dist.get_global_rank(group, nxt) if group is not None else nxt
    gp = dist.get_global_rank(group, prv) if group is not None else prv
    recv = [torch.empty_like(t) for t in tensors]
    ops = [dist.P2POp(dist.isend, t.contiguous(), gn, group) for t in tensors]
    ops += [dist.P2POp(dist.irecv, r, gp, group) for r in recv]
    reqs = dist.batch_isend_irecv(ops)
    return recv, reqs


def _visible(j: int, rank: int, causal: bool) -> bool:
    return (not causal) or j <= rank


class _RingAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, scale, group):
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        out = lse = None
        kv = (k, v)
        for step in range(world):
            j = (rank - step) % world
            pending = _ring_exchange(kv, group, rank, world) if step + 1 < world else None
            if _visible(j, rank, causal):
                o_j, lse_j = _chunk_fwd(q, kv[0], kv[1], causal and j == rank, scale)
                if out is None:
                    out, lse = o_j, lse_j
                else:
                    new = torch.logaddexp(lse, lse_j)
                    a = torch.exp(lse - new).transpose(1, 2).unsqueeze(-1)
                    b = torch.exp(lse_j - new).transpose(1, 2).unsqueeze(-1)
                    out, lse = out * a + o_j * b, new
            if pending is not None:
                recv, reqs = pending
                for r in reqs:
                    r.wait()
                kv = tuple(recv)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.causal, ctx.scale, ctx.group = causal, scale, group
        return out.to(q.dtype), lse

    @staticmethod
    def backward(ctx, dout, dlse):
        q, k, v, out, lse = ctx.saved_tensors
        group = ctx.group
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        dq = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
        dk = torch.zeros(k.shape, dtype=torch.float32, device=k.device)
        dv = torch.zeros(v.shape, dtype=torch.float32, device=v.device)
        kv = (k, v)
        for step in range(world):
            j = (rank - step) % world
            if _visible(j, rank, ctx.causal):
                gq, gk, gv = _chunk_bwd(dout, q, kv[0], kv[1], out, lse, ctx.causal and j == rank, ctx.scale)
                dq += gq
                dk += gk
                dv += gv
            # the chunk (and its gradient accumulators) moves on; after the
            # last send the accumulators are back at their owner
            send = (kv[0], kv[1], dk, dv) if step + 1 < world else (dk, dv)
            recv, reqs = _ring_exchange(send, group, rank, world)
            for r in reqs:
                r.wait()
            if step + 1 < world:
                kv, dk, dv = (recv[0], recv[1]), recv[2], recv[3]
            else:
                dk, dv = recv
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), None, None, None


def ring_attention(q, k, v, causal: bool = True, scale: float | None = None, group=None):
    """Attention of this rank's query chunk over the whole (ring-distributed)
    sequence. q/k/v: [B, Sc, H, D] with rank r holding chunk r. Returns
    (out [B, Sc, H, D], lse [B, H, Sc]); differentiable in q, k, v."""
    scale = scale if scale is not None else q.shape[-1] ** -0.5
    return _RingAttention.apply(q, k, v, causal, scale, group)
