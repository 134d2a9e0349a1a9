"""GPT decoder on the fused sm_100a kernels, split into pipeline stages.

Stage s of P runs a contiguous range of blocks; stage 0 also runs the token +
position embedding, the last stage the final LayerNorm, the tied LM head and
the softmax cross-entropy. A training step splits the batch into micro-batches
and runs them through a GPipe or 1F1B schedule (`parallel.pipeline`):

* activations [M, D] bf16 go to the next stage and gradients [M, D] bf16 to
  the previous one with NCCL point-to-point send / recv. The two directions
  use two communicators, so a send blocked on its receiver in one direction
  never holds up the other direction's transfers (with one communicator the
  1F1B order send(act i+1) -> recv(grad i) on one stage against
  recv(act i+1) <- send(grad i) on the next deadlocks once a message no
  longer fits NCCL's internal buffer).
* every in-flight micro-batch has its own preallocated activation set
  (1F1B: at most P - s of them on stage s; GPipe: all);
* the fc2 bias gradient of a stage's last block is the column sum of the
  gradient it receives (inside one stage that sum is fused into the next
  block's LayerNorm backward);
* the embedding matrix is tied to the LM head: stage 0 and the last stage
  each hold a copy and sum their gradients with one all-reduce over those two
  ranks after the backward, so both copies take identical optimizer steps;
* the global-norm clip sums the squared gradients over all stages (the tied
  matrix counted once).

Reference parity: scirs2-neural/src/training/pipeline_parallel.rs:48-380
(GPipe / 1F1B schedules, micro-batches, activation stash; a single-process
simulation there) and scirs2-autograd/src/distributed_grad.rs:603-735
(generate_1f1b_schedule).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import kernels as K
from ..parallel.pipeline import generate_1f1b_schedule, generate_gpipe_schedule
from ..utils.flat import FlatParams
from .gpt import GPTConfig, gpt_init_values
from .transformer import BlockActs, FusedTrainerMixin, add_block_params, block_backward, block_forward


def stage_bounds(num_layers: int, num_stages: int, stage: int) -> tuple[int, int]:
    """Blocks [l0, l1) of `stage`: an even split, the first stages taking one
    extra block when the count does not divide."""
    q, r = divmod(num_layers, num_stages)
    l0 = stage * q + min(stage, r)
    return l0, l0 + q + (1 if stage < r else 0)


class _StageActs(BlockActs):
    def __init__(self, cfg: GPTConfig, nblocks: int, B: int, S: int, last: bool, device):
        D, F, H = cfg.hidden_size, cfg.intermediate_size, cfg.num_attention_heads
        super().__init__(nblocks, B, S, D, F, H, device)
        M = B * S
        self.send_work = None  # outstanding send from this set's buffers
        if last:
            self.lnf = torch.empty(M, D, dtype=torch.bfloat16, device=device)
            self.muf = torch.empty(M, dtype=torch.float32, device=device)
            self.rsf = torch.empty(M, dtype=torch.float32, device=device)
            self.logits = torch.empty(M, cfg.vocab_padded, dtype=torch.bfloat16, device=device)
            self.losses = torch.empty(M, dtype=torch.float32, device=device)

    def settle(self):
        if self.send_work is not None:
            self.send_work.wait()
            self.send_work = None


class GPTPipelineStage(FusedTrainerMixin):
    """One pipeline stage of a GPT decoder. Every rank of the default group
    constructs its stage (collective: the communicators are created here).

    Usage::

        st = GPTPipelineStage(cfg, stage=rank, num_stages=world, num_micro=8)
        st.configure_adamw(lr=6e-4)
        loss = st.train_step(tokens, targets)   # last stage: mean loss; others: None
    """

    def __init__(self, cfg: GPTConfig, stage: int, num_stages: int, num_micro: int, device="cuda", seed: int = 0,
                 schedule: str = "1f1b", ranks: list[int] | None = None, bucket_align: int = 64):
        assert cfg.hidden_dropout_prob == 0 and cfg.attention_probs_dropout_prob == 0, "dropout must be 0"
        assert schedule in ("1f1b", "gpipe")
        assert 1 <= num_stages <= cfg.num_hidden_layers
        self.cfg, self.stage, self.P, self.num_micro, self.schedule = cfg, stage, num_stages, num_micro, schedule
        self.device = torch.device(device)
        self.ranks = ranks or list(range(num_stages))
        self.first, self.last = stage == 0, stage == num_stages - 1
        self.l0, self.l1 = stage_bounds(cfg.num_hidden_layers, num_stages, stage)
        D, F, Vp = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_padded
        fp = FlatParams()
        if self.first or self.last:
            fp.add("wte", (Vp, D), decay=True)
        fp.pad_to(bucket_align)
        self.wte_end = fp.mark()
        if self.first:
            fp.add("wpe", (cfg.max_position_embeddings, D), decay=True)
        for l in range(self.l0, self.l1):
            add_block_params(fp, f"h{l}.", D, F)
        if self.last:
            fp.add("ln_f.weight", (D,), False)
            fp.add("ln_f.bias", (D,), False)
        fp.pad_to(bucket_align)
        fp.allocate(self.device)
        self.fp = fp
        for name, t in gpt_init_values(cfg, seed):
            if name in fp.slots:
                fp.m(name).copy_(t)
        fp.sync_bf16()
        # communicators (collective over the default group, same order everywhere)
        self.g_fwd = dist.new_group(self.ranks) if num_stages > 1 else None
        self.g_bwd = dist.new_group(self.ranks) if num_stages > 1 else None
        self.g_all = dist.new_group(self.ranks) if num_stages > 1 else None
        tied = sorted({self.ranks[0], self.ranks[-1]})
        self.g_tied = dist.new_group(tied) if num_stages > 1 else None
        self._pool: list[_StageActs] = []
        self._pool_key = None
        self._graph = self._graph_key = self._warm_key = None
        self._last_shape = None
        self.grad_sync = None
        self.optimizer = None
        self.kernel_launches = 0

    # ------------------------------------------------------------ plumbing
    def _acts_pool(self, B: int, S: int) -> list[_StageActs]:
        n = self.num_micro if self.schedule == "gpipe" else min(self.num_micro, self.P - self.stage)
        if self._pool_key != (B, S, n):
            self._pool = [_StageActs(self.cfg, self.l1 - self.l0, B, S, self.last, self.device) for _ in range(n)]
            self._pool_key = (B, S, n)
        return self._pool

    def _send(self, t, stage, group):
        return dist.isend(t, self.ranks[stage], group=group)

    def _recv(self, t, stage, group):
        dist.irecv(t, self.ranks[stage], group=group).wait()

    # ------------------------------------------------------------- compute
    def _fwd(self, A: _StageActs, tok, tgt, scale: float) -> int:
        cfg, fp = self.cfg, self.fp
        S, H, hd, eps = A.S, cfg.num_attention_heads, cfg.head_dim, cfg.layer_norm_eps
        n = 0
        A.settle()
        if self.first:
            K.embedding_fwd(tok, fp.w("wte"), fp.w("wpe")[:S], A.x[0], S)
            n += 1
        else:
            self._recv(A.x[0], self.stage - 1, self.g_fwd)
        for j, l in enumerate(range(self.l0, self.l1)):
            n += block_forward(fp, f"h{l}.", A, j, H, hd, eps, causal=True)
        nb = self.l1 - self.l0
        if self.last:
            K.layernorm_fwd(A.x[nb], fp.w("ln_f.weight"), fp.w("ln_f.bias"), A.lnf, A.muf, A.rsf, eps)
            K.gemm(A.lnf, fp.w("wte"), A.logits)
            K.xent_fwd_bwd(A.logits, tgt, A.losses, cfg.vocab_size, scale)
            n += 3
        else:
            A.send_work = self._send(A.x[nb], self.stage + 1, self.g_fwd)
        return n

    def _bwd(self, A: _StageActs, tok) -> int:
        cfg, fp = self.cfg, self.fp
        S, H, hd = A.S, cfg.num_attention_heads, cfg.head_dim
        nb = self.l1 - self.l0
        n = 0
        A.settle()
        last_fc2 = f"h{self.l1 - 1}.mlp.c_proj.bias"
        if self.last:
            dlog = A.logits
            K.gemm(dlog, fp.w("wte"), A.dln, b_mn=True)
            K.gemm(dlog, A.lnf, fp.g("wte"), a_mn=True, b_mn=True, epi=K.EPI_F32, accumulate=True)
            K.layernorm_bwd(A.dln, A.x[nb], fp.w("ln_f.weight"), A.muf, A.rsf, A.dres, fp.g("ln_f.weight"),
                            fp.g("ln_f.bias"), A.ln_part, dsum=fp.g(last_fc2))
            n += 3
        else:
            self._recv(A.dres, self.stage + 1, self.g_bwd)
            K.bias_grad(A.dres, fp.g(last_fc2))
            n += 1
        for j in reversed(range(nb)):
            l = self.l0 + j
            n += block_backward(fp, f"h{l}.", A, j, H, hd, causal=True,
                                prev_fc2_bias=f"h{l - 1}.mlp.c_proj.bias" if j > 0 else None)
        if self.first:
            K.embedding_bwd(tok, A.dres, fp.g("wte"), fp.g("wpe")[:S], S)
            n += 1
        else:
            A.send_work = self._send(A.dres, self.stage - 1, self.g_bwd)
        return n

    # ----------------------------------------------------------------- API
    def forward_backward(self, tokens: torch.Tensor, targets: torch.Tensor, shape=None):
        """Forward + backward of all micro-batches of the step (gradients
        accumulate into the flat buffer; the tied embedding gradient is
        summed across its two stages). Returns the mean loss on the last
        stage (device scalar), None elsewhere. `tokens` / `targets` [B, S]
        are needed on the first / last stage only; a stage given neither
        takes the batch shape from `shape` (or the previous step)."""
        ref = tokens if tokens is not None else targets
        if ref is not None:
            B, S = ref.shape
        elif shape is not None:
            B, S = shape
        elif getattr(self, "_last_shape", None) is not None:
            B, S = self._last_shape
        else:
            raise ValueError("a middle stage needs the batch shape (pass shape=(B, S))")
        self._last_shape = (B, S)
        assert B % self.num_micro == 0, "batch must split into equal micro-batches"
        mb = B // self.num_micro
        pool = self._acts_pool(mb, S)
        toks = tokens.reshape(self.num_micro, mb * S) if tokens is not None else None
        tgts = targets.reshape(self.num_micro, mb * S) if targets is not None else None
        gen = generate_gpipe_schedule if self.schedule == "gpipe" else generate_1f1b_schedule
        slot_of: dict[int, _StageActs] = {}
        free = list(pool)
        loss = torch.zeros((), dtype=torch.float32, device=self.device) if self.last else None
        scale = 1.0 / (B * S)
        n = 0
        for kind, i in gen(self.P, self.num_micro, self.stage):
            tok = toks[i] if toks is not None else None
            if kind == "F":
                A = free.pop()
                slot_of[i] = A
                n += self._fwd(A, tok, tgts[i] if self.last else None, scale)
                if self.last:
                    loss += A.losses.sum() * scale
            else:
                A = slot_of.pop(i)
                n += self._bwd(A, tok)
                free.append(A)
        for A in pool:
            A.settle()
        if self.P > 1 and (self.first or self.last) and self.ranks[0] != self.ranks[-1]:
            dist.all_reduce(self.fp.g("wte"), group=self.g_tied)
        self.kernel_launches += n
        return loss

    def train_step(self, tokens, targets, shape=None):
        """zero_grad -> pipelined forward/backward -> tied-gradient sum ->
        fused AdamW with the global-norm clip taken over all stages. With
        enable_cuda_graph() the whole step of this stage (its kernels, the
        NCCL point-to-point transfers and the two all-reduces) is captured
        once per batch shape and replayed; every stage must enable it."""
        if self.optimizer is None:
            self.configure_adamw()
        if getattr(self, "use_graph", False) and self.device.type == "cuda":
            return self._step_graphed(tokens, targets, shape)
        return self._step_eager(tokens, targets, shape)

    def _step_eager(self, tokens, targets, shape=None):
        self.fp.grad.zero_()
        loss = self.forward_backward(tokens, targets, shape)
        self._optimizer_step()
        return loss

    def _step_graphed(self, tokens, targets, shape=None):
        ref = tokens if tokens is not None else targets
        key = tuple(ref.shape) if ref is not None else (tuple(shape) if shape is not None else self._last_shape)
        if self._graph is not None and self._graph_key == key:
            if tokens is not None:
                self._g_tok.copy_(tokens, non_blocking=True)
            if targets is not None:
                self._g_tgt.copy_(targets, non_blocking=True)
            self._graph.replay()
            self.optimizer.t += 1
            K.STATS.launches += self._graph_kernels
            return self._g_loss
        if self._warm_key != key:  # first step at this shape runs eagerly and allocates every buffer
            self._warm_key = key
            return self._step_eager(tokens, targets, shape)
        self._g_tok = tokens.clone() if tokens is not None else None
        self._g_tgt = targets.clone() if targets is not None else None
        torch.cuda.synchronize()
        if self.P > 1:
            dist.barrier(group=self.g_all)
        k0 = K.STATS.launches
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._g_loss = self._step_eager(self._g_tok, self._g_tgt, key)
        self._graph_kernels = K.STATS.launches - k0
        K.STATS.launches = k0
        self.optimizer.t -= 1  # the capture did not execute a step; the replay below does
        self._graph, self._graph_key = g, key
        return self._step_graphed(tokens, targets, shape)

    def _optimizer_step(self):
        o, fp = self.optimizer, self.fp
        o._hyper()
        if o.max_grad_norm > 0 and self.P > 1:
            # tied matrix counted once: the last stage leaves its copy out
            g = fp.grad[self.wte_end:] if (self.last and not self.first) else fp.grad
            n = K.grad_sumsq(g, o.part, o.hp)
            tot = o.part[:n].sum().reshape(1)
            dist.all_reduce(tot, group=self.g_all)
            o.part[:n].zero_()
            o.part[:1].copy_(tot)
            K.optim_step(o.mode, fp.master, o.state1, o.state2, fp.grad, fp.p16, fp.total, o.hp, part=o.part,
                         norm_out=o.grad_norm, decay_mask=fp.decay_mask, parts_ready=n)
        else:
            K.optim_step(o.mode, fp.master, o.state1, o.state2, fp.grad, fp.p16, fp.total, o.hp, part=o.part,
                         norm_out=o.grad_norm, decay_mask=fp.decay_mask)
        self.kernel_launches += o.launches_per_step

    def state_dict(self):
        """This stage's parameters (fp32 master copies), by global name."""
        return self.fp.state_dict()
