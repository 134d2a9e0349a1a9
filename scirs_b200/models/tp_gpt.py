"""Tensor-parallel decoder (RoPE, GELU MLP, pre-LN) on the fused
all-gather->GEMM / GEMM->reduce-scatter kernels.

Layout per rank r of a tensor-parallel group of `world` ranks (Megatron
style, sequence-parallel):

  replicated (gradients summed over ranks): token embedding wte [V, D],
      LayerNorm weights/biases, the row-parallel output biases
  column-parallel (output features split): attn.c_attn [3*D/w, D] (this
      rank's D/w query/key/value features = H/w heads), mlp.c_fc [F/w, D],
      lm_head [V/w, D] (vocabulary-parallel logits)
  row-parallel (input features split): attn.c_proj [D, D/w],
      mlp.c_proj [D, F/w]

The residual stream is split by tokens: rank r holds tokens
[r*M/w, (r+1)*M/w) of the M = batch*seq tokens of the step, so LayerNorms,
residual adds and the embedding touch only local rows. Every block:

  x_l --LN1--> ln1 (own rows of a gathered heap buffer) ==AG-GEMM==> qkv [M, 3D/w] -> RoPE -> attention over
  this rank's heads -> att [M, D/w] ==GEMM-RS==> + c_proj.bias + x_l = xm
  --LN2--> ln2 (heap) ==AG-GEMM(+bias, GELU)==> g [M, F/w] ==GEMM-RS==>
  + mlp.c_proj.bias + xm = x_{l+1}

then LN_f -> AG-GEMM with this rank's vocabulary slice -> vocabulary-
parallel softmax cross-entropy (row statistics exchanged through the heap).
The backward mirrors it (data gradients of row-parallel layers are AG-GEMMs
of the token-split residual gradient, those of column-parallel layers are
GEMM-RS; weight gradients read the gathered full-size operands locally).
The input embedding is replicated rather than vocabulary-split: it
costs 131 MB per GPU at this size and saves a reduce-scatter of [M, D] per
step.

Configuration names follow GPTConfig; the 1.3B preset is 24 layers, d=2048,
16 heads, MLP 8192, vocabulary 32000, sequence 2048 with rotary positions.
Reference parity: scirs2-neural/src/training/tensor_parallel.rs:85-385,
scirs2-neural/src/attention/rope.rs:53-250,
scirs2-neural/src/models/architectures/gpt.rs:19-62.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist

from .. import _ext
from ..ops import kernels as K
from ..utils.flat import FlatParams
from .transformer import FusedTrainerMixin


@dataclass
class DecoderConfig:
    vocab_size: int = 32000
    hidden_size: int = 2048
    num_hidden_layers: int = 24
    num_attention_heads: int = 16
    intermediate_size: int = 8192
    max_position_embeddings: int = 2048
    rope_theta: float = 10000.0
    layer_norm_eps: float = 1e-5
    initializer_range: float = 0.02

    @staticmethod
    def decoder_1_3b() -> "DecoderConfig":
        return DecoderConfig()

    @staticmethod
    def tiny(vocab: int = 1024, seq: int = 256) -> "DecoderConfig":
        return DecoderConfig(vocab, 256, 2, 2, 1024, seq)

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    def num_parameters(self) -> int:
        d, f, L, V = self.hidden_size, self.intermediate_size, self.num_hidden_layers, self.vocab_size
        per_layer = 4 * d * d + 4 * d + 2 * d * f + f + d + 4 * d
        return 2 * V * d + L * per_layer + 2 * d

    def flops_per_token(self, seq: int) -> float:
        d, f, L, V = self.hidden_size, self.intermediate_size, self.num_hidden_layers, self.vocab_size
        mm = L * (2 * d * 3 * d + 2 * d * d + 2 * 2 * d * f) + 2 * d * V
        attn = L * 2 * 2 * seq * d * 0.5
        return 3.0 * (mm + attn)


def rope_tables(seq: int, hd: int, theta: float, device):
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2, dtype=torch.float64) / hd))
    ang = torch.arange(seq, dtype=torch.float64)[:, None] * inv[None, :]
    return ang.cos().float().to(device).contiguous(), ang.sin().float().to(device).contiguous()


REPLICATED = ("ln_1.weight", "ln_1.bias", "ln_2.weight", "ln_2.bias", "attn.c_proj.bias", "mlp.c_proj.bias")


class TPDecoder(FusedTrainerMixin):
    """Usage (one process per GPU, torch.distributed initialised)::

        ctx = TPContext(TPDecoder.heap_bytes(cfg, 32, 2048, world), mode="fused")
        model = TPDecoder(cfg, ctx, batch=32)
        model.configure_adamw(lr=3e-4)
        loss = model.train_step(tokens, targets)   # full [B, S] batch on every rank
    """

    def __init__(self, cfg: DecoderConfig, ctx, batch: int, seq: int | None = None, seed: int = 0):
        self.cfg, self.ctx = cfg, ctx
        self.rank, self.world = ctx.rank, ctx.world
        w = self.world
        D, F, H, V = cfg.hidden_size, cfg.intermediate_size, cfg.num_attention_heads, cfg.vocab_size
        assert D % w == 0 and F % w == 0 and H % w == 0 and V % w == 0, "dims must split evenly"
        assert cfg.head_dim in (64, 128)
        self.S = seq or cfg.max_position_embeddings
        self.B = batch
        self.M = batch * self.S
        assert self.M % (128 * w) == 0, "tokens per rank must be a multiple of 128"
        self.Mr = self.M // w
        self.Dl, self.Fl, self.Hl, self.Vl = D // w, F // w, H // w, V // w
        assert self.Vl % 8 == 0
        self.device = ctx.device
        fp = FlatParams()
        fp.add("wte", (V, D), True)
        L = cfg.num_hidden_layers
        for l in range(L):
            for n in REPLICATED:
                fp.add(f"h{l}.{n}", (D,), False)
        fp.add("ln_f.weight", (D,), False)
        fp.add("ln_f.bias", (D,), False)
        fp.pad_to(256)
        self.rep_end = fp.mark()
        for l in range(L):
            p = f"h{l}."
            fp.add(p + "attn.c_attn.weight", (3 * self.Dl, D), True)
            fp.add(p + "attn.c_attn.bias", (3 * self.Dl,), False)
            fp.add(p + "attn.c_proj.weight", (D, self.Dl), True)
            fp.add(p + "mlp.c_fc.weight", (self.Fl, D), True)
            fp.add(p + "mlp.c_fc.bias", (self.Fl,), False)
            fp.add(p + "mlp.c_proj.weight", (D, self.Fl), True)
        fp.add("lm_head.weight", (self.Vl, D), True)
        fp.allocate(self.device)
        self.fp = fp
        self._init_weights(seed)
        self.cos, self.sin = rope_tables(self.S, cfg.head_dim, cfg.rope_theta, self.device)
        # the GEMM epilogue rotates whole 32-column halves: head_dim 64 or 128
        self.rope_fused = cfg.head_dim in (64, 128) and os.environ.get("SCIRS_ROPE_FUSED", "1") == "1"
        self._alloc()
        self.grad_sync = None
        self.optimizer = None
        self.kernel_launches = 0
        self.rep_comm = None
        if ctx.mode == "fused" and w > 1:
            from ..parallel.nvlink import NVLinkComm

            self.rep_comm = NVLinkComm(area_bytes=self.rep_end * 2 + (1 << 20), group=ctx.group)

    # ------------------------------------------------------------ weights
    def _init_weights(self, seed: int):
        """Full-size weights drawn on every rank from the same seed, then this
        rank's slice is kept (so any world size gives the same model)."""
        g = torch.Generator().manual_seed(seed)
        for name, t in self.full_init(self.cfg, g, self.cfg.initializer_range):
            if name in self.fp.slots:
                self.fp.m(name).copy_(self.shard_of(name, t))
        self.fp.sync_bf16()

    @staticmethod
    def full_init(cfg: DecoderConfig, g, std):
        D, F, V, L = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size, cfg.num_hidden_layers
        yield "wte", torch.randn(V, D, generator=g) * std
        for l in range(L):
            p = f"h{l}."
            yield p + "ln_1.weight", torch.ones(D)
            yield p + "ln_1.bias", torch.zeros(D)
            yield p + "attn.c_attn.weight", torch.randn(3 * D, D, generator=g) * std
            yield p + "attn.c_attn.bias", torch.zeros(3 * D)
            yield p + "attn.c_proj.weight", torch.randn(D, D, generator=g) * std / math.sqrt(2 * L)
            yield p + "attn.c_proj.bias", torch.zeros(D)
            yield p + "ln_2.weight", torch.ones(D)
            yield p + "ln_2.bias", torch.zeros(D)
            yield p + "mlp.c_fc.weight", torch.randn(F, D, generator=g) * std
            yield p + "mlp.c_fc.bias", torch.zeros(F)
            yield p + "mlp.c_proj.weight", torch.randn(D, F, generator=g) * std / math.sqrt(2 * L)
            yield p + "mlp.c_proj.bias", torch.zeros(D)
        yield "ln_f.weight", torch.ones(D)
        yield "ln_f.bias", torch.zeros(D)
        yield "lm_head.weight", torch.randn(V, D, generator=g) * std

    def shard_of(self, name: str, t: torch.Tensor) -> torch.Tensor:
        """This rank's slice of a full-size parameter."""
        r = self.rank
        if name.endswith("attn.c_attn.weight") or name.endswith("attn.c_attn.bias"):
            D = self.cfg.hidden_size
            parts = t.view(3, D, *t.shape[1:])  # q, k, v blocks; heads are contiguous in each
            return parts[:, r * self.Dl : (r + 1) * self.Dl].reshape(3 * self.Dl, *t.shape[1:])
        if name.endswith("attn.c_proj.weight"):
            return t[:, r * self.Dl : (r + 1) * self.Dl]
        if name.endswith("mlp.c_fc.weight") or name.endswith("mlp.c_fc.bias"):
            return t[r * self.Fl : (r + 1) * self.Fl]
        if name.endswith("mlp.c_proj.weight"):
            return t[:, r * self.Fl : (r + 1) * self.Fl]
        if name == "lm_head.weight":
            return t[r * self.Vl : (r + 1) * self.Vl]
        return t

    @staticmethod
    def heap_bytes(cfg: DecoderConfig, batch: int, seq: int, world: int) -> int:
        """Symmetric-heap bytes the model allocates from its TPContext."""
        M = batch * seq
        Mr, D, L = M // world, cfg.hidden_size, cfg.num_hidden_layers
        gathered = (2 * L + 1 + 4) * M * D * 2  # ln1 / ln2 per layer, ln_f, 2 x (dY, dYm)
        act = gathered + world * M * 16 + 2 * world * Mr * D * 2
        return act + 1024 * (2 * L + 16)

    # ------------------------------------------------------------ buffers
    def _alloc(self):
        cfg, ctx = self.cfg, self.ctx
        L, D, M, Mr = cfg.num_hidden_layers, cfg.hidden_size, self.M, self.Mr
        Dl, Fl, Vl, Hl, S, B = self.Dl, self.Fl, self.Vl, self.Hl, self.S, self.B
        bf, f32, dev = torch.bfloat16, torch.float32, self.device
        e = lambda *s, dt=bf: torch.empty(*s, dtype=dt, device=dev)  # noqa: E731
        # full-size gathered buffers (symmetric heap in fused mode); this rank
        # writes its own rows, the gather fills in the peers' rows
        self.gln1 = [ctx.alloc((M, D)) for _ in range(L)]
        self.gln2 = [ctx.alloc((M, D)) for _ in range(L)]
        self.glnf = ctx.alloc((M, D))
        self.gdY = [ctx.alloc((M, D)) for _ in range(2)]   # d loss / d x_{l+1}, slot l % 2
        self.gdYm = [ctx.alloc((M, D)) for _ in range(2)]  # d loss / d xm_l, slot l % 2
        self.ln1 = [ctx.segment(t) for t in self.gln1]
        self.ln2 = [ctx.segment(t) for t in self.gln2]
        self.lnf = ctx.segment(self.glnf)
        self.stats = ctx.alloc((self.world, M, 4), torch.float32)
        ctx.recv_buffers(Mr, D)
        # local
        self.x = [e(Mr, D) for _ in range(L + 1)]
        self.xm = [e(Mr, D) for _ in range(L)]
        self.mu = [[e(Mr, dt=f32) for _ in range(L)] for _ in range(2)]
        self.rs = [[e(Mr, dt=f32) for _ in range(L)] for _ in range(2)]
        self.muf, self.rsf = e(Mr, dt=f32), e(Mr, dt=f32)
        self.qkv = [e(M, 3 * Dl) for _ in range(L)]
        self.att = [e(M, Dl) for _ in range(L)]
        self.lse = [e(B, Hl, S, dt=f32) for _ in range(L)]
        self.h = [e(M, Fl) for _ in range(L)]
        self.g = [e(M, Fl) for _ in range(L)]
        self.logits = e(M, Vl)
        self.losses = e(M, dt=f32)
        self.dx0 = e(Mr, D)
        self.dln = e(Mr, D)
        self.dqkv = e(M, 3 * Dl)
        self.datt = e(M, Dl)
        self.dh = e(M, Fl)
        self.dq_acc = e(M * Dl, dt=f32)
        self.delta = e(B * Hl * S, dt=f32)
        self.ln_part = K.ln_partials(Mr, D, dev)
        if ctx.mode == "nccl":
            # the unfused baseline's full partial products before reduce-scatter
            self.partial = e(M, D)
            self.stats_local = e(M, 4, dt=f32)
        else:
            self.partial = None

    # ------------------------------------------------------------ forward
    def _forward(self, tok_local):
        cfg, fp, ctx = self.cfg, self.fp, self.ctx
        L, eps, S, B, Hl, hd = cfg.num_hidden_layers, cfg.layer_norm_eps, self.S, self.B, self.Hl, cfg.head_dim
        Mr, kx = self.Mr, _ext.kernels()
        ctx.begin_step()
        K.embedding_fwd(tok_local, fp.w("wte"), None, self.x[0], S)
        for l in range(L):
            p = f"h{l}."
            K.layernorm_fwd(self.x[l], fp.w(p + "ln_1.weight"), fp.w(p + "ln_1.bias"), self.ln1[l], self.mu[0][l],
                            self.rs[0][l], eps)
            s = ctx.gather(self.gln1[l])
            if self.rope_fused:
                # rotary embedding of q and k in the QKV GEMM's epilogue
                ctx.ag_gemm(self.gln1[l], s, fp.w(p + "attn.c_attn.weight"), self.qkv[l],
                            bias=fp.w(p + "attn.c_attn.bias"), epi=K.EPI_ROPE,
                            rope=(self.cos, self.sin, S, hd, 2 * Hl * hd))
            else:
                ctx.ag_gemm(self.gln1[l], s, fp.w(p + "attn.c_attn.weight"), self.qkv[l],
                            bias=fp.w(p + "attn.c_attn.bias"))
                kx.rope_apply(self.qkv[l], self.cos, self.sin, S, Hl, hd, False)
            q, k, v = self.qkv[l].view(B, S, 3, Hl, hd).unbind(2)
            K.flash_attn_fwd(q, k, v, self.att[l].view(B, S, Hl, hd), self.lse[l], causal=True)
            recv, s = ctx.gemm_rs(self.att[l], fp.w(p + "attn.c_proj.weight"), Mr, partial=self.partial)
            ctx.reduce(recv, s, self.xm[l], bias=fp.w(p + "attn.c_proj.bias"), resid=self.x[l])
            K.layernorm_fwd(self.xm[l], fp.w(p + "ln_2.weight"), fp.w(p + "ln_2.bias"), self.ln2[l], self.mu[1][l],
                            self.rs[1][l], eps)
            s = ctx.gather(self.gln2[l])
            ctx.ag_gemm(self.gln2[l], s, fp.w(p + "mlp.c_fc.weight"), self.g[l], epi=K.EPI_BIAS_GELU,
                        bias=fp.w(p + "mlp.c_fc.bias"), out2=self.h[l])
            recv, s = ctx.gemm_rs(self.g[l], fp.w(p + "mlp.c_proj.weight"), Mr, partial=self.partial)
            ctx.reduce(recv, s, self.x[l + 1], bias=fp.w(p + "mlp.c_proj.bias"), resid=self.xm[l])
        K.layernorm_fwd(self.x[L], fp.w("ln_f.weight"), fp.w("ln_f.bias"), self.lnf, self.muf, self.rsf, eps)
        s = ctx.gather(self.glnf)
        ctx.ag_gemm(self.glnf, s, fp.w("lm_head.weight"), self.logits)

    def _xent(self, tgt_full):
        ctx, kx = self.ctx, _ext.kernels()
        v0 = self.rank * self.Vl
        if ctx.mode == "fused":
            i = ctx._next()
            kx.tp_xent_stats(self.logits, tgt_full, self.Vl, v0, self.rank, ctx.heap.peer_addrs(self.stats),
                             ctx.sig, ctx.epoch, i)
            kx.tp_xent_finish(self.logits, tgt_full, self.stats, self.losses, self.Vl, v0, self.rank, 1.0 / self.M,
                              ctx.flags, ctx.epoch, i, ctx.timeout_s)
        else:
            kx.tp_xent_stats(self.logits, tgt_full, self.Vl, v0, 0, [self.stats_local.data_ptr()], [], ctx.epoch, 0)
            dist.all_gather_into_tensor(self.stats.view(-1, 4), self.stats_local, group=ctx.group)
            kx.tp_xent_finish(self.logits, tgt_full, self.stats, self.losses, self.Vl, v0, self.rank, 1.0 / self.M,
                              self.stats_local, ctx.epoch, 0, ctx.timeout_s)

    # ------------------------------------------------------------ backward
    def _backward(self, tok_local):
        cfg, fp, ctx = self.cfg, self.fp, self.ctx
        L, S, B, Hl, hd, Mr = cfg.num_hidden_layers, self.S, self.B, self.Hl, cfg.head_dim, self.Mr
        dlog = self.logits  # d loss / d logits after the cross-entropy
        recv, s = ctx.gemm_rs(dlog, fp.w("lm_head.weight"), Mr, b_mn=True, partial=self.partial)
        ctx.wgrad(dlog, self.glnf, fp.g("lm_head.weight"))
        ctx.reduce(recv, s, self.dln)
        dY = lambda l: ctx.segment(self.gdY[l % 2])  # noqa: E731
        dYm = lambda l: ctx.segment(self.gdYm[l % 2])  # noqa: E731
        K.layernorm_bwd(self.dln, self.x[L], fp.w("ln_f.weight"), self.muf, self.rsf, dY(L - 1),
                        fp.g("ln_f.weight"), fp.g("ln_f.bias"), self.ln_part,
                        dsum=fp.g(f"h{L - 1}.mlp.c_proj.bias"))
        for l in reversed(range(L)):
            p = f"h{l}."
            # fc2 (row-parallel): dh = gather(dY) @ W2 * gelu'(h); dW2 = gather(dY)^T g
            gdy = self.gdY[l % 2]
            s = ctx.gather(gdy)
            ctx.ag_gemm(gdy, s, fp.w(p + "mlp.c_proj.weight"), self.dh, b_mn=True, epi=K.EPI_DGELU, aux=self.h[l])
            ctx.wgrad(gdy, self.g[l], fp.g(p + "mlp.c_proj.weight"))
            K.bias_grad(self.dh, fp.g(p + "mlp.c_fc.bias"))
            # fc1 (column-parallel): d ln2 = RS(dh @ W1); dW1 = dh^T gather(ln2)
            recv, s = ctx.gemm_rs(self.dh, fp.w(p + "mlp.c_fc.weight"), Mr, b_mn=True, partial=self.partial)
            ctx.wgrad(self.dh, self.gln2[l], fp.g(p + "mlp.c_fc.weight"))
            ctx.reduce(recv, s, self.dln)
            K.layernorm_bwd(self.dln, self.xm[l], fp.w(p + "ln_2.weight"), self.mu[1][l], self.rs[1][l], dYm(l),
                            fp.g(p + "ln_2.weight"), fp.g(p + "ln_2.bias"), self.ln_part, dresid=dY(l),
                            dsum=fp.g(p + "attn.c_proj.bias"))
            # proj (row-parallel)
            gdym = self.gdYm[l % 2]
            s = ctx.gather(gdym)
            ctx.ag_gemm(gdym, s, fp.w(p + "attn.c_proj.weight"), self.datt, b_mn=True)
            ctx.wgrad(gdym, self.att[l], fp.g(p + "attn.c_proj.weight"))
            # attention over this rank's heads, then the inverse rotation of dq, dk
            q, k, v = self.qkv[l].view(B, S, 3, Hl, hd).unbind(2)
            dq, dk, dv = self.dqkv.view(B, S, 3, Hl, hd).unbind(2)
            K.flash_attn_bwd(self.datt.view(B, S, Hl, hd), q, k, v, self.att[l].view(B, S, Hl, hd), self.lse[l], dq,
                             dk, dv, self.dq_acc, self.delta, causal=True)
            _ext.kernels().rope_apply(self.dqkv, self.cos, self.sin, S, Hl, hd, True)
            # qkv (column-parallel)
            recv, s = ctx.gemm_rs(self.dqkv, fp.w(p + "attn.c_attn.weight"), Mr, b_mn=True, partial=self.partial)
            ctx.wgrad(self.dqkv, self.gln1[l], fp.g(p + "attn.c_attn.weight"))
            K.bias_grad(self.dqkv, fp.g(p + "attn.c_attn.bias"))
            ctx.reduce(recv, s, self.dln)
            dst = dY(l - 1) if l > 0 else self.dx0
            K.layernorm_bwd(self.dln, self.x[l], fp.w(p + "ln_1.weight"), self.mu[0][l], self.rs[0][l], dst,
                            fp.g(p + "ln_1.weight"), fp.g(p + "ln_1.bias"), self.ln_part, dresid=dYm(l),
                            dsum=fp.g(f"h{l - 1}.mlp.c_proj.bias") if l > 0 else None)
        K.embedding_bwd(tok_local, self.dx0, fp.g("wte"), None, S)
        ctx.finish()

    # ------------------------------------------------------------ API
    def forward_backward(self, tokens, targets):
        """tokens/targets: the full [B, S] batch (identical on every rank)."""
        tok = tokens.reshape(-1)
        tgt = targets.reshape(-1)
        tok_local = tok[self.rank * self.Mr : (self.rank + 1) * self.Mr]
        self._forward(tok_local)
        self._xent(tgt)
        self._backward(tok_local)
        return self.losses.mean()

    @torch.no_grad()
    def eval_loss(self, tokens, targets):
        """Forward + loss only (the logits buffer is overwritten by the loss)."""
        tok = tokens.reshape(-1)
        self._forward(tok[self.rank * self.Mr : (self.rank + 1) * self.Mr])
        self._xent(targets.reshape(-1))
        self.ctx.finish()
        return self.losses.mean()

    def configure_adamw(self, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, max_grad_norm=1.0):
        from ..optim.fused import FusedFlatOptimizer

        self.optimizer = FusedFlatOptimizer(self.fp, "adamw", lr=lr, betas=betas, eps=eps,
                                            weight_decay=weight_decay, max_grad_norm=max_grad_norm)
        self._hp0 = torch.zeros(16, dtype=torch.float32, device=self.device)  # no step-counter update
        return self.optimizer

    def _train_step_eager(self, tokens, targets):
        self.zero_grad()
        loss = self.forward_backward(tokens, targets)
        o, fp = self.optimizer, self.fp
        rep = fp.grad[: self.rep_end]
        if self.world > 1:
            # replicated parameters saw only this rank's tokens: sum over ranks
            if self.rep_comm is not None:
                self.rep_comm.allreduce_(rep, 1.0)
            else:
                dist.all_reduce(rep, group=self.ctx.group)
        # global gradient norm: sharded part on every rank, replicated part once
        o._hyper()
        o.part.zero_()
        K.grad_sumsq(fp.grad[self.rep_end :], o.part[:512], o.hp)
        if self.rank == 0:
            K.grad_sumsq(rep, o.part[512:], self._hp0)
        if self.world > 1:
            # also the step's last cross-rank synchronisation: no rank starts
            # the next step (and overwrites heap data) before all finished
            dist.all_reduce(o.part, group=self.ctx.group)
        K.optim_step(o.mode, fp.master, o.state1, o.state2, fp.grad, fp.p16, fp.total, o.hp, part=o.part,
                     norm_out=o.grad_norm, decay_mask=fp.decay_mask, parts_ready=o.part.numel())
        self.kernel_launches += 4
        return loss

    def close(self):
        self.release_cuda_graph()
        if self.rep_comm is not None:
            self.rep_comm.close()
            self.rep_comm = None
