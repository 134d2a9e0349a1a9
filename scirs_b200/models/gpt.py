"""GPT-style decoder with a hand-scheduled forward/backward on sm_100a kernels.

This is the framework's flagship training path. Instead of a tape, each
block's forward and backward are written out as a fixed sequence of fused
kernels over preallocated activation buffers:

  forward (per block)                    backward (per block, reverse)
  LN1            layernorm_fwd            fc2  dgrad*gelu' / wgrad / bias grad
  QKV            gemm (+bias)             fc1  dgrad / wgrad / bias grad
  attention      flash_attn_fwd           LN2  layernorm_bwd (+residual grad)
  proj           gemm (+bias +residual)   proj dgrad / wgrad / bias grad
  LN2            layernorm_fwd            attention flash_attn_bwd
  fc1            gemm (+bias, GELU)       QKV  dgrad / wgrad / bias grad
  fc2            gemm (+bias +residual)   LN1  layernorm_bwd (+residual grad)

then the tied LM head (gemm), the fused softmax cross-entropy (forward and
gradient in one pass, in place over the logits), its two backward GEMMs, the
embedding backward and ONE fused AdamW launch over the flat parameter
buffer. Weight gradients are accumulated in fp32 straight into the flat
gradient buffer; as soon as a block's gradients are final its slice is
handed to the gradient synchroniser (data parallel), which overlaps the
NVLink all-reduce with the rest of the backward pass.

Architecture and configuration names follow the reference GPT
(scirs2-neural/src/models/architectures/gpt.rs:19-62 GPTConfig, :627
gpt2_small; pre-LN block ln_1 -> attn -> +res -> ln_2 -> mlp(GELU) -> +res,
final ln_f). Unlike the reference (whose attention is a placeholder
`q + k + v`, gpt.rs:442-444, and whose backward is the identity, gpt.rs:456)
this is the full causal-attention model with a tied LM head and exact
gradients. Dropout is not applied (probabilities must be 0 in this engine).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from ..ops import kernels as K
from ..utils.flat import FlatParams
from .transformer import BLOCK_PARAMS, BlockActs, FusedTrainerMixin, add_block_params, block_backward, block_forward


@dataclass
class GPTConfig:
    vocab_size: int = 50257
    max_position_embeddings: int = 1024
    hidden_size: int = 768
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    intermediate_size: int = 3072
    hidden_act: str = "gelu"
    hidden_dropout_prob: float = 0.0
    attention_probs_dropout_prob: float = 0.0
    layer_norm_eps: float = 1e-5
    initializer_range: float = 0.02
    tie_word_embeddings: bool = True
    pad_vocab_to: int = 128

    @staticmethod
    def gpt2_small() -> "GPTConfig":
        return GPTConfig()

    @staticmethod
    def gpt2_medium() -> "GPTConfig":
        return GPTConfig(hidden_size=1024, num_hidden_layers=24, num_attention_heads=16, intermediate_size=4096)

    @staticmethod
    def gpt2_large() -> "GPTConfig":
        return GPTConfig(hidden_size=1280, num_hidden_layers=36, num_attention_heads=20, intermediate_size=5120)

    @staticmethod
    def tiny(vocab: int = 512, seq: int = 128) -> "GPTConfig":
        return GPTConfig(
            vocab_size=vocab,
            max_position_embeddings=seq,
            hidden_size=256,
            num_hidden_layers=2,
            num_attention_heads=4,
            intermediate_size=1024,
        )

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @property
    def vocab_padded(self) -> int:
        a = self.pad_vocab_to
        return (self.vocab_size + a - 1) // a * a

    def num_parameters(self, padded: bool = False) -> int:
        d, f, L = self.hidden_size, self.intermediate_size, self.num_hidden_layers
        v = self.vocab_padded if padded else self.vocab_size
        per_layer = 4 * d * d + 4 * d + 2 * d * f + f + d + 4 * d
        return v * d + self.max_position_embeddings * d + L * per_layer + 2 * d

    def flops_per_token(self, seq: int) -> float:
        """Training FLOPs per token (forward + backward), incl. causal attention."""
        d, f, L = self.hidden_size, self.intermediate_size, self.num_hidden_layers
        mm = L * (2 * d * 3 * d + 2 * d * d + 2 * 2 * d * f) + 2 * d * self.vocab_size
        attn = L * 2 * 2 * seq * d * 0.5  # QK^T and PV, causal half
        return 3.0 * (mm + attn)


def gpt_param_shapes(cfg: GPTConfig):
    """(name, shape) of every parameter in the canonical order: wte (padded
    vocabulary), wpe, the blocks, ln_f."""
    D, F = cfg.hidden_size, cfg.intermediate_size
    out = [("wte", (cfg.vocab_padded, D)), ("wpe", (cfg.max_position_embeddings, D))]
    for l in range(cfg.num_hidden_layers):
        out += [(f"h{l}." + n, shape(D, F)) for n, shape, _ in BLOCK_PARAMS]
    return out + [("ln_f.weight", (D,)), ("ln_f.bias", (D,))]


def gpt_init_values(cfg: GPTConfig, seed: int):
    """Initial values (CPU fp32), drawn in the canonical order from one
    generator, so a model split over pipeline stages starts from exactly the
    weights of the unsplit model: N(0, 0.02), residual projections scaled by
    1/sqrt(2 L), LayerNorm weights 1, biases 0, padded vocabulary rows 0."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    std = cfg.initializer_range
    for name, shape in gpt_param_shapes(cfg):
        if name.endswith("ln_1.weight") or name.endswith("ln_2.weight") or name == "ln_f.weight":
            t = torch.ones(shape)
        elif name.endswith("bias"):
            t = torch.zeros(shape)
        else:
            sd = std
            if name.endswith("c_proj.weight"):  # GPT-2 residual scaling
                sd = std / math.sqrt(2 * cfg.num_hidden_layers)
            t = torch.randn(shape, generator=g) * sd
            if name == "wte":
                t[cfg.vocab_size :] = 0.0  # padded rows never receive gradient
        yield name, t


class _Acts(BlockActs):
    """Preallocated activations for one micro-batch shape."""

    def __init__(self, cfg: GPTConfig, B: int, S: int, device):
        D, F, L, H = cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers, cfg.num_attention_heads
        super().__init__(L, B, S, D, F, H, device)
        M = B * S
        self.lnf = torch.empty(M, D, dtype=torch.bfloat16, device=device)
        self.muf = torch.empty(M, dtype=torch.float32, device=device)
        self.rsf = torch.empty(M, dtype=torch.float32, device=device)
        self.logits = torch.empty(M, cfg.vocab_padded, dtype=torch.bfloat16, device=device)
        self.losses = torch.empty(M, dtype=torch.float32, device=device)


class GPTModel(FusedTrainerMixin):
    """GPT decoder trained with fused sm_100a kernels (see module docstring).

    Usage::

        model = GPTModel(GPTConfig.gpt2_small(), device="cuda")
        opt = model.configure_adamw(lr=6e-4, weight_decay=0.1)
        loss = model.train_step(tokens, targets)        # tokens/targets [B, S] int64
    """

    def __init__(self, cfg: GPTConfig, device="cuda", seed: int = 0, bucket_align: int = 64):
        assert cfg.hidden_dropout_prob == 0 and cfg.attention_probs_dropout_prob == 0, "dropout must be 0"
        assert cfg.head_dim in (64, 128), "head_dim must be 64 or 128"
        self.cfg = cfg
        self.device = torch.device(device)
        D, F, Vp = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_padded
        fp = FlatParams()
        # Layout: [wte] [wpe] [block 0] ... [block L-1, ln_f]; each is a
        # contiguous gradient bucket (ln_f rides with the last block), padded
        # so buckets split evenly into per-rank shards (ZeRO). wte is a bucket
        # of its own: its LM-head gradient is final at the start of the
        # backward pass and can be reduced while the blocks run.
        fp.add("wte", (Vp, D), decay=True)
        fp.pad_to(bucket_align)
        self.bucket_bounds = [(0, fp.mark())]
        s = fp.mark()
        fp.add("wpe", (cfg.max_position_embeddings, D), decay=True)
        fp.pad_to(bucket_align)
        self.bucket_bounds.append((s, fp.mark()))
        for l in range(cfg.num_hidden_layers):
            s = fp.mark()
            add_block_params(fp, f"h{l}.", D, F)
            if l == cfg.num_hidden_layers - 1:
                fp.add("ln_f.weight", (D,), False)
                fp.add("ln_f.bias", (D,), False)
            fp.pad_to(bucket_align)
            self.bucket_bounds.append((s, fp.mark()))
        # bucket 0 is a [vocab_padded, D] table (rows may be owned by ranks)
        self.vocab_grad_spec = {"rows": Vp, "dim": D, "valid": cfg.vocab_size}
        fp.allocate(self.device)
        self.fp = fp
        self._init_weights(seed)
        self._acts: _Acts | None = None
        self.grad_sync = None  # set by parallel.DataParallel
        self.optimizer = None
        self.kernel_launches = 0

    # ------------------------------------------------------------------ init
    def _init_weights(self, seed: int):
        fp = self.fp
        for name, t in gpt_init_values(self.cfg, seed):
            fp.m(name).copy_(t)
        fp.sync_bf16()

    def parameters_count(self) -> int:
        return self.cfg.num_parameters()

    def state_dict(self):
        sd = self.fp.state_dict()
        sd["wte"] = sd["wte"][: self.cfg.vocab_size].clone()
        return sd

    def load_state_dict(self, sd):
        sd = dict(sd)
        if "wte" in sd and sd["wte"].shape[0] == self.cfg.vocab_size:
            w = torch.zeros(self.cfg.vocab_padded, self.cfg.hidden_size)
            w[: self.cfg.vocab_size] = sd["wte"]
            sd["wte"] = w
        self.fp.load_state_dict(sd)

    def acts(self, B: int, S: int) -> _Acts:
        if self._acts is None or self._acts.B != B or self._acts.S != S:
            self._acts = None
            self._acts = _Acts(self.cfg, B, S, self.device)
        return self._acts

    # --------------------------------------------------------------- forward
    def _forward(self, tokens: torch.Tensor, A: _Acts):
        cfg, fp = self.cfg, self.fp
        S, H, hd, eps = A.S, cfg.num_attention_heads, cfg.head_dim, cfg.layer_norm_eps
        n = 0
        self._params_begin()
        self._wait_params(0)
        self._wait_params(1)
        K.embedding_fwd(tokens, fp.w("wte"), fp.w("wpe")[:S], A.x[0], S)
        n += 1
        for l in range(cfg.num_hidden_layers):
            self._wait_params(l + 2)
            n += block_forward(fp, f"h{l}.", A, l, H, hd, eps, causal=True)
        L = cfg.num_hidden_layers
        K.layernorm_fwd(A.x[L], fp.w("ln_f.weight"), fp.w("ln_f.bias"), A.lnf, A.muf, A.rsf, eps)
        K.gemm(A.lnf, fp.w("wte"), A.logits)
        self._params_end()
        n += 2
        return n

    # -------------------------------------------------------------- backward
    def _backward(self, tokens: torch.Tensor, A: _Acts):
        cfg, fp = self.cfg, self.fp
        S, H, hd, L = A.S, cfg.num_attention_heads, cfg.head_dim, cfg.num_hidden_layers
        n = 0
        dlog = A.logits  # now holds dloss/dlogits
        gs = self.grad_sync
        early = gs is not None and getattr(gs, "early_vocab", False)
        # LM head (tied to wte): dx_f = dlogits @ wte ; dwte += dlogits^T @ lnf
        K.gemm(dlog, fp.w("wte"), A.dln, b_mn=True)
        K.gemm(dlog, A.lnf, fp.g("wte"), a_mn=True, b_mn=True, epi=K.EPI_F32, accumulate=True)
        if early:
            # the LM-head part of the wte gradient is final: reduce it now,
            # overlapped with the whole backward pass
            gs.bucket_ready(0)
        # colsum(d x[L]) is the bias gradient of the last block's fc2
        K.layernorm_bwd(A.dln, A.x[L], fp.w("ln_f.weight"), A.muf, A.rsf, A.dres, fp.g("ln_f.weight"),
                        fp.g("ln_f.bias"), A.ln_part, dsum=fp.g(f"h{L - 1}.mlp.c_proj.bias"))
        n += 4
        for l in reversed(range(L)):
            # d x[l+1] is in A.dres and its column sum (the fc2 bias gradient)
            # was produced by the LayerNorm backward that wrote it
            n += block_backward(fp, f"h{l}.", A, l, H, hd, causal=True,
                                prev_fc2_bias=f"h{l - 1}.mlp.c_proj.bias" if l > 0 else None)
            if gs is not None:
                gs.bucket_ready(l + 2)
        if early:
            # lookup part of the wte gradient: rows go to their shard owners
            gs.route_vocab(tokens, A.dres)
            K.embedding_bwd(tokens, A.dres, None, fp.g("wpe")[:S], S)
            gs.vocab_ready()
        else:
            K.embedding_bwd(tokens, A.dres, fp.g("wte"), fp.g("wpe")[:S], S)
            if gs is not None:
                gs.bucket_ready(0)
        n += 1
        if gs is not None:
            gs.bucket_ready(1)
        return n

    # ----------------------------------------------------------------- API
    def forward_backward(self, tokens: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        """One forward + backward; returns the mean loss (device scalar).
        Gradients are accumulated into the flat gradient buffer."""
        B, S = tokens.shape
        A = self.acts(B, S)
        tok = tokens.reshape(-1)
        with self._phase("forward"):
            n = self._forward(tok, A)
        with self._phase("loss"):
            K.xent_fwd_bwd(A.logits, targets.reshape(-1), A.losses, self.cfg.vocab_size, 1.0 / A.M)
        n += 1
        with self._phase("backward"):
            n += self._backward(tok, A)
        self.kernel_launches += n
        return A.losses.mean()

    @torch.no_grad()
    def logits(self, tokens: torch.Tensor) -> torch.Tensor:
        """Forward only; returns logits [B, S, vocab_size] (a view)."""
        B, S = tokens.shape
        A = self.acts(B, S)
        self._forward(tokens.reshape(-1), A)
        return A.logits.view(B, S, -1)[..., : self.cfg.vocab_size]

    @torch.no_grad()
    def eval_loss(self, tokens: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        B, S = tokens.shape
        A = self.acts(B, S)
        self._forward(tokens.reshape(-1), A)
        K.xent_fwd(A.logits, targets.reshape(-1), A.losses, self.cfg.vocab_size)
        return A.losses.mean()
