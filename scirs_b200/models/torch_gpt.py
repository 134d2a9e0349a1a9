"""Plain-PyTorch GPT (nn.Module, cuBLAS GEMMs, SDPA attention, autograd).

Two roles:
  * numerical oracle for :class:`scirs_b200.models.gpt.GPTModel` (same
    parameter names and layout, loadable from its state_dict);
  * the PyTorch + cuBLAS + NCCL baseline arm of the benchmark (wrapped in
    DistributedDataParallel with a bf16 gradient compression hook, autocast
    bf16 compute over fp32 master weights, fused torch AdamW).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .gpt import GPTConfig


class TorchBlock(nn.Module):
    """Pre-LN transformer block (GPT-2 parameter names)."""

    def __init__(self, D: int, H: int, Fd: int, eps: float, causal: bool = True, rope=None):
        super().__init__()
        self.rope = rope  # (cos, sin) tables [S, hd/2] or None
        self.ln_1 = nn.LayerNorm(D, eps=eps)
        self.attn = nn.Module()
        self.attn.c_attn = nn.Linear(D, 3 * D)
        self.attn.c_proj = nn.Linear(D, D)
        self.ln_2 = nn.LayerNorm(D, eps=eps)
        self.mlp = nn.Module()
        self.mlp.c_fc = nn.Linear(D, Fd)
        self.mlp.c_proj = nn.Linear(Fd, D)
        self.H = H
        self.causal = causal

    def forward(self, x):
        B, S, D = x.shape
        h = self.ln_1(x)
        qkv = self.attn.c_attn(h).view(B, S, 3, self.H, D // self.H)
        q, k, v = qkv.unbind(2)
        if self.rope is not None:
            q, k = _rotate(q, *self.rope), _rotate(k, *self.rope)
        a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                           is_causal=self.causal)
        x = x + self.attn.c_proj(a.transpose(1, 2).reshape(B, S, D))
        x = x + self.mlp.c_proj(F.gelu(self.mlp.c_fc(self.ln_2(x)), approximate="tanh"))
        return x


def Block(cfg: GPTConfig) -> TorchBlock:
    return TorchBlock(cfg.hidden_size, cfg.num_attention_heads, cfg.intermediate_size, cfg.layer_norm_eps, True)


class TorchGPT(nn.Module):
    """`pad_vocab=True` stores the tied embedding with cfg.vocab_padded rows
    (a multiple of 128, so the LM-head GEMM has an aligned N) and slices the
    logits back to the real vocabulary before the loss: the same function,
    the usual way PyTorch GPT-2 trainers lay the head out."""

    def __init__(self, cfg: GPTConfig, pad_vocab: bool = False):
        super().__init__()
        self.cfg = cfg
        self.V = cfg.vocab_size
        self.wte = nn.Embedding(cfg.vocab_padded if pad_vocab else cfg.vocab_size, cfg.hidden_size)
        self.wpe = nn.Embedding(cfg.max_position_embeddings, cfg.hidden_size)
        self.h = nn.ModuleList([Block(cfg) for _ in range(cfg.num_hidden_layers)])
        self.ln_f = nn.LayerNorm(cfg.hidden_size, eps=cfg.layer_norm_eps)
        self.apply(self._init)
        with torch.no_grad():
            self.wte.weight[cfg.vocab_size:] = 0.0  # padded vocabulary rows (never looked up, no loss gradient)
        for n, p in self.named_parameters():
            if n.endswith("c_proj.weight"):
                nn.init.normal_(p, 0.0, cfg.initializer_range / math.sqrt(2 * cfg.num_hidden_layers))

    def _init(self, m):
        if isinstance(m, nn.Linear):
            nn.init.normal_(m.weight, 0.0, self.cfg.initializer_range)
            nn.init.zeros_(m.bias)
        elif isinstance(m, nn.Embedding):
            nn.init.normal_(m.weight, 0.0, self.cfg.initializer_range)

    def forward(self, tokens, targets=None):
        B, S = tokens.shape
        x = self.wte(tokens) + self.wpe(torch.arange(S, device=tokens.device))
        for blk in self.h:
            x = blk(x)
        x = self.ln_f(x)
        logits = x @ self.wte.weight.t()
        if logits.shape[-1] != self.V:
            logits = logits[..., : self.V]
        if targets is None:
            return logits
        return F.cross_entropy(logits.reshape(-1, self.V).float(), targets.reshape(-1))

    def load_flat_state(self, sd: dict):
        """Load a GPTModel.state_dict() (names map 1:1; `wte`/`wpe` are the
        embedding weights)."""
        own = dict(self.named_parameters())
        with torch.no_grad():
            for k, v in sd.items():
                name = _to_torch_name(k)
                n = min(own[name].shape[0], v.shape[0]) if own[name].dim() == 2 else own[name].shape[0]
                own[name][:n].copy_(v[:n].reshape(own[name][:n].shape))

    def flat_grads(self) -> dict:
        out = {_from_torch_name(n): p.grad for n, p in self.named_parameters()}
        out["wte"] = out["wte"][: self.V]
        return out


def _to_torch_name(k: str) -> str:
    """Engine parameter name -> nn.Module parameter name."""
    if k in ("wte", "wpe"):
        return k + ".weight"
    if k.startswith("h") and "." in k and k[1 : k.index(".")].isdigit():
        return "h." + k[1:]
    return k


def _from_torch_name(n: str) -> str:
    if n in ("wte.weight", "wpe.weight"):
        return n[:-7]
    if n.startswith("h."):
        return "h" + n[2:]
    return n


def _rotate(x, cos, sin):
    """Half-rotation rotary embedding of x [B, S, H, hd] with tables [S, hd/2]."""
    S, half = x.shape[1], x.shape[-1] // 2
    c = cos[:S].view(1, S, 1, half).to(x.dtype)
    s = sin[:S].view(1, S, 1, half).to(x.dtype)
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


class TorchDecoder(nn.Module):
    """Plain-PyTorch rotary-position decoder with an untied LM head: oracle for
    the tensor-parallel engine (same full-size parameter names) and the
    cuBLAS + NCCL baseline of the 1.3B configuration."""

    def __init__(self, cfg, seq: int | None = None):
        super().__init__()
        from .tp_gpt import rope_tables

        self.cfg = cfg
        S = seq or cfg.max_position_embeddings
        cos, sin = rope_tables(S, cfg.head_dim, cfg.rope_theta, "cpu")
        self.register_buffer("cos", cos, persistent=False)
        self.register_buffer("sin", sin, persistent=False)
        self.wte = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.h = nn.ModuleList([TorchBlock(cfg.hidden_size, cfg.num_attention_heads, cfg.intermediate_size,
                                           cfg.layer_norm_eps, True) for _ in range(cfg.num_hidden_layers)])
        self.ln_f = nn.LayerNorm(cfg.hidden_size, eps=cfg.layer_norm_eps)
        self.lm_head = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)
        with torch.no_grad():
            for n, p in self.named_parameters():
                if p.dim() == 2:
                    p.normal_(0.0, cfg.initializer_range)

    def forward(self, tokens, targets=None):
        x = self.wte(tokens)
        for blk in self.h:
            blk.rope = (self.cos, self.sin)
            x = blk(x)
        logits = self.lm_head(self.ln_f(x))
        if targets is None:
            return logits
        return F.cross_entropy(logits.float().view(-1, logits.shape[-1]), targets.reshape(-1))

    @torch.no_grad()
    def load_full(self, named):
        """Load (name, tensor) pairs named like TPDecoder.full_init."""
        own = dict(self.named_parameters())
        for k, v in named:
            own["wte.weight" if k == "wte" else _to_torch_name(k)].copy_(v)

    def full_grads(self) -> dict:
        return {("wte" if n == "wte.weight" else _from_torch_name(n)): p.grad for n, p in self.named_parameters()}
