"""Encoder-decoder transformer with cross-attention on the framework's
kernels.

Every matrix product is the tcgen05 GEMM (bias, and GELU when chosen, in its
epilogue), LayerNorm is the fused LayerNorm kernel, self-attention (causal in
the decoder) and cross-attention (decoder queries over encoder keys / values,
another sequence length) are the flash-attention kernels, the loss is the
fused softmax cross-entropy; autograd chains their backward kernels.

    layer (post-LN, the reference's order; norm_first=True gives pre-LN)
      encoder:  x = LN1(x + SelfAttn(x));  x = LN2(x + FFN(x))
      decoder:  x = LN1(x + CausalSelfAttn(x))
                x = LN2(x + CrossAttn(x, memory))
                x = LN3(x + FFN(x))

Attention projections: self-attention uses one fused QKV GEMM [3d, d];
cross-attention a Q GEMM on the decoder stream and one fused KV GEMM [2d, d]
on the encoder output (computed once per layer). Inputs are token ids
(embedding + sinusoidal positions) or ready [B, S, d_model] features as in
the reference's forward_train(src, tgt).

Reference parity: scirs2-neural/src/transformer/model.rs:19-340
(TransformerConfig{d_model, n_encoder_layers, n_decoder_layers, n_heads,
d_ff, max_seq_len, dropout, pos_encoding_type, epsilon}; forward_train /
forward_inference), encoder.rs:21-700, decoder.rs:22-470 (decoder layer with
self-attention, cross-attention over the encoder output and the ReLU
feed-forward). The reference's layers have no working backward.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn

from ..ops import functional as FN


@dataclass
class TransformerConfig:
    d_model: int = 512
    n_encoder_layers: int = 6
    n_decoder_layers: int = 6
    n_heads: int = 8
    d_ff: int = 2048
    max_seq_len: int = 1024
    dropout: float = 0.0
    pos_encoding_type: str = "sinusoidal"  # sinusoidal | learned
    epsilon: float = 1e-5
    activation: str = "relu"  # relu (the reference's) | gelu (fused into the GEMM epilogue)
    norm_first: bool = False
    src_vocab: int = 0  # > 0: token-id inputs with an embedding table
    tgt_vocab: int = 0

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads


def sinusoidal_table(n: int, d: int) -> torch.Tensor:
    pos = torch.arange(n, dtype=torch.float64)[:, None]
    i = torch.arange(0, d, 2, dtype=torch.float64)[None, :]
    ang = pos / torch.pow(10000.0, i / d)
    t = torch.zeros(n, d, dtype=torch.float64)
    t[:, 0::2] = torch.sin(ang)
    t[:, 1::2] = torch.cos(ang)
    return t.float()


def _w(gen, out_f, in_f):
    return nn.Parameter(torch.randn(out_f, in_f, generator=gen) * (1.0 / math.sqrt(in_f)))


class _Attention(nn.Module):
    """Multi-head attention; `cross=True` projects queries from x and keys /
    values from the memory with a fused KV weight."""

    def __init__(self, cfg: TransformerConfig, gen, cross: bool, causal: bool):
        super().__init__()
        d = cfg.d_model
        self.cfg, self.cross, self.causal = cfg, cross, causal
        if cross:
            self.w_q, self.b_q = _w(gen, d, d), nn.Parameter(torch.zeros(d))
            self.w_kv, self.b_kv = _w(gen, 2 * d, d), nn.Parameter(torch.zeros(2 * d))
        else:
            self.w_qkv, self.b_qkv = _w(gen, 3 * d, d), nn.Parameter(torch.zeros(3 * d))
        self.w_o, self.b_o = _w(gen, d, d), nn.Parameter(torch.zeros(d))

    def forward(self, x, memory=None):
        B, S, d = x.shape
        H, hd = self.cfg.n_heads, self.cfg.head_dim
        if self.cross:
            q = FN.linear(x, self.w_q.t(), self.b_q).view(B, S, H, hd)
            Sk = memory.shape[1]
            kv = FN.linear(memory, self.w_kv.t(), self.b_kv).view(B, Sk, 2, H, hd)
            k, v = kv[:, :, 0], kv[:, :, 1]
        else:
            qkv = FN.linear(x, self.w_qkv.t(), self.b_qkv).view(B, S, 3, H, hd)
            q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
        o = FN.attention(q, k, v, causal=self.causal)
        return FN.linear(o.reshape(B, S, d), self.w_o.t(), self.b_o)


class _FFN(nn.Module):
    def __init__(self, cfg: TransformerConfig, gen):
        super().__init__()
        self.act = cfg.activation
        self.w1, self.b1 = _w(gen, cfg.d_ff, cfg.d_model), nn.Parameter(torch.zeros(cfg.d_ff))
        self.w2, self.b2 = _w(gen, cfg.d_model, cfg.d_ff), nn.Parameter(torch.zeros(cfg.d_model))

    def forward(self, x):
        return FN.linear(FN.linear(x, self.w1.t(), self.b1, activation=self.act), self.w2.t(), self.b2)


class _Norm(nn.Module):
    def __init__(self, d, eps):
        super().__init__()
        self.weight, self.bias, self.eps = nn.Parameter(torch.ones(d)), nn.Parameter(torch.zeros(d)), eps

    def forward(self, x):
        return FN.layer_norm(x, self.weight, self.bias, self.eps)


class TransformerEncoderLayer(nn.Module):
    def __init__(self, cfg: TransformerConfig, gen):
        super().__init__()
        self.cfg = cfg
        self.self_attn = _Attention(cfg, gen, cross=False, causal=False)
        self.ffn = _FFN(cfg, gen)
        self.norm1, self.norm2 = _Norm(cfg.d_model, cfg.epsilon), _Norm(cfg.d_model, cfg.epsilon)

    def forward(self, x):
        if self.cfg.norm_first:
            x = x + self.self_attn(self.norm1(x))
            return x + self.ffn(self.norm2(x))
        x = self.norm1(x + self.self_attn(x))
        return self.norm2(x + self.ffn(x))


class TransformerDecoderLayer(nn.Module):
    def __init__(self, cfg: TransformerConfig, gen):
        super().__init__()
        self.cfg = cfg
        self.self_attn = _Attention(cfg, gen, cross=False, causal=True)
        self.cross_attn = _Attention(cfg, gen, cross=True, causal=False)
        self.ffn = _FFN(cfg, gen)
        self.norm1, self.norm2, self.norm3 = (_Norm(cfg.d_model, cfg.epsilon) for _ in range(3))

    def forward_with_encoder(self, x, memory):
        if self.cfg.norm_first:
            x = x + self.self_attn(self.norm1(x))
            x = x + self.cross_attn(self.norm2(x), memory)
            return x + self.ffn(self.norm3(x))
        x = self.norm1(x + self.self_attn(x))
        x = self.norm2(x + self.cross_attn(x, memory))
        return self.norm3(x + self.ffn(x))

    forward = forward_with_encoder


class Transformer(nn.Module):
    """Encoder-decoder transformer (see the module docstring).

        model = Transformer(TransformerConfig(d_model=512, n_heads=8, src_vocab=V, tgt_vocab=V))
        loss = model.loss(src_ids, tgt_in_ids, tgt_out_ids)
        feats = model.forward_train(src_features, tgt_features)   # [B, S_tgt, d_model]
    """

    def __init__(self, cfg: TransformerConfig, seed: int = 0):
        super().__init__()
        assert cfg.dropout == 0.0, "dropout must be 0 in this engine"
        self.cfg = cfg
        g = torch.Generator().manual_seed(seed)
        self.encoder = nn.ModuleList([TransformerEncoderLayer(cfg, g) for _ in range(cfg.n_encoder_layers)])
        self.decoder = nn.ModuleList([TransformerDecoderLayer(cfg, g) for _ in range(cfg.n_decoder_layers)])
        if cfg.pos_encoding_type == "learned":
            self.pos = nn.Parameter(torch.randn(cfg.max_seq_len, cfg.d_model, generator=g) * 0.02)
        else:
            self.register_buffer("pos", sinusoidal_table(cfg.max_seq_len, cfg.d_model), persistent=False)
        self.src_emb = nn.Parameter(torch.randn(cfg.src_vocab, cfg.d_model, generator=g) * 0.02) \
            if cfg.src_vocab else None
        self.tgt_emb = nn.Parameter(torch.randn(cfg.tgt_vocab, cfg.d_model, generator=g) * 0.02) \
            if cfg.tgt_vocab else None
        if cfg.norm_first:
            self.enc_norm, self.dec_norm = _Norm(cfg.d_model, cfg.epsilon), _Norm(cfg.d_model, cfg.epsilon)

    def _add_pos(self, x):
        return x + self.pos[: x.shape[1]].to(x.dtype)

    def encode(self, src):
        x = self._add_pos(src)
        for layer in self.encoder:
            x = layer(x)
        return self.enc_norm(x) if self.cfg.norm_first else x

    def decode(self, tgt, memory):
        x = self._add_pos(tgt)
        for layer in self.decoder:
            x = layer.forward_with_encoder(x, memory)
        return self.dec_norm(x) if self.cfg.norm_first else x

    def forward_train(self, src, tgt):
        """src [B, S_src, d_model], tgt [B, S_tgt, d_model] -> [B, S_tgt, d_model]."""
        self._memory = self.encode(src)
        return self.decode(tgt, self._memory)

    def forward_inference(self, src, tgt):
        """Reuses the encoder output of the last forward_train on `src`
        (recomputed when src changed shape)."""
        mem = getattr(self, "_memory", None)
        if mem is None or mem.shape[:2] != src.shape[:2]:
            mem = self._memory = self.encode(src)
        return self.decode(tgt, mem)

    def forward(self, src, tgt):
        return self.forward_train(src, tgt)

    # ------------------------------------------------------------ token ids
    def embed(self, ids, table):
        return FN.embedding(ids, table)

    def logits(self, src_ids, tgt_ids):
        out = self.forward_train(self.embed(src_ids, self.src_emb), self.embed(tgt_ids, self.tgt_emb))
        return FN.linear(out, self.tgt_emb.t())  # tied output head

    def loss(self, src_ids, tgt_in, tgt_out):
        lg = self.logits(src_ids, tgt_in)
        return FN.cross_entropy(lg.reshape(-1, lg.shape[-1]), tgt_out.reshape(-1))
