"""Plain PyTorch ViT: the fp32 numerical oracle for the fused ViT engine and
the cuBLAS/cuDNN + NCCL baseline. Parameter names match ViTModel's flat
layout (blocks{l}.attn.c_attn.weight ... classifier.bias)."""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .torch_gpt import TorchBlock


class TorchViT(nn.Module):
    def __init__(self, cfg):
        super().__init__()
        self.cfg = cfg
        D, P = cfg.embed_dim, cfg.patch_size[0]
        self.patch_embed = nn.Conv2d(cfg.in_channels, D, P, stride=P)
        self.cls_token = nn.Parameter(torch.zeros(D))
        self.pos_embed = nn.Parameter(torch.zeros(cfg.seq_len, D))
        self.blocks = nn.ModuleList(
            [TorchBlock(D, cfg.num_heads, cfg.mlp_dim, cfg.layer_norm_eps, causal=False) for _ in range(cfg.num_layers)]
        )
        self.norm = nn.LayerNorm(D, eps=cfg.layer_norm_eps)
        self.classifier = nn.Linear(D, cfg.num_classes)

    def forward(self, images, labels=None):
        B = images.shape[0]
        x = self.patch_embed(images).flatten(2).transpose(1, 2)
        x = torch.cat([self.cls_token.view(1, 1, -1).expand(B, 1, -1).to(x.dtype), x], dim=1) + self.pos_embed.to(x.dtype)
        for b in self.blocks:
            x = b(x)
        logits = self.classifier(self.norm(x[:, 0]))
        if labels is None:
            return logits
        return F.cross_entropy(logits.float(), labels)

    # ------------------------------------------------------------ flat names
    def _pairs(self):
        D = self.cfg.embed_dim
        out = {
            "patch_embed.weight": (self.patch_embed.weight, (D, -1)),
            "patch_embed.bias": (self.patch_embed.bias, None),
            "cls_token": (self.cls_token, None),
            "pos_embed": (self.pos_embed, None),
            "norm.weight": (self.norm.weight, None),
            "norm.bias": (self.norm.bias, None),
            "classifier.weight": (self.classifier.weight, None),
            "classifier.bias": (self.classifier.bias, None),
        }
        for l, b in enumerate(self.blocks):
            for name, p in b.named_parameters():
                out[f"blocks{l}.{name}"] = (p, None)
        return out

    @torch.no_grad()
    def load_flat_state(self, sd):
        for name, (p, _) in self._pairs().items():
            p.copy_(sd[name].reshape(p.shape).to(p.dtype))

    def flat_grads(self):
        out = {}
        for name, (p, shp) in self._pairs().items():
            if p.grad is not None:
                out[name] = p.grad.detach().reshape(shp) if shp else p.grad.detach()
        return out
