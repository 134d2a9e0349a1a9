"""Multimodal models: feature fusion of several modalities and CLIP.

Feature fusion: every modality is aligned to `hidden_dim` (Linear + LayerNorm,
eps 1e-6), then fused by concatenation, sum, product, cross-modal attention
(modality 0 attends to modality 1), low-rank bilinear fusion (rank
hidden_dim / 4) or FiLM (modality 1 produces gamma and beta for modality 0),
then a GELU MLP (2 hidden_dim -> hidden_dim, optional dropout) and an optional
classifier. CLIP: a causal transformer text encoder (token + position
embeddings, pre-LN blocks, final LayerNorm, projection of the end-of-text
token, i.e. the highest token id of each sequence) and a ViT image encoder
(the [CLS] state, projected), with a learned temperature; `forward_contrastive`
gives image-text logits and the symmetric InfoNCE loss, `forward_classification`
zero-shot class scores against class-prompt embeddings.

Both are built from torch.nn layers and put on the framework's kernels
(`models.architectures.use_framework_kernels`): Linear, LayerNorm and the ViT
patch convolution run on the tcgen05 GEMM / LayerNorm / im2col kernels on CUDA.

Reference parity: scirs2-neural/src/models/architectures/fusion.rs:16-800
(FusionMethod, FeatureFusionConfig, FeatureAlignment, CrossModalAttention,
FiLMModule, BilinearFusion, FeatureFusion), clip.rs:25-460 (CLIPTextConfig,
CLIPConfig, CLIPTextEncoder; the image tower and the full model, which the
reference leaves commented out, follow the published CLIP design).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from enum import Enum

import torch
import torch.nn as nn
import torch.nn.functional as F

from .architectures import CLIPConfig, clip_contrastive_loss, use_framework_kernels
from .torch_gpt import TorchBlock


class FusionMethod(Enum):
    CONCATENATION = "concatenation"
    SUM = "sum"
    PRODUCT = "product"
    ATTENTION = "attention"
    BILINEAR = "bilinear"
    FILM = "film"


@dataclass
class FeatureFusionConfig:
    input_dims: list = field(default_factory=lambda: [512, 512])
    hidden_dim: int = 256
    fusion_method: FusionMethod = FusionMethod.CONCATENATION
    dropout_rate: float = 0.0
    num_classes: int = 10
    include_head: bool = True


class FeatureAlignment(nn.Module):
    def __init__(self, input_dim: int, output_dim: int):
        super().__init__()
        self.projection = nn.Linear(input_dim, output_dim)
        self.norm = nn.LayerNorm(output_dim, eps=1e-6)

    def forward(self, x):
        return self.norm(self.projection(x))


class CrossModalAttention(nn.Module):
    """Queries from one modality attend to another: softmax(q k^T / sqrt(h)) v. 2-D inputs are
    treated as one-token sequences."""

    def __init__(self, query_dim: int, key_dim: int, hidden_dim: int):
        super().__init__()
        self.query_proj = nn.Linear(query_dim, hidden_dim)
        self.key_proj = nn.Linear(key_dim, hidden_dim)
        self.value_proj = nn.Linear(key_dim, hidden_dim)
        self.scale = 1.0 / math.sqrt(hidden_dim)

    def forward(self, query, context):
        squeeze = query.dim() == 2
        q = self.query_proj(query if not squeeze else query[:, None])
        c = context if context.dim() == 3 else context[:, None]
        k, v = self.key_proj(c), self.value_proj(c)
        w = torch.softmax(q @ k.transpose(1, 2) * self.scale, dim=-1)
        out = w @ v
        return out[:, 0] if squeeze else out


class FiLMModule(nn.Module):
    def __init__(self, feature_dim: int, cond_dim: int):
        super().__init__()
        self.gamma_proj = nn.Linear(cond_dim, feature_dim)
        self.beta_proj = nn.Linear(cond_dim, feature_dim)

    def forward(self, features, conditioning):
        return self.gamma_proj(conditioning) * features + self.beta_proj(conditioning)


class BilinearFusion(nn.Module):
    def __init__(self, dim_a: int, dim_b: int, output_dim: int, rank: int):
        super().__init__()
        self.proj_a = nn.Linear(dim_a, rank)
        self.proj_b = nn.Linear(dim_b, rank)
        self.low_rank_proj = nn.Linear(rank, output_dim)

    def forward(self, a, b):
        return self.low_rank_proj(self.proj_a(a) * self.proj_b(b))


class FeatureFusion(nn.Module):
    def __init__(self, config: FeatureFusionConfig, kernels: bool = True):
        super().__init__()
        c = config
        n = len(c.input_dims)
        if c.fusion_method is FusionMethod.ATTENTION and n < 2:
            raise ValueError("Attention fusion requires at least two modalities")
        if c.fusion_method in (FusionMethod.BILINEAR, FusionMethod.FILM) and n != 2:
            raise ValueError(f"{c.fusion_method.value} fusion requires exactly two modalities")
        self.config = c
        self.aligners = nn.ModuleList([FeatureAlignment(d, c.hidden_dim) for d in c.input_dims])
        h = c.hidden_dim
        self.fusion_module = {
            FusionMethod.ATTENTION: lambda: CrossModalAttention(h, h, h),
            FusionMethod.BILINEAR: lambda: BilinearFusion(h, h, h, max(1, h // 4)),
            FusionMethod.FILM: lambda: FiLMModule(h, h),
        }.get(c.fusion_method, lambda: None)()
        fin = h * n if c.fusion_method is FusionMethod.CONCATENATION else h
        layers = [nn.Linear(fin, 2 * h), nn.GELU(approximate="tanh")]
        if c.dropout_rate > 0:
            layers.append(nn.Dropout(c.dropout_rate))
        layers += [nn.Linear(2 * h, h), nn.GELU(approximate="tanh")]
        self.post_fusion = nn.Sequential(*layers)
        self.classifier = nn.Linear(h, c.num_classes) if c.include_head else None
        if kernels:
            use_framework_kernels(self)

    def forward_multi(self, inputs):
        if len(inputs) != len(self.config.input_dims):
            raise ValueError(f"expected {len(self.config.input_dims)} modalities, got {len(inputs)}")
        a = [al(x) for al, x in zip(self.aligners, inputs)]
        m = self.config.fusion_method
        if m is FusionMethod.CONCATENATION:
            fused = torch.cat(a, dim=-1)
        elif m is FusionMethod.SUM:
            fused = torch.stack(a).sum(0)
        elif m is FusionMethod.PRODUCT:
            fused = a[0]
            for t in a[1:]:
                fused = fused * t
        elif m is FusionMethod.ATTENTION:
            fused = self.fusion_module(a[0], a[1])
        else:
            fused = self.fusion_module(a[0], a[1])
        y = self.post_fusion(fused)
        return self.classifier(y) if self.classifier is not None else y

    def forward(self, *inputs):
        return self.forward_multi(list(inputs))


# ---------------------------------------------------------------------------- CLIP
class CLIPTextEncoder(nn.Module):
    def __init__(self, cfg, projection_dim: int):
        super().__init__()
        D = cfg.hidden_size
        self.token_embedding = nn.Embedding(cfg.vocab_size, D)
        self.position_embedding = nn.Parameter(torch.zeros(cfg.max_position_embeddings, D))
        nn.init.normal_(self.position_embedding, std=0.01)
        self.blocks = nn.ModuleList([TorchBlock(D, cfg.num_heads, 4 * D, 1e-5, causal=True)
                                     for _ in range(cfg.num_layers)])
        self.final_ln = nn.LayerNorm(D)
        self.projection = nn.Linear(D, projection_dim, bias=False)

    def forward(self, tokens):
        B, S = tokens.shape
        x = self.token_embedding(tokens) + self.position_embedding[:S]
        for b in self.blocks:
            x = b(x)
        x = self.final_ln(x)
        eot = tokens.argmax(dim=-1)  # the end-of-text token has the largest id
        return self.projection(x[torch.arange(B, device=tokens.device), eot])


class CLIPVisionEncoder(nn.Module):
    def __init__(self, image_size: int, patch_size: int, width: int, layers: int, heads: int, projection_dim: int,
                 in_channels: int = 3):
        super().__init__()
        self.patch_embed = nn.Conv2d(in_channels, width, patch_size, stride=patch_size, bias=False)
        n = (image_size // patch_size) ** 2
        self.cls_token = nn.Parameter(torch.zeros(width))
        self.pos_embed = nn.Parameter(torch.randn(n + 1, width) * 0.01)
        self.pre_ln = nn.LayerNorm(width)
        self.blocks = nn.ModuleList([TorchBlock(width, heads, 4 * width, 1e-5, causal=False) for _ in range(layers)])
        self.post_ln = nn.LayerNorm(width)
        self.projection = nn.Linear(width, projection_dim, bias=False)

    def forward(self, images):
        B = images.shape[0]
        x = self.patch_embed(images).flatten(2).transpose(1, 2)
        x = torch.cat([self.cls_token.view(1, 1, -1).expand(B, 1, -1).to(x.dtype), x], 1) + self.pos_embed.to(x.dtype)
        x = self.pre_ln(x)
        for b in self.blocks:
            x = b(x)
        return self.projection(self.post_ln(x[:, 0]))


class CLIPModel(nn.Module):
    def __init__(self, config: CLIPConfig | None = None, image_size: int = 224, patch_size: int = 16,
                 vision_width: int = 768, vision_layers: int = 12, vision_heads: int = 12, kernels: bool = True):
        super().__init__()
        c = config or CLIPConfig()
        self.text = CLIPTextEncoder(c.text, c.projection_dim)
        self.vision = CLIPVisionEncoder(image_size, patch_size, vision_width, vision_layers, vision_heads,
                                        c.projection_dim)
        self.logit_scale = nn.Parameter(torch.tensor(float(c.logit_scale_init)))
        if kernels:
            use_framework_kernels(self)

    def encode_image(self, images):
        return F.normalize(self.vision(images), dim=-1)

    def encode_text(self, tokens):
        return F.normalize(self.text(tokens), dim=-1)

    def forward_contrastive(self, images, tokens):
        """(logits_per_image [B, B], logits_per_text [B, B], symmetric InfoNCE loss)."""
        ie, te = self.vision(images), self.text(tokens)
        loss = clip_contrastive_loss(ie, te, self.logit_scale)
        li = self.logit_scale.exp() * F.normalize(ie, dim=-1) @ F.normalize(te, dim=-1).t()
        return li, li.t(), loss

    def forward_classification(self, images, class_tokens):
        """Zero-shot class probabilities [B, n_classes] against class-prompt token sequences."""
        logits = self.logit_scale.exp() * self.encode_image(images) @ self.encode_text(class_tokens).t()
        return logits.softmax(dim=-1)
