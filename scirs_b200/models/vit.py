"""Vision Transformer (ViT) encoder on the fused sm_100a kernels.

Same engine design as the GPT decoder: the pre-LN transformer blocks are the
shared fused schedule (non-causal attention here), all parameters live in
one flat buffer with one gradient bucket per block, and the whole training
step (patch gather -> patch GEMM -> [CLS]+position assembly -> blocks ->
final LayerNorm on the [CLS] token -> classifier GEMM -> fused softmax
cross-entropy -> backward -> fused AdamW) is a fixed kernel sequence that can
be captured as one CUDA graph.

Configuration names follow the reference's ViTConfig
(scirs2-neural/src/models/architectures/vit.rs:21-42; presets vit_base /
vit_large / vit_huge at :46-108). The reference's VisionTransformer itself
is commented out pending a PatchEmbedding layer (vit.rs:296-470); this one
is complete, trains, and is checked against an fp32 PyTorch restatement.
Dropout is not applied (rates must be 0 in this engine).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..ops import kernels as K
from ..utils.flat import FlatParams
from .transformer import BlockActs, FusedTrainerMixin, add_block_params, block_backward, block_forward


@dataclass
class ViTConfig:
    image_size: tuple = (224, 224)
    patch_size: tuple = (16, 16)
    in_channels: int = 3
    num_classes: int = 1000
    embed_dim: int = 768
    num_layers: int = 12
    num_heads: int = 12
    mlp_dim: int = 3072
    dropout_rate: float = 0.0
    attention_dropout_rate: float = 0.0
    layer_norm_eps: float = 1e-6
    pad_classes_to: int = 128

    @staticmethod
    def vit_base(image_size=(224, 224), patch_size=(16, 16), in_channels=3, num_classes=1000) -> "ViTConfig":
        return ViTConfig(image_size, patch_size, in_channels, num_classes, 768, 12, 12, 3072)

    @staticmethod
    def vit_large(image_size=(224, 224), patch_size=(16, 16), in_channels=3, num_classes=1000) -> "ViTConfig":
        return ViTConfig(image_size, patch_size, in_channels, num_classes, 1024, 24, 16, 4096)

    @staticmethod
    def vit_huge(image_size=(224, 224), patch_size=(14, 14), in_channels=3, num_classes=1000) -> "ViTConfig":
        return ViTConfig(image_size, patch_size, in_channels, num_classes, 1280, 32, 16, 5120)

    @staticmethod
    def tiny(num_classes=10) -> "ViTConfig":
        return ViTConfig((32, 32), (8, 8), 3, num_classes, 256, 2, 4, 1024)

    @property
    def num_patches(self) -> int:
        return (self.image_size[0] // self.patch_size[0]) * (self.image_size[1] // self.patch_size[1])

    @property
    def seq_len(self) -> int:
        return self.num_patches + 1

    @property
    def patch_dim(self) -> int:
        return self.in_channels * self.patch_size[0] * self.patch_size[1]

    @property
    def head_dim(self) -> int:
        return self.embed_dim // self.num_heads

    @property
    def classes_padded(self) -> int:
        a = self.pad_classes_to
        return (self.num_classes + a - 1) // a * a

    def num_parameters(self) -> int:
        d, f, L = self.embed_dim, self.mlp_dim, self.num_layers
        per_layer = 4 * d * d + 4 * d + 2 * d * f + f + d + 4 * d
        return (self.patch_dim * d + d + d + self.seq_len * d + L * per_layer + 2 * d
                + d * self.num_classes + self.num_classes)

    def flops_per_image(self) -> float:
        """Training FLOPs per image (forward + backward, patch GEMM without dgrad)."""
        d, f, L, T = self.embed_dim, self.mlp_dim, self.num_layers, self.seq_len
        blk = T * (2 * d * 3 * d + 2 * d * d + 2 * 2 * d * f) + 2 * 2 * T * T * d
        patch = self.num_patches * 2 * self.patch_dim * d
        head = 2 * d * self.num_classes
        return 3.0 * (L * blk + head) + 2.0 * patch


class _Acts(BlockActs):
    def __init__(self, cfg: ViTConfig, B: int, device):
        D, F, L, H, T = cfg.embed_dim, cfg.mlp_dim, cfg.num_layers, cfg.num_heads, cfg.seq_len
        super().__init__(L, B, T, D, F, H, device)
        bf, f32 = torch.bfloat16, torch.float32
        NP = cfg.num_patches
        self.patches = torch.empty(B * NP, cfg.patch_dim, dtype=bf, device=device)
        self.pe = torch.empty(B * NP, D, dtype=bf, device=device)
        self.dpe = torch.empty(B * NP, D, dtype=bf, device=device)
        self.xcls = torch.empty(B, D, dtype=bf, device=device)
        self.lnf = torch.empty(B, D, dtype=bf, device=device)
        self.muf = torch.empty(B, dtype=f32, device=device)
        self.rsf = torch.empty(B, dtype=f32, device=device)
        self.dlnf = torch.empty(B, D, dtype=bf, device=device)
        self.dxcls = torch.empty(B, D, dtype=bf, device=device)
        self.logits = torch.empty(B, cfg.classes_padded, dtype=bf, device=device)
        self.losses = torch.empty(B, dtype=f32, device=device)


class ViTModel(FusedTrainerMixin):
    """ViT classifier trained with fused sm_100a kernels.

    Usage::

        model = ViTModel(ViTConfig.vit_base(), device="cuda")
        model.configure_adamw(lr=1e-3, weight_decay=0.05)
        loss = model.train_step(images, labels)   # images [B,3,224,224] fp32/bf16, labels [B] int64
    """

    def __init__(self, cfg: ViTConfig, device="cuda", seed: int = 0, bucket_align: int = 64):
        assert cfg.dropout_rate == 0 and cfg.attention_dropout_rate == 0, "dropout must be 0"
        assert cfg.head_dim in (64, 128), "head_dim must be 64 or 128"
        assert cfg.patch_size[0] == cfg.patch_size[1], "square patches only"
        self.cfg = cfg
        self.device = torch.device(device)
        D, F, T = cfg.embed_dim, cfg.mlp_dim, cfg.seq_len
        fp = FlatParams()
        fp.add("patch_embed.weight", (D, cfg.patch_dim), True)
        fp.add("patch_embed.bias", (D,), False)
        fp.add("cls_token", (D,), False)
        fp.add("pos_embed", (T, D), False)
        fp.pad_to(bucket_align)
        self.bucket_bounds = [(0, fp.mark())]
        for l in range(cfg.num_layers):
            s = fp.mark()
            add_block_params(fp, f"blocks{l}.", D, F)
            if l == cfg.num_layers - 1:
                fp.add("norm.weight", (D,), False)
                fp.add("norm.bias", (D,), False)
                fp.add("classifier.weight", (cfg.classes_padded, D), True)
                fp.add("classifier.bias", (cfg.classes_padded,), False)
            fp.pad_to(bucket_align)
            self.bucket_bounds.append((s, fp.mark()))
        fp.allocate(self.device)
        self.fp = fp
        self._init_weights(seed)
        self._acts: _Acts | None = None
        self.grad_sync = None
        self.param_sync = None
        self.optimizer = None
        self.kernel_launches = 0

    def _init_weights(self, seed: int):
        cfg, fp = self.cfg, self.fp
        g = torch.Generator(device="cpu").manual_seed(seed)
        for name in fp.order:
            s = fp.slots[name]
            if name.endswith("ln_1.weight") or name.endswith("ln_2.weight") or name == "norm.weight":
                t = torch.ones(s.shape)
            elif name.endswith("bias"):
                t = torch.zeros(s.shape)
            elif name in ("cls_token", "pos_embed"):
                t = torch.randn(s.shape, generator=g) * 0.02
            elif name == "patch_embed.weight":
                t = (torch.rand(s.shape, generator=g) * 2 - 1) / math.sqrt(cfg.patch_dim)
            else:
                t = torch.randn(s.shape, generator=g) * 0.02
                if name == "classifier.weight":
                    t[cfg.num_classes :] = 0.0
            fp.m(name).copy_(t)
        fp.sync_bf16()

    def state_dict(self):
        sd = self.fp.state_dict()
        n = self.cfg.num_classes
        sd["classifier.weight"] = sd["classifier.weight"][:n].clone()
        sd["classifier.bias"] = sd["classifier.bias"][:n].clone()
        return sd

    def load_state_dict(self, sd):
        sd = dict(sd)
        cp, D = self.cfg.classes_padded, self.cfg.embed_dim
        for k in ("classifier.weight", "classifier.bias"):
            if k in sd and sd[k].shape[0] != cp:
                w = torch.zeros((cp, D) if k.endswith("weight") else (cp,))
                w[: sd[k].shape[0]] = sd[k]
                sd[k] = w
        self.fp.load_state_dict(sd)

    def acts(self, B: int) -> _Acts:
        if self._acts is None or self._acts.B != B:
            self._acts = None
            self._acts = _Acts(self.cfg, B, self.device)
        return self._acts

    # --------------------------------------------------------------- forward
    def _forward(self, images: torch.Tensor, A: _Acts) -> int:
        cfg, fp = self.cfg, self.fp
        H, hd, eps, B, L = cfg.num_heads, cfg.head_dim, cfg.layer_norm_eps, A.B, cfg.num_layers
        self._params_begin()
        self._wait_params(0)
        K.patchify(images, A.patches, cfg.patch_size[0])
        K.gemm(A.patches, fp.w("patch_embed.weight"), A.pe, bias=fp.w("patch_embed.bias"))
        K.vit_embed_fwd(A.pe, fp.w("cls_token"), fp.w("pos_embed"), A.x[0], B)
        n = 3
        for l in range(L):
            self._wait_params(l + 1)
            n += block_forward(fp, f"blocks{l}.", A, l, H, hd, eps, causal=False)
        A.xcls.copy_(A.x[L].view(B, cfg.seq_len, -1)[:, 0])
        K.layernorm_fwd(A.xcls, fp.w("norm.weight"), fp.w("norm.bias"), A.lnf, A.muf, A.rsf, eps)
        K.gemm(A.lnf, fp.w("classifier.weight"), A.logits, bias=fp.w("classifier.bias"))
        self._params_end()
        return n + 2

    # -------------------------------------------------------------- backward
    def _backward(self, A: _Acts) -> int:
        cfg, fp = self.cfg, self.fp
        H, hd, B, L, T = cfg.num_heads, cfg.head_dim, A.B, cfg.num_layers, cfg.seq_len
        dlog = A.logits  # holds dloss/dlogits
        K.gemm(dlog, fp.w("classifier.weight"), A.dlnf, b_mn=True)
        K.gemm(dlog, A.lnf, fp.g("classifier.weight"), a_mn=True, b_mn=True, epi=K.EPI_F32, accumulate=True)
        K.bias_grad(dlog, fp.g("classifier.bias"))
        # only the [CLS] rows of the last residual stream receive gradient;
        # their column sum is the last block's fc2 bias gradient
        K.layernorm_bwd(A.dlnf, A.xcls, fp.w("norm.weight"), A.muf, A.rsf, A.dxcls, fp.g("norm.weight"),
                        fp.g("norm.bias"), A.ln_part, dsum=fp.g(f"blocks{L - 1}.mlp.c_proj.bias"))
        A.dres.zero_()
        A.dres.view(B, T, -1)[:, 0].copy_(A.dxcls)
        n = 4
        for l in reversed(range(L)):
            n += block_backward(fp, f"blocks{l}.", A, l, H, hd, causal=False,
                                prev_fc2_bias=f"blocks{l - 1}.mlp.c_proj.bias" if l > 0 else None)
            if self.grad_sync is not None:
                self.grad_sync.bucket_ready(l + 1)
        K.vit_embed_bwd(A.dres, A.dpe, fp.g("pos_embed"), fp.g("cls_token"), B)
        K.gemm(A.dpe, A.patches, fp.g("patch_embed.weight"), a_mn=True, b_mn=True, epi=K.EPI_F32, accumulate=True)
        K.bias_grad(A.dpe, fp.g("patch_embed.bias"))
        n += 3
        if self.grad_sync is not None:
            self.grad_sync.bucket_ready(0)
        return n

    # ----------------------------------------------------------------- API
    def forward_backward(self, images: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        A = self.acts(images.shape[0])
        n = self._forward(images, A)
        K.xent_fwd_bwd(A.logits, labels.reshape(-1), A.losses, self.cfg.num_classes, 1.0 / A.B)
        n += 1 + self._backward(A)
        self.kernel_launches += n
        return A.losses.mean()

    @torch.no_grad()
    def logits(self, images: torch.Tensor) -> torch.Tensor:
        A = self.acts(images.shape[0])
        self._forward(images, A)
        return A.logits[:, : self.cfg.num_classes]

    @torch.no_grad()
    def eval_loss(self, images: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        A = self.acts(images.shape[0])
        self._forward(images, A)
        K.xent_fwd(A.logits, labels.reshape(-1), A.losses, self.cfg.num_classes)
        return A.losses.mean()
