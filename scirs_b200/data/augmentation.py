"""Batched image augmentation on the tensors' own device ([N, C, H, W]),
seeded and reproducible.

Transforms: RandomCrop (with padding), RandomHorizontalFlip,
RandomVerticalFlip, RandomRotation, ColorJitter (brightness / contrast /
saturation), Normalize, RandomErasing, GaussianNoise, Cutout, RandomAffine
(rotation, translation, scale through one sampling grid); batch mixing:
mixup, cutmix. Presets: cifar10_train, imagenet_train, basic_eval.

Reference parity: scirs2-neural/src/training/augmentation.rs:34-800
(AugmentationType, AugmentationPipeline add / with_seed / presets / apply,
apply_mixup, apply_cutmix).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass
class Aug:
    kind: str
    params: dict


def RandomCrop(size, padding=0):
    return Aug("crop", {"size": size, "padding": padding})


def RandomHorizontalFlip(p=0.5):
    return Aug("hflip", {"p": p})


def RandomVerticalFlip(p=0.5):
    return Aug("vflip", {"p": p})


def RandomRotation(degrees):
    return Aug("affine", {"degrees": degrees, "translate": 0.0, "scale": (1.0, 1.0)})


def RandomAffine(degrees=0.0, translate=0.0, scale=(1.0, 1.0)):
    return Aug("affine", {"degrees": degrees, "translate": translate, "scale": scale})


def ColorJitter(brightness=0.0, contrast=0.0, saturation=0.0):
    return Aug("jitter", {"brightness": brightness, "contrast": contrast, "saturation": saturation})


def Normalize(mean, std):
    return Aug("normalize", {"mean": mean, "std": std})


def RandomErasing(p=0.5, scale=(0.02, 0.33), value=0.0):
    return Aug("erase", {"p": p, "scale": scale, "value": value})


def GaussianNoise(std=0.1):
    return Aug("noise", {"std": std})


def Cutout(size):
    return Aug("cutout", {"size": size})


class AugmentationPipeline:
    def __init__(self, seed: int = 0):
        self.transforms: list[Aug] = []
        self.seed = seed
        self._calls = 0

    def add(self, t: Aug) -> "AugmentationPipeline":
        self.transforms.append(t)
        return self

    def with_seed(self, seed: int) -> "AugmentationPipeline":
        self.seed = seed
        return self

    @classmethod
    def cifar10_train(cls):
        return (cls().add(RandomCrop(32, 4)).add(RandomHorizontalFlip())
                .add(Normalize((0.4914, 0.4822, 0.4465), (0.2470, 0.2435, 0.2616))))

    @classmethod
    def imagenet_train(cls):
        return (cls().add(RandomAffine(0.0, 0.0, (0.8, 1.0))).add(RandomHorizontalFlip())
                .add(ColorJitter(0.4, 0.4, 0.4)).add(Normalize((0.485, 0.456, 0.406), (0.229, 0.224, 0.225))))

    @classmethod
    def basic_eval(cls):
        return cls().add(Normalize((0.485, 0.456, 0.406), (0.229, 0.224, 0.225)))

    def apply(self, x: torch.Tensor) -> torch.Tensor:
        g = torch.Generator(device=x.device).manual_seed(self.seed * 1_000_003 + self._calls)
        self._calls += 1
        for t in self.transforms:
            x = _apply(t, x, g)
        return x

    __call__ = apply

    def apply_single(self, img: torch.Tensor) -> torch.Tensor:
        return self.apply(img.unsqueeze(0))[0]


def _u(n, g, device):
    return torch.rand(n, generator=g, device=device)


def _apply(t: Aug, x: torch.Tensor, g) -> torch.Tensor:
    N, C, H, W = x.shape
    dev, p = x.device, t.params
    if t.kind == "hflip":
        m = (_u(N, g, dev) < p["p"]).view(N, 1, 1, 1)
        return torch.where(m, x.flip(-1), x)
    if t.kind == "vflip":
        m = (_u(N, g, dev) < p["p"]).view(N, 1, 1, 1)
        return torch.where(m, x.flip(-2), x)
    if t.kind == "crop":
        s, pad = p["size"], p["padding"]
        xp = F.pad(x, (pad, pad, pad, pad)) if pad else x
        oy = (_u(N, g, dev) * (xp.shape[-2] - s + 1)).long()
        ox = (_u(N, g, dev) * (xp.shape[-1] - s + 1)).long()
        ar = torch.arange(s, device=dev)
        rows = (oy[:, None] + ar[None]).view(N, 1, s, 1).expand(N, C, s, xp.shape[-1])
        xr = xp.gather(2, rows)
        cols = (ox[:, None] + ar[None]).view(N, 1, 1, s).expand(N, C, s, s)
        return xr.gather(3, cols)
    if t.kind == "affine":
        ang = (_u(N, g, dev) * 2 - 1) * math.radians(p["degrees"])
        lo, hi = p["scale"]
        sc = lo + _u(N, g, dev) * (hi - lo)
        tx = (_u(N, g, dev) * 2 - 1) * p["translate"] * 2
        ty = (_u(N, g, dev) * 2 - 1) * p["translate"] * 2
        cos, sin = torch.cos(ang) / sc, torch.sin(ang) / sc
        theta = torch.stack([torch.stack([cos, -sin, tx], -1), torch.stack([sin, cos, ty], -1)], 1)
        grid = F.affine_grid(theta.to(x.dtype), list(x.shape), align_corners=False)
        return F.grid_sample(x, grid, align_corners=False, padding_mode="zeros")
    if t.kind == "jitter":
        out = x
        if p["brightness"]:
            out = out * (1 + (_u(N, g, dev) * 2 - 1) * p["brightness"]).view(N, 1, 1, 1)
        if p["contrast"]:
            m = out.mean((1, 2, 3), keepdim=True)
            out = (out - m) * (1 + (_u(N, g, dev) * 2 - 1) * p["contrast"]).view(N, 1, 1, 1) + m
        if p["saturation"] and C == 3:
            gray = out.mean(1, keepdim=True)
            out = (out - gray) * (1 + (_u(N, g, dev) * 2 - 1) * p["saturation"]).view(N, 1, 1, 1) + gray
        return out
    if t.kind == "normalize":
        m = torch.tensor(p["mean"], device=dev, dtype=x.dtype).view(1, -1, 1, 1)
        s = torch.tensor(p["std"], device=dev, dtype=x.dtype).view(1, -1, 1, 1)
        return (x - m) / s
    if t.kind == "noise":
        return x + torch.randn(x.shape, generator=g, device=dev, dtype=x.dtype) * p["std"]
    if t.kind in ("erase", "cutout"):
        if t.kind == "erase":
            apply = _u(N, g, dev) < p["p"]
            area = p["scale"][0] + _u(N, g, dev) * (p["scale"][1] - p["scale"][0])
            hh = (torch.sqrt(area) * H).long().clamp(1, H)
            ww = (torch.sqrt(area) * W).long().clamp(1, W)
            val = p["value"]
        else:
            apply = torch.ones(N, dtype=torch.bool, device=dev)
            hh = torch.full((N,), min(p["size"], H), device=dev)
            ww = torch.full((N,), min(p["size"], W), device=dev)
            val = 0.0
        y0 = (_u(N, g, dev) * (H - hh + 1)).long()
        x0 = (_u(N, g, dev) * (W - ww + 1)).long()
        yy = torch.arange(H, device=dev).view(1, H, 1)
        xx = torch.arange(W, device=dev).view(1, 1, W)
        box = ((yy >= y0.view(N, 1, 1)) & (yy < (y0 + hh).view(N, 1, 1)) & (xx >= x0.view(N, 1, 1))
               & (xx < (x0 + ww).view(N, 1, 1)) & apply.view(N, 1, 1))
        return torch.where(box.unsqueeze(1), torch.full_like(x, val), x)
    raise ValueError(t.kind)


def apply_mixup(x: torch.Tensor, y: torch.Tensor, num_classes: int, alpha: float = 0.2, seed: int = 0):
    """Returns (mixed images, soft labels [N, num_classes])."""
    g = torch.Generator().manual_seed(seed)
    lam = float(torch.distributions.Beta(alpha, alpha).sample()) if alpha > 0 else 1.0
    perm = torch.randperm(x.shape[0], generator=g).to(x.device)
    yo = F.one_hot(y.long(), num_classes).to(x.dtype)
    return lam * x + (1 - lam) * x[perm], lam * yo + (1 - lam) * yo[perm]


def apply_cutmix(x: torch.Tensor, y: torch.Tensor, num_classes: int, alpha: float = 1.0, seed: int = 0):
    g = torch.Generator().manual_seed(seed)
    N, C, H, W = x.shape
    lam = float(torch.distributions.Beta(alpha, alpha).sample()) if alpha > 0 else 1.0
    perm = torch.randperm(N, generator=g).to(x.device)
    ch, cw = int(H * math.sqrt(1 - lam)), int(W * math.sqrt(1 - lam))
    cy, cx = int(torch.randint(H, (1,), generator=g)), int(torch.randint(W, (1,), generator=g))
    y0, y1 = max(cy - ch // 2, 0), min(cy + ch // 2, H)
    x0, x1 = max(cx - cw // 2, 0), min(cx + cw // 2, W)
    out = x.clone()
    out[:, :, y0:y1, x0:x1] = x[perm][:, :, y0:y1, x0:x1]
    lam_eff = 1 - (y1 - y0) * (x1 - x0) / (H * W)
    yo = F.one_hot(y.long(), num_classes).to(x.dtype)
    return out, lam_eff * yo + (1 - lam_eff) * yo[perm]
