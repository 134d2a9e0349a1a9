"""Model families of the reference's architecture zoo, as PyTorch modules
with the reference's configuration names and presets.

Each `*Config` mirrors the reference's struct fields and named presets;
`build()` returns an nn.Module. They run on any device; the flagship
training paths (GPT, ViT, tensor-parallel decoder) have dedicated fused
engines elsewhere in the package.

Reference parity (scirs2-neural/src/models/architectures/): bert.rs:21-120,
resnet.rs:39-250, vgg.rs:69-200, mobilenet.rs:56-370, mlp_mixer.rs:49-150,
autoencoder.rs:26-120, unet.rs:24-120, efficientnet.rs:24-230,
convnext.rs:21-120, mamba.rs:23-120, t5.rs:26-220, swin.rs:26-150,
clip.rs:25-120, seq2seq.rs:39-120.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn as nn
import torch.nn.functional as F

from .torch_gpt import TorchBlock


# ------------------------------------------------------------------- BERT
@dataclass
class BertConfig:
    vocab_size: int = 30522
    hidden_size: int = 768
    num_hidden_layers: int = 12
    num_attention_heads: int = 12
    intermediate_size: int = 3072
    hidden_act: str = "gelu"
    hidden_dropout_prob: float = 0.1
    attention_probs_dropout_prob: float = 0.1
    max_position_embeddings: int = 512
    type_vocab_size: int = 2
    initializer_range: float = 0.02
    layer_norm_eps: float = 1e-12

    @staticmethod
    def bert_base_uncased() -> "BertConfig":
        return BertConfig()

    @staticmethod
    def bert_large_uncased() -> "BertConfig":
        return BertConfig(hidden_size=1024, num_hidden_layers=24, num_attention_heads=16, intermediate_size=4096)

    @staticmethod
    def custom(vocab_size, hidden_size, num_hidden_layers, num_attention_heads) -> "BertConfig":
        return BertConfig(vocab_size, hidden_size, num_hidden_layers, num_attention_heads, 4 * hidden_size)

    def build(self):
        return BertModel(self)


class BertModel(nn.Module):
    def __init__(self, c: BertConfig):
        super().__init__()
        D = c.hidden_size
        self.word = nn.Embedding(c.vocab_size, D)
        self.pos = nn.Embedding(c.max_position_embeddings, D)
        self.token_type = nn.Embedding(c.type_vocab_size, D)
        self.ln = nn.LayerNorm(D, eps=c.layer_norm_eps)
        self.drop = nn.Dropout(c.hidden_dropout_prob)
        self.layers = nn.ModuleList([TorchBlock(D, c.num_attention_heads, c.intermediate_size, c.layer_norm_eps,
                                                causal=False) for _ in range(c.num_hidden_layers)])
        self.pool = nn.Linear(D, D)

    def forward(self, ids, token_type=None):
        S = ids.shape[1]
        tt = torch.zeros_like(ids) if token_type is None else token_type
        x = self.drop(self.ln(self.word(ids) + self.pos(torch.arange(S, device=ids.device)) + self.token_type(tt)))
        for blk in self.layers:
            x = blk(x)
        return x, torch.tanh(self.pool(x[:, 0]))


# ------------------------------------------------------------------- ResNet
@dataclass
class ResNetConfig:
    layers: list = field(default_factory=lambda: [2, 2, 2, 2])
    bottleneck: bool = False
    input_channels: int = 3
    num_classes: int = 1000
    dropout_rate: float = 0.0

    @staticmethod
    def resnet18(input_channels=3, num_classes=1000):
        return ResNetConfig([2, 2, 2, 2], False, input_channels, num_classes)

    @staticmethod
    def resnet34(input_channels=3, num_classes=1000):
        return ResNetConfig([3, 4, 6, 3], False, input_channels, num_classes)

    @staticmethod
    def resnet50(input_channels=3, num_classes=1000):
        return ResNetConfig([3, 4, 6, 3], True, input_channels, num_classes)

    @staticmethod
    def resnet101(input_channels=3, num_classes=1000):
        return ResNetConfig([3, 4, 23, 3], True, input_channels, num_classes)

    @staticmethod
    def resnet152(input_channels=3, num_classes=1000):
        return ResNetConfig([3, 8, 36, 3], True, input_channels, num_classes)

    def with_dropout(self, rate):
        self.dropout_rate = rate
        return self

    def build(self):
        return ResNet(self)


class _Basic(nn.Module):
    expansion = 1

    def __init__(self, cin, c, stride):
        super().__init__()
        self.c1 = nn.Conv2d(cin, c, 3, stride, 1, bias=False)
        self.b1 = nn.BatchNorm2d(c)
        self.c2 = nn.Conv2d(c, c, 3, 1, 1, bias=False)
        self.b2 = nn.BatchNorm2d(c)
        self.sc = (nn.Sequential(nn.Conv2d(cin, c, 1, stride, bias=False), nn.BatchNorm2d(c))
                   if stride != 1 or cin != c else nn.Identity())

    def forward(self, x):
        return F.relu(self.b2(self.c2(F.relu(self.b1(self.c1(x))))) + self.sc(x))


class _Bottleneck(nn.Module):
    expansion = 4

    def __init__(self, cin, c, stride):
        super().__init__()
        o = 4 * c
        self.body = nn.Sequential(nn.Conv2d(cin, c, 1, bias=False), nn.BatchNorm2d(c), nn.ReLU(),
                                  nn.Conv2d(c, c, 3, stride, 1, bias=False), nn.BatchNorm2d(c), nn.ReLU(),
                                  nn.Conv2d(c, o, 1, bias=False), nn.BatchNorm2d(o))
        self.sc = (nn.Sequential(nn.Conv2d(cin, o, 1, stride, bias=False), nn.BatchNorm2d(o))
                   if stride != 1 or cin != o else nn.Identity())

    def forward(self, x):
        return F.relu(self.body(x) + self.sc(x))


class ResNet(nn.Module):
    def __init__(self, c: ResNetConfig):
        super().__init__()
        blk = _Bottleneck if c.bottleneck else _Basic
        self.stem = nn.Sequential(nn.Conv2d(c.input_channels, 64, 7, 2, 3, bias=False), nn.BatchNorm2d(64),
                                  nn.ReLU(), nn.MaxPool2d(3, 2, 1))
        layers, cin = [], 64
        for i, n in enumerate(c.layers):
            ch = 64 * 2 ** i
            for j in range(n):
                layers.append(blk(cin, ch, 2 if (j == 0 and i > 0) else 1))
                cin = ch * blk.expansion
        self.layers = nn.Sequential(*layers)
        self.drop = nn.Dropout(c.dropout_rate)
        self.fc = nn.Linear(cin, c.num_classes)

    def forward(self, x):
        return self.fc(self.drop(self.layers(self.stem(x)).mean((2, 3))))


# ------------------------------------------------------------------- VGG
_VGG = {"vgg11": [64, "M", 128, "M", 256, 256, "M", 512, 512, "M", 512, 512, "M"],
        "vgg13": [64, 64, "M", 128, 128, "M", 256, 256, "M", 512, 512, "M", 512, 512, "M"],
        "vgg16": [64, 64, "M", 128, 128, "M", 256, 256, 256, "M", 512, 512, 512, "M", 512, 512, 512, "M"],
        "vgg19": [64, 64, "M", 128, 128, "M", 256, 256, 256, 256, "M", 512, 512, 512, 512, "M", 512, 512, 512, 512,
                  "M"]}


@dataclass
class VGGConfig:
    variant: str = "vgg16"
    batch_norm: bool = False
    input_channels: int = 3
    num_classes: int = 1000
    dropout_rate: float = 0.5

    def name(self) -> str:
        return self.variant + ("_bn" if self.batch_norm else "")

    def num_conv_layers(self) -> int:
        return sum(1 for v in _VGG[self.variant] if v != "M")

    def build(self):
        layers, cin = [], self.input_channels
        for v in _VGG[self.variant]:
            if v == "M":
                layers.append(nn.MaxPool2d(2))
            else:
                layers += [nn.Conv2d(cin, v, 3, padding=1)] + ([nn.BatchNorm2d(v)] if self.batch_norm else []) + [
                    nn.ReLU()]
                cin = v
        return nn.Sequential(*layers, nn.AdaptiveAvgPool2d(7), nn.Flatten(), nn.Linear(512 * 49, 4096), nn.ReLU(),
                             nn.Dropout(self.dropout_rate), nn.Linear(4096, 4096), nn.ReLU(),
                             nn.Dropout(self.dropout_rate), nn.Linear(4096, self.num_classes))


for _n in ("vgg11", "vgg13", "vgg16", "vgg19"):
    setattr(VGGConfig, _n, staticmethod(lambda input_channels=3, num_classes=1000, _n=_n:
                                        VGGConfig(_n, False, input_channels, num_classes)))
    setattr(VGGConfig, _n + "_bn", staticmethod(lambda input_channels=3, num_classes=1000, _n=_n:
                                                VGGConfig(_n, True, input_channels, num_classes)))


# ------------------------------------------------------------------- MobileNet
@dataclass
class MobileNetConfig:
    version: int = 2
    width_multiplier: float = 1.0
    input_channels: int = 3
    num_classes: int = 1000
    dropout_rate: float = 0.2

    @staticmethod
    def mobilenet_v1(input_channels=3, num_classes=1000):
        return MobileNetConfig(1, 1.0, input_channels, num_classes)

    @staticmethod
    def mobilenet_v2(input_channels=3, num_classes=1000):
        return MobileNetConfig(2, 1.0, input_channels, num_classes)

    def scale_channels(self, c: int) -> int:
        return max(8, int(c * self.width_multiplier + 4) // 8 * 8)

    def build(self):
        return MobileNet(self)


class _InvRes(nn.Module):
    def __init__(self, cin, cout, stride, expand):
        super().__init__()
        h = cin * expand
        self.use_res = stride == 1 and cin == cout
        self.body = nn.Sequential(
            *([nn.Conv2d(cin, h, 1, bias=False), nn.BatchNorm2d(h), nn.ReLU6()] if expand != 1 else []),
            nn.Conv2d(h, h, 3, stride, 1, groups=h, bias=False), nn.BatchNorm2d(h), nn.ReLU6(),
            nn.Conv2d(h, cout, 1, bias=False), nn.BatchNorm2d(cout))

    def forward(self, x):
        y = self.body(x)
        return x + y if self.use_res else y


class MobileNet(nn.Module):
    def __init__(self, c: MobileNetConfig):
        super().__init__()
        s = c.scale_channels
        layers = [nn.Conv2d(c.input_channels, s(32), 3, 2, 1, bias=False), nn.BatchNorm2d(s(32)), nn.ReLU6()]
        cin = s(32)
        if c.version == 1:
            for cout, st in [(64, 1), (128, 2), (128, 1), (256, 2), (256, 1), (512, 2)] + [(512, 1)] * 5 + [
                    (1024, 2), (1024, 1)]:
                layers += [nn.Conv2d(cin, cin, 3, st, 1, groups=cin, bias=False), nn.BatchNorm2d(cin), nn.ReLU(),
                           nn.Conv2d(cin, s(cout), 1, bias=False), nn.BatchNorm2d(s(cout)), nn.ReLU()]
                cin = s(cout)
        else:
            for t, ch, n, st in [(1, 16, 1, 1), (6, 24, 2, 2), (6, 32, 3, 2), (6, 64, 4, 2), (6, 96, 3, 1),
                                 (6, 160, 3, 2), (6, 320, 1, 1)]:
                for i in range(n):
                    layers.append(_InvRes(cin, s(ch), st if i == 0 else 1, t))
                    cin = s(ch)
            layers += [nn.Conv2d(cin, 1280, 1, bias=False), nn.BatchNorm2d(1280), nn.ReLU6()]
            cin = 1280
        self.features = nn.Sequential(*layers)
        self.head = nn.Sequential(nn.Dropout(c.dropout_rate), nn.Linear(cin, c.num_classes))

    def forward(self, x):
        return self.head(self.features(x).mean((2, 3)))


# ------------------------------------------------------------------- MLP-Mixer
@dataclass
class MLPMixerConfig:
    image_size: int = 224
    patch_size: int = 16
    in_channels: int = 3
    num_classes: int = 1000
    hidden_dim: int = 512
    num_layers: int = 8
    token_mlp_dim: int = 256
    channel_mlp_dim: int = 2048
    dropout_rate: float = 0.0

    @staticmethod
    def mixer_s_32(num_classes=1000):
        return MLPMixerConfig(224, 32, 3, num_classes, 512, 8, 256, 2048)

    @staticmethod
    def mixer_s_16(num_classes=1000):
        return MLPMixerConfig(224, 16, 3, num_classes, 512, 8, 256, 2048)

    @staticmethod
    def mixer_b_32(num_classes=1000):
        return MLPMixerConfig(224, 32, 3, num_classes, 768, 12, 384, 3072)

    @staticmethod
    def mixer_b_16(num_classes=1000):
        return MLPMixerConfig(224, 16, 3, num_classes, 768, 12, 384, 3072)

    def num_patches(self) -> int:
        return (self.image_size // self.patch_size) ** 2

    def build(self):
        return MLPMixer(self)


class _MixerBlock(nn.Module):
    def __init__(self, n, d, tok, ch):
        super().__init__()
        self.n1, self.n2 = nn.LayerNorm(d), nn.LayerNorm(d)
        self.tok = nn.Sequential(nn.Linear(n, tok), nn.GELU(), nn.Linear(tok, n))
        self.ch = nn.Sequential(nn.Linear(d, ch), nn.GELU(), nn.Linear(ch, d))

    def forward(self, x):
        x = x + self.tok(self.n1(x).transpose(1, 2)).transpose(1, 2)
        return x + self.ch(self.n2(x))


class MLPMixer(nn.Module):
    def __init__(self, c: MLPMixerConfig):
        super().__init__()
        self.stem = nn.Conv2d(c.in_channels, c.hidden_dim, c.patch_size, c.patch_size)
        self.blocks = nn.Sequential(*[_MixerBlock(c.num_patches(), c.hidden_dim, c.token_mlp_dim, c.channel_mlp_dim)
                                      for _ in range(c.num_layers)])
        self.norm = nn.LayerNorm(c.hidden_dim)
        self.head = nn.Linear(c.hidden_dim, c.num_classes)

    def forward(self, x):
        x = self.stem(x).flatten(2).transpose(1, 2)
        return self.head(self.norm(self.blocks(x)).mean(1))


# ------------------------------------------------------------------- Autoencoders
@dataclass
class AutoencoderConfig:
    input_dim: int = 784
    hidden_dims: list = field(default_factory=lambda: [512, 256])
    latent_dim: int = 32
    dropout_rate: float = 0.0
    activation: str = "relu"

    @staticmethod
    def standard(input_dim, latent_dim):
        return AutoencoderConfig(input_dim, [512, 256], latent_dim)

    @staticmethod
    def tiny(input_dim, latent_dim):
        return AutoencoderConfig(input_dim, [64], latent_dim)

    @staticmethod
    def custom(input_dim, hidden_dims, latent_dim):
        return AutoencoderConfig(input_dim, list(hidden_dims), latent_dim)

    def with_dropout(self, rate):
        self.dropout_rate = rate
        return self

    def with_activation(self, act):
        self.activation = act
        return self

    def _act(self):
        return {"relu": nn.ReLU, "tanh": nn.Tanh, "gelu": nn.GELU, "sigmoid": nn.Sigmoid}[self.activation]()

    def _mlp(self, dims):
        out = []
        for a, b in zip(dims[:-1], dims[1:]):
            out += [nn.Linear(a, b), self._act(), nn.Dropout(self.dropout_rate)]
        return out[:-2]

    def build(self):
        enc = nn.Sequential(*self._mlp([self.input_dim] + self.hidden_dims + [self.latent_dim]))
        dec = nn.Sequential(*self._mlp([self.latent_dim] + self.hidden_dims[::-1] + [self.input_dim]))
        return Autoencoder(enc, dec)


class Autoencoder(nn.Module):
    def __init__(self, enc, dec):
        super().__init__()
        self.encoder, self.decoder = enc, dec

    def forward(self, x):
        return self.decoder(self.encoder(x))


@dataclass
class VAEConfig:
    input_dim: int = 784
    hidden_dims: list = field(default_factory=lambda: [512, 256])
    latent_dim: int = 32

    @staticmethod
    def standard(input_dim, latent_dim):
        return VAEConfig(input_dim, [512, 256], latent_dim)

    def build(self):
        return VAE(self)


class VAE(nn.Module):
    def __init__(self, c: VAEConfig):
        super().__init__()
        dims = [c.input_dim] + c.hidden_dims
        self.enc = nn.Sequential(*[m for a, b in zip(dims[:-1], dims[1:]) for m in (nn.Linear(a, b), nn.ReLU())])
        self.mu = nn.Linear(dims[-1], c.latent_dim)
        self.logvar = nn.Linear(dims[-1], c.latent_dim)
        rd = [c.latent_dim] + c.hidden_dims[::-1]
        self.dec = nn.Sequential(*[m for a, b in zip(rd[:-1], rd[1:]) for m in (nn.Linear(a, b), nn.ReLU())],
                                 nn.Linear(rd[-1], c.input_dim))

    def forward(self, x):
        h = self.enc(x)
        mu, lv = self.mu(h), self.logvar(h)
        z = mu + torch.randn_like(mu) * (0.5 * lv).exp()
        return self.dec(z), mu, lv

    @staticmethod
    def loss(recon, x, mu, lv):
        return F.mse_loss(recon, x, reduction="sum") / x.shape[0] - 0.5 * (1 + lv - mu ** 2 - lv.exp()).sum(1).mean()


# ------------------------------------------------------------------- U-Net
@dataclass
class UNetConfig:
    input_channels: int = 3
    output_channels: int = 1
    base_channels: int = 64
    depth: int = 4
    dropout_rate: float = 0.0
    batch_norm: bool = True
    kernel_size: int = 3

    @staticmethod
    def standard(input_channels, output_channels):
        return UNetConfig(input_channels, output_channels, 64, 4)

    @staticmethod
    def tiny(input_channels, output_channels):
        return UNetConfig(input_channels, output_channels, 8, 2)

    def with_dropout(self, r):
        self.dropout_rate = r
        return self

    def with_batch_norm(self, bn):
        self.batch_norm = bn
        return self

    def build(self):
        return UNet(self)


class UNet(nn.Module):
    def __init__(self, c: UNetConfig):
        super().__init__()
        k = c.kernel_size

        def block(a, b):
            bn = (lambda n: nn.BatchNorm2d(n)) if c.batch_norm else (lambda n: nn.Identity())
            return nn.Sequential(nn.Conv2d(a, b, k, padding=k // 2), bn(b), nn.ReLU(),
                                 nn.Conv2d(b, b, k, padding=k // 2), bn(b), nn.ReLU())

        chs = [c.base_channels * 2 ** i for i in range(c.depth + 1)]
        self.down = nn.ModuleList([block(c.input_channels if i == 0 else chs[i - 1], chs[i]) for i in range(c.depth)])
        self.mid = block(chs[c.depth - 1], chs[c.depth])
        self.up = nn.ModuleList([nn.ConvTranspose2d(chs[i + 1], chs[i], 2, 2) for i in reversed(range(c.depth))])
        self.dec = nn.ModuleList([block(2 * chs[i], chs[i]) for i in reversed(range(c.depth))])
        self.out = nn.Conv2d(chs[0], c.output_channels, 1)
        self.drop = nn.Dropout2d(c.dropout_rate)

    def forward(self, x):
        skips = []
        for d in self.down:
            x = d(x)
            skips.append(x)
            x = F.max_pool2d(x, 2)
        x = self.drop(self.mid(x))
        for up, dec, s in zip(self.up, self.dec, reversed(skips)):
            x = dec(torch.cat([up(x), s], 1))
        return self.out(x)


# ------------------------------------------------------------------- EfficientNet / ConvNeXt
@dataclass
class EfficientNetConfig:
    width: float = 1.0
    depth: float = 1.0
    resolution: int = 224
    dropout_rate: float = 0.2
    input_channels: int = 3
    num_classes: int = 1000

    @staticmethod
    def efficientnet_b0(input_channels=3, num_classes=1000):
        return EfficientNetConfig(1.0, 1.0, 224, 0.2, input_channels, num_classes)

    @staticmethod
    def efficientnet_b1(input_channels=3, num_classes=1000):
        return EfficientNetConfig(1.0, 1.1, 240, 0.2, input_channels, num_classes)

    @staticmethod
    def efficientnet_b2(input_channels=3, num_classes=1000):
        return EfficientNetConfig(1.1, 1.2, 260, 0.3, input_channels, num_classes)

    @staticmethod
    def efficientnet_b3(input_channels=3, num_classes=1000):
        return EfficientNetConfig(1.2, 1.4, 300, 0.3, input_channels, num_classes)

    def build(self):
        return EfficientNet(self)


class _SE(nn.Module):
    def __init__(self, c, s):
        super().__init__()
        self.f = nn.Sequential(nn.Conv2d(c, s, 1), nn.SiLU(), nn.Conv2d(s, c, 1), nn.Sigmoid())

    def forward(self, x):
        return x * self.f(x.mean((2, 3), keepdim=True))


class _MBConv(nn.Module):
    def __init__(self, cin, cout, k, stride, expand):
        super().__init__()
        h = cin * expand
        self.res = stride == 1 and cin == cout
        self.body = nn.Sequential(
            *([nn.Conv2d(cin, h, 1, bias=False), nn.BatchNorm2d(h), nn.SiLU()] if expand != 1 else []),
            nn.Conv2d(h, h, k, stride, k // 2, groups=h, bias=False), nn.BatchNorm2d(h), nn.SiLU(),
            _SE(h, max(1, cin // 4)), nn.Conv2d(h, cout, 1, bias=False), nn.BatchNorm2d(cout))

    def forward(self, x):
        y = self.body(x)
        return x + y if self.res else y


class EfficientNet(nn.Module):
    BASE = [(1, 3, 1, 16, 1), (6, 3, 2, 24, 2), (6, 5, 2, 40, 2), (6, 3, 2, 80, 3), (6, 5, 1, 112, 3),
            (6, 5, 2, 192, 4), (6, 3, 1, 320, 1)]

    def __init__(self, c: EfficientNetConfig):
        super().__init__()
        w = lambda n: max(8, int(n * c.width + 4) // 8 * 8)  # noqa: E731
        layers = [nn.Conv2d(c.input_channels, w(32), 3, 2, 1, bias=False), nn.BatchNorm2d(w(32)), nn.SiLU()]
        cin = w(32)
        for e, k, s, ch, n in self.BASE:
            for i in range(int(math.ceil(n * c.depth))):
                layers.append(_MBConv(cin, w(ch), k, s if i == 0 else 1, e))
                cin = w(ch)
        layers += [nn.Conv2d(cin, w(1280), 1, bias=False), nn.BatchNorm2d(w(1280)), nn.SiLU()]
        self.features = nn.Sequential(*layers)
        self.head = nn.Sequential(nn.Dropout(c.dropout_rate), nn.Linear(w(1280), c.num_classes))

    def forward(self, x):
        return self.head(self.features(x).mean((2, 3)))


@dataclass
class ConvNeXtConfig:
    depths: list = field(default_factory=lambda: [3, 3, 9, 3])
    dims: list = field(default_factory=lambda: [96, 192, 384, 768])
    num_classes: int = 1000
    layer_scale_init_value: float = 1e-6

    @staticmethod
    def convnext_tiny(num_classes=1000):
        return ConvNeXtConfig([3, 3, 9, 3], [96, 192, 384, 768], num_classes)

    @staticmethod
    def convnext_small(num_classes=1000):
        return ConvNeXtConfig([3, 3, 27, 3], [96, 192, 384, 768], num_classes)

    @staticmethod
    def convnext_base(num_classes=1000):
        return ConvNeXtConfig([3, 3, 27, 3], [128, 256, 512, 1024], num_classes)

    def build(self):
        return ConvNeXt(self)


class _CNBlock(nn.Module):
    def __init__(self, d, ls):
        super().__init__()
        self.dw = nn.Conv2d(d, d, 7, padding=3, groups=d)
        self.ln = nn.LayerNorm(d, eps=1e-6)
        self.pw = nn.Sequential(nn.Linear(d, 4 * d), nn.GELU(), nn.Linear(4 * d, d))
        self.gamma = nn.Parameter(torch.full((d,), ls))

    def forward(self, x):
        y = self.dw(x).permute(0, 2, 3, 1)
        return x + (self.gamma * self.pw(self.ln(y))).permute(0, 3, 1, 2)


class ConvNeXt(nn.Module):
    def __init__(self, c: ConvNeXtConfig):
        super().__init__()
        layers = [nn.Conv2d(3, c.dims[0], 4, 4)]
        for i, (n, d) in enumerate(zip(c.depths, c.dims)):
            if i > 0:
                layers += [_ChannelsLN(c.dims[i - 1]), nn.Conv2d(c.dims[i - 1], d, 2, 2)]
            layers += [_CNBlock(d, c.layer_scale_init_value) for _ in range(n)]
        self.features = nn.Sequential(*layers)
        self.norm = nn.LayerNorm(c.dims[-1], eps=1e-6)
        self.head = nn.Linear(c.dims[-1], c.num_classes)

    def forward(self, x):
        return self.head(self.norm(self.features(x).mean((2, 3))))


class _ChannelsLN(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.ln = nn.LayerNorm(d, eps=1e-6)

    def forward(self, x):
        return self.ln(x.permute(0, 2, 3, 1)).permute(0, 3, 1, 2)


# ------------------------------------------------------------------- Mamba
@dataclass
class MambaConfig:
    d_model: int = 256
    d_state: int = 16
    d_conv: int = 4
    expand: int = 2
    n_layers: int = 4
    dropout_prob: float = 0.0
    vocab_size: int | None = None
    num_classes: int | None = None

    @staticmethod
    def new(d_model):
        return MambaConfig(d_model)

    def with_d_state(self, n):
        self.d_state = n
        return self

    def with_n_layers(self, n):
        self.n_layers = n
        return self

    def with_expand(self, e):
        self.expand = e
        return self

    def with_vocab_size(self, v):
        self.vocab_size = v
        return self

    def with_num_classes(self, c):
        self.num_classes = c
        return self

    def build(self):
        return Mamba(self)


class _MambaBlock(nn.Module):
    """Selective state-space block: input-dependent (dt, B, C), diagonal A,
    causal depthwise conv, gated output; sequential scan over time."""

    def __init__(self, c: MambaConfig):
        super().__init__()
        di, n = c.expand * c.d_model, c.d_state
        self.norm = nn.LayerNorm(c.d_model)
        self.inp = nn.Linear(c.d_model, 2 * di)
        self.conv = nn.Conv1d(di, di, c.d_conv, padding=c.d_conv - 1, groups=di)
        self.xproj = nn.Linear(di, 1 + 2 * n)
        self.dt = nn.Linear(1, di)
        self.A_log = nn.Parameter(torch.log(torch.arange(1, n + 1, dtype=torch.float32)).repeat(di, 1))
        self.D = nn.Parameter(torch.ones(di))
        self.out = nn.Linear(di, c.d_model)
        self.n = n

    def forward(self, x):
        B, L, _ = x.shape
        xz = self.inp(self.norm(x))
        u, z = xz.chunk(2, -1)
        u = F.silu(self.conv(u.transpose(1, 2))[..., :L].transpose(1, 2))
        p = self.xproj(u)
        dt = F.softplus(self.dt(p[..., :1]))
        Bm, Cm = p[..., 1 : 1 + self.n], p[..., 1 + self.n :]
        A = -torch.exp(self.A_log)
        h = torch.zeros(B, u.shape[-1], self.n, device=x.device, dtype=u.dtype)
        ys = []
        for t in range(L):
            h = torch.exp(dt[:, t, :, None] * A) * h + dt[:, t, :, None] * Bm[:, t, None, :] * u[:, t, :, None]
            ys.append((h * Cm[:, t, None, :]).sum(-1))
        y = torch.stack(ys, 1) + u * self.D
        return x + self.out(y * F.silu(z))


class Mamba(nn.Module):
    def __init__(self, c: MambaConfig):
        super().__init__()
        self.emb = nn.Embedding(c.vocab_size, c.d_model) if c.vocab_size else None
        self.layers = nn.ModuleList([_MambaBlock(c) for _ in range(c.n_layers)])
        self.norm = nn.LayerNorm(c.d_model)
        self.head = nn.Linear(c.d_model, c.num_classes or c.vocab_size or c.d_model)

    def forward(self, x):
        if self.emb is not None:
            x = self.emb(x)
        for blk in self.layers:
            x = blk(x)
        return self.head(self.norm(x))


# ------------------------------------------------------------------- Seq2Seq / T5
@dataclass
class Seq2SeqConfig:
    src_vocab_size: int = 32000
    tgt_vocab_size: int = 32000
    d_model: int = 512
    num_heads: int = 8
    num_encoder_layers: int = 6
    num_decoder_layers: int = 6
    d_ff: int = 2048
    dropout: float = 0.1
    max_len: int = 512

    def build(self):
        return Seq2Seq(self)


class Seq2Seq(nn.Module):
    def __init__(self, c: Seq2SeqConfig):
        super().__init__()
        self.src = nn.Embedding(c.src_vocab_size, c.d_model)
        self.tgt = nn.Embedding(c.tgt_vocab_size, c.d_model)
        self.pos = nn.Embedding(c.max_len, c.d_model)
        self.tf = nn.Transformer(c.d_model, c.num_heads, c.num_encoder_layers, c.num_decoder_layers, c.d_ff,
                                 c.dropout, batch_first=True, norm_first=True)
        self.out = nn.Linear(c.d_model, c.tgt_vocab_size)

    def forward(self, src, tgt):
        ps = self.pos(torch.arange(src.shape[1], device=src.device))
        pt = self.pos(torch.arange(tgt.shape[1], device=tgt.device))
        mask = nn.Transformer.generate_square_subsequent_mask(tgt.shape[1], device=tgt.device)
        return self.out(self.tf(self.src(src) + ps, self.tgt(tgt) + pt, tgt_mask=mask, tgt_is_causal=True))


@dataclass
class T5Config:
    vocab_size: int = 32128
    d_model: int = 512
    d_kv: int = 64
    d_ff: int = 2048
    num_layers: int = 6
    num_heads: int = 8
    relative_attention_num_buckets: int = 32
    relative_attention_max_distance: int = 128
    dropout_rate: float = 0.1

    @staticmethod
    def t5_small():
        return T5Config()

    @staticmethod
    def t5_base():
        return T5Config(d_model=768, d_ff=3072, num_layers=12, num_heads=12)

    @staticmethod
    def t5_large():
        return T5Config(d_model=1024, d_ff=4096, num_layers=24, num_heads=16)


def t5_relative_bucket(rel: torch.Tensor, bidirectional: bool, num_buckets: int, max_distance: int) -> torch.Tensor:
    """T5 relative-position bucketing: exact buckets for small offsets,
    logarithmically wider ones up to max_distance."""
    ret = torch.zeros_like(rel)
    n = -rel
    if bidirectional:
        num_buckets //= 2
        ret = ret + (n < 0).long() * num_buckets
        n = n.abs()
    else:
        n = n.clamp(min=0)
    max_exact = num_buckets // 2
    large = max_exact + (torch.log(n.float().clamp(min=1) / max_exact) / math.log(max_distance / max_exact)
                         * (num_buckets - max_exact)).long()
    large = large.clamp(max=num_buckets - 1)
    return ret + torch.where(n < max_exact, n, large)


# ------------------------------------------------------------------- Swin / CLIP
@dataclass
class SwinConfig:
    img_size: tuple = (224, 224)
    patch_size: int = 4
    embed_dim: int = 96
    depths: list = field(default_factory=lambda: [2, 2, 6, 2])
    num_heads: list = field(default_factory=lambda: [3, 6, 12, 24])
    window_size: int = 7
    num_classes: int = 1000

    @staticmethod
    def swin_tiny(img_size=(224, 224), num_classes=1000):
        return SwinConfig(img_size, 4, 96, [2, 2, 6, 2], [3, 6, 12, 24], 7, num_classes)

    @staticmethod
    def swin_small(img_size=(224, 224), num_classes=1000):
        return SwinConfig(img_size, 4, 96, [2, 2, 18, 2], [3, 6, 12, 24], 7, num_classes)

    @staticmethod
    def swin_base(img_size=(224, 224), num_classes=1000):
        return SwinConfig(img_size, 4, 128, [2, 2, 18, 2], [4, 8, 16, 32], 7, num_classes)

    def num_stages(self) -> int:
        return len(self.depths)

    def stage_dim(self, stage: int) -> int:
        return self.embed_dim * 2 ** stage

    def num_patches(self):
        return (self.img_size[0] // self.patch_size, self.img_size[1] // self.patch_size)


@dataclass
class CLIPTextConfig:
    vocab_size: int = 49408
    hidden_size: int = 512
    num_layers: int = 12
    num_heads: int = 8
    max_position_embeddings: int = 77


@dataclass
class CLIPConfig:
    text: CLIPTextConfig = field(default_factory=CLIPTextConfig)
    projection_dim: int = 512
    logit_scale_init: float = math.log(1 / 0.07)


def clip_contrastive_loss(image_emb: torch.Tensor, text_emb: torch.Tensor, logit_scale: torch.Tensor) -> torch.Tensor:
    """Symmetric InfoNCE over the batch."""
    i = F.normalize(image_emb, dim=-1)
    t = F.normalize(text_emb, dim=-1)
    logits = logit_scale.exp() * i @ t.t()
    y = torch.arange(i.shape[0], device=i.device)
    return 0.5 * (F.cross_entropy(logits, y) + F.cross_entropy(logits.t(), y))


# ---------------------------------------------------------------------------- framework kernels
# The zoo's layers are declared with torch.nn; `use_framework_kernels` swaps the
# ones the framework has kernels for (Linear, Conv2d, LayerNorm, max / average
# pooling) for modules that call scirs_b200.ops.functional, so on CUDA the
# model runs on the tcgen05 GEMM, the im2col convolution, the LayerNorm and the
# pooling kernels. The new modules hold the same Parameter objects under the same
# names, so state dicts are unchanged. Grouped or padded-mode convolutions,
# ceil-mode / dilated pooling and non-last-dim LayerNorms stay on PyTorch.
class KernelLinear(nn.Module):
    def __init__(self, lin: nn.Linear):
        super().__init__()
        self.in_features, self.out_features = lin.in_features, lin.out_features
        self.weight, self.bias = lin.weight, lin.bias

    def forward(self, x):
        from ..ops import functional as OF

        return OF.linear(x, self.weight.t(), self.bias)


class KernelConv2d(nn.Module):
    def __init__(self, conv: nn.Conv2d):
        super().__init__()
        self.in_channels, self.out_channels, self.kernel_size = conv.in_channels, conv.out_channels, conv.kernel_size
        self.stride, self.padding, self.dilation = conv.stride, conv.padding, conv.dilation
        self.weight, self.bias = conv.weight, conv.bias

    def forward(self, x):
        from ..ops import functional as OF

        return OF.conv2d(x, self.weight, self.bias, self.stride, self.padding, self.dilation)


class KernelLayerNorm(nn.Module):
    def __init__(self, ln: nn.LayerNorm):
        super().__init__()
        self.normalized_shape, self.eps = ln.normalized_shape, ln.eps
        self.weight, self.bias = ln.weight, ln.bias

    def forward(self, x):
        from ..ops import functional as OF

        return OF.layer_norm(x, self.weight, self.bias, self.eps)


class KernelPool2d(nn.Module):
    def __init__(self, pool, is_max: bool):
        super().__init__()
        self.kernel_size, self.stride, self.padding = pool.kernel_size, pool.stride, pool.padding
        self.is_max = is_max
        self.count_include_pad = getattr(pool, "count_include_pad", True)

    def forward(self, x):
        from ..ops import functional as OF

        if self.is_max:
            return OF.max_pool2d(x, self.kernel_size, self.stride, self.padding)
        return OF.avg_pool2d(x, self.kernel_size, self.stride, self.padding, self.count_include_pad)


def _kernel_module(m: nn.Module):
    if type(m) is nn.Linear:
        return KernelLinear(m)
    if type(m) is nn.Conv2d and m.groups == 1 and m.padding_mode == "zeros" and not isinstance(m.padding, str):
        return KernelConv2d(m)
    if (type(m) is nn.LayerNorm and len(m.normalized_shape) == 1 and m.elementwise_affine
            and m.weight is not None and m.bias is not None):
        return KernelLayerNorm(m)
    if type(m) is nn.MaxPool2d and not m.ceil_mode and m.dilation in (1, (1, 1)) and not m.return_indices:
        return KernelPool2d(m, True)
    if type(m) is nn.AvgPool2d and not m.ceil_mode and m.divisor_override is None:
        return KernelPool2d(m, False)
    return None


def use_framework_kernels(model: nn.Module) -> nn.Module:
    """Replace, in place, every layer of `model` that has a framework kernel
    (see above) and return the model."""
    for name, child in list(model.named_children()):
        rep = _kernel_module(child)
        if rep is not None:
            setattr(model, name, rep)
        else:
            use_framework_kernels(child)
    return model


def _with_kernels(cls):
    raw = cls.build

    def build(self, kernels: bool = True):
        """Build the model; with `kernels` (default) its Linear / Conv2d / LayerNorm /
        pooling layers run on the framework's kernels (use_framework_kernels)."""
        m = raw(self)
        return use_framework_kernels(m) if kernels else m

    cls.build = build
    return cls


for _n, _c in list(globals().items()):
    if isinstance(_c, type) and _n.endswith("Config") and callable(getattr(_c, "build", None)):
        _with_kernels(_c)
