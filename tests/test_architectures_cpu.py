"""Shapes and a training step of each model family in the architecture zoo
(small inputs, CPU)."""
import math

import pytest
import torch

from scirs_b200.models import architectures as A


def _step(model, x, y_fn):
    opt = torch.optim.SGD(model.parameters(), lr=1e-3)
    out = model(*x) if isinstance(x, tuple) else model(x)
    loss = y_fn(out)
    loss.backward()
    opt.step()
    assert torch.isfinite(loss)
    return out


def test_bert_presets_and_forward():
    assert A.BertConfig.bert_large_uncased().hidden_size == 1024
    c = A.BertConfig.custom(100, 32, 2, 4)
    m = c.build()
    ids = torch.randint(0, 100, (2, 9))
    seq, pooled = m(ids)
    assert seq.shape == (2, 9, 32) and pooled.shape == (2, 32)
    _step(m, ids, lambda o: o[0].square().mean())


@pytest.mark.parametrize("name,blocks", [("resnet18", 8), ("resnet50", 16)])
def test_resnet(name, blocks):
    c = getattr(A.ResNetConfig, name)(3, 10)
    m = c.build()
    assert len(m.layers) == blocks
    out = _step(m, torch.randn(2, 3, 32, 32), lambda o: o.square().mean())
    assert out.shape == (2, 10)


def test_resnet_param_count_matches_torchvision_layout():
    # ResNet-18 for 1000 classes has 11,689,512 parameters.
    m = A.ResNetConfig.resnet18().build()
    assert sum(p.numel() for p in m.parameters()) == 11689512


def test_vgg():
    c = A.VGGConfig.vgg11_bn(3, 5)
    assert c.name() == "vgg11_bn" and c.num_conv_layers() == 8
    assert A.VGGConfig.vgg16().num_conv_layers() == 13
    m = c.build()
    assert m(torch.randn(1, 3, 32, 32)).shape == (1, 5)


@pytest.mark.parametrize("ver", [1, 2])
def test_mobilenet(ver):
    c = A.MobileNetConfig(ver, 0.5, 3, 7)
    m = c.build()
    out = _step(m, torch.randn(2, 3, 32, 32), lambda o: o.square().mean())
    assert out.shape == (2, 7)


def test_mlp_mixer():
    c = A.MLPMixerConfig(32, 8, 3, 4, 16, 2, 8, 32)
    assert A.MLPMixerConfig.mixer_b_16().num_patches() == 196
    m = c.build()
    out = _step(m, torch.randn(2, 3, 32, 32), lambda o: o.square().mean())
    assert out.shape == (2, 4)


def test_autoencoder_and_vae():
    ae = A.AutoencoderConfig.tiny(20, 4).with_activation("tanh").build()
    x = torch.randn(3, 20)
    _step(ae, x, lambda o: (o - x).square().mean())
    assert ae.encoder(x).shape == (3, 4)
    vae = A.VAEConfig(20, [16], 4).build()
    recon, mu, lv = vae(x)
    loss = A.VAE.loss(recon, x, mu, lv)
    loss.backward()
    assert recon.shape == x.shape and torch.isfinite(loss)


def test_unet_preserves_spatial_size():
    m = A.UNetConfig.tiny(1, 2).build()
    out = _step(m, torch.randn(1, 1, 16, 16), lambda o: o.square().mean())
    assert out.shape == (1, 2, 16, 16)


def test_efficientnet_convnext():
    e = A.EfficientNetConfig(0.25, 0.5, 32, 0.0, 3, 3).build()
    assert e(torch.randn(2, 3, 32, 32)).shape == (2, 3)
    c = A.ConvNeXtConfig([1, 1, 1, 1], [8, 16, 32, 64], 3).build()
    out = _step(c, torch.randn(2, 3, 32, 32), lambda o: o.square().mean())
    assert out.shape == (2, 3)


def test_mamba_is_causal():
    c = A.MambaConfig.new(16).with_n_layers(2).with_d_state(4).with_vocab_size(50)
    m = c.build().eval()
    ids = torch.randint(0, 50, (1, 10))
    full = m(ids)
    prefix = m(ids[:, :6])
    torch.testing.assert_close(full[:, :6], prefix, rtol=1e-4, atol=1e-5)
    assert full.shape == (1, 10, 50)


def test_seq2seq():
    c = A.Seq2SeqConfig(30, 40, 16, 2, 1, 1, 32, 0.0, 16)
    m = c.build()
    out = _step(m, (torch.randint(0, 30, (2, 7)), torch.randint(0, 40, (2, 5))), lambda o: o.square().mean())
    assert out.shape == (2, 5, 40)


def test_t5_relative_buckets():
    rel = torch.arange(-200, 201)
    b = A.t5_relative_bucket(rel, True, 32, 128)
    assert b.min() >= 0 and b.max() < 32
    # exact buckets near zero, monotone magnitude within each direction
    assert b[200] == 0 and b[201] != b[199]
    uni = A.t5_relative_bucket(rel, False, 32, 128)
    assert (uni[rel > 0] == 0).all()
    assert A.T5Config.t5_base().d_model == 768


def test_swin_clip():
    s = A.SwinConfig.swin_tiny()
    assert s.num_stages() == 4 and s.stage_dim(3) == 768 and s.num_patches() == (56, 56)
    img, txt = torch.randn(4, 8), torch.randn(4, 8)
    loss = A.clip_contrastive_loss(img, img.clone(), torch.tensor(math.log(100.0)))
    loss_rand = A.clip_contrastive_loss(img, txt, torch.tensor(math.log(100.0)))
    assert loss < loss_rand


def test_zoo_layers_run_on_framework_kernels():
    """build() swaps Linear / Conv2d / LayerNorm / pooling for the framework's kernel-backed
    modules (same parameters, same state-dict keys); on the CPU they compute what torch.nn does."""
    from scirs_b200.models import architectures as A

    torch.manual_seed(0)
    for cfg, x in ((A.ResNetConfig.resnet18(num_classes=10), torch.randn(2, 3, 64, 64)),
                   (A.MLPMixerConfig(image_size=32, patch_size=8, hidden_dim=64, num_layers=2,
                                     token_mlp_dim=32, channel_mlp_dim=128, num_classes=10),
                    torch.randn(2, 3, 32, 32))):
        torch.manual_seed(1)
        ref = cfg.build(kernels=False).eval()
        torch.manual_seed(1)
        m = cfg.build().eval()
        kinds = {type(mod).__name__ for mod in m.modules()}
        assert "KernelLinear" in kinds
        assert not any(type(mod) is torch.nn.Linear for mod in m.modules())
        assert list(m.state_dict()) == list(ref.state_dict())
        m.load_state_dict(ref.state_dict())
        with torch.no_grad():
            assert torch.allclose(m(x), ref(x), atol=1e-5, rtol=1e-4)
