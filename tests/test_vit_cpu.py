"""ViT engine (CPU reference path of every kernel) vs the PyTorch oracle."""
import torch

from scirs_b200.models.torch_vit import TorchViT
from scirs_b200.models.vit import ViTConfig, ViTModel


def _cfg():
    c = ViTConfig.tiny(num_classes=10)
    c.embed_dim, c.num_heads, c.mlp_dim, c.num_layers = 128, 2, 256, 2
    return c


def test_vit_engine_matches_oracle_cpu():
    cfg = _cfg()
    m = ViTModel(cfg, device="cpu", seed=3)
    sd = {k: v.to(torch.bfloat16).float() for k, v in m.state_dict().items()}
    m.load_state_dict(sd)
    ref = TorchViT(cfg)
    ref.load_flat_state(sd)
    g = torch.Generator().manual_seed(0)
    img = torch.randn(3, 3, 32, 32, generator=g)
    lab = torch.randint(0, cfg.num_classes, (3,), generator=g)
    m.zero_grad()
    loss = m.forward_backward(img, lab)
    lref = ref(img, lab)
    lref.backward()
    assert abs(float(loss) - float(lref)) < 2e-2
    for name, gr in ref.flat_grads().items():
        mine = m.fp.g(name)
        if name.startswith("classifier"):
            mine = mine[: cfg.num_classes]
        err = float((mine - gr).norm() / (gr.norm() + 1e-8))
        assert err < 5e-2, (name, err)


def test_vit_config_presets():
    b = ViTConfig.vit_base()
    assert (b.embed_dim, b.num_layers, b.num_heads, b.mlp_dim) == (768, 12, 12, 3072)
    assert b.seq_len == 197 and b.patch_dim == 768
    assert ViTConfig.vit_large().embed_dim == 1024
    assert 85e6 < b.num_parameters() < 88e6
