import pytest
import torch

from scirs_b200.models import multimodal as M
from scirs_b200.models.architectures import CLIPConfig, CLIPTextConfig


@pytest.mark.parametrize("method", list(M.FusionMethod))
def test_feature_fusion_methods(method):
    torch.manual_seed(0)
    dims = [12, 20]
    cfg = M.FeatureFusionConfig(input_dims=dims, hidden_dim=16, fusion_method=method, num_classes=5)
    model = M.FeatureFusion(cfg)
    a, b = torch.randn(3, 12), torch.randn(3, 20)
    out = model(a, b)
    assert out.shape == (3, 5) and torch.isfinite(out).all()
    out.sum().backward()
    ref = M.FeatureFusion(cfg, kernels=False)
    ref.load_state_dict(model.state_dict())
    assert torch.allclose(ref(a, b), model(a, b), atol=1e-5)


def test_fusion_validation_and_modules():
    with pytest.raises(ValueError):
        M.FeatureFusion(M.FeatureFusionConfig(input_dims=[4, 4, 4], fusion_method=M.FusionMethod.FILM))
    film = M.FiLMModule(4, 3)
    f, c = torch.randn(2, 4), torch.randn(2, 3)
    assert torch.allclose(film(f, c), film.gamma_proj(c) * f + film.beta_proj(c))
    att = M.CrossModalAttention(4, 6, 8)
    q, ctx = torch.randn(2, 5, 4), torch.randn(2, 7, 6)
    w = torch.softmax(att.query_proj(q) @ att.key_proj(ctx).transpose(1, 2) / 8 ** 0.5, -1)
    assert torch.allclose(att(q, ctx), w @ att.value_proj(ctx), atol=1e-6)


def test_clip_contrastive_and_zero_shot():
    torch.manual_seed(0)
    cfg = CLIPConfig(text=CLIPTextConfig(vocab_size=100, hidden_size=32, num_layers=2, num_heads=4,
                                         max_position_embeddings=16), projection_dim=24)
    model = M.CLIPModel(cfg, image_size=32, patch_size=8, vision_width=32, vision_layers=2, vision_heads=4)
    imgs, toks = torch.randn(3, 3, 32, 32), torch.randint(0, 99, (3, 10))
    li, lt, loss = model.forward_contrastive(imgs, toks)
    assert li.shape == (3, 3) and torch.allclose(lt, li.t()) and loss.item() > 0
    loss.backward()
    assert model.logit_scale.grad is not None
    probs = model.forward_classification(imgs, torch.randint(0, 99, (4, 10)))
    assert probs.shape == (3, 4) and torch.allclose(probs.sum(-1), torch.ones(3), atol=1e-5)
