"""Model-zoo layers on the framework's kernels (CUDA, bf16) against the same
models built from torch.nn (fp32), with equal weights."""
import pytest
import torch

from scirs_b200.models import architectures as A

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12))


@pytest.mark.parametrize("name", ["resnet18", "mixer"])
def test_zoo_kernels_match_torch(name):
    torch.manual_seed(0)
    if name == "resnet18":
        cfg, x = A.ResNetConfig.resnet18(num_classes=16), torch.randn(4, 3, 64, 64)
    else:
        cfg = A.MLPMixerConfig(image_size=32, patch_size=8, hidden_dim=64, num_layers=2, token_mlp_dim=32,
                               channel_mlp_dim=128, num_classes=16)
        x = torch.randn(4, 3, 32, 32)
    ref = cfg.build(kernels=False).cuda().eval()
    m = cfg.build().cuda().eval()
    m.load_state_dict(ref.state_dict())
    xc = x.cuda()
    with torch.no_grad():
        y_ref = ref(xc)
        y = m.to(torch.bfloat16)(xc.to(torch.bfloat16))
    assert _rel(y, y_ref) < 5e-2
    m.train()
    out = m(xc.to(torch.bfloat16))
    out.float().pow(2).mean().backward()
    grads = [p.grad for p in m.parameters() if p.grad is not None]
    assert grads and all(torch.isfinite(g.float()).all() for g in grads)
