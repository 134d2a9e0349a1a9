"""New functional / model APIs on the framework's kernels (CUDA, bf16) against fp32 references."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12))


def test_functional_attention_on_flash_kernels():
    from scirs_b200 import linalg as L
    from scirs_b200.ops import kernels as K

    torch.manual_seed(0)
    q, k, v = (torch.randn(2, 256, 64, device="cuda") for _ in range(3))
    n0 = K.STATS.launches
    out = L.causal_attention(q.bfloat16(), k.bfloat16(), v.bfloat16())
    assert K.STATS.launches > n0  # the flash kernels ran
    ref = L.causal_attention(q.double().cpu(), k.double().cpu(), v.double().cpu())
    assert _rel(out.cpu(), ref) < 2e-2
    mha = L.multi_head_attention(q.bfloat16(), k.bfloat16(), v.bfloat16(),
                                 *[(torch.randn(64, 64, device="cuda") * 0.1).bfloat16() for _ in range(4)],
                                 None, L.AttentionConfig(num_heads=1, head_dim=64))
    assert mha.shape == (2, 256, 64) and torch.isfinite(mha.float()).all()


def test_fusion_and_static_graph_on_kernels():
    from scirs_b200.models import multimodal as M
    from scirs_b200.nn import tracing as T

    torch.manual_seed(1)
    cfg = M.FeatureFusionConfig(input_dims=[64, 128], hidden_dim=64, fusion_method=M.FusionMethod.FILM,
                                num_classes=16)
    ref = M.FeatureFusion(cfg, kernels=False).cuda()
    m = M.FeatureFusion(cfg).cuda()
    m.load_state_dict(ref.state_dict())
    a, b = torch.randn(32, 64, device="cuda"), torch.randn(32, 128, device="cuda")
    with torch.no_grad():
        assert _rel(m.to(torch.bfloat16)(a.bfloat16(), b.bfloat16()), ref(a, b)) < 5e-2
    seq = torch.nn.Sequential(torch.nn.Linear(64, 128), torch.nn.ReLU(), torch.nn.Linear(128, 32)).double()
    g, wm = T.trace_sequential(seq, [16, 64])
    x = torch.randn(16, 64, dtype=torch.float64)
    out = T.GraphExecutor(g, wm, device="cuda", dtype=torch.bfloat16).run([x])[0]
    with torch.no_grad():
        assert _rel(out.cpu(), seq(x)) < 5e-2
