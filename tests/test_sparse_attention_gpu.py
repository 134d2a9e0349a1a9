"""Sparse, windowed and cross attention on the tcgen05 kernels (block lists
+ element predicate, separate key length) against the fp32 dense-mask
reference: outputs, log-sum-exp and all three input gradients."""
import pytest
import torch

from scirs_b200.ops import functional as FN
from scirs_b200.ops import kernels as K
from scirs_b200.ops import sparse_attention as SA

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


def _run(pattern, B, H, Sq, Sk, hd, plan=True, causal=False):
    g = torch.Generator().manual_seed(Sq + Sk + hd)
    q = torch.randn(B, Sq, H, hd, generator=g).cuda().bfloat16().requires_grad_(True)
    k = torch.randn(B, Sk, H, hd, generator=g).cuda().bfloat16().requires_grad_(True)
    v = torch.randn(B, Sk, H, hd, generator=g).cuda().bfloat16().requires_grad_(True)
    scale = hd ** -0.5
    pl = pattern.plan(Sq, Sk, hd, q.device) if plan else None
    o = FN.attention(q, k, v, causal, scale, plan=pl)
    qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    if plan:
        ref, lse_ref = SA.reference_attention(qf, kf, vf, pattern, scale)
    else:
        ref, lse_ref = K.attention_reference(qf, kf, vf, causal, scale)
    assert _rel(o, ref) < 1e-2, _rel(o, ref)
    # forward log-sum-exp straight from the kernel
    lse = torch.empty(B, H, Sq, device="cuda")
    K.flash_attn_fwd(q.detach(), k.detach(), v.detach(), torch.empty_like(q), lse, causal, scale, plan=pl)
    assert float((lse - lse_ref).abs().max()) < 2e-2
    do = torch.randn(o.shape, generator=g).cuda().bfloat16()
    gq, gk, gv = torch.autograd.grad(o, (q, k, v), do)
    rq, rk, rv = torch.autograd.grad(ref, (qf, kf, vf), do.float())
    for n, a, b in (("dq", gq, rq), ("dk", gk, rk), ("dv", gv, rv)):
        assert _rel(a, b) < 2e-2, (n, _rel(a, b))
    torch.cuda.synchronize()
    from scirs_b200 import _ext

    _ext.check_status(0)
    return pl


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("name,pattern", [
    ("window_global", SA.sliding_window(150, num_global=5)),
    ("causal_window", SA.sliding_window(300, causal=True)),
    ("asym_window", SA.AttentionPattern(window_left=64, window_right=260)),
    ("block_strided", SA.block_sparse(SA.strided_bitmap(8, 8, local=1, stride=3), key="bs8")),
    ("bigbird", SA.AttentionPattern(window_left=100, num_global=2,
                                     bitmap=SA.strided_bitmap(8, 8, 1, 5), bitmap_key="bb8")),
])
def test_sparse_attention_matches_reference(name, pattern, hd):
    pl = _run(pattern, 2, 3, 1000, 1000, hd)
    if name in ("window_global", "causal_window"):
        assert pl.density < 0.9


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("Sq,Sk", [(700, 1300), (1024, 256), (200, 900)])
def test_cross_attention_lengths(hd, Sq, Sk):
    _run(SA.AttentionPattern(), 2, 2, Sq, Sk, hd, plan=False)


def test_cross_attention_windowed():
    _run(SA.sliding_window(128), 2, 2, 600, 900, 64)


def test_long_window_sparsity_speed():
    """A 256-token window at 8K tokens visits ~1/16 of the key blocks and
    runs several times faster than dense attention (timed with events)."""
    B, H, S, hd = 1, 8, 8192, 64
    q, k, v = (torch.randn(B, S, H, hd, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    out = torch.empty_like(q)
    lse = torch.empty(B, H, S, device="cuda")
    pl = SA.sliding_window(256).plan(S, S, hd, q.device)

    def t(fn):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(10):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 10

    dense = t(lambda: K.flash_attn_fwd(q, k, v, out, lse, False, hd ** -0.5))
    sparse = t(lambda: K.flash_attn_fwd(q, k, v, out, lse, False, hd ** -0.5, plan=pl))
    assert sparse < dense / 3, (sparse, dense)
