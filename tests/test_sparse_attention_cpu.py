"""Sparse / windowed attention plans: every allowed (query, key) pair lies
in a listed block (forward and backward lists), the work shrinks with the
window, and the CPU path of the layers equals the dense-mask reference."""
import pytest
import torch

from scirs_b200.nn.attention import SlidingWindowAttention, SlidingWindowConfig, SparseAttention
from scirs_b200.ops import sparse_attention as SA


def _covered(plan, pattern, Sq, Sk, hd):
    m = pattern.allowed_dense(Sq, Sk)
    for c in range(plan.fwd_ptr.numel() - 1):
        blocks = set(plan.fwd_idx[plan.fwd_ptr[c]:plan.fwd_ptr[c + 1]].tolist())
        need = set((m[c * 256:(c + 1) * 256].any(0).nonzero()[:, 0] // 128).tolist())
        assert need <= blocks, ("fwd", c, need - blocks)
    BQ = 128 if hd == 64 else 64
    for t in range(plan.bwd_ptr.numel() - 1):
        blocks = set(plan.bwd_idx[plan.bwd_ptr[t]:plan.bwd_ptr[t + 1]].tolist())
        need = set((m[:, t * 128:(t + 1) * 128].any(1).nonzero()[:, 0] // BQ).tolist())
        assert need <= blocks, ("bwd", t, need - blocks)


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("pattern", [
    SA.sliding_window(100, num_global=3),
    SA.sliding_window(300, causal=True),
    SA.AttentionPattern(window_left=50, window_right=200),
    SA.block_sparse(SA.strided_bitmap(8, 8, local=1, stride=3)),
    SA.AttentionPattern(causal=True, window_left=128, num_global=1,
                        bitmap=SA.strided_bitmap(8, 8, 1, 4), bitmap_key="t1"),
])
def test_plan_covers_every_allowed_pair(pattern, hd):
    S = 1000
    plan = pattern.plan(S, S, hd, "cpu")
    _covered(plan, pattern, S, S, hd)


def test_window_plan_is_sparse():
    p = SA.sliding_window(256).plan(16384, 16384, 64, "cpu")
    assert p.density < 0.06  # ~5 of 128 key blocks per CTA
    assert SA.AttentionPattern().plan(2048, 2048, 64, "cpu").density == 1.0


def test_cross_attention_plan_shapes():
    p = SA.sliding_window(64).plan(300, 700, 128, "cpu")
    assert p.fwd_ptr.numel() == 2 + 1 and p.bwd_ptr.numel() == 6 + 1


def test_layers_cpu_match_dense_reference():
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(2, 300, 2, 16, generator=g) for _ in range(3))
    sw = SlidingWindowAttention(SlidingWindowConfig(window_size=20, global_tokens=2))
    o = sw.forward(q, k, v)
    ref, _ = SA.reference_attention(q, k, v, sw.pattern(), 16 ** -0.5)
    assert torch.allclose(o.float(), ref, atol=1e-4)
    m = sw.mask(300)
    assert m[50, 30] and m[50, 70] and not m[50, 71] and m[299, 1] and m[0, 299]
    sp = SparseAttention("bigbird", window=16, num_global=1, num_random=1)
    o2 = sp.forward(q, k, v)
    ref2, _ = SA.reference_attention(q, k, v, sp.block_pattern(300, 300), 16 ** -0.5)
    assert torch.allclose(o2.float(), ref2, atol=1e-4)
