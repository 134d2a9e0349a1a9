"""Property-based tests (hypothesis) of host-side components: invariants
that must hold for every shape / size, not only the hand-picked cases."""
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from scirs_b200 import linalg as L
from scirs_b200.data.transforms import KFold, create_batches
from scirs_b200.nn import tracing as T
from scirs_b200.utils.logging import RateLimiter, RateLimitStrategy

SET = settings(max_examples=25, deadline=None)


@SET
@given(st.integers(1, 3), st.integers(1, 9), st.integers(1, 9), st.integers(1, 6), st.integers(1, 10),
       st.booleans(), st.integers(0, 10_000))
def test_flash_attention_block_size_invariance(b, lq, lk, d, bs, causal, seed):
    g = torch.Generator().manual_seed(seed)
    if causal:
        lk = lq
    q, k, v = (torch.randn(b, n, d, generator=g, dtype=torch.float64) for n in (lq, lk, lk))
    mask = L.AttentionMask.causal() if causal else None
    ref = L.scaled_dot_product_attention(q, k, v, mask, 0.7)
    assert torch.allclose(L.flash_attention(q, k, v, mask, 0.7, block_size=bs), ref, atol=1e-10)


@SET
@given(st.integers(2, 40), st.integers(2, 12), st.booleans(), st.integers(0, 99))
def test_kfold_partitions(n, k, shuffle, seed):
    if k > n:
        k = n
    folds = KFold(k, shuffle, seed).split(n)
    tests = sorted(i for _, te in folds for i in te)
    assert tests == list(range(n))
    assert max(len(te) for _, te in folds) - min(len(te) for _, te in folds) <= 1
    assert all(sorted(tr + te) == list(range(n)) for tr, te in folds)


@SET
@given(st.integers(1, 30), st.integers(1, 8))
def test_create_batches_cover_everything(n, bs):
    x = torch.arange(n)
    got = torch.cat([bx for bx, _ in create_batches(x, x, bs, shuffle=True)])
    assert sorted(got.tolist()) == list(range(n))


@SET
@given(st.integers(1, 5), st.floats(0.5, 5.0), st.lists(st.floats(0.0, 2.0), min_size=1, max_size=40))
def test_sliding_window_limit(maxev, window, gaps):
    t = [0.0]
    rl = RateLimiter(RateLimitStrategy("sliding_window", max_events=maxev, window_s=window), clock=lambda: t[0])
    allowed = []
    for dt in gaps:
        t[0] += dt
        if rl.allow("k"):
            allowed.append(t[0])
    for i, a in enumerate(allowed):
        assert sum(1 for x in allowed[: i + 1] if a - x < window) <= maxev


@SET
@given(st.lists(st.sampled_from(["relu", "tanh", "sigmoid"]), min_size=1, max_size=4), st.integers(1, 6),
       st.integers(0, 1000))
def test_traced_mlp_matches_module(acts, width, seed):
    torch.manual_seed(seed)
    layers, d = [], 5
    for a in acts:
        layers += [torch.nn.Linear(d, width), {"relu": torch.nn.ReLU, "tanh": torch.nn.Tanh,
                                               "sigmoid": torch.nn.Sigmoid}[a]()]
        d = width
    model = torch.nn.Sequential(*layers).double()
    x = torch.randn(3, 5, dtype=torch.float64)
    g, wm = T.trace_sequential(model, [3, 5])
    with torch.no_grad():
        assert torch.allclose(T.GraphExecutor(g, wm).run([x])[0], model(x))
