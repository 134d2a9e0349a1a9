"""Hand-written decomposition gradients (scirs_b200.autograd.linalg) against
central finite differences in float64 (GradientChecker) and against
torch.autograd.gradcheck, plus a finite-difference sweep of the extended
op table through the graph API."""
import numpy as np
import pytest
import torch

from scirs_b200.autograd import GradientChecker, grad, run
from scirs_b200.autograd import linalg as LA
from scirs_b200.autograd import ops as T

torch.manual_seed(0)


def _spd(n, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(n, n, generator=g, dtype=torch.float64)
    return a @ a.T + n * torch.eye(n, dtype=torch.float64)


def _sym(a):
    return 0.5 * (a + a.T)


def _rand(*s, seed=1):
    return torch.randn(*s, generator=torch.Generator().manual_seed(seed), dtype=torch.float64)


C5 = _rand(5, 5, seed=7)
C64 = _rand(6, 4, seed=8)
W4 = _rand(4, seed=9)

# (name, fn over float64 inputs, inputs): every loss depends on eigen / singular
# vectors only through sign-invariant products
CASES = [
    ("inverse", lambda a: (LA.inverse(a) * C5).sum(), [_spd(5, 1)]),
    ("det", lambda a: LA.det(a), [_spd(4, 2) / 4]),
    ("logabsdet", lambda a: LA.logabsdet(a), [_rand(4, 4, seed=3) + 3 * torch.eye(4, dtype=torch.float64)]),
    ("cholesky", lambda a: (LA.cholesky(_sym(a)) * C5).sum(), [_spd(5, 4)]),
    ("eigh", lambda a: (LA.eigh(_sym(a))[0] * torch.arange(5.0, dtype=torch.float64)).sum()
     + ((LA.eigh(_sym(a))[1] ** 2) * C5).sum(), [_spd(5, 5)]),
    ("qr", lambda a: (LA.qr(a)[0] * C64).sum() + (LA.qr(a)[1] * C5[:4, :4]).sum(), [_rand(6, 4, seed=6)]),
    ("svd", lambda a: (LA.svd(a)[1] * W4).sum() + ((LA.svd(a)[0] @ LA.svd(a)[2].T) * C64).sum(),
     [_rand(6, 4, seed=10)]),
    ("cholesky_solve", lambda b, l: (LA.cholesky_solve(b, torch.tril(l)) * _rand(4, 3, seed=11)).sum(),
     [_rand(4, 3, seed=12), torch.linalg.cholesky(_spd(4, 13))]),
    ("pinv", lambda a: (LA.pinv(a) * C64.T).sum(), [_rand(6, 4, seed=14)]),
    ("lstsq", lambda a, b: LA.lstsq(a, b).sum(), [_rand(6, 4, seed=15), _rand(6, 2, seed=16)]),
    ("matrix_power", lambda a: LA.matrix_power(a, 3).sum() + LA.matrix_power(a, -2).sum(),
     [_spd(4, 17) / 4]),
]


@pytest.mark.parametrize("name,fn,inputs", CASES, ids=[c[0] for c in CASES])
def test_decomposition_gradients_match_finite_differences(name, fn, inputs):
    res = GradientChecker(eps=1e-6, rtol=1e-5, atol=1e-7).check(fn, *inputs)
    assert res.passed, (name, res)
    xs = [x.clone().requires_grad_(True) for x in inputs]
    assert torch.autograd.gradcheck(fn, xs, eps=1e-6, atol=1e-5, rtol=1e-4)


def test_decomposition_forward_matches_torch():
    a = _rand(6, 4, seed=20)
    q, r = LA.qr(a)
    assert torch.allclose(q @ r, a)
    u, s, v = LA.svd(a)
    assert torch.allclose(u @ torch.diag(s) @ v.T, a)
    sp = _spd(5, 21)
    w, vv = LA.eigh(sp)
    assert torch.allclose(vv @ torch.diag(w) @ vv.T, sp)
    assert torch.allclose(LA.cholesky(sp) @ LA.cholesky(sp).T, sp)
    assert torch.allclose(LA.det(sp), torch.linalg.det(sp))


def test_second_order_through_inverse():
    a = _spd(4, 30).requires_grad_(True)
    g1, = torch.autograd.grad(LA.inverse(a).sum(), a, create_graph=True)
    g2, = torch.autograd.grad(g1.sum(), a)
    g1t, = torch.autograd.grad(torch.linalg.inv(a).sum(), a, create_graph=True)
    g2t, = torch.autograd.grad(g1t.sum(), a)
    assert torch.allclose(g2, g2t, atol=1e-10)


def test_graph_api_decompositions_and_grad():
    a0 = _spd(4, 31).numpy()

    def body(ctx):
        a = ctx.placeholder("a", [4, 4])
        q, r = T.qr(a)
        u, s, v = T.svd(a)
        w, vecs = T.eigh(a)
        loss = T.reduce_sum(s) + T.reduce_sum(w) + T.determinant(a) * 0.0 + T.reduce_sum(T.square(T.cholesky(a)))
        g, = grad([loss], [a])
        return ctx.evaluator().push(loss).push(g).push(q).push(r).feed("a", a0).run()

    loss, g, q, r = run(body)
    assert np.allclose(q @ r, a0)
    assert g.shape == (4, 4) and np.isfinite(g).all()


UNARY_SMOOTH = ["tan", "asin", "acos", "atan", "sinh", "cosh", "asinh", "atanh", "exp2", "expm1", "log2",
                "log10", "log1p", "rsqrt", "reciprocal", "erf", "erfc", "lgamma", "digamma", "sinc", "logit",
                "mish", "selu", "softsign", "log_sigmoid", "silu", "gelu_exact", "tanhshrink", "cube",
                "l2_normalize", "frobenius_norm", "nuclear_norm", "matrix_exp"]


@pytest.mark.parametrize("op", UNARY_SMOOTH)
def test_op_table_gradients_by_finite_differences(op):
    x0 = (torch.rand(3, 3, generator=torch.Generator().manual_seed(3), dtype=torch.float64) * 0.5 + 0.25)

    def f(x):
        def body(ctx):
            xp = ctx.placeholder("x", [3, 3])
            y = T.reduce_sum(getattr(T, op)(xp))
            return ctx.evaluator().torch().push(y).feed("x", x).run()[0]

        return run(body)

    def body(ctx):
        xp = ctx.placeholder("x", [3, 3])
        y = T.reduce_sum(getattr(T, op)(xp))
        g, = grad([y], [xp])
        return ctx.evaluator().torch().push(g).feed("x", x0).run()[0]

    g = run(body)
    eps = 1e-6
    num = torch.zeros_like(x0)
    for j in range(9):
        xp, xm = x0.clone(), x0.clone()
        xp.view(-1)[j] += eps
        xm.view(-1)[j] -= eps
        num.view(-1)[j] = (f(xp) - f(xm)) / (2 * eps)
    assert torch.allclose(g.double(), num, rtol=1e-4, atol=1e-6), (op, g, num)


def test_op_table_size():
    assert len(T.op_names()) >= 230
