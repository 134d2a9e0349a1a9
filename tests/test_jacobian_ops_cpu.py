"""Jacobian / JVP / VJP operations and domain validation (CPU, float64)."""
import pytest
import torch

from scirs_b200.autograd import jacobian_ops as J

D = torch.float64


def f(x):
    return torch.stack([x[0] * x[1], torch.sin(x[2]) + x[0] ** 2, x.sum()])


def test_jacobians_agree():
    x = torch.tensor([0.3, -1.2, 0.7], dtype=D)
    exact = torch.tensor([[x[1], x[0], 0.0], [2 * x[0], 0.0, torch.cos(x[2])], [1.0, 1.0, 1.0]], dtype=D)
    for fn in (J.jacobian_reverse, J.jacobian_forward, J.jacobian_auto):
        assert torch.allclose(fn(f, x), exact)
    assert torch.allclose(J.numerical_jacobian(f, x), exact, atol=1e-8)
    v, u = torch.tensor([1.0, 2.0, -1.0], dtype=D), torch.tensor([0.5, -1.0, 2.0], dtype=D)
    assert torch.allclose(J.jvp_forward(f, x, v), exact @ v)
    assert torch.allclose(J.vjp_reverse(f, x, u), u @ exact)
    g1, g2 = J.vjp_multi(lambda a, b: a * b + a, [x, v], u)
    assert torch.allclose(g1, u * (v + 1)) and torch.allclose(g2, u * x)
    assert J.jacobian_check(f, x) < 1e-6
    with pytest.raises(ValueError):
        J.jacobian_check(lambda z: torch.floor(z * 1e6), x, tolerance=1e-12)
    sq = lambda z: z ** 3 + z  # noqa: E731
    assert torch.allclose(J.jacobian_diagonal(sq, x), 3 * x ** 2 + 1)
    batch = torch.randn(4, 3, dtype=D)
    bj = J.batch_jacobian(f, batch)
    assert bj.shape == (4, 3, 3) and torch.allclose(bj[2], J.jacobian_reverse(f, batch[2]))
    with pytest.raises(ValueError):
        J.jvp_forward(f, x, torch.ones(2, dtype=D))


def test_validation():
    J.validate_sqrt_domain(torch.tensor([0.0, 1.0]))
    J.validate_log_domain(torch.tensor([0.1, 1.0]))
    J.validate_arcfunc_domain(torch.tensor([-1.0, 0.5]))
    for fn, bad in ((J.validate_sqrt_domain, [-1.0]), (J.validate_log_domain, [0.0]),
                    (J.validate_arcfunc_domain, [1.5]), (J.validate_finite, [float("inf")]),
                    (J.validate_non_nan, [float("nan")])):
        with pytest.raises(ValueError):
            fn(torch.tensor(bad))
