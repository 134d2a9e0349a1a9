"""RAdam / LAMB / LARS / Adafactor / Sophia against element-wise restatements
of their update rules and (where torch has one) torch.optim."""
import math

import torch

from scirs_b200.optim.extra import Adafactor, Lamb, Lars, RAdam, Sophia


def _params(seed=0, shape=(6, 5)):
    g = torch.Generator().manual_seed(seed)
    p = torch.randn(shape, generator=g, dtype=torch.float64).requires_grad_(True)
    grads = [torch.randn(shape, generator=g, dtype=torch.float64) for _ in range(8)]
    return p, grads


def test_radam_matches_torch_and_rectified_rule():
    p, grads = _params()
    q = p.detach().clone().requires_grad_(True)
    a = RAdam([p], lr=0.01, weight_decay=0.01)
    b = torch.optim.RAdam([q], lr=0.01, weight_decay=0.01, eps=1e-8)
    # steps 1-4: rho_t <= 4, both take the un-adapted momentum step
    for g in grads[:4]:
        p.grad, q.grad = g.clone(), g.clone()
        a.step()
        b.step()
    torch.testing.assert_close(p, q)
    # step 5 onwards: rectified, restated element-wise
    st = a.state[p]
    m, v, w = st["m"].clone(), st["v"].clone(), p.detach().clone()
    for t, g in enumerate(grads[4:], start=5):
        gg = g + 0.01 * w
        m = 0.9 * m + 0.1 * gg
        v = 0.999 * v + 0.001 * gg * gg
        rho_inf = 2 / 0.001 - 1
        rho = rho_inf - 2 * t * 0.999 ** t / (1 - 0.999 ** t)
        r = math.sqrt((rho - 4) * (rho - 2) * rho_inf / ((rho_inf - 4) * (rho_inf - 2) * rho))
        w = w - 0.01 * r * (m / (1 - 0.9 ** t)) / ((v / (1 - 0.999 ** t)).sqrt() + 1e-8)
        p.grad = g.clone()
        a.step()
    torch.testing.assert_close(p.detach(), w)


def test_radam_reference_rectification_differs():
    p, grads = _params()
    q = p.detach().clone().requires_grad_(True)
    a, b = RAdam([p], lr=0.01, beta2=0.9), RAdam([q], lr=0.01, beta2=0.9, rectification="reference")
    for g in grads:
        p.grad, q.grad = g.clone(), g.clone()
        a.step()
        b.step()
    assert not torch.allclose(p, q)


def test_lamb_trust_ratio():
    p, grads = _params()
    p0 = p.detach().clone()
    opt = Lamb([p], lr=0.1, weight_decay=0.01)
    p.grad = grads[0]
    opt.step()
    m = 0.1 * grads[0] / 0.1
    v = 0.001 * grads[0] ** 2 / 0.001
    u = m / (v.sqrt() + 1e-6) + 0.01 * p0
    trust = p0.norm() / u.norm()
    torch.testing.assert_close(p.detach(), p0 - 0.1 * trust * u)


def test_lars_and_larc():
    p, grads = _params()
    p0 = p.detach().clone()
    opt = Lars([p], lr=0.1, momentum=0.9, weight_decay=1e-4)
    p.grad = grads[0]
    opt.step()
    llr = 0.001 * p0.norm() / (grads[0].norm() + 1e-4 * p0.norm() + 1e-8)
    torch.testing.assert_close(p.detach(), p0 - llr * (grads[0] + 1e-4 * p0))
    assert Lars.local_lr(1e-5, 0.001, 0, 1e-8, True, 100.0, 1.0) == 1e-5


def test_adafactor_factored_and_full():
    torch.manual_seed(0)
    big = torch.randn(130, 140, requires_grad=True)
    small = torch.randn(7, requires_grad=True)
    opt = Adafactor([big, small])
    for _ in range(3):
        big.grad, small.grad = torch.randn_like(big), torch.randn_like(small)
        opt.step()
    st = opt.state[big]
    assert set(st) == {"row", "col"} and st["row"].shape == (130,)
    assert "v" in opt.state[small]
    assert math.isclose(opt.relative_step_size(), 1 / math.sqrt(3))


def test_adafactor_single_step_rule():
    p = torch.randn(4, 3, dtype=torch.float64, requires_grad=True)
    p0 = p.detach().clone()
    g = torch.randn(4, 3, dtype=torch.float64) * 0.1
    opt = Adafactor([p], clipping_threshold=None)
    p.grad = g
    opt.step()
    # t = 1: beta2 = 0, v = g^2, update = sign(g), lr = 1
    torch.testing.assert_close(p.detach(), p0 - torch.sign(g))


def test_sophia_rule():
    p, grads = _params()
    p0 = p.detach().clone()
    opt = Sophia([p], lr=0.5, weight_decay=0.0, rho=0.04)
    p.grad = grads[0]
    opt.update_hessian(torch.Generator().manual_seed(1))
    h = opt.state[p]["h"].clone()
    torch.testing.assert_close(h, 0.01 * grads[0] ** 2)
    opt.step()
    m = 0.035 * grads[0]
    d = (0.04 * h).clamp_min(1e-8)
    torch.testing.assert_close(p.detach(), p0 - 0.5 * (m / d).clamp(-1, 1) * d)
    assert opt.get_learning_rate() == 0.5


def test_optimizers_reduce_quadratic():
    for cls, kw in [(RAdam, dict(lr=0.05)), (Lamb, dict(lr=0.05)), (Lars, dict(lr=5.0, trust_coefficient=0.02)),
                    (Adafactor, dict(lr=0.05)), (Sophia, dict(lr=1.0, rho=10.0, weight_decay=0.0))]:
        torch.manual_seed(0)
        w = torch.randn(10, 10, requires_grad=True)
        opt = cls([w], **kw)
        l0 = None
        for i in range(60):
            loss = (w - 1).square().sum()
            l0 = l0 or float(loss.detach())
            opt.zero_grad()
            loss.backward()
            if cls is Sophia and i % 10 == 0:
                opt.update_hessian()
            opt.step()
        assert float((w - 1).square().sum()) < 0.5 * l0, cls.__name__
