"""Graph-mode autodiff API: placeholders/variables, evaluator + feeds,
symbolic gradients (incl. second order), graph optimizers, env persistence,
transforms and the finite-difference checker."""
import numpy as np
import torch

from scirs_b200 import autograd as ag
from scirs_b200.autograd import ops as T


def test_graph_forward_and_grad():
    env = ag.VariableEnvironment()
    w0 = np.array([[1.0, -1.0], [0.5, 2.0], [0.0, 1.0]], dtype=np.float32)
    env.name("w").set(w0)

    def body(ctx):
        x = ctx.placeholder("x", [-1, 3])
        w = ctx.variable("w")
        y = T.matmul(x, w)
        loss = T.reduce_sum(T.square(y))
        (gw,) = ag.grad([loss], [w])
        return ctx.evaluator().push(loss).push(gw).feed(x, np.ones((2, 3), np.float32)).run()

    loss, gw = env.run(body)
    xs = np.ones((2, 3), np.float32)
    y = xs @ w0
    assert np.isclose(loss, (y**2).sum())
    assert np.allclose(gw, xs.T @ (2 * y))


def test_second_order_gradient():
    def body(ctx):
        x = ctx.placeholder("x")
        y = x * x * x
        (g,) = ag.grad([y], [x])
        (gg,) = ag.grad([g], [x])
        return ctx.evaluator().push(g).push(gg).feed("x", np.array(2.0, np.float32)).run()

    g, gg = ag.run(body)
    assert np.isclose(g, 12.0) and np.isclose(gg, 12.0)


def test_graph_optimizer_trains_and_env_roundtrip(tmp_path):
    rng = np.random.default_rng(0)
    X = rng.normal(size=(64, 4)).astype(np.float32)
    true_w = np.array([[1.0], [-2.0], [0.5], [3.0]], np.float32)
    Y = X @ true_w
    env = ag.VariableEnvironment()
    env.name("w").set(np.zeros((4, 1), np.float32))
    opt = ag.Adam(["w"], env, lr=0.1)

    def step(ctx):
        x, yt = ctx.placeholder("x"), ctx.placeholder("y")
        w = ctx.variable("w")
        loss = T.reduce_mean(T.square(T.matmul(x, w) - yt))
        grads = ag.grad([loss], [w])
        opt.update([w], grads, ctx, ag.Feeder().push(x, X).push(yt, Y))
        return loss.eval({"x": X, "y": Y})

    first = env.run(step)
    for _ in range(200):
        last = env.run(step)
    assert last < first * 1e-2
    env.save(tmp_path / "env.json")
    env2 = ag.VariableEnvironment.load(tmp_path / "env.json")
    assert np.allclose(env2.get_array_by_name("w"), env.get_array_by_name("w"))
    import json

    obj = json.load(open(tmp_path / "env.json"))
    assert set(obj) == {"array_list", "name_to_id"} and obj["array_list"][0]["dim"] == [4, 1]


def test_custom_gradient_ops_and_export():
    def body(ctx):
        x = ctx.placeholder("x")
        y = T.reduce_sum(T.scale_gradient(x, 3.0) * 2.0)
        z = T.reduce_sum(T.stop_gradient(x) * x)
        (gy,) = ag.grad([y], [x])
        (gz,) = ag.grad([z], [x])
        dot = ag.to_dot(ctx)
        return ctx.evaluator().push(gy).push(gz).feed(x, np.array([1.0, 2.0], np.float32)).run(), dot

    (gy, gz), dot = ag.run(body)
    assert np.allclose(gy, [6.0, 6.0]) and np.allclose(gz, [1.0, 2.0])
    assert dot.startswith("digraph") and "scale_gradient" in dot


def test_transforms_and_gradient_checker():
    f = lambda x: (x**3).sum()  # noqa: E731
    x = torch.tensor([1.0, 2.0], dtype=torch.float64)
    v, g = ag.value_and_grad(f)(x)
    assert float(v) == 9.0 and torch.allclose(g, 3 * x**2)
    assert torch.allclose(ag.hessian(f, x), torch.diag(6 * x))
    assert torch.allclose(ag.hessian_vector_product(f, x, torch.ones(2, dtype=torch.float64)), 6 * x)
    _, t = ag.jvp(lambda x: x * x, (x,), (torch.ones(2, dtype=torch.float64),))
    assert torch.allclose(t, 2 * x)
    assert torch.allclose(ag.vmap(lambda r: r.sum())(torch.ones(3, 4)), torch.full((3,), 4.0))
    carry, ys = ag.scan(lambda c, x: (c + x, c * x), torch.tensor(0.0), torch.arange(4.0))
    assert float(carry) == 6.0
    assert ag.check_grad(lambda a, b: (a * b).sin(), torch.randn(3, 2), torch.randn(3, 2))
