"""Autograd edge cases and concurrency: deep graphs (thousands of nodes) in
serial and parallel evaluation, NaN / Inf propagation, empty tensors, and the
same / separate graphs evaluated from 2, 4 and 8 threads at once."""
import threading

import numpy as np
import pytest

from scirs_b200 import autograd as ag
from scirs_b200.autograd import ops as T


@pytest.mark.parametrize("parallel", [False, True])
def test_deep_chain_values_and_gradients(parallel):
    def body(ctx):
        x = ctx.placeholder("x", (3,))
        y = x
        for _ in range(3000):
            y = y * 1.0 + 1.0
        (g,) = ag.grad([T.reduce_sum(y)], [x])
        ev = ctx.evaluator().extend([y, g]).feed(x, np.zeros(3, np.float32))
        if parallel:
            ev.parallel(4)
        out, grad = ev.run()
        np.testing.assert_allclose(out, [3000.0] * 3)
        np.testing.assert_allclose(grad, [1.0] * 3)

    ag.run(body)


def test_nan_and_inf_propagate():
    def body(ctx):
        x = ctx.placeholder("x", (4,))
        y = T.relu(x) * 2.0
        s = T.reduce_sum(y)
        (g,) = ag.grad([s], [x])
        out, tot, grad = ctx.evaluator().extend([y, s, g]).feed(
            x, np.array([np.nan, np.inf, -np.inf, 1.0], np.float32)).run()
        assert np.isnan(out[0]) and out[1] == np.inf and out[2] == 0.0 and out[3] == 2.0
        assert np.isnan(tot)
        assert grad[1] == 2.0 and grad[2] == 0.0 and grad[3] == 2.0

    ag.run(body)


def test_empty_tensors():
    def body(ctx):
        x = ctx.placeholder("x", (0, 3))
        w = ctx.constant(np.ones((3, 2), np.float32))
        y = x @ w
        s = T.reduce_sum(y)
        (g,) = ag.grad([s], [x])
        out, tot, grad = ctx.evaluator().extend([y, s, g]).feed(x, np.zeros((0, 3), np.float32)).run()
        assert out.shape == (0, 2) and tot == 0.0 and grad.shape == (0, 3)

    ag.run(body)


def _one_graph(seed: int):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((16, 16)).astype(np.float32)
    res = {}

    def body(ctx):
        x = ctx.placeholder("x", (16, 16))
        y = T.reduce_sum(T.tanh(x @ x))
        (g,) = ag.grad([y], [x])
        res["y"], res["g"] = ctx.evaluator().extend([y, g]).feed(x, a).run()

    ag.run(body)
    return a, res


@pytest.mark.parametrize("n_threads", [2, 4, 8])
def test_separate_graphs_in_threads(n_threads):
    expected = {i: _one_graph(i)[1] for i in range(n_threads)}
    got, errors = {}, []

    def worker(i):
        try:
            got[i] = _one_graph(i)[1]
        except Exception as e:  # noqa: BLE001 - reported below
            errors.append(e)

    ts = [threading.Thread(target=worker, args=(i,)) for i in range(n_threads)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errors
    for i in range(n_threads):
        np.testing.assert_allclose(got[i]["y"], expected[i]["y"], rtol=1e-5)
        np.testing.assert_allclose(got[i]["g"], expected[i]["g"], rtol=1e-5)


@pytest.mark.parametrize("n_threads", [2, 4, 8])
def test_shared_graph_evaluated_from_threads(n_threads):
    def body(ctx):
        x = ctx.placeholder("x", (8,))
        y = T.reduce_sum(T.sigmoid(x) * x)
        (g,) = ag.grad([y], [x])
        feeds = [np.full(8, i, np.float32) for i in range(n_threads)]
        ref = [ctx.evaluator().extend([y, g]).feed(x, f).run() for f in feeds]
        got = [None] * n_threads

        def worker(i):
            got[i] = ctx.evaluator().extend([y, g]).feed(x, feeds[i]).run()

        ts = [threading.Thread(target=worker, args=(i,)) for i in range(n_threads)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
        for r, o in zip(ref, got):
            np.testing.assert_allclose(o[0], r[0], rtol=1e-6)
            np.testing.assert_allclose(o[1], r[1], rtol=1e-6)

    ag.run(body)
