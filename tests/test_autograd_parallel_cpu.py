"""Parallel evaluation of autograd graphs on the native dataflow scheduler:
same values and gradients as the serial evaluator, and independent branches
overlap."""
import time

import numpy as np

from scirs_b200 import autograd as ag


def _graph(ctx, n_branches=4):
    x = ctx.placeholder("x", (8, 8))
    outs = []
    for i in range(n_branches):
        w = ctx.constant(np.eye(8) * (i + 1))
        h = ag.ops.tanh(x @ w) * (i + 1.0)
        outs.append(ag.ops.reduce_sum(h))
    total = outs[0]
    for o in outs[1:]:
        total = total + o
    return x, outs, total


def test_parallel_matches_serial_values_and_gradients():
    feed = np.random.default_rng(0).standard_normal((8, 8)).astype(np.float32)

    def body(ctx):
        x, outs, total = _graph(ctx)
        (g,) = ag.grad([total], [x])
        serial = ctx.evaluator().extend([total, g] + outs).feed(x, feed).run()
        par = ctx.evaluator().extend([total, g] + outs).feed(x, feed).parallel(4).run()
        for a, b in zip(serial, par):
            np.testing.assert_allclose(a, b, rtol=1e-6)

    ag.run(body)


def test_independent_branches_overlap():
    def body(ctx):
        x = ctx.placeholder("x", (2,))
        branches = []
        for i in range(6):
            b = x * float(i + 1)
            b.register_hook(lambda v: time.sleep(0.15))  # releases the interpreter lock
            branches.append(b)
        s = branches[0]
        for b in branches[1:]:
            s = s + b
        t0 = time.perf_counter()
        (out,) = ctx.evaluator().push(s).feed(x, np.ones(2, np.float32)).parallel(6).run()
        dt = time.perf_counter() - t0
        np.testing.assert_allclose(out, [21.0, 21.0])
        assert dt < 0.6  # serial: 0.9 s

    ag.run(body)
