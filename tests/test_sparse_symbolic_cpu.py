"""Sparse gradients and symbolic differentiation / tapes."""
import math

import torch

from scirs_b200.autograd import sparse as SP
from scirs_b200.autograd import symbolic as S


def test_sparse_grad_roundtrip_and_accumulate():
    d = torch.tensor([0.0, 3.0, 0.0, -0.01, 5.0])
    g = SP.SparseGrad.from_dense(d, threshold=0.1)
    assert g.nnz() == 2 and abs(g.sparsity() - 0.6) < 1e-9
    torch.testing.assert_close(g.to_dense(), torch.tensor([0.0, 3.0, 0.0, 0.0, 5.0]))
    g.accumulate(SP.SparseGrad([1, 2], [1.0, 2.0], 5))
    torch.testing.assert_close(g.to_dense(), torch.tensor([0.0, 4.0, 2.0, 0.0, 5.0]))
    dense = torch.ones(5)
    g.add_to_dense(dense)
    assert float(dense.sum()) == 16.0
    g.clip(3.0)
    assert g.l1_norm() == 8.0 and abs(g.scaled(2).l2_norm() - 2 * math.sqrt(22)) < 1e-5
    r = SP.GradientRepr(SP.SparseGrad([0], [1.0], 5))
    r.accumulate(SP.GradientRepr(torch.ones(5)))
    assert not r.is_sparse() and float(r.to_dense()[0]) == 2.0


def test_symbolic_differentiate_simplify_evaluate():
    x, y = S.SymExpr.variable("x"), S.SymExpr.variable("y")
    f = x ** 3 * y + S.sin(x) / y + S.exp(x * 0) * 2
    df = f.differentiate("x").simplify()
    vals = {"x": 0.7, "y": 1.3}
    want = 3 * 0.7 ** 2 * 1.3 + math.cos(0.7) / 1.3
    assert abs(df.evaluate(vals) - want) < 1e-12
    assert str((x * 1 + 0).simplify()) == "x"
    assert S.ExprBuilder.var("z").pow(2).add(1).build().differentiate("z").simplify().evaluate({"z": 3}) == 6


def test_symbolic_tape_reverse_mode():
    t = S.SymbolicTape()
    a, b = t.input("a"), t.input("b")
    out = t.log(t.add(t.mul(a, b), t.exp(a)))
    g = t.gradient({"a": 0.5, "b": 2.0}, out)
    s = 0.5 * 2.0 + math.exp(0.5)
    assert abs(g["a"] - (2.0 + math.exp(0.5)) / s) < 1e-12 and abs(g["b"] - 0.5 / s) < 1e-12
