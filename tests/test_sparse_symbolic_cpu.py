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


def test_sparse_tensor_nd_and_products():
    d = torch.zeros(3, 4, 5)
    d[0, 1, 2], d[2, 3, 4], d[1, 0, 0] = 1.5, -2.0, 0.25
    st = SP.SparseTensor.from_dense(d)
    assert st.nnz() == 3 and st.total_size() == 60 and torch.equal(st.to_dense(), d)
    f = st.coords_to_flat([2, 3, 4])
    assert st.flat_to_coords(f) == [2, 3, 4]
    assert torch.equal(st.reshape((12, 5)).to_dense(), d.reshape(12, 5))
    assert torch.equal(st.slice_first_dim(1, 3).to_dense(), d[1:3])
    st.accumulate(SP.SparseTensor.from_dense(d))
    assert torch.equal(st.to_dense(), 2 * d)
    m = SP.SparseTensor.from_dense(torch.tensor([[0.0, 2.0], [1.0, 0.0], [0.0, 0.0]]))
    x = torch.randn(2, 3, requires_grad=True)
    y = m.matmul(x)
    assert torch.allclose(y, m.to_dense() @ x)
    y.sum().backward()
    assert torch.allclose(x.grad, m.to_dense().t() @ torch.ones(3, 3))


def test_embedding_backward_and_accumulator():
    ids = torch.tensor([3, 1, 3])
    go = torch.arange(6.0).reshape(3, 2)
    g = SP.embedding_backward(ids, go, num_embeddings=5)
    dense = g.to_dense()
    assert torch.equal(dense[3], go[0] + go[2]) and torch.equal(dense[1], go[1]) and dense[0].abs().sum() == 0
    acc = SP.SparseGradAccumulator()
    acc.accumulate_sparse("emb", g.to_sparse_grad())
    acc.step()
    acc.accumulate_sparse("emb", g.to_sparse_grad())
    acc.step()
    assert acc.raw_grad("emb").is_sparse()
    assert torch.allclose(acc.averaged_grad("emb"), dense.reshape(-1))
    acc.accumulate_dense("w", torch.ones(4))
    assert acc.param_names() == ["emb", "w"]
