"""The numpy-facing API honours the contract of the reference's Python
bindings (behaviours exercised by scirs2-python/tests/test_neural.py and
test_autograd.py): shapes, accessors, losses, optimizers, training, autograd."""
import numpy as np
import pytest

import scirs_b200.api as sc


def test_sequential_build_forward_compile():
    m = sc.Sequential()
    assert m.num_layers() == 0
    m.add(sc.Dense(3, 6, activation="relu"))
    m.add(sc.Dense(6, 2, activation="sigmoid"))
    assert m.num_layers() == 2
    out = m.forward(np.arange(6, dtype=np.float64).reshape(2, 3))
    assert out.shape == (2, 2) and np.all((out >= 0) & (out <= 1))
    m.compile(optimizer="sgd", loss="mse", learning_rate=0.05)
    assert m.is_compiled()


def test_dense_accessors_and_activations():
    d = sc.Dense(input_dim=7, output_dim=4, activation="tanh")
    assert (d.input_dim(), d.output_dim(), d.activation()) == (7, 4, "tanh")
    y = d.forward(np.random.randn(5, 7))
    assert y.shape == (5, 4) and np.all(np.abs(y) <= 1)
    for act in ["relu", "sigmoid", "softmax", "gelu", None]:
        assert sc.Dense(3, 3, activation=act).forward(np.ones((2, 3))).shape == (2, 3)


def test_conv_and_pool_shapes():
    c = sc.Conv2D(in_channels=3, out_channels=5, kernel_size=3, stride=1, padding=1)
    assert (c.in_channels(), c.out_channels(), c.kernel_size()) == (3, 5, 3)
    assert c.forward(np.random.randn(2, 3, 12, 12)).shape == (2, 5, 12, 12)
    assert sc.Conv2D(3, 4, kernel_size=3, stride=2).forward(np.random.randn(1, 3, 16, 16)).shape[2] <= 8
    mp = sc.MaxPool2D(kernel_size=2, stride=2)
    assert (mp.kernel_size(), mp.stride()) == (2, 2)
    x = np.arange(16, dtype=np.float64).reshape(1, 1, 4, 4)
    o = mp.forward(x)
    assert o.shape == (1, 1, 2, 2) and o.max() == 15
    assert np.allclose(sc.AvgPool2D(2, 2).forward(np.full((1, 1, 4, 4), 3.0)), 3.0)


def test_activation_layers():
    x = np.array([[-2.0, 0.0, 3.0]])
    assert np.allclose(sc.ReLU().forward(x), [[0, 0, 3]])
    assert np.allclose(sc.Sigmoid().forward(np.zeros((1, 1))), 0.5)
    assert np.allclose(sc.Tanh().forward(np.zeros((1, 2))), 0.0)
    s = sc.Softmax().forward(x)
    assert np.allclose(s.sum(1), 1.0) and np.all(s > 0)


def test_losses():
    assert np.isclose(sc.MSELoss().compute(np.ones((1, 3)), np.ones((1, 3))), 0.0)
    assert sc.MSELoss().compute(np.array([[0.0, 1.0]]), np.array([[1.0, 3.0]])) > 0
    ce = sc.CrossEntropyLoss().compute(np.array([[3.0, 0.5, -1.0]]), np.array([0]))
    assert 0 <= ce < 0.2
    bce = sc.BinaryCrossEntropyLoss().compute(np.array([[0.95, 0.05]]), np.array([[1.0, 0.0]]))
    assert bce < 0.1


@pytest.mark.parametrize("opt", [sc.SGD(learning_rate=0.1), sc.Adam(learning_rate=0.01, beta1=0.9, beta2=0.999),
                                 sc.RMSprop(learning_rate=0.01, decay_rate=0.9), sc.AdamW(0.01), sc.Adagrad(0.1)])
def test_optimizers_step(opt):
    w = np.array([[1.0, -2.0], [0.5, 4.0]])
    g = np.full_like(w, 0.3)
    w2 = opt.step(w, g)
    assert w2.shape == w.shape and np.all(w2 < w)


def test_sgd_matches_reference_rule():
    w = np.array([1.0, 2.0])
    g = np.array([0.5, -1.0])
    assert np.allclose(sc.SGD(learning_rate=0.1).step(w, g), w - 0.1 * g)


def test_adam_first_step_is_lr_sign():
    # bias-corrected Adam's first step moves each weight by ~lr * sign(g)
    w = np.array([1.0, 1.0])
    w2 = sc.Adam(learning_rate=0.01).step(w, np.array([3.0, -0.2]))
    assert np.allclose(w - w2, [0.01, -0.01], atol=1e-5)


def test_training_reduces_loss():
    np.random.seed(0)
    m = sc.Sequential()
    m.add(sc.Dense(2, 8, activation="relu", seed=1))
    m.add(sc.Dense(8, 1, activation="sigmoid", seed=2))
    m.compile(optimizer="adam", loss="bce", learning_rate=0.05)
    X = np.array([[0, 0], [0, 1], [1, 0], [1, 1]], dtype=np.float64)
    y = np.array([[0], [1], [1], [0]], dtype=np.float64)
    l0 = m.evaluate(X, y)
    for _ in range(200):
        m.train_step(X, y)
    assert m.evaluate(X, y) < l0


def test_minibatch_regression_and_edge_cases():
    m = sc.Sequential()
    m.add(sc.Dense(5, 3, activation="relu"))
    m.add(sc.Dense(3, 1))
    m.compile(optimizer="sgd", loss="mse", learning_rate=0.01)
    X, y = np.random.randn(20, 5), np.random.randn(20, 1)
    for i in range(0, 20, 4):
        m.train_step(X[i : i + 4], y[i : i + 4])
    assert m.forward(X[:5]).shape == (5, 1)
    one = sc.Sequential()
    one.add(sc.Dense(3, 1))
    one.compile(optimizer="sgd", loss="mse")
    one.train_step(np.array([[1.0, 2.0, 3.0]]), np.array([[1.0]]))
    assert sc.Sequential().num_layers() == 0
    big = sc.Sequential()
    big.add(sc.Dense(10, 5))
    assert big.forward(np.random.randn(1000, 10)).shape == (1000, 5)


def test_dropout_batchnorm_resnet_cnn():
    d = sc.Dropout(rate=0.5)
    x = np.ones((10, 10))
    d.training(True)
    assert not np.allclose(d.forward(x), x)
    d.training(False)
    assert np.allclose(d.forward(x), x)
    bn = sc.BatchNorm(num_features=5)
    bn.training(True)
    o = bn.forward(np.random.randn(64, 5) * 10 + 5)
    assert np.allclose(o.mean(0), 0, atol=0.1) and np.allclose(o.std(0), 1, atol=0.1)
    rb = sc.ResNetBlock(channels=8, stride=1)
    xi = np.random.randn(2, 8, 10, 10)
    assert rb.forward(xi).shape == xi.shape
    cnn = sc.Sequential()
    cnn.add(sc.Conv2D(1, 4, kernel_size=3, padding=1))
    cnn.add(sc.ReLU())
    cnn.add(sc.MaxPool2D(kernel_size=2, stride=2))
    cnn.add(sc.Flatten())
    cnn.add(sc.Dense(4 * 14 * 14, 10))
    assert cnn.forward(np.random.randn(2, 1, 28, 28)).shape == (2, 10)


# ----------------------------------------------------------------------------- autograd
def test_tensor_creation_and_ops():
    t = sc.Tensor(np.array([[1.0, 2.0], [3.0, 4.0]]), requires_grad=True)
    assert t.shape == (2, 2) and t.requires_grad is True
    assert sc.Tensor(5.0, requires_grad=True).shape in ((), (1,))
    assert sc.Tensor(np.array([1.0]), requires_grad=False).requires_grad is False
    a, b = sc.Tensor(np.array([1.0, 2.0, 6.0])), sc.Tensor(np.array([4.0, 5.0, 3.0]))
    assert np.allclose((a + b).data, [5, 7, 9]) and np.allclose((a - b).data, [-3, -3, 3])
    assert np.allclose((a * b).data, [4, 10, 18]) and np.allclose((a / b).data, [0.25, 0.4, 2.0])
    m = sc.Tensor(np.array([[1.0, 2.0]])) @ sc.Tensor(np.array([[3.0], [4.0]]))
    assert np.allclose(m.data, [[11.0]])
    assert np.allclose(sc.Tensor(np.array([0.0, 1.0])).exp().data, [1.0, np.e])
    assert np.allclose(sc.Tensor(np.array([1.0, np.e])).log().data, [0.0, 1.0])
    assert np.isclose(sc.Tensor(np.array([[1.0, 2.0], [3.0, 4.0]])).sum().data, 10.0)
    assert np.isclose(sc.Tensor(np.array([1.0, 2.0, 3.0, 4.0])).mean().data, 2.5)


def test_tensor_gradients():
    x = sc.Tensor(np.array([2.0]), requires_grad=True)
    (x * x).backward()
    assert np.allclose(x.grad, [4.0])
    a, b = sc.Tensor(np.array([2.0]), requires_grad=True), sc.Tensor(np.array([3.0]), requires_grad=True)
    (a * b).backward()
    assert np.allclose(a.grad, [3.0]) and np.allclose(b.grad, [2.0])
    x = sc.Tensor(np.array([2.0]), requires_grad=True)
    (x * x * x + x * 2 + 1).backward()  # d/dx = 3x^2 + 2 = 14
    assert np.allclose(x.grad, [14.0])
    a = sc.Tensor(np.array([[1.0, 2.0]]), requires_grad=True)
    b = sc.Tensor(np.array([[3.0], [4.0]]), requires_grad=True)
    (a @ b).backward()
    assert a.grad.shape == (1, 2) and b.grad.shape == (2, 1) and np.allclose(a.grad, [[3.0, 4.0]])
    x = sc.Tensor(np.array([-1.0, 0.5, 2.0]), requires_grad=True)
    x.relu().backward(np.ones(3))
    assert np.allclose(x.grad, [0.0, 1.0, 1.0])
    x = sc.Tensor(np.array([0.0]), requires_grad=True)
    x.sigmoid().backward()
    assert np.allclose(x.grad, [0.25])
    x = sc.Tensor(np.array([0.0]), requires_grad=True)
    x.tanh().backward()
    assert np.allclose(x.grad, [1.0])
    x = sc.Tensor(np.array([3.0]), requires_grad=True)
    y = x.detach() * 2
    assert not y.requires_grad
    with sc.no_grad():
        z = sc.Tensor(np.array([1.0]), requires_grad=True) * 3
    assert not z.requires_grad
