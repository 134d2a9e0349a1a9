"""Recurrent layers: the time-loop autograd Function (run here through the
kernels' CPU reference paths) and the PyTorch-math loop both reproduce
torch.nn.RNN / LSTM / GRU with the same weights, outputs and gradients."""
import pytest
import torch

from scirs_b200.nn import recurrent as R

TORCH = {"rnn": torch.nn.RNN, "lstm": torch.nn.LSTM, "gru": torch.nn.GRU}
G = {"rnn": 1, "lstm": 4, "gru": 3}


def _weights(kind, I, H, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(G[kind] * H, I, generator=g) * 0.3, torch.randn(G[kind] * H, H, generator=g) * 0.3,
            torch.randn(G[kind] * H, generator=g) * 0.1, torch.randn(G[kind] * H, generator=g) * 0.1]


@pytest.mark.parametrize("kind", ["rnn", "lstm", "gru"])
@pytest.mark.parametrize("use_fn", [True, False])
def test_recurrence_matches_torch(kind, use_fn):
    B, S, I, H = 3, 7, 8, 16
    w = [t.requires_grad_(True) for t in _weights(kind, I, H, 1)]
    x = torch.randn(B, S, I, generator=torch.Generator().manual_seed(2), requires_grad=True)
    h0 = torch.randn(B, H, generator=torch.Generator().manual_seed(3))
    c0 = torch.randn(B, H, generator=torch.Generator().manual_seed(4)) if kind == "lstm" else None
    if use_fn:
        y, h, c = R._RecurrentFn.apply(kind, x, h0, c0, *w)
    else:
        y, h, c = R._loop_reference(kind, x, h0, c0, *w)
    ref = TORCH[kind](I, H, batch_first=True)
    with torch.no_grad():
        for p, v in zip((ref.weight_ih_l0, ref.weight_hh_l0, ref.bias_ih_l0, ref.bias_hh_l0), w):
            p.copy_(v)
    xr = x.detach().clone().requires_grad_(True)
    st = (h0[None], c0[None]) if kind == "lstm" else h0[None]
    yr, _ = ref(xr, st)
    assert torch.allclose(y, yr, atol=1e-5)
    gy = torch.randn_like(y)
    grads = torch.autograd.grad(y, [x] + w, gy)
    rgrads = torch.autograd.grad(yr, [xr, ref.weight_ih_l0, ref.weight_hh_l0, ref.bias_ih_l0, ref.bias_hh_l0], gy)
    for a, b in zip(grads, rgrads):
        assert torch.allclose(a, b, atol=1e-4), (a - b).abs().max()


def test_layers_stack_and_bidirectional():
    torch.manual_seed(0)
    m = R.LSTM(8, 16, num_layers=2, seed=3)
    x = torch.randn(2, 5, 8)
    y = m(x)
    assert y.shape == (2, 5, 16) and m.last_state[0].shape == (2, 2, 16)
    assert torch.allclose(m.bias_ih_l0[16:32], torch.ones(16))  # forget-gate bias init
    bi = R.Bidirectional(R.GRU(8, 16, return_sequences=True, seed=4))
    assert bi(x).shape == (2, 5, 32)
    last = R.RNN(8, 16, return_sequences=False, seed=5)(x)
    assert last.shape == (2, 16)


def test_recurrent_fn_without_initial_state():
    """No h0 / c0: the Function returns no gradient for them."""
    w = [t.requires_grad_(True) for t in _weights("lstm", 8, 16, 7)]
    x = torch.randn(2, 4, 8, requires_grad=True)
    y, h, c = R._RecurrentFn.apply("lstm", x, None, None, *w)
    y.sum().backward()
    assert x.grad is not None and w[0].grad is not None
