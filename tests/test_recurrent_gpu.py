"""Recurrent layers on the framework's kernels (tcgen05 GEMMs + cell
kernels) against the PyTorch-math recurrence in fp32 on the same
bf16-rounded inputs and weights."""
import pytest
import torch

from scirs_b200.nn import recurrent as R
from scirs_b200.ops import kernels as K

pytestmark = pytest.mark.gpu
G = {"rnn": 1, "lstm": 4, "gru": 3}


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


@pytest.mark.parametrize("kind", ["rnn", "lstm", "gru"])
def test_recurrent_kernels_match_fp32(kind):
    B, S, I, H = 8, 16, 64, 128
    g = torch.Generator().manual_seed(0)
    bf = lambda *s, sc=1.0: (torch.randn(*s, generator=g) * sc).cuda().bfloat16()  # noqa: E731
    w = [bf(G[kind] * H, I, sc=0.1), bf(G[kind] * H, H, sc=0.1), bf(G[kind] * H, sc=0.1), bf(G[kind] * H, sc=0.1)]
    x = bf(B, S, I)
    h0 = bf(B, H, sc=0.5)
    c0 = bf(B, H, sc=0.5).float() if kind == "lstm" else None
    ws = [t.clone().requires_grad_(True) for t in w]
    xs = x.clone().requires_grad_(True)
    k0 = K.STATS.launches
    y, h, c = R.recurrent(kind, xs, h0, c0, *ws)
    assert K.STATS.launches - k0 >= 2 * S  # a GEMM and a cell kernel per step: the native path ran
    wf = [t.float().requires_grad_(True) for t in w]
    xf = x.float().requires_grad_(True)
    yr, hr, cr = R._loop_reference(kind, xf, h0.float(), c0, *wf)
    assert _rel(y, yr) < 2e-2 and _rel(h, hr) < 2e-2
    gy = torch.randn(y.shape, generator=g).cuda().bfloat16()
    grads = torch.autograd.grad(y, [xs] + ws, gy)
    rgrads = torch.autograd.grad(yr, [xf] + wf, gy.float())
    for name, a, b in zip(["x", "w_ih", "w_hh", "b_ih", "b_hh"], grads, rgrads):
        assert _rel(a, b) < 4e-2, (kind, name, _rel(a, b))
    torch.cuda.synchronize()


def test_lstm_layer_on_gpu_trains():
    torch.manual_seed(0)
    m = R.LSTM(32, 64, num_layers=2, seed=1).cuda()
    opt = torch.optim.Adam(m.parameters(), lr=1e-2)
    x = torch.randn(16, 12, 32, device="cuda")
    tgt = torch.randn(16, 12, 64, device="cuda") * 0.1
    losses = []
    for _ in range(20):
        opt.zero_grad()
        loss = ((m(x) - tgt) ** 2).mean()
        loss.backward()
        opt.step()
        losses.append(float(loss))
    assert losses[-1] < 0.5 * losses[0], losses
