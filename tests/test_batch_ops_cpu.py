"""Batched operations with explicit backward functions (CPU, float64): each
backward against autograd of a plain restatement, layouts against loops."""
import math

import torch

from scirs_b200.ops import batch_ops as O

torch.manual_seed(0)
D = torch.float64


def _grad(fn, inputs, dout):
    xs = [t.clone().requires_grad_(True) for t in inputs]
    fn(*xs).backward(dout)
    return [x.grad for x in xs]


def test_matmul_and_conv_family():
    a, b = torch.randn(3, 4, 5, dtype=D), torch.randn(3, 5, 2, dtype=D)
    assert torch.allclose(O.batch_matmul(a, b), a @ b)
    go = torch.randn(3, 4, 2, dtype=D)
    ga, gb = O.batch_matmul_backward(a, b, go)
    ra, rb = _grad(lambda x, y: x @ y, (a, b), go)
    assert torch.allclose(ga, ra) and torch.allclose(gb, rb)
    v = torch.randn(3, 5, dtype=D)
    assert torch.allclose(O.batch_vecmat(v, b), torch.einsum("bk,bkn->bn", v, b))
    x, w, bias = torch.randn(2, 3, 7, 6, dtype=D), torch.randn(4, 3, 3, 3, dtype=D), torch.randn(4, dtype=D)
    y = O.conv2d(x, w, bias, 2, 1)
    assert torch.allclose(y, torch.nn.functional.conv2d(x, w, bias, 2, 1))
    go = torch.randn_like(y)
    gi, gw, gbias = O.conv2d_backward(go, x, w, 2, 1)
    ri, rw, rbias = _grad(lambda a, b, c: torch.nn.functional.conv2d(a, b, c, 2, 1), (x, w, bias), go)
    assert torch.allclose(gi, ri) and torch.allclose(gw, rw) and torch.allclose(gbias, rbias)
    cols = O.im2col(x, 3, 3, 2, 1)
    oh, ow = 4, 3
    assert cols.shape == (3 * 9, 2 * oh * ow)
    xp = torch.nn.functional.pad(x, (1, 1, 1, 1))
    assert torch.allclose(cols[1 * 9 + 2 * 3 + 1, 1 * oh * ow + 2 * ow + 1], xp[1, 1, 2 * 2 + 2, 1 * 2 + 1])
    # col2im is the adjoint of im2col: <im2col(x), c> = <x, col2im(c)>
    c = torch.randn_like(cols)
    lhs = (O.im2col(x, 3, 3, 2, 1) * c).sum()
    rhs = (x * O.col2im(c, 2, 3, 7, 6, 3, 3, 2, 1)).sum()
    assert torch.allclose(lhs, rhs)
    out, idx = O.max_pool2d(x, 2, 2)
    go = torch.randn_like(out)
    assert torch.allclose(O.max_pool2d_backward(go, x, idx, 2, 2),
                          _grad(lambda t: torch.nn.functional.max_pool2d(t, 2, 2), (x,), go)[0])
    ap = O.adaptive_avg_pool2d(x, 2, 3)
    go = torch.randn_like(ap)
    assert torch.allclose(O.adaptive_avg_pool2d_backward(go, x, 2, 3),
                          _grad(lambda t: torch.nn.functional.adaptive_avg_pool2d(t, (2, 3)), (x,), go)[0])


def test_norms_lstm_dropout_adam():
    x, g, b = torch.randn(8, 5, dtype=D), torch.rand(5, dtype=D) + 0.5, torch.randn(5, dtype=D)
    rm, rv = torch.zeros(5, dtype=D), torch.ones(5, dtype=D)
    y, cache = O.batch_norm_forward(x, g, b, 1e-5, 0.9, rm, rv, True)
    assert torch.allclose(rm, 0.1 * x.mean(0)) and torch.allclose(rv, 0.9 + 0.1 * x.var(0, unbiased=False))
    go = torch.randn_like(y)
    dx, dg, db = O.batch_norm_backward(go, cache)
    bn = lambda t, gg, bb: (t - t.mean(0)) / torch.sqrt(t.var(0, unbiased=False) + 1e-5) * gg + bb  # noqa: E731
    r = _grad(bn, (x, g, b), go)
    assert torch.allclose(dx, r[0]) and torch.allclose(dg, r[1]) and torch.allclose(db, r[2])
    y2, c2 = O.layer_norm(x, g, b, 1e-5)
    assert torch.allclose(y2, torch.nn.functional.layer_norm(x, (5,), g, b, 1e-5))
    dx, dg, db = O.layer_norm_backward(go, c2)
    r = _grad(lambda t, gg, bb: torch.nn.functional.layer_norm(t, (5,), gg, bb, 1e-5), (x, g, b), go)
    assert torch.allclose(dx, r[0]) and torch.allclose(dg, r[1]) and torch.allclose(db, r[2])
    H, I, B = 3, 4, 2
    w_ih, w_hh = torch.randn(4 * H, I, dtype=D), torch.randn(4 * H, H, dtype=D)
    b_ih, b_hh = torch.randn(4 * H, dtype=D), torch.randn(4 * H, dtype=D)
    xi, h0, c0 = torch.randn(B, I, dtype=D), torch.randn(B, H, dtype=D), torch.randn(B, H, dtype=D)
    h1, c1, _ = O.lstm_cell(xi, h0, c0, w_ih, w_hh, b_ih, b_hh)
    cell = torch.nn.LSTMCell(I, H).double()
    with torch.no_grad():
        cell.weight_ih.copy_(w_ih), cell.weight_hh.copy_(w_hh), cell.bias_ih.copy_(b_ih), cell.bias_hh.copy_(b_hh)
        rh, rc = cell(xi, (h0, c0))
    assert torch.allclose(h1, rh) and torch.allclose(c1, rc)
    y, m = O.dropout(torch.ones(1000, dtype=D), 0.25, torch.Generator().manual_seed(1))
    assert set(torch.unique(m).tolist()) <= {0.0, 1 / 0.75} and 0.65 < float((m > 0).double().mean()) < 0.85
    assert torch.equal(O.dropout_backward(torch.ones(1000, dtype=D), m, 0.25), m)
    gr = torch.tensor([3.0, 4.0], dtype=D)
    assert torch.allclose(O.clip_grad_norm(gr, 1.0), gr / 5)
    w, dw = torch.randn(6, dtype=D), torch.randn(6, dtype=D)
    wn, mn, vn = O.adam_update(w, dw, torch.zeros(6, dtype=D), torch.zeros(6, dtype=D), 0.1, 0.9, 0.999, 1e-8, 1)
    assert torch.allclose(wn, w - 0.1 * dw / (dw.abs() + 1e-8))
    assert torch.allclose(O.log_softmax(x, 1), torch.log_softmax(x, 1))


def test_attention_transformer_and_positions():
    q, k, v = torch.randn(2, 3, 4, dtype=D), torch.randn(2, 5, 4, dtype=D), torch.randn(2, 5, 6, dtype=D)
    mask = torch.ones(2, 3, 5, dtype=D)
    mask[:, :, 3:] = 0
    o, p = O.scaled_dot_product_attention(q, k, v, mask)
    ref = torch.softmax((q @ k.transpose(1, 2)) / 2 + torch.where(mask == 0, -1e9, 0.0), -1)
    assert torch.allclose(p, ref) and torch.allclose(o, ref @ v) and float(p[..., 3:].abs().max()) < 1e-12
    d, H = 8, 2
    qq = torch.randn(2, 3, d, dtype=D)
    ws = [torch.randn(d, d, dtype=D) for _ in range(4)]
    out = O.multi_head_attention(qq, qq, qq, *ws, H)
    Q, K, V = qq @ ws[0], qq @ ws[1], qq @ ws[2]
    heads = [torch.softmax(Q[..., h * 4:(h + 1) * 4] @ K[..., h * 4:(h + 1) * 4].transpose(1, 2) / 2, -1)
             @ V[..., h * 4:(h + 1) * 4] for h in range(H)]
    assert torch.allclose(out, torch.cat(heads, -1) @ ws[3])
    pe = O.positional_encoding(5, 6)
    assert abs(float(pe[3, 2]) - math.sin(3 / 10000 ** (2 / 6))) < 1e-12
    assert abs(float(pe[3, 5]) - math.cos(3 / 10000 ** (4 / 6))) < 1e-12
    x = torch.randn(2, 3, 4, dtype=D)
    w1, b1, w2, b2 = torch.randn(4, 7, dtype=D), torch.randn(7, dtype=D), torch.randn(7, 4, dtype=D), torch.randn(4, dtype=D)
    y = O.transformer_ffn(x, w1, b1, w2, b2)
    go = torch.randn_like(y)
    grads = O.transformer_ffn_backward(go, x, w1, b1, w2, b2)
    ref = _grad(lambda a, b, c, d2, e: torch.relu(a @ b + c) @ d2 + e, (x, w1, b1, w2, b2), go)
    assert all(torch.allclose(g1, g2) for g1, g2 in zip(grads, ref))
