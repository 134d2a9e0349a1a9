"""Functional attention (scirs_b200.linalg) against float64 restatements of
the reference's definitions (scirs2-linalg/src/attention/*), on the CPU."""
import math

import pytest
import torch

from scirs_b200 import linalg as L

torch.manual_seed(0)


def _t(*s):
    return torch.randn(*s, dtype=torch.float64)


def _softmax_rows(s):
    m = s.max(-1, keepdim=True).values
    e = torch.exp(s - m)
    return e / e.sum(-1, keepdim=True)


def _loop_attention(q, k, v, scale, bias=None, allowed=None):
    B, Lq, _ = q.shape
    out = torch.zeros(B, Lq, v.shape[-1], dtype=q.dtype)
    for b in range(B):
        for i in range(Lq):
            idx = [j for j in range(k.shape[1]) if allowed is None or allowed[i][j]]
            if not idx:
                continue
            sc = torch.stack([(q[b, i] * k[b, j]).sum() * scale + (0 if bias is None else bias[i][j]) for j in idx])
            p = _softmax_rows(sc[None])[0]
            out[b, i] = sum(p[n] * v[b, j] for n, j in enumerate(idx))
    return out


def test_sdpa_masks_and_flash_blocks():
    q, k, v = _t(2, 5, 8), _t(2, 7, 8), _t(2, 7, 6)
    sc = 0.3
    ref = _loop_attention(q, k, v, sc)
    assert torch.allclose(L.scaled_dot_product_attention(q, k, v, scale=sc), ref, atol=1e-10)
    for bs in (1, 3, 64):
        assert torch.allclose(L.flash_attention(q, k, v, scale=sc, block_size=bs), ref, atol=1e-10)
    allowed = torch.rand(5, 7) > 0.4
    allowed[:, 0] = True
    ref_b = _loop_attention(q, k, v, sc, allowed=allowed.tolist())
    m = L.AttentionMask.boolean(allowed[None])
    assert torch.allclose(L.masked_attention(q, k, v, m, sc), ref_b, atol=1e-10)
    assert torch.allclose(L.flash_attention(q, k, v, m, sc, block_size=2), ref_b, atol=1e-10)
    add = _t(1, 5, 7)
    ref_a = _loop_attention(q, k, v, sc, bias=add[0].tolist())
    assert torch.allclose(L.masked_attention(q, k, v, L.AttentionMask.additive(add), sc), ref_a, atol=1e-10)
    mul = torch.rand(1, 5, 7, dtype=torch.float64)
    p = _softmax_rows(torch.matmul(q, k.transpose(-1, -2)) * sc) * mul
    assert torch.allclose(L.masked_attention(q, k, v, L.AttentionMask.multiplicative(mul), sc), p @ v, atol=1e-10)
    qc, kc, vc = _t(2, 6, 8), _t(2, 6, 8), _t(2, 6, 8)
    tri = [[j <= i for j in range(6)] for i in range(6)]
    ref_c = _loop_attention(qc, kc, vc, sc, allowed=tri)
    assert torch.allclose(L.causal_attention(qc, kc, vc, sc), ref_c, atol=1e-10)
    assert torch.allclose(L.flash_attention(qc, kc, vc, L.AttentionMask.causal(), sc, 4), ref_c, atol=1e-10)


def test_sparse_alibi_rotary():
    q, k, v = _t(1, 4, 6), _t(1, 5, 6), _t(1, 5, 3)
    pat = torch.tensor([[1, 0, 1, 0, 0], [0, 0, 0, 0, 0], [1, 1, 1, 1, 1], [0, 0, 0, 1, 0]], dtype=torch.bool)
    out = L.sparse_attention(q, k, v, pat, 0.5)
    assert torch.allclose(out, _loop_attention(q, k, v, 0.5, allowed=pat.tolist()), atol=1e-10)
    assert torch.all(out[0, 1] == 0)  # a row with no attended key is zero
    slopes = torch.tensor([0.25, 0.5], dtype=torch.float64)
    bias = [[-0.25 * abs(i - j) for j in range(5)] for i in range(4)]
    assert torch.allclose(L.attention_with_alibi(q, k, v, slopes, 0.5), _loop_attention(q, k, v, 0.5, bias=bias),
                          atol=1e-10)
    tri = [[j <= i for j in range(5)] for i in range(4)]
    assert torch.allclose(L.attention_with_alibi(q, k, v, slopes, 0.5, causal=True),
                          _loop_attention(q, k, v, 0.5, bias=bias, allowed=tri), atol=1e-10)
    x = _t(2, 3, 6)
    r = L.rotary_embedding(x, 100.0)
    for pos in range(3):
        for i in range(3):
            th = pos * 100.0 ** (-2.0 * i / 6)
            a, b = x[:, pos, 2 * i], x[:, pos, 2 * i + 1]
            assert torch.allclose(r[:, pos, 2 * i], a * math.cos(th) - b * math.sin(th))
            assert torch.allclose(r[:, pos, 2 * i + 1], a * math.sin(th) + b * math.cos(th))
    with pytest.raises(ValueError):
        L.rotary_embedding(_t(1, 2, 5))


def test_linear_and_relative_position():
    q, k, v = _t(2, 4, 5), _t(2, 6, 5), _t(2, 6, 3)
    sc = 0.7
    fm = lambda x: torch.where(x > 0, x + 1, torch.exp(x))  # noqa: E731  elu(x) + 1
    out = L.linear_attention(q, k, v, sc)
    for b in range(2):
        qp, kp = fm(q[b]), fm(k[b] * sc)
        for i in range(4):
            z = (qp[i] * kp.sum(0)).sum()
            num = sum(qp[i][j] * (kp[:, j:j + 1] * v[b]).sum(0) for j in range(5))
            assert torch.allclose(out[b, i], num / z, atol=1e-10)
    rel = _t(2 * 6 - 1, 5)
    bias_out = L.relative_position_attention(q, k, v, rel, sc)
    for b in range(2):
        for i in range(4):
            s = torch.stack([((q[b, i] * k[b, j]).sum() + (q[b, i] * rel[(6 - 1) + i - j]).sum()) * sc
                             for j in range(6)])
            p = _softmax_rows(s[None])[0]
            assert torch.allclose(bias_out[b, i], (p[:, None] * v[b]).sum(0), atol=1e-10)
    assert torch.allclose(L.attention_with_rpe(q, k, v, rel, sc), bias_out)
    with pytest.raises(ValueError):
        L.relative_position_attention(q, k, v, _t(3, 5), sc)
    xq = q * torch.tensor([[(p + 1) ** (-(j / 5)) for j in range(5)] for p in range(4)], dtype=torch.float64)
    xk = k * torch.tensor([[(p + 1) ** (-(j / 5)) for j in range(5)] for p in range(6)], dtype=torch.float64)
    assert torch.allclose(L.attention_with_rpe(q, k, v, rel, sc, use_xpos=True), _loop_attention(xq, xk, v, sc),
                          atol=1e-10)


def test_multi_head_and_grouped_query():
    B, Lq, Lk, d, H = 2, 3, 4, 8, 2
    q, k, v = _t(B, Lq, d), _t(B, Lk, d), _t(B, Lk, d)
    wq, wk, wv, wo = _t(d, d), _t(d, d), _t(d, d), _t(d, d)
    cfg = L.AttentionConfig(num_heads=H, head_dim=d // H)
    out = L.multi_head_attention(q, k, v, wq, wk, wv, wo, None, cfg)
    Q, K, V = q @ wq, k @ wk, v @ wv
    heads = [_loop_attention(Q[..., h * 4:(h + 1) * 4], K[..., h * 4:(h + 1) * 4], V[..., h * 4:(h + 1) * 4], 0.5)
             for h in range(H)]
    assert torch.allclose(out, torch.cat(heads, -1) @ wo, atol=1e-10)
    # grouped: 4 query heads over 2 kv heads, head_dim 2
    Hq, Hkv, hd = 4, 2, 2
    wk2, wv2 = _t(d, Hkv * hd), _t(d, Hkv * hd)
    out = L.grouped_query_attention(q, k, v, wq, wk2, wv2, wo, None, Hq, Hkv, 0.4)
    Q, K, V = q @ wq, k @ wk2, v @ wv2
    heads = []
    for h in range(Hq):
        g = h // (Hq // Hkv)
        heads.append(_loop_attention(Q[..., h * hd:(h + 1) * hd], K[..., g * hd:(g + 1) * hd],
                                     V[..., g * hd:(g + 1) * hd], 0.4))
    assert torch.allclose(out, torch.cat(heads, -1) @ wo, atol=1e-10)
    with pytest.raises(ValueError):
        L.grouped_query_attention(q, k, v, wq, wk2, wv2, wo, None, 3, 2, 0.4)


def test_gradients_flow():
    q, k, v = (_t(1, 5, 4).requires_grad_(True) for _ in range(3))
    for fn in (lambda: L.linear_attention(q, k, v), lambda: L.flash_attention(q, k, v, block_size=2),
               lambda: L.relative_position_attention(q, k, v, _t(9, 4))):
        q.grad = k.grad = v.grad = None
        fn().sum().backward()
        assert all(t.grad is not None and torch.isfinite(t.grad).all() for t in (q, k, v))
