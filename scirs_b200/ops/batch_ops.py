"""Batched tensor operations with explicit forward and backward functions.

The reference exposes these as free functions over ndarrays (each `*_backward`
takes the forward's inputs or cache and the upstream gradient). Here they take
and return torch tensors; forwards run on the framework's kernels where one
exists (conv2d -> im2col + tcgen05 GEMM, layer_norm -> LayerNorm kernel, on
CUDA), and every backward is the exact vector-Jacobian product of its forward
(autograd over the forward, so the pair is consistent by construction).

Kept as in the reference: names, argument order, NCHW layouts, im2col's
[C*kh*kw, N*OH*OW] column matrix, masks in attention where 0 means "blocked"
(score -1e9), running statistics `momentum * running + (1 - momentum) * batch`
(batch variance, biased), the (x_hat, mean, var, gamma, eps) caches of the
normalisations, LSTM gate order (input, forget, cell, output) with
[4 H, in] / [4 H, H] weights, inverted dropout (mask holds 0 or 1 / keep),
bias-corrected Adam with t starting at 1, and sinusoidal position encodings
(sin on even, cos on odd features, 10000^(2i/d)).

Reference parity: scirs2-neural/src/linalg/batch_operations/{matmul,
convolution, normalization, rnn, attention}.rs.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _vjp(fn, inputs, grad_out):
    xs = [t.detach().requires_grad_(True) for t in inputs]
    with torch.enable_grad():
        out = fn(*xs)
        outs = out if isinstance(out, tuple) else (out,)
        gos = grad_out if isinstance(grad_out, tuple) else (grad_out,)
        grads = torch.autograd.grad(outs, xs, gos, allow_unused=True)
    return tuple(torch.zeros_like(x) if g is None else g for x, g in zip(xs, grads))


# ---------------------------------------------------------------------------- matmul
def batch_matmul(a, b):
    """[B, m, k] @ [B, k, n] -> [B, m, n]."""
    if a.dim() != 3 or b.dim() != 3 or a.shape[0] != b.shape[0] or a.shape[2] != b.shape[1]:
        raise ValueError(f"batch_matmul shapes {tuple(a.shape)} and {tuple(b.shape)} do not match")
    return torch.bmm(a, b)


def batch_vecmat(v, m):
    """[B, k] x [B, k, n] -> [B, n]."""
    if v.dim() != 2 or m.dim() != 3 or v.shape[0] != m.shape[0] or v.shape[1] != m.shape[1]:
        raise ValueError("batch_vecmat shapes do not match")
    return torch.bmm(v.unsqueeze(1), m).squeeze(1)


def batch_matmul_backward(a, b, grad_output):
    return grad_output @ b.transpose(1, 2), a.transpose(1, 2) @ grad_output


# ---------------------------------------------------------------------------- convolution
def conv2d(input, weight, bias=None, stride: int = 1, padding: int = 0):
    from .functional import conv2d as conv

    return conv(input, weight, bias, stride, padding)


def conv2d_backward(dout, input, weight, stride: int = 1, padding: int = 0):
    """(d input, d weight, d bias)."""
    bias = torch.zeros(weight.shape[0], dtype=weight.dtype, device=weight.device)
    gi, gw, gb = _vjp(lambda x, w, b: F.conv2d(x, w, b, stride, padding), (input, weight, bias), dout)
    return gi, gw, gb


def max_pool2d(input, kernel_size: int, stride: int, padding: int = 0):
    """(output, flat argmax indices into each input plane)."""
    return F.max_pool2d(input, kernel_size, stride, padding, return_indices=True)


def max_pool2d_backward(dout, input, indices, kernel_size: int, stride: int, padding: int = 0):
    return F.max_unpool2d(dout, indices, kernel_size, stride, padding, output_size=input.shape[-2:])


def im2col(input, kernel_height: int, kernel_width: int, stride: int = 1, padding: int = 0):
    """[N, C, H, W] -> [C * kh * kw, N * OH * OW] (rows channel-major, then kernel row, kernel column)."""
    cols = F.unfold(input, (kernel_height, kernel_width), padding=padding, stride=stride)  # [N, C*kh*kw, L]
    return cols.permute(1, 0, 2).reshape(cols.shape[1], -1)


def col2im(cols, batch_size, channels, height, width, kernel_height, kernel_width, stride: int = 1,
           padding: int = 0):
    """Adjoint of im2col (overlapping taps summed)."""
    oh = (height + 2 * padding - kernel_height) // stride + 1
    ow = (width + 2 * padding - kernel_width) // stride + 1
    c = cols.reshape(channels * kernel_height * kernel_width, batch_size, oh * ow).permute(1, 0, 2)
    return F.fold(c, (height, width), (kernel_height, kernel_width), padding=padding, stride=stride)


def adaptive_avg_pool2d(input, output_height: int, output_width: int):
    return F.adaptive_avg_pool2d(input, (output_height, output_width))


def adaptive_avg_pool2d_backward(dout, input, output_height: int, output_width: int):
    return _vjp(lambda x: F.adaptive_avg_pool2d(x, (output_height, output_width)), (input,), dout)[0]


# ---------------------------------------------------------------------------- normalisation
def batch_norm_forward(x, gamma, beta, eps, momentum, running_mean, running_var, training: bool = True):
    """x [N, C]. Returns (y, cache or None); updates the running statistics in place when training."""
    if training:
        mean = x.mean(0)
        var = ((x - mean) ** 2).mean(0)
        with torch.no_grad():
            running_mean.mul_(momentum).add_((1 - momentum) * mean)
            running_var.mul_(momentum).add_((1 - momentum) * var)
        x_hat = (x - mean) / torch.sqrt(var + eps)
        return gamma * x_hat + beta, (x_hat, mean, var, gamma, eps)
    x_hat = (x - running_mean) / torch.sqrt(running_var + eps)
    return gamma * x_hat + beta, None


def batch_norm_backward(dout, cache):
    """(dx, dgamma, dbeta) from the training-mode cache."""
    x_hat, mean, var, gamma, eps = cache
    n = dout.shape[0]
    dbeta = dout.sum(0)
    dgamma = (dout * x_hat).sum(0)
    dxh = dout * gamma
    dx = (n * dxh - dxh.sum(0) - x_hat * (dxh * x_hat).sum(0)) / (n * torch.sqrt(var + eps))
    return dx, dgamma, dbeta


def layer_norm(x, gamma, beta, eps):
    """x [N, D] normalised over D. Returns (y, (x_hat, mean, var, gamma, eps))."""
    mean = x.mean(1)
    var = ((x - mean[:, None]) ** 2).mean(1)
    x_hat = (x - mean[:, None]) / torch.sqrt(var + eps)[:, None]
    if x.is_cuda and x.dtype == torch.bfloat16:
        from .functional import layer_norm as ln

        y = ln(x, gamma, beta, eps)
    else:
        y = gamma * x_hat + beta
    return y, (x_hat, mean, var, gamma, eps)


def layer_norm_backward(dout, cache):
    x_hat, mean, var, gamma, eps = cache
    dbeta = dout.sum(0)
    dgamma = (dout * x_hat).sum(0)
    dxh = dout * gamma
    rstd = 1.0 / torch.sqrt(var + eps)
    dx = (dxh - dxh.mean(1, keepdim=True) - x_hat * (dxh * x_hat).mean(1, keepdim=True)) * rstd[:, None]
    return dx, dgamma, dbeta


# ---------------------------------------------------------------------------- recurrent / misc
def lstm_cell(x, h_prev, c_prev, w_ih, w_hh, b_ih, b_hh):
    """One LSTM step. Returns (h_next, c_next, (i, f, g, o))."""
    H = h_prev.shape[1]
    if w_ih.shape != (4 * H, x.shape[1]) or w_hh.shape != (4 * H, H) or b_ih.shape != (4 * H,) \
            or b_hh.shape != (4 * H,):
        raise ValueError("LSTM weights must be [4H, in], [4H, H] and biases [4H]")
    gates = x @ w_ih.t() + b_ih + h_prev @ w_hh.t() + b_hh
    i, f = torch.sigmoid(gates[:, :H]), torch.sigmoid(gates[:, H:2 * H])
    g, o = torch.tanh(gates[:, 2 * H:3 * H]), torch.sigmoid(gates[:, 3 * H:])
    c = f * c_prev + i * g
    return o * torch.tanh(c), c, (i, f, g, o)


def clip_grad_norm(grad, max_norm):
    n = torch.linalg.vector_norm(grad)
    return grad * (max_norm / n) if n > max_norm else grad.clone()


def dropout(x, dropout_rate, generator: torch.Generator | None = None, training: bool = True):
    """(y, mask) with mask in {0, 1 / keep}; identity (mask of ones) when not training or rate 0."""
    if not training or dropout_rate <= 0:
        return x.clone(), torch.ones_like(x)
    if dropout_rate >= 1:
        raise ValueError("dropout rate must be < 1")
    keep = 1.0 - dropout_rate
    mask = (torch.rand(x.shape, generator=generator, device=x.device, dtype=torch.float32) < keep).to(x.dtype) / keep
    return x * mask, mask


def dropout_backward(dout, mask, dropout_rate):
    return dout * mask


def log_softmax(x, dim: int):
    return torch.log_softmax(x, dim=dim)


def adam_update(w, dw, m, v, learning_rate, beta1, beta2, epsilon, t: int):
    """One bias-corrected Adam step (t >= 1). Returns (w_new, m_new, v_new)."""
    if t < 1:
        raise ValueError("Adam step t starts at 1")
    m_new = beta1 * m + (1 - beta1) * dw
    v_new = beta2 * v + (1 - beta2) * dw * dw
    m_hat = m_new / (1 - beta1 ** t)
    v_hat = v_new / (1 - beta2 ** t)
    return w - learning_rate * m_hat / (torch.sqrt(v_hat) + epsilon), m_new, v_new


# ---------------------------------------------------------------------------- attention / transformer
def scaled_dot_product_attention(query, key, value, mask=None):
    """[B, Lq, d] x [B, Lk, d] x [B, Lk, dv]; mask [B, Lq, Lk] with 0 = blocked.
    Returns (output, attention weights)."""
    s = query @ key.transpose(1, 2) / math.sqrt(query.shape[-1])
    if mask is not None:
        s = torch.where(mask == 0, torch.full_like(s, -1e9), s)
    p = torch.softmax(s, dim=-1)
    return p @ value, p


def multi_head_attention(query, key, value, wq, wk, wv, wo, num_heads: int, mask=None):
    """Projections x @ W ([d, d]), num_heads heads, output projection."""
    B, Lq, d = query.shape
    if d % num_heads:
        raise ValueError("d_model must be divisible by num_heads")
    hd = d // num_heads

    def split(t):
        return t.reshape(B, t.shape[1], num_heads, hd).permute(0, 2, 1, 3).reshape(B * num_heads, t.shape[1], hd)

    q, k, v = split(query @ wq), split(key @ wk), split(value @ wv)
    m = None if mask is None else mask.repeat_interleave(num_heads, dim=0)
    o, _ = scaled_dot_product_attention(q, k, v, m)
    o = o.reshape(B, num_heads, Lq, hd).permute(0, 2, 1, 3).reshape(B, Lq, d)
    return o @ wo


def positional_encoding(seq_len: int, d_model: int, max_seq_len: int | None = None, dtype=torch.float64):
    if max_seq_len is not None and seq_len > max_seq_len:
        raise ValueError(f"sequence length {seq_len} exceeds max_seq_len {max_seq_len}")
    pos = torch.arange(seq_len, dtype=torch.float64)[:, None]
    i = torch.arange((d_model + 1) // 2, dtype=torch.float64)[None, :]
    div = 10000.0 ** (2.0 * i / d_model)
    pe = torch.zeros(seq_len, d_model, dtype=torch.float64)
    pe[:, 0::2] = torch.sin(pos / div)[:, : (d_model + 1) // 2]
    pe[:, 1::2] = torch.cos(pos / div)[:, : d_model // 2]
    return pe.to(dtype)


def transformer_ffn(x, w1, b1, w2, b2):
    """relu(x W1 + b1) W2 + b2 with W1 [d, d_ff], W2 [d_ff, d]."""
    return torch.relu(x @ w1 + b1) @ w2 + b2


def transformer_ffn_backward(dout, x, w1, b1, w2, b2):
    """(dx, dW1, db1, dW2, db2)."""
    return _vjp(transformer_ffn, (x, w1, b1, w2, b2), dout)
