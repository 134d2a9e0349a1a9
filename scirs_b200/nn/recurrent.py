"""Recurrent layers: RNN (tanh), LSTM, GRU and Bidirectional.

Batch-first [B, S, F] inputs. Each layer and direction runs one
`_RecurrentFn` whose forward is

    gx = X W_ih^T + b_ih                         one GEMM over all S steps
    for t in 0..S-1:  gh = h_{t-1} W_hh^T + b_hh   (GEMM, [B, H] x [H, G*H])
                      h_t (, c_t) = cell(gx_t, gh)  (pointwise kernel)

and whose backward walks the steps in reverse with the cell-backward kernel
and one [B, G*H] x [G*H, H] GEMM per step for the recurrent gradient, then
computes dX, dW_ih, dW_hh and both bias gradients as whole-sequence GEMMs
and column sums. On CUDA the products run on the framework's tcgen05 GEMM
and the cells on scirs_b200/csrc/rnn.cu (bf16 activations, fp32 cell state;
inputs of other dtypes are computed in bf16 and cast back). Shapes the GEMM
cannot take (hidden or input size not a multiple of 8) and CPU tensors use
the same loop with PyTorch math.

Gate order and semantics follow the reference and PyTorch: LSTM [i, f, g, o],
GRU [r, z, n] with n = tanh(W_in x + b_in + r * (W_hn h + b_hn)). Parameters
per layer k: weight_ih_l{k} [G*H, in], weight_hh_l{k} [G*H, H], bias_ih_l{k},
bias_hh_l{k}; initialisation U(-1/sqrt(H), 1/sqrt(H)), LSTM forget-gate
input bias 1.

Reference parity: scirs2-neural/src/layers/recurrent/{rnn,lstm,gru,cells,
bidirectional}.rs.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from ..ops import kernels as K
from .base import Layer

_GATES = {"rnn": 1, "lstm": 4, "gru": 3}


class _RecurrentFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, kind, x, h0, c0, w_ih, w_hh, b_ih, b_hh):
        B, S, I = x.shape
        GH, H = w_hh.shape
        dev, dt = x.device, x.dtype
        xt = x.transpose(0, 1).contiguous().view(S * B, I)  # time-major rows
        gx = torch.empty(S * B, GH, device=dev, dtype=dt)
        K.gemm(xt, w_ih, gx, bias=b_ih)
        gx = gx.view(S, B, GH)
        hs = torch.empty(S + 1, B, H, device=dev, dtype=dt)
        hs[0] = h0 if h0 is not None else 0
        cs = None
        if kind == "lstm":
            cs = torch.empty(S + 1, B, H, device=dev, dtype=torch.float32)
            cs[0] = c0 if c0 is not None else 0
        acts = torch.empty(S, B, 4 * H, device=dev, dtype=dt) if kind != "rnn" else None
        gh = torch.empty(B, GH, device=dev, dtype=dt)
        for t in range(S):
            K.gemm(hs[t], w_hh, gh, bias=b_hh)
            if kind == "lstm":
                K.lstm_cell_fwd(gx[t], gh, cs[t], cs[t + 1], hs[t + 1], acts[t])
            elif kind == "gru":
                K.gru_cell_fwd(gx[t], gh, hs[t], hs[t + 1], acts[t])
            else:
                K.rnn_cell_fwd(gx[t], gh, hs[t + 1])
        ctx.kind = kind
        ctx.has_b = b_ih is not None
        ctx.has_h0, ctx.has_c0 = h0 is not None, c0 is not None
        ctx.save_for_backward(xt, hs, cs if cs is not None else torch.empty(0, device=dev),
                              acts if acts is not None else torch.empty(0, device=dev), w_ih, w_hh)
        y = hs[1:].transpose(0, 1).contiguous()
        h_last = hs[S].clone()
        c_last = cs[S].clone() if cs is not None else torch.empty(0, device=dev)
        return y, h_last, c_last

    @staticmethod
    def backward(ctx, gy, g_hlast, g_clast):
        kind = ctx.kind
        xt, hs, cs, acts, w_ih, w_hh = ctx.saved_tensors
        S, B, H = hs.shape[0] - 1, hs.shape[1], hs.shape[2]
        GH = w_hh.shape[0]
        dev, dt = hs.device, hs.dtype
        gy_t = (gy if gy is not None else torch.zeros(B, S, H, device=dev, dtype=dt)).transpose(0, 1).contiguous()
        dgx = torch.empty(S, B, GH, device=dev, dtype=dt)
        dgh = torch.empty(S, B, GH, device=dev, dtype=dt) if kind == "gru" else dgx
        dh_next = torch.zeros(B, H, device=dev, dtype=torch.float32)
        if g_hlast is not None:
            dh_next += g_hlast.float()
        dc = None
        if kind == "lstm":
            dc = torch.zeros(B, H, device=dev, dtype=torch.float32)
            if g_clast is not None and g_clast.numel():
                dc += g_clast.float()
        dh_t = torch.empty(B, H, device=dev, dtype=dt)
        dc_new = torch.empty_like(dc) if dc is not None else None
        for t in reversed(range(S)):
            K.add_bf16_f32(gy_t[t], dh_next, dh_t)
            if kind == "lstm":
                K.lstm_cell_bwd(dh_t, dc, acts[t], cs[t], cs[t + 1], dc_new, dgx[t])
                dc, dc_new = dc_new, dc
                K.gemm(dgx[t], w_hh, dh_next, b_mn=True, epi=K.EPI_F32)
            elif kind == "gru":
                K.gru_cell_bwd(dh_t, acts[t], hs[t], dgx[t], dgh[t], dh_next)
                K.gemm(dgh[t], w_hh, dh_next, b_mn=True, epi=K.EPI_F32, accumulate=True)
            else:
                K.rnn_cell_bwd(dh_t, hs[t + 1], dgx[t])
                K.gemm(dgx[t], w_hh, dh_next, b_mn=True, epi=K.EPI_F32)
        dgx2, dgh2 = dgx.view(S * B, GH), dgh.view(S * B, GH)
        dxt = torch.empty_like(xt)
        K.gemm(dgx2, w_ih, dxt, b_mn=True)
        dw_ih = torch.zeros(GH, xt.shape[1], device=dev, dtype=torch.float32)
        K.gemm(dgx2, xt, dw_ih, a_mn=True, b_mn=True, epi=K.EPI_F32)
        dw_hh = torch.zeros(GH, H, device=dev, dtype=torch.float32)
        K.gemm(dgh2, hs[:S].reshape(S * B, H), dw_hh, a_mn=True, b_mn=True, epi=K.EPI_F32)
        db_ih = db_hh = None
        if ctx.has_b:
            db_ih = torch.zeros(GH, device=dev, dtype=torch.float32)
            K.bias_grad(dgx2, db_ih)
            db_hh = torch.zeros(GH, device=dev, dtype=torch.float32)
            K.bias_grad(dgh2, db_hh)
            db_ih, db_hh = db_ih.to(w_ih.dtype), db_hh.to(w_ih.dtype)
        dx = dxt.view(S, B, -1).transpose(0, 1)
        dh0 = dh_next.to(dt) if ctx.has_h0 else None
        dc0 = dc if (kind == "lstm" and ctx.has_c0) else None
        return None, dx, dh0, dc0, dw_ih.to(w_ih.dtype), dw_hh.to(w_hh.dtype), db_ih, db_hh


def _loop_reference(kind, x, h0, c0, w_ih, w_hh, b_ih, b_hh):
    """The same recurrence in PyTorch math (CPU, other shapes)."""
    B, S, _ = x.shape
    H = w_hh.shape[1]
    h = h0 if h0 is not None else x.new_zeros(B, H)
    c = c0 if c0 is not None else x.new_zeros(B, H)
    gx_all = x @ w_ih.t() + (b_ih if b_ih is not None else 0)
    ys = []
    for t in range(S):
        gx = gx_all[:, t]
        gh = h @ w_hh.t() + (b_hh if b_hh is not None else 0)
        if kind == "lstm":
            i, f, g, o = (gx + gh).chunk(4, -1)
            c = torch.sigmoid(f) * c + torch.sigmoid(i) * torch.tanh(g)
            h = torch.sigmoid(o) * torch.tanh(c)
        elif kind == "gru":
            xr, xz, xn = gx.chunk(3, -1)
            hr, hz, hn = gh.chunk(3, -1)
            r, z = torch.sigmoid(xr + hr), torch.sigmoid(xz + hz)
            n = torch.tanh(xn + r * hn)
            h = (1 - z) * n + z * h
        else:
            h = torch.tanh(gx + gh)
        ys.append(h)
    return torch.stack(ys, 1), h, c


def recurrent(kind, x, h0, c0, w_ih, w_hh, b_ih, b_hh):
    """One layer, one direction. Returns (y [B, S, H], h_S, c_S or None)."""
    H, I = w_hh.shape[1], w_ih.shape[1]
    native = x.is_cuda and H % 8 == 0 and I % 8 == 0
    if native:
        dt = x.dtype
        bf = torch.bfloat16
        cast = (lambda t: None if t is None else t.to(bf).contiguous())  # noqa: E731
        y, h, c = _RecurrentFn.apply(kind, cast(x), cast(h0), None if c0 is None else c0.float(), cast(w_ih),
                                     cast(w_hh), cast(b_ih), cast(b_hh))
        return y.to(dt), h.to(dt), (c.to(dt) if kind == "lstm" else None)
    if x.is_cuda:
        from ..ops.functional import _fallback

        _fallback("recurrent", x)
    y, h, c = _loop_reference(kind, x, h0, c0, w_ih, w_hh, b_ih, b_hh)
    return y, h, (c if kind == "lstm" else None)


class _Rec(Layer):
    kind = "rnn"

    def __init__(self, input_size: int, hidden_size: int, num_layers: int = 1, return_sequences: bool = True,
                 bias: bool = True, dtype=torch.float32, device=None, seed=None):
        super().__init__()
        G = _GATES[self.kind]
        self.input_size, self.hidden_size, self.num_layers = input_size, hidden_size, num_layers
        self.return_sequences = return_sequences
        g = torch.Generator().manual_seed(seed) if seed is not None else None
        k = 1.0 / math.sqrt(hidden_size)
        for l in range(num_layers):
            inp = input_size if l == 0 else hidden_size
            u = lambda *s: ((torch.rand(*s, generator=g) * 2 - 1) * k).to(dtype=dtype, device=device)  # noqa: E731
            setattr(self, f"weight_ih_l{l}", nn.Parameter(u(G * hidden_size, inp)))
            setattr(self, f"weight_hh_l{l}", nn.Parameter(u(G * hidden_size, hidden_size)))
            if bias:
                bi = u(G * hidden_size)
                if self.kind == "lstm":  # forget-gate bias 1 (the reference's initialisation)
                    bi[hidden_size:2 * hidden_size] = 1.0
                setattr(self, f"bias_ih_l{l}", nn.Parameter(bi))
                setattr(self, f"bias_hh_l{l}", nn.Parameter(u(G * hidden_size)))
            else:
                setattr(self, f"bias_ih_l{l}", None)
                setattr(self, f"bias_hh_l{l}", None)

    def forward(self, x, state=None):
        h0s = c0s = None
        if state is not None:
            if self.kind == "lstm":
                h0s, c0s = state
            else:
                h0s = state
        hs, cs = [], []
        y = x
        for l in range(self.num_layers):
            h0 = h0s[l] if h0s is not None else None
            c0 = c0s[l] if c0s is not None else None
            y, h, c = recurrent(self.kind, y, h0, c0, getattr(self, f"weight_ih_l{l}"),
                                getattr(self, f"weight_hh_l{l}"), getattr(self, f"bias_ih_l{l}"),
                                getattr(self, f"bias_hh_l{l}"))
            hs.append(h)
            cs.append(c)
        h_n = torch.stack(hs)
        self.last_state = (h_n, torch.stack(cs)) if self.kind == "lstm" else h_n
        return y if self.return_sequences else y[:, -1]


class RNN(_Rec):
    kind = "rnn"


class LSTM(_Rec):
    kind = "lstm"


class GRU(_Rec):
    kind = "gru"


class Bidirectional(Layer):
    """Runs a recurrent layer forward and on the time-reversed input and
    concatenates (or sums) the two output sequences."""

    def __init__(self, forward_layer: _Rec, backward_layer: _Rec | None = None, merge: str = "concat"):
        super().__init__()
        import copy

        self.fwd = forward_layer
        self.bwd = backward_layer if backward_layer is not None else copy.deepcopy(forward_layer)
        self.merge = merge

    def forward(self, x):
        a = self.fwd(x)
        b = self.bwd(torch.flip(x, [1]))
        if b.dim() == 3:
            b = torch.flip(b, [1])
        return torch.cat([a, b], -1) if self.merge == "concat" else a + b
