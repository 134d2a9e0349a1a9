"""Differentiable ops (torch.autograd.Function) routed to the sm_100a kernels.

These are what the general layer API (:mod:`scirs_b200.nn`) calls. On CUDA
bf16 tensors every forward and backward goes through the native kernels
(tcgen05 GEMM with fused epilogues, flash attention, LayerNorm,
softmax-cross-entropy, embedding). Other dtypes / devices use PyTorch
(fp32 CPU is the reference semantics of the original library).
"""
from __future__ import annotations

import os

import torch
import torch.nn.functional as F

from . import kernels as K


def _native(*ts) -> bool:
    if os.environ.get("SCIRS_KERNELS", "custom") == "torch":  # explicitly requested: no warning
        return False
    return all(t is None or (t.is_cuda and t.dtype == torch.bfloat16) for t in ts)


_warned: set = set()


def _fallback(op: str, *ts):
    """Record (and warn once per op) that a CUDA call is served by PyTorch
    instead of the framework's kernels (dtype other than bf16, or a shape the
    kernels do not take). CPU calls are the reference semantics, not a
    fallback."""
    if os.environ.get("SCIRS_KERNELS", "custom") == "torch":
        return
    if any(t is not None and t.is_cuda for t in ts):
        K.STATS.fallbacks[op] = K.STATS.fallbacks.get(op, 0) + 1
        if op not in _warned:
            import warnings

            _warned.add(op)
            warnings.warn(f"scirs_b200.{op}: CUDA call served by PyTorch (needs bf16 and aligned shapes for the "
                          f"native kernels); counted in ops.kernels.STATS.fallbacks", stacklevel=3)


def _aligned(*dims) -> bool:
    return all(d % 8 == 0 for d in dims)


# ---------------------------------------------------------------------------- linear
class _LinearFn(torch.autograd.Function):
    """y = x @ W (+ b), optional fused GELU. W is [in, out] (the reference
    Dense layout, scirs2-neural/src/layers/dense.rs:82-139) given either as a
    contiguous [in, out] tensor or as the transpose view of a contiguous
    [out, in] (torch Linear layout) tensor; both map onto the GEMM without a
    copy (MN-major or K-major B operand)."""

    @staticmethod
    def forward(ctx, x, w, b, gelu):
        shp = x.shape
        x2 = x.reshape(-1, shp[-1]).contiguous()
        M, N = x2.shape[0], w.shape[1]
        kmaj = not w.is_contiguous()  # w = W_oi.t() with W_oi [out, in] contiguous
        bw = w.t() if kmaj else w
        out = torch.empty(M, N, device=x.device, dtype=x.dtype)
        pre = None
        if gelu:
            pre = torch.empty_like(out)
            K.gemm(x2, bw, out, b_mn=not kmaj, epi=K.EPI_BIAS_GELU, bias=b, out2=pre)
        else:
            K.gemm(x2, bw, out, b_mn=not kmaj, bias=b)
        ctx.save_for_backward(x2, bw, pre)
        ctx.has_b, ctx.kmaj, ctx.shp = b is not None, kmaj, shp
        return out.reshape(*shp[:-1], N)

    @staticmethod
    def backward(ctx, gy):
        x2, bw, pre = ctx.saved_tensors
        kmaj = ctx.kmaj
        n_out = bw.shape[0] if kmaj else bw.shape[1]
        g2 = gy.reshape(-1, n_out).contiguous()
        if pre is not None:  # gradient w.r.t. the pre-activation of the fused bias+GELU epilogue
            g2 = K.dgelu_mul(g2, pre, torch.empty_like(g2))
        dx = torch.empty_like(x2)
        # dX = dY W^T: W[in,out] is a K-major [N=in, K=out] operand; W_oi [out,in] an MN-major one.
        K.gemm(g2, bw, dx, b_mn=kmaj)
        if kmaj:  # grad w.r.t. W_oi [out, in] = dY^T X
            dw32 = torch.zeros(bw.shape, device=bw.device, dtype=torch.float32)
            K.gemm(g2, x2, dw32, a_mn=True, b_mn=True, epi=K.EPI_F32)
            dw = dw32.to(bw.dtype).t()
        else:  # grad w.r.t. W [in, out] = X^T dY
            dw32 = torch.zeros(bw.shape, device=bw.device, dtype=torch.float32)
            K.gemm(x2, g2, dw32, a_mn=True, b_mn=True, epi=K.EPI_F32)
            dw = dw32.to(bw.dtype)
        db = None
        if ctx.has_b:
            db32 = torch.zeros(n_out, device=bw.device, dtype=torch.float32)
            K.bias_grad(g2, db32)
            db = db32.to(bw.dtype)
        return dx.reshape(ctx.shp), dw, db, None


def linear(x, w, b=None, activation: str | None = None):
    """x @ w (+ b), w is [in, out] (contiguous, or the .t() view of an [out, in] tensor)."""
    gelu = activation == "gelu"
    layout_ok = w.dim() == 2 and (w.is_contiguous() or w.t().is_contiguous())
    if _native(x, w, b) and layout_ok and _aligned(w.shape[0], w.shape[1]) and x.shape[-1] == w.shape[0]:
        y = _LinearFn.apply(x, w, b, gelu)
        return y if gelu or activation is None else apply_activation(y, activation)
    _fallback("linear", x, w)
    y = x @ w
    if b is not None:
        y = y + b
    return apply_activation(y, activation)


def apply_activation(y, activation):
    if activation is None or activation == "linear" or activation == "none":
        return y
    a = activation.lower()
    if a == "relu":
        return torch.relu(y)
    if a == "sigmoid":
        return torch.sigmoid(y)
    if a == "tanh":
        return torch.tanh(y)
    if a == "softmax":
        return torch.softmax(y, -1)
    if a == "gelu":
        return F.gelu(y, approximate="tanh")
    if a in ("swish", "silu"):
        return F.silu(y)
    if a == "mish":
        return F.mish(y)
    if a in ("leaky_relu", "leakyrelu"):
        return F.leaky_relu(y, 0.01)
    if a == "elu":
        return F.elu(y)
    raise ValueError(f"unknown activation {activation}")


# ---------------------------------------------------------------------------- layer norm
class _LayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, eps):
        D = x.shape[-1]
        x2 = x.reshape(-1, D).contiguous()
        y = torch.empty_like(x2)
        mu = torch.empty(x2.shape[0], device=x.device, dtype=torch.float32)
        rs = torch.empty_like(mu)
        K.layernorm_fwd(x2, w, b, y, mu, rs, eps)
        ctx.save_for_backward(x2, w, mu, rs)
        ctx.shp = x.shape
        return y.reshape(x.shape)

    @staticmethod
    def backward(ctx, gy):
        x2, w, mu, rs = ctx.saved_tensors
        D = x2.shape[1]
        dx = torch.empty_like(x2)
        dw = torch.zeros(D, device=x2.device, dtype=torch.float32)
        db = torch.zeros_like(dw)
        part = K.ln_partials(x2.shape[0], D, x2.device)
        K.layernorm_bwd(gy.reshape(-1, D).contiguous(), x2, w, mu, rs, dx, dw, db, part)
        return dx.reshape(ctx.shp), dw.to(w.dtype), db.to(w.dtype), None


def layer_norm(x, w, b, eps=1e-5):
    if _native(x, w, b) and _aligned(x.shape[-1]):
        return _LayerNormFn.apply(x, w, b, eps)
    _fallback("layer_norm", x)
    return F.layer_norm(x, (x.shape[-1],), w, b, eps)


# ---------------------------------------------------------------------------- attention
class _AttnFn(torch.autograd.Function):
    """Flash attention on the tcgen05 kernels; q [B, S, H, D], k / v
    [B, Sk, H, D] (Sk may differ: cross-attention); `plan` selects the
    block-sparse / windowed kernels."""

    @staticmethod
    def forward(ctx, q, k, v, causal, scale, plan):
        B, S, H, D = q.shape
        fix = lambda t: t if t.stride(-1) == 1 and t.stride(2) == D and t.stride(0) == t.shape[1] * t.stride(1) \
            else t.contiguous()  # noqa: E731
        q, k, v = fix(q), fix(k), fix(v)
        out = torch.empty(B, S, H, D, device=q.device, dtype=q.dtype)
        lse = torch.empty(B, H, S, device=q.device, dtype=torch.float32)
        K.flash_attn_fwd(q, k, v, out, lse, causal, scale, plan=plan)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.causal, ctx.scale, ctx.plan = causal, scale, plan
        return out

    @staticmethod
    def backward(ctx, do):
        q, k, v, out, lse = ctx.saved_tensors
        B, S, H, D = q.shape
        do = do.contiguous()
        dq = torch.empty_like(q)
        dk = torch.empty(k.shape, device=k.device, dtype=k.dtype)
        dv = torch.empty(v.shape, device=v.device, dtype=v.dtype)
        dq_acc = torch.empty(B * S * H * D, device=q.device, dtype=torch.float32)
        delta = torch.empty(B * H * S, device=q.device, dtype=torch.float32)
        K.flash_attn_bwd(do, q, k, v, out, lse, dq, dk, dv, dq_acc, delta, ctx.causal, ctx.scale, plan=ctx.plan)
        return dq, dk, dv, None, None, None


def attention(q, k, v, causal: bool = False, scale: float | None = None, plan=None):
    """Scaled dot-product attention on [B, S, H, D] tensors (token-major);
    k / v may have another sequence length (cross-attention). `plan`
    (ops.sparse_attention.AttentionPlan) restricts it to a sparse / windowed
    pattern without building a dense mask."""
    scale = scale if scale is not None else q.shape[-1] ** -0.5
    same_kv = k.shape == v.shape and k.shape[0] == q.shape[0] and k.shape[2:] == q.shape[2:]
    if _native(q, k, v) and q.shape[-1] in (64, 128) and same_kv and (not causal or k.shape[1] == q.shape[1]):
        return _AttnFn.apply(q, k, v, causal, scale, plan)
    _fallback("attention", q)
    if plan is not None:
        from .sparse_attention import reference_attention

        o, _ = reference_attention(q, k, v, plan.pattern, scale)
        return o.to(q.dtype)
    o = F.scaled_dot_product_attention(
        q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=causal, scale=scale
    )
    return o.transpose(1, 2)


# ---------------------------------------------------------------------------- cross entropy
class _XentFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, targets, ignore_index):
        M, V = logits.shape
        lg = logits.contiguous().clone()
        loss = torch.empty(M, device=logits.device, dtype=torch.float32)
        valid = (targets != ignore_index).sum().clamp(min=1)
        K.xent_fwd_bwd(lg, targets, loss, V, 1.0, ignore_index)
        ctx.save_for_backward(lg, valid)
        return loss.sum() / valid

    @staticmethod
    def backward(ctx, g):
        lg, valid = ctx.saved_tensors
        dl = K.scale_by(lg, g.float().reshape(1), valid.float().reshape(1), torch.empty_like(lg))
        return dl, None, None


def cross_entropy(logits, targets, ignore_index: int = -100):
    """Mean softmax cross-entropy of logits [M, V] against class indices."""
    if _native(logits) and logits.dim() == 2 and _aligned(logits.shape[1]):
        return _XentFn.apply(logits, targets.long(), ignore_index)
    _fallback("cross_entropy", logits)
    return F.cross_entropy(logits.float(), targets.long(), ignore_index=ignore_index)


# ---------------------------------------------------------------------------- embedding
class _EmbFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tok, w):
        t = tok.reshape(-1).long().contiguous()
        out = torch.empty(t.numel(), w.shape[1], device=w.device, dtype=w.dtype)
        K.embedding_fwd(t, w, None, out, 1)
        ctx.save_for_backward(t)
        ctx.wshape = w.shape
        ctx.shp = tok.shape
        return out.reshape(*tok.shape, w.shape[1])

    @staticmethod
    def backward(ctx, g):
        (t,) = ctx.saved_tensors
        dw = torch.zeros(ctx.wshape, device=g.device, dtype=torch.float32)
        K.embedding_bwd(t, g.reshape(-1, ctx.wshape[1]).contiguous(), dw, None, 1)
        return None, dw.to(g.dtype)


def embedding(tok, w):
    if _native(w) and tok.is_cuda and _aligned(w.shape[1]):
        return _EmbFn.apply(tok, w)
    _fallback("embedding", w)
    return F.embedding(tok.long(), w)


# ---------------------------------------------------------------------------- convolution
def _pair(v):
    return (int(v), int(v)) if isinstance(v, int) else (int(v[0]), int(v[1]))


class _Conv2dFn(torch.autograd.Function):
    """2-D convolution (NCHW, weight [Cout, Cin, KH, KW]) as im2col + the
    tcgen05 GEMM; backward: dgrad GEMM + col2im, wgrad GEMM (fp32), bias
    column sums. Output channels are padded to a multiple of 8 for the GEMM
    (zero weight rows) and sliced off again."""

    @staticmethod
    def forward(ctx, x, w, b, stride, padding, dilation):
        x = x.contiguous()
        N, C, H, W = x.shape
        Cout, _, KH, KW = w.shape
        OH, OW = K.conv_out_hw(H, W, KH, KW, stride, padding, dilation)
        Kd = C * KH * KW
        Kp = (Kd + 7) // 8 * 8
        Np = (Cout + 7) // 8 * 8
        M = N * OH * OW
        cols = torch.empty(M, Kp, device=x.device, dtype=x.dtype)
        K.conv_im2col(x, cols, KH, KW, stride, padding, dilation)
        wp = torch.zeros(Np, Kp, device=w.device, dtype=w.dtype)
        wp[:Cout, :Kd] = w.reshape(Cout, Kd)
        bp = None
        if b is not None:
            bp = torch.zeros(Np, device=b.device, dtype=b.dtype)
            bp[:Cout] = b
        rows = torch.empty(M, Np, device=x.device, dtype=x.dtype)
        K.gemm(cols, wp, rows, bias=bp)
        y = torch.empty(N, Cout, OH, OW, device=x.device, dtype=x.dtype)
        K.conv_rows_to_nchw(rows, y)
        ctx.save_for_backward(cols, wp)
        ctx.geom = (x.shape, w.shape, stride, padding, dilation, Np, Kp)
        ctx.has_b = b is not None
        return y

    @staticmethod
    def backward(ctx, gy):
        cols, wp = ctx.saved_tensors
        xshape, wshape, stride, padding, dilation, Np, Kp = ctx.geom
        N, C, H, W = xshape
        Cout, _, KH, KW = wshape
        gy = gy.contiguous()
        M = cols.shape[0]
        grows = torch.empty(M, Np, device=gy.device, dtype=gy.dtype)
        K.conv_nchw_to_rows(gy, grows)
        dcols = torch.empty(M, Kp, device=gy.device, dtype=gy.dtype)
        K.gemm(grows, wp, dcols, b_mn=True)  # [M, Np] @ [Np, Kp]
        dx = torch.empty(xshape, device=gy.device, dtype=gy.dtype)
        K.conv_col2im(dcols, dx, KH, KW, stride, padding, dilation)
        dw32 = torch.zeros(Np, Kp, device=gy.device, dtype=torch.float32)
        K.gemm(grows, cols, dw32, a_mn=True, b_mn=True, epi=K.EPI_F32)  # [Np, M] @ [M, Kp]
        dw = dw32[:Cout, : C * KH * KW].reshape(wshape).to(wp.dtype)
        db = None
        if ctx.has_b:
            db32 = torch.zeros(Np, device=gy.device, dtype=torch.float32)
            K.bias_grad(grows, db32)
            db = db32[:Cout].to(wp.dtype)
        return dx, dw, db, None, None, None


def conv2d(x, w, b=None, stride=1, padding=0, dilation=1):
    """2-D convolution on the framework's kernels for CUDA tensors (computed
    in bf16, returned in the input dtype); PyTorch on the CPU (the oracle)."""
    stride, padding, dilation = _pair(stride), _pair(padding), _pair(dilation)
    if x.is_cuda and x.dim() == 4:
        dt = x.dtype
        cast = (lambda t: None if t is None else t.to(torch.bfloat16))  # noqa: E731
        y = _Conv2dFn.apply(cast(x), cast(w), cast(b), stride, padding, dilation)
        return y if dt == torch.bfloat16 else y.to(dt)
    return F.conv2d(x, w, b, stride, padding, dilation)


class _Pool2dFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, kernel, stride, padding, is_max, count_pad):
        x = x.contiguous()
        N, C, H, W = x.shape
        OH, OW = K.conv_out_hw(H, W, kernel[0], kernel[1], stride, padding, (1, 1))
        y = torch.empty(N, C, OH, OW, device=x.device, dtype=x.dtype)
        arg = torch.empty(N, C, OH, OW, device=x.device, dtype=torch.int32) if is_max else None
        K.pool2d_fwd(x, y, arg, kernel, stride, padding, is_max, count_pad)
        if arg is not None:
            ctx.save_for_backward(arg)
        ctx.cfg = (x.shape, kernel, stride, padding, is_max, count_pad)
        return y

    @staticmethod
    def backward(ctx, gy):
        xshape, kernel, stride, padding, is_max, count_pad = ctx.cfg
        gy = gy.contiguous()
        if is_max:
            (arg,) = ctx.saved_tensors
            dx = torch.empty(xshape, device=gy.device, dtype=torch.float32)
            K.pool2d_bwd(gy, dx, arg, kernel, stride, padding, True, count_pad)
            dx = dx.to(gy.dtype)
        else:
            dx = torch.empty(xshape, device=gy.device, dtype=gy.dtype)
            K.pool2d_bwd(gy, dx, None, kernel, stride, padding, False, count_pad)
        return dx, None, None, None, None, None


def _pool(x, kernel, stride, padding, is_max, count_pad=True):
    kernel = _pair(kernel)
    stride = _pair(stride if stride is not None else kernel)
    padding = _pair(padding)
    if x.is_cuda and x.dim() == 4:
        dt = x.dtype
        y = _Pool2dFn.apply(x.to(torch.bfloat16), kernel, stride, padding, is_max, count_pad)
        return y if dt == torch.bfloat16 else y.to(dt)
    if is_max:
        return F.max_pool2d(x, kernel, stride, padding)
    return F.avg_pool2d(x, kernel, stride, padding, count_include_pad=count_pad)


def max_pool2d(x, kernel, stride=None, padding=0):
    return _pool(x, kernel, stride, padding, True)


def avg_pool2d(x, kernel, stride=None, padding=0, count_include_pad=True):
    return _pool(x, kernel, stride, padding, False, count_include_pad)
