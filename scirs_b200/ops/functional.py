"""Differentiable ops (torch.autograd.Function) routed to the sm_100a kernels.

These are what the general layer API (:mod:`scirs_b200.nn`) calls. On CUDA
bf16 tensors every forward and backward goes through the native kernels
(tcgen05 GEMM with fused epilogues, flash attention, LayerNorm,
softmax-cross-entropy, embedding). Other dtypes / devices use PyTorch
(fp32 CPU is the reference semantics of the original library).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import kernels as K


def _native(*ts) -> bool:
    return all(t is None or (t.is_cuda and t.dtype == torch.bfloat16) for t in ts)


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
        if pre is not None:
            g2 = (g2.float() * K.gelu_tanh_grad(pre.float())).to(g2.dtype)
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
    return F.layer_norm(x, (x.shape[-1],), w, b, eps)


# ---------------------------------------------------------------------------- attention
class _AttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, scale):
        B, S, H, D = q.shape
        q, k, v = (t if t.stride(-1) == 1 and t.stride(2) == D else t.contiguous() for t in (q, k, v))
        out = torch.empty(B, S, H, D, device=q.device, dtype=q.dtype)
        lse = torch.empty(B, H, S, device=q.device, dtype=torch.float32)
        K.flash_attn_fwd(q, k, v, out, lse, causal, scale)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.causal, ctx.scale = causal, scale
        return out

    @staticmethod
    def backward(ctx, do):
        q, k, v, out, lse = ctx.saved_tensors
        B, S, H, D = q.shape
        do = do.contiguous()
        dq, dk, dv = (torch.empty(B, S, H, D, device=q.device, dtype=q.dtype) for _ in range(3))
        dq_acc = torch.empty(B * S * H * D, device=q.device, dtype=torch.float32)
        delta = torch.empty(B * H * S, device=q.device, dtype=torch.float32)
        K.flash_attn_bwd(do, q, k, v, out, lse, dq, dk, dv, dq_acc, delta, ctx.causal, ctx.scale)
        return dq, dk, dv, None, None


def attention(q, k, v, causal: bool = False, scale: float | None = None):
    """Scaled dot-product attention on [B, S, H, D] tensors (token-major)."""
    scale = scale if scale is not None else q.shape[-1] ** -0.5
    if _native(q, k, v) and q.shape[-1] in (64, 128) and q.shape == k.shape == v.shape:
        return _AttnFn.apply(q, k, v, causal, scale)
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
        return (lg.float() * (g / valid)).to(lg.dtype), None, None


def cross_entropy(logits, targets, ignore_index: int = -100):
    """Mean softmax cross-entropy of logits [M, V] against class indices."""
    if _native(logits) and logits.dim() == 2 and _aligned(logits.shape[1]):
        return _XentFn.apply(logits, targets.long(), ignore_index)
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
    return F.embedding(tok.long(), w)
