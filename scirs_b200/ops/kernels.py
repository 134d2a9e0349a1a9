"""Thin, shape-checked wrappers around the sm_100a kernels.

Every function takes preallocated outputs where the hot path wants them
(no allocation inside a captured CUDA graph) and has a pure-PyTorch path for
CPU tensors. The CPU path is the numerical oracle used by the tests.
"""
from __future__ import annotations

import math
import os

import torch

from .. import _ext

# GEMM epilogues (must match gemm_sm100.cu)
EPI_BF16 = 0
EPI_BIAS_GELU = 1
EPI_RESID = 2
EPI_DGELU = 3
EPI_F32 = 4
EPI_ROPE = 5

OPT_MODES = {"adam": 0, "adamw": 1, "sgd": 2, "rmsprop": 3, "adagrad": 4}

# Attention forward implementation: "tcgen05" (TMEM/TMA kernel) or "mma"
# (warp-level mma.sync kernel). Both are sm_100a kernels of this library.
# Attention forward: "tcgen05" (one 128-query tile per CTA, O in registers),
# "pingpong" (two tiles per CTA, O in TMEM, P through TMEM) or "mma".
ATTN_FWD_IMPL = os.environ.get("SCIRS_ATTN_FWD", "pingpong_x2")
# Attention backward: "tcgen05" (tcgen05 kernels, serial schedule), "tcgen05_pipe"
# (tcgen05 kernels; the tensor core overlaps the softmax-gradient warps),
# "tcgen05_persist" (pipelined; head_dim 64 dense patterns as one persistent CTA
# per SM), "tcgen05_auto" (persistent up to 1,024 keys, pipelined above) or "mma".
ATTN_BWD_IMPL = os.environ.get("SCIRS_ATTN_BWD", "tcgen05_auto")
_BWD_CODES = {"mma": 0, "tcgen05": 1, "tcgen05_pipe": 2, "tcgen05_persist": 3, "tcgen05_auto": 4}


def _shared_sms() -> bool:
    """True inside a multi-rank process group: collective kernels then run next to the attention
    kernels, and the persistent schedules (a fixed work list per CTA, one CTA per SM) would wait
    for whole SMs; the per-tile grids spread over whatever SMs are free."""
    import torch.distributed as dist

    return dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1


def _bwd_code(sparse: bool = False) -> int:
    code = _BWD_CODES.get(ATTN_BWD_IMPL)
    if code is None:
        raise ValueError(f"unknown attention backward implementation {ATTN_BWD_IMPL!r}")
    if code == 4 and _shared_sms():
        code = 2
    return max(code, 1) if sparse else code


def _fwd_persist() -> int:
    """-1: the kernel chooses by size; 0: per-item grid (multi-rank runs, see _shared_sms)."""
    return 0 if _shared_sms() else -1


class _Stats:
    """Counts native kernel launches issued through these wrappers, and the
    layer-API calls on CUDA tensors that PyTorch served instead (per op)."""

    def __init__(self):
        self.launches = 0
        self.fallbacks: dict[str, int] = {}


STATS = _Stats()


def _count(n: int = 1):
    STATS.launches += n


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    """GELU, tanh approximation (the form the reference's CUDA kernel uses,
    scirs2-core/src/gpu/kernels/ml/activation.rs:440-457)."""
    return 0.5 * x * (1.0 + torch.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x * x * x)))


def gelu_tanh_grad(x: torch.Tensor) -> torch.Tensor:
    k0 = math.sqrt(2.0 / math.pi)
    u = k0 * (x + 0.044715 * x**3)
    t = torch.tanh(u)
    return 0.5 * (1 + t) + 0.5 * x * (1 - t * t) * k0 * (1 + 3 * 0.044715 * x * x)


# ---------------------------------------------------------------------------
# GEMM
# ---------------------------------------------------------------------------
def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    out: torch.Tensor,
    *,
    a_mn: bool = False,
    b_mn: bool = False,
    epi: int = EPI_BF16,
    bias: torch.Tensor | None = None,
    aux: torch.Tensor | None = None,
    out2: torch.Tensor | None = None,
    accumulate: bool = False,
    splits: int = 0,
    bn: int = 0,
    bias_grad: torch.Tensor | None = None,
    rope: tuple | None = None,
) -> torch.Tensor:
    """out[M,N] = op(a) @ op(b) with a fused epilogue.

    a: [M,K] (a_mn=False) or [K,M] (a_mn=True); b: [N,K] (b_mn=False, i.e.
    out = a @ b.T) or [K,N] (b_mn=True, out = a @ b).

    Epilogues: EPI_BF16 (+bias), EPI_BIAS_GELU (out2 = pre-activation,
    out = gelu(out2)), EPI_RESID (+bias +aux), EPI_DGELU (out = acc *
    gelu'(aux)), EPI_F32 (fp32 out, optionally accumulated), EPI_ROPE
    (+bias, then the rotary embedding of the first `cols` columns, a fused
    [rows, 3, H, hd] q/k/v output; rope = (cos, sin, S, hd, cols) with fp32
    [S, hd/2] tables, position = row % S). With EPI_DGELU, `bias_grad` (fp32
    [N]) accumulates the column sums of out.
    """
    if a.is_cuda:
        rc, rsn, rS, rhd, rcols = rope if rope is not None else (None, None, 0, 0, 0)
        _ext.kernels().gemm(a, b, out, int(a_mn), int(b_mn), int(epi), bias, aux, out2, accumulate, splits, bn,
                            bias_grad, rc, rsn, int(rS), int(rhd), int(rcols))
        _count(1)
        return out
    A = (a.t() if a_mn else a).float()
    B = (b if b_mn else b.t()).float()
    acc = A @ B
    if epi == EPI_F32:
        if accumulate:
            out.add_(acc)
        else:
            out.copy_(acc)
        return out
    if bias is not None and epi != EPI_DGELU:
        acc = acc + bias.float()
    if epi == EPI_RESID:
        acc = acc + aux.float()
    elif epi == EPI_DGELU:
        acc = acc * gelu_tanh_grad(aux.float())
        if bias_grad is not None:
            bias_grad.add_(acc.sum(0))
    elif epi == EPI_BIAS_GELU:
        out2.copy_(acc)
        acc = gelu_tanh(acc)
    elif epi == EPI_ROPE:
        acc = rope_rotate(acc, *rope)
    out.copy_(acc)
    return out


def rope_rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, S: int, hd: int, cols: int,
                inverse: bool = False) -> torch.Tensor:
    """Half-rotation RoPE of columns [0, cols) of x [rows, N] (heads of hd
    columns; position = row % S): (x1, x2) -> (x1 c - x2 s, x2 c + x1 s)."""
    rows = x.shape[0]
    y = x.float().clone()
    half = hd // 2
    pos = torch.arange(rows, device=x.device) % S
    c = cos.reshape(-1, half)[pos].float()[:, None, :]
    sn = sin.reshape(-1, half)[pos].float()[:, None, :]
    if inverse:
        sn = -sn
    part = y[:, :cols].view(rows, cols // hd, hd)
    x1, x2 = part[..., :half].clone(), part[..., half:].clone()
    part[..., :half] = x1 * c - x2 * sn
    part[..., half:] = x2 * c + x1 * sn
    return y


# ---------------------------------------------------------------------------
# LayerNorm
# ---------------------------------------------------------------------------
def layernorm_fwd(x, w, b, y, mean, rstd, eps=1e-5):
    if x.is_cuda:
        _ext.kernels().layernorm_fwd(x, w, b, y, mean, rstd, float(eps))
        _count(1)
        return y
    xf = x.float()
    mu = xf.mean(-1)
    var = ((xf - mu[..., None]) ** 2).mean(-1)
    rs = torch.rsqrt(var + eps)
    y.copy_((xf - mu[..., None]) * rs[..., None] * w.float() + b.float())
    mean.copy_(mu.reshape(mean.shape))
    rstd.copy_(rs.reshape(rstd.shape))
    return y


def layernorm_bwd(dy, x, w, mean, rstd, dx, dw, db, part, dresid=None, dsum=None):
    """dx = LN backward (+ dresid); dw/db (fp32) are accumulated into, and
    so is dsum (fp32 [D], optional) with the column sums of dx."""
    if x.is_cuda:
        _ext.kernels().layernorm_bwd(dy, x, w, mean, rstd, dresid, dx, dw, db, part, dsum)
        _count(2)
        return dx
    D = x.shape[-1]
    xf = x.float().reshape(-1, D)
    g = dy.float().reshape(-1, D)
    mu = mean.reshape(-1, 1)
    rs = rstd.reshape(-1, 1)
    xh = (xf - mu) * rs
    dw.add_((g * xh).sum(0))
    db.add_(g.sum(0))
    gw = g * w.float()
    o = rs * (gw - gw.mean(-1, keepdim=True) - xh * (gw * xh).mean(-1, keepdim=True))
    if dresid is not None:
        o = o + dresid.float().reshape(-1, D)
    if dsum is not None:
        dsum.add_(o.sum(0))
    dx.copy_(o.reshape(dx.shape))
    return dx


def ln_partials(n_rows: int, D: int, device) -> torch.Tensor:
    """Scratch for LayerNorm backward's per-block partial column sums."""
    if device is not None and torch.device(device).type == "cuda":
        sms = _ext.kernels().num_sms(torch.device(device).index or 0)
        nb = max(1, min(2 * sms, (n_rows + 7) // 8))
    else:
        nb = 1
    return torch.empty(nb * 3 * D, dtype=torch.float32, device=device)


# ---------------------------------------------------------------------------
# Cross entropy
# ---------------------------------------------------------------------------
def xent_fwd_bwd(logits, targets, loss, V, grad_scale, ignore_index=-100):
    """In place: logits <- d(mean loss)/d logits * grad_scale; loss[row] = CE."""
    if logits.is_cuda:
        _ext.kernels().xent_fwd_bwd(logits, targets, loss, int(V), float(grad_scale), int(ignore_index))
        _count(1)
        return loss
    lf = logits[:, :V].float()
    lse = torch.logsumexp(lf, -1)
    valid = (targets != ignore_index) & (targets >= 0) & (targets < V)
    t = targets.clamp(0, V - 1)
    l = lse - lf.gather(1, t[:, None])[:, 0]
    loss.copy_(torch.where(valid, l, torch.zeros_like(l)))
    p = torch.softmax(lf, -1)
    p[torch.arange(p.shape[0]), t] -= 1.0
    p = p * (grad_scale * valid.float())[:, None]
    logits.zero_()
    logits[:, :V].copy_(p)
    return loss


def xent_fwd(logits, targets, loss, V, ignore_index=-100):
    if logits.is_cuda:
        _ext.kernels().xent_fwd(logits, targets, loss, int(V), int(ignore_index))
        _count(1)
        return loss
    lf = logits[:, :V].float()
    lse = torch.logsumexp(lf, -1)
    valid = (targets != ignore_index) & (targets >= 0) & (targets < V)
    t = targets.clamp(0, V - 1)
    l = lse - lf.gather(1, t[:, None])[:, 0]
    loss.copy_(torch.where(valid, l, torch.zeros_like(l)))
    return loss


# ---------------------------------------------------------------------------
# Embedding
# ---------------------------------------------------------------------------
def embedding_fwd(tok, wte, wpe, out, S):
    if tok.is_cuda:
        _ext.kernels().embedding_fwd(tok, wte, wpe, out, int(S))
        _count(1)
        return out
    e = wte.float()[tok.reshape(-1)]
    if wpe is not None:
        pos = torch.arange(tok.numel(), device=tok.device) % S
        e = e + wpe.float()[pos]
    out.copy_(e.reshape(out.shape))
    return out


def embedding_bwd(tok, dout, dwte, dwpe, S):
    if tok.is_cuda:
        _ext.kernels().embedding_bwd(tok, dout, dwte, dwpe, int(S))
        _count(1)
        return
    D = dout.shape[-1]
    g = dout.float().reshape(-1, D)
    if dwte is not None:
        dwte.index_add_(0, tok.reshape(-1), g)
    if dwpe is not None:
        pos = torch.arange(tok.numel(), device=tok.device) % S
        dwpe.index_add_(0, pos, g)


def bias_grad(dy, out):
    """out (fp32, [N]) += column sums of dy [M, N]."""
    if dy.is_cuda:
        _ext.kernels().bias_grad(dy, out)
        _count(1)
        return out
    out.add_(dy.float().sum(0))
    return out


# ---------------------------------------------------------------------------
# Attention
# ---------------------------------------------------------------------------
def attention_reference(q, k, v, causal, scale):
    """fp32 reference: q/k/v [B, S, H, D] -> (o [B,S,H,D], lse [B,H,S])."""
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    s = (qf @ kf.transpose(-1, -2)) * scale
    if causal:
        S = s.shape[-1]
        mask = torch.ones(S, S, dtype=torch.bool, device=s.device).triu(1)
        s = s.masked_fill(mask, float("-inf"))
    lse = torch.logsumexp(s, -1)
    p = torch.softmax(s, -1)
    o = (p @ vf).transpose(1, 2)
    return o, lse


def flash_attn_fwd(q, k, v, out, lse, causal=True, scale=None, plan=None):
    """q/out: [B, S, H, D], k/v: [B, Sk, H, D] token-major views (heads
    contiguous). `plan` (ops.sparse_attention.AttentionPlan) selects the
    sparse / windowed kernels, which visit only the planned key blocks."""
    scale = scale if scale is not None else q.shape[-1] ** -0.5
    if q.is_cuda:
        if plan is not None:
            _ext.kernels().flash_attn_fwd_pp(q, k, v, out, lse, bool(plan.pattern.causal), float(scale), False, None,
                                             False, **plan.kernel_args(), persist=_fwd_persist())
        elif ATTN_FWD_IMPL in ("pingpong", "pingpong_poly", "pingpong_x2", "pingpong_bf2"):
            _ext.kernels().flash_attn_fwd_pp(q, k, v, out, lse, bool(causal), float(scale),
                                             ATTN_FWD_IMPL == "pingpong_poly", None, ATTN_FWD_IMPL == "pingpong_x2",
                                             bf2=ATTN_FWD_IMPL == "pingpong_bf2", persist=_fwd_persist())
        elif ATTN_FWD_IMPL == "tcgen05":
            _ext.kernels().flash_attn_fwd_tc(q, k, v, out, lse, bool(causal), float(scale))
        else:
            _ext.kernels().flash_attn_fwd(q, k, v, out, lse, bool(causal), float(scale))
        _count(1)
        return out
    if plan is not None:
        from .sparse_attention import reference_attention

        o, l = reference_attention(q, k, v, plan.pattern, scale)
    else:
        o, l = attention_reference(q, k, v, causal, scale)
    out.copy_(o)
    lse.copy_(l.reshape(lse.shape))
    return out


def flash_attn_fwd_impl(impl, q, k, v, out, lse, causal=True, scale=None):
    """flash_attn_fwd with an explicit implementation ("pingpong", "tcgen05", "mma")."""
    global ATTN_FWD_IMPL
    old, ATTN_FWD_IMPL = ATTN_FWD_IMPL, impl
    try:
        return flash_attn_fwd(q, k, v, out, lse, causal, scale)
    finally:
        ATTN_FWD_IMPL = old


def flash_attn_bwd(dout, q, k, v, out, lse, dq, dk, dv, dq_acc, delta, causal=True, scale=None, plan=None):
    scale = scale if scale is not None else q.shape[-1] ** -0.5
    if q.is_cuda:
        if plan is not None:
            _ext.kernels().flash_attn_bwd(dout, q, k, v, out, lse, dq, dk, dv, dq_acc, delta,
                                          bool(plan.pattern.causal), float(scale), _bwd_code(True),
                                          **plan.kernel_args(True))
        else:
            _ext.kernels().flash_attn_bwd(dout, q, k, v, out, lse, dq, dk, dv, dq_acc, delta, bool(causal),
                                          float(scale), _bwd_code())
        _count(3)
        return
    with torch.enable_grad():
        qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
        if plan is not None:
            from .sparse_attention import reference_attention

            o, _ = reference_attention(qf, kf, vf, plan.pattern, scale)
        else:
            o, _ = attention_reference(qf, kf, vf, causal, scale)
        gq, gk, gv = torch.autograd.grad(o, (qf, kf, vf), dout.float())
    dq.copy_(gq)
    dk.copy_(gk)
    dv.copy_(gv)


# ---------------------------------------------------------------------------
# Fused optimizer step over flat buffers
# ---------------------------------------------------------------------------
def grad_sumsq(grads, part, hp) -> int:
    """Partial sums of squares of `grads` into part[:n]; returns n. Also
    advances the device-managed step counter (hp[9] when hp[10] != 0), as
    the fused optimizer's own norm pass would."""
    if grads.is_cuda:
        n = _ext.kernels().grad_sumsq(grads, part, hp)
        _count(1)
        return int(n)
    if float(hp[10]) != 0:
        hp[9] += 1
    part[0] = grads.float().pow(2).sum()
    return 1


def optim_step(mode, params, state1, state2, grads, params16, n_decay, hp, part=None, norm_out=None, decay_mask=None,
               parts_ready: int = 0):
    """One fused step; hp (fp32, >= 11 entries) = lr, beta1|momentum|rho, beta2,
    eps, wd, bias_corr1, bias_corr2, grad multiplier, max_norm, step counter,
    device-managed flag. With the flag set (and `part` given) the step counter
    is incremented on the device and the bias corrections derived from it."""
    m = OPT_MODES[mode] if isinstance(mode, str) else int(mode)
    if hp.numel() < 11:
        hp = torch.cat([hp.reshape(-1), torch.zeros(11 - hp.numel(), dtype=hp.dtype, device=hp.device)])
    if params.is_cuda:
        _ext.kernels().optim_step(
            m, params, state1, state2, grads, params16, int(n_decay), decay_mask, hp, part, norm_out, int(parts_ready)
        )
        _count(2 if part is not None and not parts_ready else 1)
        return
    h = hp.tolist()
    lr, b1, b2, eps, wd, bc1, bc2, gmul, max_norm = h[:9]
    if h[10] != 0 and part is not None:
        if not parts_ready:
            hp[9] += 1
        bc1, bc2 = 1 - b1 ** float(hp[9]), 1 - b2 ** float(hp[9])
    g = grads.float() * gmul
    if part is not None:
        if parts_ready:
            norm = math.sqrt(max(float(part[:parts_ready].sum()), 0.0)) * abs(gmul)
        else:
            norm = float(grads.float().norm()) * abs(gmul)
        if norm_out is not None:
            norm_out.fill_(norm)
        if not math.isfinite(norm):
            return
        if max_norm > 0 and norm > max_norm:
            g = g * (max_norm / (norm + 1e-6))
    n = params.numel()
    wdv = torch.zeros(n, dtype=torch.float32, device=params.device)
    if decay_mask is not None:
        wdv = decay_mask.repeat_interleave(64)[:n].float() * wd
    else:
        wdv[:n_decay] = wd
    p = params
    if m in (0, 1):
        if m == 0:
            g = g + wdv * p
        state1.mul_(b1).add_((1 - b1) * g)
        state2.mul_(b2).add_((1 - b2) * g * g)
        mh = state1 / bc1
        vh = state2 / bc2
        if m == 1:
            p.mul_(1 - lr * wdv)
        p.sub_(lr * mh / (vh.sqrt() + eps))
    elif m == 2:
        g = g + wdv * p
        if b1 > 0:
            state1.mul_(b1).add_(lr * g)
            p.sub_(state1)
        else:
            p.sub_(lr * g)
    elif m == 3:
        g = g + wdv * p
        state1.mul_(b1).add_((1 - b1) * g * g)
        p.sub_(lr * g / (state1.sqrt() + eps))
    else:
        g = g + wdv * p
        state1.add_(g * g)
        p.sub_(lr * g / (state1.sqrt() + eps))
    if params16 is not None:
        params16.copy_(p)


# ---------------------------------------------------------------------------
# Vision transformer input
# ---------------------------------------------------------------------------
def patchify(images: torch.Tensor, out: torch.Tensor, patch: int) -> torch.Tensor:
    """images [B, C, H, W] (fp32/bf16) -> out [B*(H/P)*(W/P), C*P*P] bf16,
    columns ordered (c, ky, kx) like a flattened conv weight [E, C, P, P]."""
    if images.is_cuda:
        _ext.kernels().patchify(images, out, int(patch))
        _count(1)
        return out
    B, C, H, W = images.shape
    P = patch
    t = images.reshape(B, C, H // P, P, W // P, P).permute(0, 2, 4, 1, 3, 5)
    out.copy_(t.reshape(out.shape))
    return out


def vit_embed_fwd(pe, cls, pos, x, B: int):
    """x[b, 0] = cls + pos[0]; x[b, 1 + i] = pe[b, i] + pos[1 + i]."""
    if x.is_cuda:
        _ext.kernels().vit_embed_fwd(pe, cls, pos, x, int(B))
        _count(1)
        return x
    T, D = pos.shape
    xv = x.view(B, T, D)
    xv[:, 0] = (cls.float() + pos[0].float()).to(x.dtype)
    xv[:, 1:] = (pe.view(B, T - 1, D).float() + pos[1:].float()).to(x.dtype)
    return x


def vit_embed_bwd(dx, dpe, dpos, dcls, B: int):
    """dpe = dx[:, 1:]; dpos += sum_b dx; dcls += sum_b dx[:, 0]."""
    if dx.is_cuda:
        _ext.kernels().vit_embed_bwd(dx, dpe, dpos, dcls, int(B))
        _count(1)
        return
    T, D = dpos.shape
    d = dx.view(B, T, D).float()
    dpe.copy_(d[:, 1:].reshape(dpe.shape))
    dpos.add_(d.sum(0))
    dcls.add_(d[:, 0].sum(0))


# ---------------------------------------------------------------------------
# Elementwise helpers of the layer API's backward passes
# ---------------------------------------------------------------------------
def dgelu_mul(gy, pre, out):
    """out = gy * gelu'(pre) (tanh form)."""
    if gy.is_cuda:
        _ext.kernels().dgelu_mul(gy, pre, out)
        _count(1)
        return out
    out.copy_(gy.float() * gelu_tanh_grad(pre.float()))
    return out


def scale_by(x, g, count, out):
    """out = x * g / max(count, 1) with g, count fp32 device scalars."""
    if x.is_cuda:
        _ext.kernels().scale_by(x, g, count, out)
        _count(1)
        return out
    out.copy_(x.float() * (g.float() / count.float().clamp(min=1)))
    return out


# ---------------------------------------------------------------------------
# Convolution (implicit GEMM around the tcgen05 GEMM) and pooling
# ---------------------------------------------------------------------------
def conv_out_hw(H, W, KH, KW, stride, padding, dilation):
    sh, sw = stride
    ph, pw = padding
    dh, dw = dilation
    return (H + 2 * ph - dh * (KH - 1) - 1) // sh + 1, (W + 2 * pw - dw * (KW - 1) - 1) // sw + 1


def conv_im2col(x, cols, KH, KW, stride, padding, dilation):
    """cols [N*OH*OW, Kp] (Kp = C*KH*KW rounded up to 8; pad columns zero)."""
    if x.is_cuda:
        _ext.kernels().conv_im2col(x, cols, KH, KW, stride[0], stride[1], padding[0], padding[1], dilation[0],
                                   dilation[1])
        _count(1)
        return cols
    u = torch.nn.functional.unfold(x.float(), (KH, KW), dilation=dilation, padding=padding, stride=stride)
    r = u.transpose(1, 2).reshape(-1, u.shape[1])
    cols.zero_()
    cols[:, : r.shape[1]] = r.to(cols.dtype)
    return cols


def conv_col2im(dcols, dx, KH, KW, stride, padding, dilation):
    if dx.is_cuda:
        _ext.kernels().conv_col2im(dcols, dx, KH, KW, stride[0], stride[1], padding[0], padding[1], dilation[0],
                                   dilation[1])
        _count(1)
        return dx
    N, C, H, W = dx.shape
    OH, OW = conv_out_hw(H, W, KH, KW, stride, padding, dilation)
    K = C * KH * KW
    u = dcols[:, :K].float().reshape(N, OH * OW, K).transpose(1, 2)
    dx.copy_(torch.nn.functional.fold(u, (H, W), (KH, KW), dilation=dilation, padding=padding, stride=stride))
    return dx


def conv_rows_to_nchw(rows, y):
    if y.is_cuda:
        _ext.kernels().conv_rows_nchw(rows, y, True)
        _count(1)
        return y
    N, C, H, W = y.shape
    y.copy_(rows[:, :C].reshape(N, H, W, C).permute(0, 3, 1, 2))
    return y


def conv_nchw_to_rows(y, rows):
    if y.is_cuda:
        _ext.kernels().conv_rows_nchw(rows, y, False)
        _count(1)
        return rows
    N, C, H, W = y.shape
    rows.zero_()
    rows[:, :C] = y.permute(0, 2, 3, 1).reshape(-1, C)
    return rows


def pool2d_fwd(x, y, arg, kernel, stride, padding, is_max, count_pad=True):
    if x.is_cuda:
        _ext.kernels().pool2d_fwd(x, y, arg, kernel[0], kernel[1], stride[0], stride[1], padding[0], padding[1],
                                  bool(is_max), bool(count_pad))
        _count(1)
        return y
    F_ = torch.nn.functional
    if is_max:
        v, i = F_.max_pool2d(x.float(), kernel, stride, padding, return_indices=True)
        y.copy_(v)
        arg.copy_(i)
    else:
        y.copy_(F_.avg_pool2d(x.float(), kernel, stride, padding, count_include_pad=count_pad))
    return y


def pool2d_bwd(dy, dx, arg, kernel, stride, padding, is_max, count_pad=True):
    if dy.is_cuda:
        _ext.kernels().pool2d_bwd(dy, dx, arg, kernel[0], kernel[1], stride[0], stride[1], padding[0], padding[1],
                                  bool(is_max), bool(count_pad))
        _count(1)
        return dx
    N, C, H, W = dx.shape
    if is_max:
        dx.zero_()
        dx.view(N, C, -1).scatter_add_(2, arg.view(N, C, -1).long(), dy.float().view(N, C, -1))
    else:
        with torch.enable_grad():
            xx = torch.zeros(N, C, H, W, requires_grad=True)
            yy = torch.nn.functional.avg_pool2d(xx, kernel, stride, padding, count_include_pad=count_pad)
            (g,) = torch.autograd.grad(yy, xx, dy.float())
        dx.copy_(g)
    return dx


# ---------------------------------------------------------------------------
# Recurrent cells (pointwise part of one time step; see csrc/rnn.cu). The CPU
# branches are the same math in PyTorch and serve as the test oracle.
# ---------------------------------------------------------------------------
def _chk_bf16(*ts):
    for t in ts:
        if t is not None and (t.dtype != torch.bfloat16 or not t.is_contiguous()):
            raise ValueError("recurrent-cell kernels take contiguous bf16 tensors")


def lstm_cell_fwd(gx, gh, c_prev, c_out, h_out, acts):
    if gx.is_cuda:
        _chk_bf16(gx, gh, h_out, acts)
        _ext.kernels().lstm_cell_fwd(gx, gh, c_prev, c_out, h_out, acts)
        _count(1)
        return
    g = gx.float() + (gh.float() if gh is not None else 0.0)
    i, f, gg, o = g.chunk(4, -1)
    i, f, gg, o = torch.sigmoid(i), torch.sigmoid(f), torch.tanh(gg), torch.sigmoid(o)
    c = f * (c_prev if c_prev is not None else 0.0) + i * gg
    c_out.copy_(c)
    h_out.copy_(o * torch.tanh(c))
    acts.copy_(torch.cat([i, f, gg, o], -1))


def lstm_cell_bwd(dh, dc_in, acts, c_prev, c, dc_out, dgates):
    if dh.is_cuda:
        _chk_bf16(dh, acts, dgates)
        _ext.kernels().lstm_cell_bwd(dh, dc_in, acts, c_prev, c, dc_out, dgates)
        _count(1)
        return
    i, f, gg, o = acts.float().chunk(4, -1)
    tc = torch.tanh(c)
    g = dh.float()
    dct = (dc_in if dc_in is not None else 0.0) + g * o * (1 - tc * tc)
    cp = c_prev if c_prev is not None else torch.zeros_like(c)
    dgates.copy_(torch.cat([dct * gg * i * (1 - i), dct * cp * f * (1 - f), dct * i * (1 - gg * gg),
                            g * tc * o * (1 - o)], -1))
    dc_out.copy_(dct * f)


def gru_cell_fwd(gx, gh, h_prev, h_out, acts):
    if gx.is_cuda:
        _chk_bf16(gx, gh, h_prev, h_out, acts)
        _ext.kernels().gru_cell_fwd(gx, gh, h_prev, h_out, acts)
        _count(1)
        return
    xr, xz, xn = gx.float().chunk(3, -1)
    if gh is not None:
        hr, hz, hn = gh.float().chunk(3, -1)
    else:
        hr = hz = hn = torch.zeros_like(xr)
    r, z = torch.sigmoid(xr + hr), torch.sigmoid(xz + hz)
    n = torch.tanh(xn + r * hn)
    hp = h_prev.float() if h_prev is not None else 0.0
    h_out.copy_((1 - z) * n + z * hp)
    acts.copy_(torch.cat([r, z, n, hn], -1))


def gru_cell_bwd(dh, acts, h_prev, dgx, dgh, dh_prev):
    if dh.is_cuda:
        _chk_bf16(dh, acts, h_prev, dgx, dgh)
        _ext.kernels().gru_cell_bwd(dh, acts, h_prev, dgx, dgh, dh_prev)
        _count(1)
        return
    r, z, n, hn = acts.float().chunk(4, -1)
    g = dh.float()
    hp = h_prev.float() if h_prev is not None else torch.zeros_like(g)
    dn = g * (1 - z) * (1 - n * n)
    dz = g * (hp - n) * z * (1 - z)
    dr = dn * hn * r * (1 - r)
    dgx.copy_(torch.cat([dr, dz, dn], -1))
    dgh.copy_(torch.cat([dr, dz, dn * r], -1))
    dh_prev.copy_(g * z)


def rnn_cell_fwd(gx, gh, h_out):
    if gx.is_cuda:
        _chk_bf16(gx, gh, h_out)
        _ext.kernels().rnn_cell_fwd(gx, gh, h_out)
        _count(1)
        return
    h_out.copy_(torch.tanh(gx.float() + (gh.float() if gh is not None else 0.0)))


def rnn_cell_bwd(dh, h, dg):
    if dh.is_cuda:
        _chk_bf16(dh, h, dg)
        _ext.kernels().rnn_cell_bwd(dh, h, dg)
        _count(1)
        return
    y = h.float()
    dg.copy_(dh.float() * (1 - y * y))


def add_bf16_f32(a, b, out):
    """out (bf16) = a (bf16) + b (fp32, or None)."""
    if a.is_cuda:
        _chk_bf16(a, out)
        _ext.kernels().add_bf16_f32(a, b, out)
        _count(1)
        return out
    out.copy_(a.float() + (b if b is not None else 0.0))
    return out
