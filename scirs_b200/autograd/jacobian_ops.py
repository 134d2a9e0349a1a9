"""Jacobian / JVP / VJP operations and input-domain validation.

Functions take plain callables over torch tensors (the framework layer is
PyTorch: reverse mode is autograd, forward mode is torch.func.jvp, which
carries a tangent through the ops like the reference's dual numbers):

  jacobian_reverse(f, x)     [m, n] by one VJP per output row
  jacobian_forward(f, x)     [m, n] by one JVP per input column
  jacobian_auto(f, x)        forward mode when n <= m, else reverse mode
  jvp_forward(f, x, v)       J v in one forward pass
  vjp_reverse(f, x, u)       u^T J in one backward pass
  vjp_multi(f, xs, u)        u^T J for every input of a multi-input f
  batch_jacobian(f, batch)   per-row Jacobians of a batched f
  numerical_jacobian(f, x, eps)   central differences
  jacobian_check(f, x, tol)  max relative error |a - n| / (1 + |n|) of the
                             analytical against the numerical Jacobian; raises
                             ValueError above tol, returns the error otherwise
  jacobian_diagonal(f, x)    d f_i / d x_i (square f), one JVP per entry

Reference parity: scirs2-autograd/src/jacobian_ops.rs:82-470.
"""
from __future__ import annotations

import torch
from torch.func import jacfwd, jacrev, jvp, vjp, vmap


def _flat(f, shape):
    return lambda z: f(z.reshape(shape)).reshape(-1)


def jacobian_reverse(f, x):
    return jacrev(_flat(f, x.shape))(x.reshape(-1))


def jacobian_forward(f, x):
    return jacfwd(_flat(f, x.shape))(x.reshape(-1))


def jacobian_auto(f, x):
    m = f(x).numel()
    return jacobian_forward(f, x) if x.numel() <= m else jacobian_reverse(f, x)


def jvp_forward(f, x, v):
    if x.shape != v.shape:
        raise ValueError(f"x shape {tuple(x.shape)} != v shape {tuple(v.shape)}")
    return jvp(f, (x,), (v,))[1]


def vjp_reverse(f, x, u):
    y, pull = vjp(f, x)
    if y.shape != u.shape:
        raise ValueError(f"output shape {tuple(y.shape)} != cotangent shape {tuple(u.shape)}")
    return pull(u)[0]


def vjp_multi(f, xs, u):
    y, pull = vjp(f, *xs)
    if y.shape != u.shape:
        raise ValueError(f"output shape {tuple(y.shape)} != cotangent shape {tuple(u.shape)}")
    return list(pull(u))


def batch_jacobian(f, batch):
    """f maps one row [n] to [m]; returns [B, m, n]."""
    return vmap(jacrev(f))(batch)


def numerical_jacobian(f, x, epsilon=1e-6):
    x = x.detach()
    m = f(x).numel()
    flat = x.reshape(-1)
    jac = torch.zeros(m, flat.numel(), dtype=x.dtype, device=x.device)
    for j in range(flat.numel()):
        e = torch.zeros_like(flat)
        e[j] = epsilon
        jac[:, j] = (f((flat + e).reshape(x.shape)).reshape(-1) - f((flat - e).reshape(x.shape)).reshape(-1)) \
            / (2 * epsilon)
    return jac


def jacobian_check(f, x, tolerance=1e-4, epsilon=1e-5):
    a = jacobian_forward(f, x)
    n = numerical_jacobian(f, x, epsilon)
    if a.shape != n.shape:
        raise ValueError(f"analytical shape {tuple(a.shape)} != numerical shape {tuple(n.shape)}")
    err = float(((a - n).abs() / (1 + n.abs())).max()) if a.numel() else 0.0
    if err > tolerance:
        raise ValueError(f"Jacobian check failed: max relative error {err} exceeds tolerance {tolerance}")
    return err


def jacobian_diagonal(f, x):
    flat = x.reshape(-1)
    out = torch.empty_like(flat)
    g = _flat(f, x.shape)
    for i in range(flat.numel()):
        e = torch.zeros_like(flat)
        e[i] = 1
        out[i] = jvp(g, (flat,), (e,))[1][i]
    return out.reshape(x.shape)


# ---------------------------------------------------------------------------- validation
def _finite(t, name, what):
    if not torch.isfinite(t).all():
        raise ValueError(f"{name}: contains non-finite value for {what}")


def validate_sqrt_domain(t, name="tensor"):
    _finite(t, name, "sqrt")
    if (t < 0).any():
        raise ValueError(f"{name}: requires non-negative values for sqrt, found {float(t.min())}")


def validate_log_domain(t, name="tensor"):
    _finite(t, name, "log")
    if (t <= 0).any():
        raise ValueError(f"{name}: requires positive values for log, found {float(t.min())}")


def validate_arcfunc_domain(t, name="tensor", func="asin"):
    _finite(t, name, func)
    if (t.abs() > 1).any():
        raise ValueError(f"{name}: requires values in [-1, 1] for {func}, found {float(t.abs().max())}")


def validate_finite(t, name="tensor"):
    if not torch.isfinite(t).all():
        raise ValueError(f"{name}: contains non-finite values")


def validate_non_nan(t, name="tensor"):
    if torch.isnan(t).any():
        raise ValueError(f"{name}: contains NaN")
