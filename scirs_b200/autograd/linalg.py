"""Differentiable matrix decompositions and solvers for the graph API.

The forward passes call the LAPACK / cuSOLVER routines behind
``torch.linalg``; the backward passes are written out here from the
matrix-calculus identities below (each is a differentiable composition of
torch ops, so grad-of-grad works through them):

  inverse        Y = A^-1:            dA = -Y^T dY Y^T
  determinant    d = det A:           dA = dd * d * A^-T
  slogdet        l = log|det A|:      dA = dl * A^-T
  cholesky       A = L L^T:           S = L^-T Phi(L^T dL) L^-1, dA = (S + S^T) / 2
                 (Phi keeps the lower triangle and halves the diagonal)
  eigh           A = V diag(w) V^T:   dA = V (diag(dw) + F o (V^T dV)) V^T, symmetrised,
                 F_ij = 1 / (w_j - w_i) off the diagonal
  qr (m >= n)    A = Q R:             M = R dR^T - dQ^T Q,
                 dA = (dQ + Q copyltu(M)) R^-T, copyltu(M) = tril(M) + tril(M, -1)^T
  svd (reduced)  A = U diag(s) V^T:   F_ij = 1 / (s_j^2 - s_i^2) off the diagonal,
                 dA = U [(F o (U^T dU - dU^T U)) S + diag(ds) + S (F o (V^T dV - dV^T V))] V^T
                      + (I - U U^T) dU S^-1 V^T + U S^-1 dV^T (I - V V^T)
  cholesky_solve X = (L L^T)^-1 B:    dB = (L L^T)^-1 dX, dL = -(dB X^T + X dB^T) L

Eigen- and singular-vector gradients assume distinct eigen / singular
values (the formulas divide by their differences); losses that depend on
the vectors only up to sign (products like U V^T or V o V) are well defined.

Reference parity: scirs2-autograd/src/tensor_ops/decomposition_ops.rs:534
(qr), :562 (svd), :749 (cholesky); eigen_ops.rs:783 (eigen);
matrix_ops.rs:855,882 (matrix_inverse, determinant); matrix_solvers.rs:862
(cholesky_solve). Gradients are checked by finite differences in float64.
"""
from __future__ import annotations

import torch


def _t(x: torch.Tensor) -> torch.Tensor:
    return x.transpose(-1, -2)


def _sym(x: torch.Tensor) -> torch.Tensor:
    return 0.5 * (x + _t(x))


def _offdiag_inv_diff(v: torch.Tensor) -> torch.Tensor:
    """F_ij = 1 / (v_j - v_i) for i != j, 0 on the diagonal."""
    d = v.unsqueeze(-2) - v.unsqueeze(-1)
    eye = torch.eye(v.shape[-1], dtype=torch.bool, device=v.device)
    return torch.where(eye, torch.zeros_like(d), 1.0 / torch.where(eye, torch.ones_like(d), d))


class Inverse(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a):
        y = torch.linalg.inv(a)
        ctx.save_for_backward(y)
        return y

    @staticmethod
    def backward(ctx, gy):
        (y,) = ctx.saved_tensors
        return -_t(y) @ gy @ _t(y)


class Determinant(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a):
        d = torch.linalg.det(a)
        ctx.save_for_backward(a, d)
        return d

    @staticmethod
    def backward(ctx, gd):
        a, d = ctx.saved_tensors
        return (gd * d).unsqueeze(-1).unsqueeze(-1) * _t(torch.linalg.inv(a))


class LogAbsDet(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a):
        _, la = torch.linalg.slogdet(a)
        ctx.save_for_backward(a)
        return la

    @staticmethod
    def backward(ctx, gl):
        (a,) = ctx.saved_tensors
        return gl.unsqueeze(-1).unsqueeze(-1) * _t(torch.linalg.inv(a))


class Cholesky(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a):
        low = torch.linalg.cholesky(a)
        ctx.save_for_backward(low)
        return low

    @staticmethod
    def backward(ctx, gl):
        (low,) = ctx.saved_tensors
        p = _t(low) @ gl
        p = torch.tril(p) - 0.5 * torch.diag_embed(torch.diagonal(p, dim1=-2, dim2=-1))
        # S = L^-T P L^-1 via two triangular solves
        s = torch.linalg.solve_triangular(_t(low), p, upper=True)
        s = _t(torch.linalg.solve_triangular(_t(low), _t(s), upper=True))
        return _sym(s)


class Eigh(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a):
        w, v = torch.linalg.eigh(a)
        ctx.save_for_backward(w, v)
        return w, v

    @staticmethod
    def backward(ctx, gw, gv):
        w, v = ctx.saved_tensors
        inner = torch.zeros_like(v)
        if gw is not None:
            inner = inner + torch.diag_embed(gw)
        if gv is not None:
            inner = inner + _offdiag_inv_diff(w) * (_t(v) @ gv)
        return _sym(v @ inner @ _t(v))


class QR(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a):
        if a.shape[-2] < a.shape[-1]:
            raise ValueError("qr gradient is implemented for m >= n (reduced factorisation)")
        q, r = torch.linalg.qr(a, mode="reduced")
        ctx.save_for_backward(q, r)
        return q, r

    @staticmethod
    def backward(ctx, gq, gr):
        q, r = ctx.saved_tensors
        gq = torch.zeros_like(q) if gq is None else gq
        gr = torch.zeros_like(r) if gr is None else gr
        m = r @ _t(gr) - _t(gq) @ q
        copyltu = torch.tril(m) + _t(torch.tril(m, -1))
        rhs = gq + q @ copyltu
        # dA = rhs R^-T  <=>  dA R^T = rhs  <=>  R dA^T = rhs^T
        return _t(torch.linalg.solve_triangular(r, _t(rhs), upper=True))


class SVD(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a):
        u, s, vh = torch.linalg.svd(a, full_matrices=False)
        v = _t(vh)
        ctx.save_for_backward(u, s, v)
        return u, s, v

    @staticmethod
    def backward(ctx, gu, gs, gv):
        u, s, v = ctx.saved_tensors
        k = s.shape[-1]
        f = _offdiag_inv_diff(s * s)
        smat = torch.diag_embed(s)
        sinv = torch.diag_embed(1.0 / s)
        inner = torch.zeros(u.shape[:-2] + (k, k), dtype=u.dtype, device=u.device)
        out = 0.0
        if gs is not None:
            inner = inner + torch.diag_embed(gs)
        if gu is not None:
            utgu = _t(u) @ gu
            inner = inner + (f * (utgu - _t(utgu))) @ smat
            eye_m = torch.eye(u.shape[-2], dtype=u.dtype, device=u.device)
            out = out + (eye_m - u @ _t(u)) @ gu @ sinv @ _t(v)
        if gv is not None:
            vtgv = _t(v) @ gv
            inner = inner + smat @ (f * (vtgv - _t(vtgv)))
            eye_n = torch.eye(v.shape[-2], dtype=v.dtype, device=v.device)
            out = out + u @ sinv @ _t(gv) @ (eye_n - v @ _t(v))
        return u @ inner @ _t(v) + out


class CholeskySolve(torch.autograd.Function):
    """X = (L L^T)^-1 B for a lower-triangular Cholesky factor L."""

    @staticmethod
    def forward(ctx, b, low):
        x = torch.cholesky_solve(b, low, upper=False)
        ctx.save_for_backward(low, x)
        return x

    @staticmethod
    def backward(ctx, gx):
        low, x = ctx.saved_tensors
        gb = CholeskySolve.apply(gx, low)
        gl = -(gb @ _t(x) + x @ _t(gb)) @ low
        return gb, torch.tril(gl)


def inverse(a):
    return Inverse.apply(a)


def det(a):
    return Determinant.apply(a)


def logabsdet(a):
    return LogAbsDet.apply(a)


def cholesky(a):
    return Cholesky.apply(a)


def eigh(a):
    return Eigh.apply(a)


def qr(a):
    return QR.apply(a)


def svd(a):
    return SVD.apply(a)


def cholesky_solve(b, low):
    return CholeskySolve.apply(b, low)


def pinv(a):
    """Moore-Penrose pseudo-inverse through the SVD above (V S^-1 U^T)."""
    u, s, v = svd(a)
    return v @ torch.diag_embed(1.0 / s) @ _t(u)


def lstsq(a, b):
    """Least-squares solution of A X = B (m >= n) through the QR above:
    X = R^-1 Q^T B."""
    q, r = qr(a)
    return torch.linalg.solve_triangular(r, _t(q) @ b, upper=True)


def matrix_power(a, n: int):
    if n < 0:
        return matrix_power(inverse(a), -n)
    out = torch.eye(a.shape[-1], dtype=a.dtype, device=a.device).expand_as(a)
    base = a
    while n:
        if n & 1:
            out = out @ base
        base = base @ base
        n >>= 1
    return out
