"""CPU path of the GEMM's RoPE epilogue: the half-rotation against a
complex-number statement of RoPE, the inverse rotation, and K.gemm with
EPI_ROPE against GEMM + rotation."""
import torch

from scirs_b200.ops import kernels as K


def _tables(S, hd, theta=10000.0):
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2, dtype=torch.float64) / hd))
    ang = torch.arange(S, dtype=torch.float64)[:, None] * inv[None, :]
    return ang.cos().float(), ang.sin().float(), ang


def test_rotation_matches_complex_form():
    S, H, hd = 16, 3, 8
    rows = 2 * S
    cos, sin, ang = _tables(S, hd)
    x = torch.randn(rows, 3 * H * hd, dtype=torch.float64)
    y = K.rope_rotate(x, cos, sin, S, hd, 2 * H * hd).double()
    half = hd // 2
    pos = torch.arange(rows) % S
    for part in range(3):
        for h in range(H):
            c0 = (part * H + h) * hd
            z = torch.complex(x[:, c0:c0 + half], x[:, c0 + half:c0 + hd])
            if part < 2:
                z = z * torch.polar(torch.ones_like(ang[pos]), ang[pos])
            assert torch.allclose(y[:, c0:c0 + half], z.real, atol=1e-5)
            assert torch.allclose(y[:, c0 + half:c0 + hd], z.imag, atol=1e-5)


def test_inverse_undoes_rotation():
    S, hd = 32, 16
    cos, sin, _ = _tables(S, hd)
    x = torch.randn(64, 3 * 2 * hd)
    y = K.rope_rotate(x, cos, sin, S, hd, 4 * hd)
    back = K.rope_rotate(y, cos, sin, S, hd, 4 * hd, inverse=True)
    assert torch.allclose(back, x, atol=1e-5)


def test_gemm_rope_cpu_path():
    S, H, hd, Kd = 8, 2, 16, 24
    cos, sin, _ = _tables(S, hd)
    a = torch.randn(3 * S, Kd).bfloat16()
    w = torch.randn(3 * H * hd, Kd).bfloat16()
    b = torch.randn(3 * H * hd).bfloat16()
    out = torch.empty(3 * S, 3 * H * hd, dtype=torch.bfloat16)
    K.gemm(a, w, out, epi=K.EPI_ROPE, bias=b, rope=(cos, sin, S, hd, 2 * H * hd))
    want = K.rope_rotate(a.float() @ w.float().t() + b.float(), cos, sin, S, hd, 2 * H * hd)
    assert torch.allclose(out.float(), want, atol=2e-2, rtol=2e-2)
