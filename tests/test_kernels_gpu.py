"""Numerics of the sm_100a kernels against PyTorch fp32 references."""
import math

import pytest
import torch

from scirs_b200.ops import kernels as K

pytestmark = pytest.mark.gpu

DEV = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-12))


def rnd(*s, scale=1.0, dtype=torch.bfloat16, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*s, generator=g) * scale).to(DEV, dtype)


# ---------------------------------------------------------------------------- GEMM
@pytest.mark.parametrize("M,N,K_", [(128, 256, 64), (256, 768, 768), (384, 2304, 768), (200, 136, 72), (1024, 50304, 128)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
def test_gemm_layouts(M, N, K_, a_mn, b_mn):
    a = rnd(K_, M, seed=1) if a_mn else rnd(M, K_, seed=1)
    b = rnd(K_, N, seed=2) if b_mn else rnd(N, K_, seed=2)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    K.gemm(a, b, out, a_mn=a_mn, b_mn=b_mn)
    A = (a.t() if a_mn else a).float()
    B = (b if b_mn else b.t()).float()
    ref = A @ B
    torch.cuda.synchronize()
    assert rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("bn", [128, 256])
def test_gemm_epilogues(bn):
    M, N, K_ = 512, 768, 256
    a, w = rnd(M, K_, seed=3), rnd(N, K_, scale=0.1, seed=4)
    bias, aux = rnd(N, seed=5), rnd(M, N, seed=6)
    acc = a.float() @ w.float().t()
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    K.gemm(a, w, out, bias=bias, bn=bn)
    assert rel_err(out, acc + bias.float()) < 1e-2
    K.gemm(a, w, out, epi=K.EPI_RESID, bias=bias, aux=aux, bn=bn)
    assert rel_err(out, acc + bias.float() + aux.float()) < 1e-2
    pre = torch.empty_like(out)
    K.gemm(a, w, out, epi=K.EPI_BIAS_GELU, bias=bias, out2=pre, bn=bn)
    h = acc + bias.float()
    assert rel_err(pre, h) < 1e-2
    assert rel_err(out, K.gelu_tanh(h)) < 1e-2
    K.gemm(a, w, out, epi=K.EPI_DGELU, aux=aux, bn=bn)
    assert rel_err(out, acc * K.gelu_tanh_grad(aux.float())) < 1e-2


@pytest.mark.parametrize("splits", [0, 1, 3])
def test_gemm_f32_wgrad_accumulate(splits):
    Mtok, N, K_ = 4096, 768, 384
    dy, x = rnd(Mtok, N, seed=7), rnd(Mtok, K_, seed=8)
    out = torch.zeros(N, K_, device=DEV, dtype=torch.float32)
    K.gemm(dy, x, out, a_mn=True, b_mn=True, epi=K.EPI_F32, splits=splits)
    ref = dy.float().t() @ x.float()
    assert rel_err(out, ref) < 5e-3
    K.gemm(dy, x, out, a_mn=True, b_mn=True, epi=K.EPI_F32, accumulate=True, splits=splits)
    assert rel_err(out, 2 * ref) < 5e-3


def test_gemm_large_m_persistent():
    M, N, K_ = 8192, 3072, 768
    a, b = rnd(M, K_, seed=9), rnd(N, K_, scale=0.05, seed=10)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    K.gemm(a, b, out)
    assert rel_err(out, a.float() @ b.float().t()) < 1e-2


# Shapes large enough for the 2-SM (cta_group::2) tiles: >= 74 tiles of 256 x 256.
@pytest.mark.parametrize("M,N,K_", [(4096, 3072, 768), (4224, 3000, 512), (2304, 8192, 256)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
def test_gemm_pair_layouts(M, N, K_, a_mn, b_mn):
    a = rnd(K_, M, seed=11) if a_mn else rnd(M, K_, seed=11)
    b = rnd(K_, N, scale=0.1, seed=12) if b_mn else rnd(N, K_, scale=0.1, seed=12)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    K.gemm(a, b, out, a_mn=a_mn, b_mn=b_mn)
    ref = (a.t() if a_mn else a).float() @ (b if b_mn else b.t()).float()
    torch.cuda.synchronize()
    assert rel_err(out, ref) < 1e-2
    single = torch.empty_like(out)
    K.gemm(a, b, single, a_mn=a_mn, b_mn=b_mn, bn=128)  # the single-CTA kernel
    assert rel_err(out, single) < 5e-3


def test_gemm_pair_epilogues():
    M, N, K_ = 4096, 3072, 768
    a, w = rnd(M, K_, seed=13), rnd(N, K_, scale=0.05, seed=14)
    bias, aux = rnd(N, seed=15), rnd(M, N, seed=16)
    acc = a.float() @ w.float().t()
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    K.gemm(a, w, out, bias=bias)
    assert rel_err(out, acc + bias.float()) < 1e-2
    K.gemm(a, w, out, epi=K.EPI_RESID, bias=bias, aux=aux)
    assert rel_err(out, acc + bias.float() + aux.float()) < 1e-2
    pre = torch.empty_like(out)
    K.gemm(a, w, out, epi=K.EPI_BIAS_GELU, bias=bias, out2=pre)
    h = acc + bias.float()
    assert rel_err(pre, h) < 1e-2 and rel_err(out, K.gelu_tanh(h)) < 1e-2
    bg = torch.zeros(N, device=DEV)
    K.gemm(a, w, out, epi=K.EPI_DGELU, aux=aux, bias_grad=bg)
    want = acc * K.gelu_tanh_grad(aux.float())
    assert rel_err(out, want) < 1e-2
    assert rel_err(bg, out.float().sum(0)) < 1e-2
    # fp32 weight gradient over a long token dimension (split-K with TMA reduce-add)
    dy, x = rnd(16384, 768, seed=17), rnd(16384, 3072, seed=18)
    g = torch.zeros(768, 3072, device=DEV)
    K.gemm(dy, x, g, a_mn=True, b_mn=True, epi=K.EPI_F32)
    assert rel_err(g, dy.float().t() @ x.float()) < 5e-3
    K.gemm(dy, x, g, a_mn=True, b_mn=True, epi=K.EPI_F32, accumulate=True)
    assert rel_err(g, 2 * (dy.float().t() @ x.float())) < 5e-3
    torch.cuda.synchronize()
    from scirs_b200 import _ext

    _ext.check_status()


# ---------------------------------------------------------------------------- LayerNorm
@pytest.mark.parametrize("D", [256, 768, 1024, 2048, 96])
def test_layernorm(D):
    M = 1000
    x, w, b = rnd(M, D, seed=1), rnd(D, seed=2) * 0.5 + 1, rnd(D, seed=3)
    y = torch.empty_like(x)
    mu = torch.empty(M, device=DEV)
    rs = torch.empty(M, device=DEV)
    K.layernorm_fwd(x, w, b, y, mu, rs, 1e-5)
    xf = x.float().requires_grad_(True)
    wf = w.float().requires_grad_(True)
    bf = b.float().requires_grad_(True)
    ref = torch.nn.functional.layer_norm(xf, (D,), wf, bf, 1e-5)
    assert rel_err(y, ref) < 1e-2
    dy, dres = rnd(M, D, seed=4), rnd(M, D, seed=5)
    ref.backward(dy.float())
    dx = torch.empty_like(x)
    dw = torch.zeros(D, device=DEV)
    db = torch.zeros(D, device=DEV)
    part = K.ln_partials(M, D, DEV)
    K.layernorm_bwd(dy, x, w, mu, rs, dx, dw, db, part, dresid=dres)
    assert rel_err(dx, xf.grad + dres.float()) < 1e-2
    assert rel_err(dw, wf.grad) < 1e-3
    assert rel_err(db, bf.grad) < 1e-3


# ---------------------------------------------------------------------------- cross entropy
@pytest.mark.parametrize("V,Vp", [(50257, 50304), (1000, 1024), (10, 16)])
def test_xent(V, Vp):
    M = 64
    logits = rnd(M, Vp, scale=2.0, seed=1)
    tgt = torch.randint(0, V, (M,), device=DEV)
    tgt[3] = -100
    ref_in = logits[:, :V].float().requires_grad_(True)
    ref = torch.nn.functional.cross_entropy(ref_in, tgt, reduction="none", ignore_index=-100)
    ref.sum().backward()
    loss = torch.empty(M, device=DEV)
    lg = logits.clone()
    K.xent_fwd_bwd(lg, tgt, loss, V, 1.0)
    assert torch.allclose(loss, ref, atol=2e-2, rtol=1e-2)
    assert rel_err(lg[:, :V], ref_in.grad) < 1e-2
    assert float(lg[:, V:].float().abs().max()) == 0.0
    loss2 = torch.empty(M, device=DEV)
    K.xent_fwd(logits, tgt, loss2, V)
    assert torch.allclose(loss2, ref, atol=2e-2, rtol=1e-2)


# ---------------------------------------------------------------------------- embedding / bias grad
def test_embedding_and_bias_grad():
    V, D, S, B = 1000, 768, 128, 4
    wte, wpe = rnd(V, D, seed=1), rnd(S, D, seed=2)
    tok = torch.randint(0, V, (B * S,), device=DEV)
    out = torch.empty(B * S, D, device=DEV, dtype=torch.bfloat16)
    K.embedding_fwd(tok, wte, wpe, out, S)
    ref = wte.float()[tok] + wpe.float()[torch.arange(B * S, device=DEV) % S]
    assert rel_err(out, ref) < 1e-2
    dout = rnd(B * S, D, seed=3)
    dwte = torch.zeros(V, D, device=DEV)
    dwpe = torch.zeros(S, D, device=DEV)
    K.embedding_bwd(tok, dout, dwte, dwpe, S)
    r1 = torch.zeros(V, D, device=DEV).index_add_(0, tok, dout.float())
    r2 = torch.zeros(S, D, device=DEV).index_add_(0, torch.arange(B * S, device=DEV) % S, dout.float())
    assert rel_err(dwte, r1) < 1e-4 and rel_err(dwpe, r2) < 1e-4
    bg = torch.zeros(D, device=DEV)
    K.bias_grad(dout, bg)
    assert rel_err(bg, dout.float().sum(0)) < 1e-4


# ---------------------------------------------------------------------------- attention
@pytest.mark.parametrize("bwd_impl", ["tcgen05", "tcgen05_pipe", "tcgen05_persist", "tcgen05_auto", "mma"])
@pytest.mark.parametrize("B,S,H,HD,causal", [(2, 256, 4, 64, True), (1, 197, 3, 64, False), (1, 384, 2, 128, True),
                                             (2, 1024, 2, 64, True), (1, 300, 2, 64, True), (1, 300, 2, 128, True),
                                             (2, 197, 2, 128, False), (1, 1024, 2, 128, True)])
def test_flash_attention(B, S, H, HD, causal, bwd_impl, monkeypatch):
    from scirs_b200 import _ext

    monkeypatch.setattr(K, "ATTN_BWD_IMPL", bwd_impl)
    qkv = rnd(B, S, 3, H, HD, seed=11)
    q, k, v = qkv.unbind(2)
    out = torch.empty(B, S, H, HD, device=DEV, dtype=torch.bfloat16)
    lse = torch.empty(B, H, S, device=DEV)
    scale = HD ** -0.5
    K.flash_attn_fwd(q, k, v, out, lse, causal, scale)
    qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
    o_ref, lse_ref = K.attention_reference(qf, kf, vf, causal, scale)
    assert rel_err(out, o_ref) < 1e-2
    assert torch.allclose(lse, lse_ref, atol=1e-2)
    dout = rnd(B, S, H, HD, seed=12)
    o_ref.backward(dout.float())
    dqkv = torch.empty_like(qkv)
    dq, dk, dv = dqkv.unbind(2)
    dq_acc = torch.empty(B * S * H * HD, device=DEV)
    delta = torch.empty(B * H * S, device=DEV)
    K.flash_attn_bwd(dout, q, k, v, out, lse, dq, dk, dv, dq_acc, delta, causal, scale)
    assert rel_err(dq, qf.grad) < 2e-2
    assert rel_err(dk, kf.grad) < 2e-2
    assert rel_err(dv, vf.grad) < 2e-2
    _ext.check_status()


@pytest.mark.parametrize("impl", ["pingpong", "pingpong_poly", "pingpong_x2", "pingpong_bf2", "tcgen05", "mma"])
@pytest.mark.parametrize("B,S,H,HD,causal", [(2, 256, 4, 64, True), (1, 197, 3, 64, False), (1, 384, 2, 128, True),
                                             (2, 1024, 2, 64, True), (1, 300, 2, 128, False)])
def test_flash_attention_fwd_impls(impl, B, S, H, HD, causal, monkeypatch):
    from scirs_b200 import _ext

    monkeypatch.setattr(K, "ATTN_FWD_IMPL", impl)
    qkv = rnd(B * S, 3 * H * HD, seed=21).view(B, S, 3, H, HD)  # fused-QKV layout
    q, k, v = qkv.unbind(2)
    out = torch.empty(B, S, H, HD, device=DEV, dtype=torch.bfloat16)
    lse = torch.empty(B, H, S, device=DEV)
    K.flash_attn_fwd(q, k, v, out, lse, causal, HD**-0.5)
    torch.cuda.synchronize()
    _ext.check_status()
    o_ref, lse_ref = K.attention_reference(q, k, v, causal, HD**-0.5)
    assert rel_err(out, o_ref) < 1e-2
    assert torch.allclose(lse, lse_ref, atol=1e-2)


@pytest.mark.parametrize("impl", ["pingpong", "pingpong_poly", "pingpong_x2", "pingpong_bf2"])
@pytest.mark.parametrize("HD,causal", [(64, True), (128, True), (64, False), (128, False)])
def test_flash_attention_fwd_pingpong_rescale(HD, causal, impl, monkeypatch):
    """Large scores: the running reference max is raised (and O rescaled in
    TMEM) several times per row."""
    from scirs_b200 import _ext

    monkeypatch.setattr(K, "ATTN_FWD_IMPL", impl)
    B, S, H = 1, 1536, 2
    qkv = rnd(B * S, 3 * H * HD, seed=5).view(B, S, 3, H, HD)
    ramp = torch.linspace(0.5, 4.0, S, device=DEV).view(1, S, 1, 1, 1).to(torch.bfloat16)
    qkv = (qkv * ramp).contiguous()  # later keys score higher: the max keeps growing
    q, k, v = qkv.unbind(2)
    out = torch.empty(B, S, H, HD, device=DEV, dtype=torch.bfloat16)
    lse = torch.empty(B, H, S, device=DEV)
    K.flash_attn_fwd(q, k, v, out, lse, causal, HD**-0.5)
    torch.cuda.synchronize()
    _ext.check_status()
    o_ref, lse_ref = K.attention_reference(q, k, v, causal, HD**-0.5)
    assert rel_err(out, o_ref) < 1e-2
    assert torch.allclose(lse, lse_ref, atol=2e-2, rtol=1e-3)


# ---------------------------------------------------------------------------- optimizer
@pytest.mark.parametrize("mode", ["adam", "adamw", "sgd", "rmsprop", "adagrad"])
def test_fused_optimizer(mode):
    n = 10000 + 64 * 3
    p = torch.randn(n, device=DEV)
    g = torch.randn(n, device=DEV)
    s1, s2 = torch.rand(n, device=DEV), torch.rand(n, device=DEV)
    hp = torch.tensor([1e-2, 0.9, 0.99, 1e-8, 0.05, 1 - 0.9**3, 1 - 0.99**3, 0.5, 0.0], device=DEV)
    ref = [t.cpu().clone() for t in (p, s1, s2)]
    p16 = torch.empty(n, device=DEV, dtype=torch.bfloat16)
    K.optim_step(mode, p, s1, s2, g, p16, n // 2, hp)
    rp, r1, r2 = ref
    K.optim_step(mode, rp, r1, r2, g.cpu(), None, n // 2, hp.cpu())
    assert torch.allclose(p.cpu(), rp, atol=1e-5, rtol=1e-5)
    assert torch.allclose(p16.float().cpu(), rp, atol=1e-2, rtol=1e-2)


def test_fused_optimizer_clip_and_skip():
    n = 4096
    p = torch.randn(n, device=DEV)
    g = torch.randn(n, device=DEV) * 10
    s1, s2 = torch.zeros(n, device=DEV), torch.zeros(n, device=DEV)
    hp = torch.tensor([1e-2, 0.9, 0.99, 1e-8, 0.0, 0.1, 0.01, 1.0, 1.0], device=DEV)
    part = torch.zeros(1024, device=DEV)
    norm = torch.zeros(1, device=DEV)
    ref = [t.cpu().clone() for t in (p, s1, s2)]
    K.optim_step("adamw", p, s1, s2, g, None, n, hp, part=part, norm_out=norm)
    rn = torch.zeros(1)
    K.optim_step("adamw", ref[0], ref[1], ref[2], g.cpu(), None, n, hp.cpu(), part=torch.zeros(1), norm_out=rn)
    assert abs(float(norm) - float(g.norm())) / float(g.norm()) < 1e-4
    assert torch.allclose(p.cpu(), ref[0], atol=1e-5)
    g[5] = float("inf")
    before = p.clone()
    K.optim_step("adamw", p, s1, s2, g, None, n, hp, part=part, norm_out=norm)
    assert torch.equal(p, before)


# ------------------------------------------------------------ RoPE in the GEMM epilogue
def _rope_tables(S, hd, theta=10000.0):
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2, dtype=torch.float64) / hd))
    ang = torch.arange(S, dtype=torch.float64)[:, None] * inv[None, :]
    return ang.cos().float().to(DEV).contiguous(), ang.sin().float().to(DEV).contiguous()


@pytest.mark.parametrize("M,H,hd,bn", [(1000, 4, 64, 0), (512, 2, 128, 128), (512, 4, 128, 256), (4096, 16, 128, 0),
                                       (8192, 12, 64, 0)])
def test_gemm_rope_epilogue(M, H, hd, bn):
    """EPI_ROPE (bias, then half-rotation RoPE of the q and k heads of a
    fused [rows, 3, H, hd] output) against an fp32 reference; the last two
    shapes run on 2-SM pair tiles."""
    Kd, S = 256, 256
    N = 3 * H * hd
    a, w, bias = rnd(M, Kd, seed=41), rnd(N, Kd, scale=0.1, seed=42), rnd(N, seed=43)
    cos, sin = _rope_tables(S, hd)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    K.gemm(a, w, out, epi=K.EPI_ROPE, bias=bias, bn=bn, rope=(cos, sin, S, hd, 2 * H * hd))
    acc = a.float() @ w.float().t() + bias.float()
    want = K.rope_rotate(acc, cos, sin, S, hd, 2 * H * hd)
    torch.cuda.synchronize()
    assert rel_err(out, want) < 1e-2
    # v columns untouched by the rotation
    assert rel_err(out[:, 2 * H * hd:], acc[:, 2 * H * hd:]) < 1e-2
    # same result as the separate RoPE kernel on the plain GEMM output
    ref2 = torch.empty_like(out)
    K.gemm(a, w, ref2, bias=bias, bn=bn)
    from scirs_b200 import _ext

    _ext.kernels().rope_apply(ref2, cos, sin, S, H, hd, False)
    assert rel_err(out, ref2) < 1e-2


@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("M,N,K_", [(2048, 768, 3072), (6304, 768, 2304), (8192, 768, 50304 // 8 * 8)])
def test_gemm_bf16_split_k(M, N, K_, b_mn):
    """Small M, long K, few output tiles: the bf16 output goes through the
    split-K fp32 workspace and the finalize pass (bias; bias + residual)."""
    a = rnd(M, K_, scale=0.5, seed=51)
    b = rnd(K_, N, scale=0.05, seed=52) if b_mn else rnd(N, K_, scale=0.05, seed=52)
    bias, res = rnd(N, seed=53), rnd(M, N, seed=54)
    acc = a.float() @ (b.float() if b_mn else b.float().t())
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    K.gemm(a, b, out, b_mn=b_mn)
    assert rel_err(out, acc) < 1e-2
    K.gemm(a, b, out, b_mn=b_mn, bias=bias)
    assert rel_err(out, acc + bias.float()) < 1e-2
    K.gemm(a, b, out, b_mn=b_mn, epi=K.EPI_RESID, bias=bias, aux=res)
    assert rel_err(out, acc + bias.float() + res.float()) < 1e-2
    # twice in a row inside a CUDA graph (the workspace is allocated and zeroed in stream order)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        K.gemm(a, b, out, b_mn=b_mn, epi=K.EPI_RESID, bias=bias, aux=res)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            K.gemm(a, b, out, b_mn=b_mn, epi=K.EPI_RESID, bias=bias, aux=res)
    out.zero_()
    g.replay()
    g.replay()
    torch.cuda.synchronize()
    assert rel_err(out, acc + bias.float() + res.float()) < 1e-2
