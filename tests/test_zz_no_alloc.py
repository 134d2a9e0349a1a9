"""The no-allocation LayerNorm-backward entry point.

Some callers of this library cannot allocate device memory at the point of
the call: C or other-language hosts that drive the kernels inside a fixed
memory budget with no allocator of their own, and code that must not call
cudaMalloc where it runs (cudaMalloc can synchronise the device).
`scirs_layernorm_bwd_noalloc` (declared in scirs_b200/csrc/scirs_noalloc.h)
serves them: it is exported with C linkage from the extension library and
keeps its scratch in a fixed-size array inside the library.

The GPU tests call it through that C symbol (ctypes), twice in a row on the
shared array, and compare each result with the regular entry point
(`layernorm_bwd`, which takes caller-provided scratch) and with a plain
PyTorch fp32 LayerNorm backward. The argument checks run on the host only.
This file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

HDR_MAX_D = (1 << 20) // 3  # SCIRS_NOALLOC_LN_MAX_D


def _lib():
    import scirs_b200._C as C

    lib = ctypes.CDLL(C.__file__)
    f = lib.scirs_layernorm_bwd_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 10 + [ctypes.c_longlong, ctypes.c_int, ctypes.c_void_p]
    lib.scirs_noalloc_last_error.restype = ctypes.c_char_p
    return lib, f


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _case(D, M, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    mk = lambda *s: torch.randn(*s, generator=g).to("cuda", torch.bfloat16)  # noqa: E731
    x, dy, dres = mk(M, D), mk(M, D), mk(M, D)
    w = (torch.rand(D, generator=g) + 0.5).to("cuda", torch.bfloat16)
    xf = x.float()
    mean = xf.mean(-1).contiguous()
    rstd = torch.rsqrt(((xf - mean[:, None]) ** 2).mean(-1) + 1e-5).contiguous()
    return x, dy, dres, w, mean, rstd


def _regular(x, dy, dres, w, mean, rstd):
    from scirs_b200.ops import kernels as K

    M, D = x.shape
    dx = torch.empty_like(x)
    dw = torch.zeros(D, device="cuda")
    db = torch.zeros(D, device="cuda")
    ds = torch.zeros(D, device="cuda")
    K.layernorm_bwd(dy, x, w, mean, rstd, dx, dw, db, K.ln_partials(M, D, "cuda"), dresid=dres, dsum=ds)
    return dx, dw, db, ds


def _torch_fp32(x, dy, dres, w):
    """LayerNorm backward by PyTorch autograd in fp32 (the oracle)."""
    D = x.shape[1]
    xf = x.float().requires_grad_(True)
    wf = w.float().requires_grad_(True)
    bf = torch.zeros(D, device="cuda", requires_grad=True)
    y = torch.nn.functional.layer_norm(xf, (D,), wf, bf, eps=1e-5)
    y.backward(dy.float())
    dx = xf.grad + (dres.float() if dres is not None else 0.0)
    return dx, wf.grad, bf.grad, dx.sum(0)


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


def _call(f, lib, dy, x, w, mean, rstd, dres, D, M, stream):
    dx = torch.empty_like(x)
    dw = torch.zeros(D, device="cuda")
    db = torch.zeros(D, device="cuda")
    ds = torch.zeros(D, device="cuda")
    rc = f(_ptr(dy), _ptr(x), _ptr(w), _ptr(mean), _ptr(rstd), _ptr(dres), _ptr(dx), _ptr(dw), _ptr(db), _ptr(ds),
           M, D, stream)
    assert rc == 0, (rc, lib.scirs_noalloc_last_error())
    return dx, dw, db, ds


# (D, M): vectorised widths, a width for the generic kernel, and D=4096 with
# M=4096, where 2 blocks per SM x 3 x 4096 floats exceed the 4 MiB array and
# the entry point has to use fewer blocks.
@pytest.mark.gpu
@pytest.mark.parametrize("D,M", [(768, 4096), (2048, 1000), (96, 333), (4096, 4096)])
@pytest.mark.parametrize("with_dresid", [True, False])
def test_noalloc_matches_regular_entry_and_fp32_two_calls(D, M, with_dresid):
    lib, f = _lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call, seed in enumerate((1, 2)):  # two calls in a row share the library's scratch
        x, dy, dres, w, mean, rstd = _case(D, M, seed + 10 * D)
        if not with_dresid:
            dres = None
        dx, dw, db, ds = _call(f, lib, dy, x, w, mean, rstd, dres, D, M, stream)
        torch.cuda.synchronize()
        # against the regular entry point (same kernels, caller-provided scratch)
        rdx, rdw, rdb, rds = _regular(x, dy, dres, w, mean, rstd)
        torch.cuda.synchronize()
        assert torch.allclose(dx.float(), rdx.float(), atol=1e-2, rtol=1e-2), call
        for a, b in ((dw, rdw), (db, rdb), (ds, rds)):
            assert _rel(a, b) < 1e-3, call
        # against PyTorch fp32
        tdx, tdw, tdb, tds = _torch_fp32(x, dy, dres, w)
        assert _rel(dx, tdx) < 1e-2, (call, _rel(dx, tdx))
        for name, a, b in (("dw", dw, tdw), ("db", db, tdb), ("dsum", ds, tds)):
            assert _rel(a, b) < 1e-3, (call, name, _rel(a, b))


@pytest.mark.gpu
def test_noalloc_misaligned_rows_use_scalar_kernel():
    """Row-offset pointers (2-byte but not 16-byte aligned) still give the
    right answer (the entry point serves them with scalar loads)."""
    lib, f = _lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    D, M = 768, 257
    x, dy, dres, w, mean, rstd = _case(D, M + 1, 7)
    # views starting one element into a buffer: not 16-byte aligned
    flat = lambda t: t.reshape(-1)[1 : 1 + M * D].view(M, D)  # noqa: E731
    xs, dys, dress = flat(x), flat(dy), flat(dres)
    assert xs.data_ptr() % 16 != 0
    xf = xs.float()
    mean = xf.mean(-1).contiguous()
    rstd = torch.rsqrt(((xf - mean[:, None]) ** 2).mean(-1) + 1e-5).contiguous()
    out = torch.empty(M * D + 1, dtype=torch.bfloat16, device="cuda")
    dx = out[1:].view(M, D)
    dw = torch.zeros(D, device="cuda")
    db = torch.zeros(D, device="cuda")
    rc = f(_ptr(dys), _ptr(xs), _ptr(w), _ptr(mean), _ptr(rstd), _ptr(dress), _ptr(dx), _ptr(dw), _ptr(db),
           ctypes.c_void_p(0), M, D, stream)
    assert rc == 0, (rc, lib.scirs_noalloc_last_error())
    tdx, tdw, tdb, _ = _torch_fp32(xs, dys, dress, w)
    assert _rel(dx, tdx) < 1e-2
    assert _rel(dw, tdw) < 1e-3 and _rel(db, tdb) < 1e-3


@pytest.mark.gpu
def test_noalloc_call_allocates_nothing():
    """After a first call (which does the per-device set-up), a call changes
    neither PyTorch's allocation count nor the device's free memory."""
    lib, f = _lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    D, M = 1024, 2048
    x, dy, dres, w, mean, rstd = _case(D, M, 3)
    dx = torch.empty_like(x)
    dw, db, ds = (torch.zeros(D, device="cuda") for _ in range(3))
    args = [_ptr(dy), _ptr(x), _ptr(w), _ptr(mean), _ptr(rstd), _ptr(dres), _ptr(dx), _ptr(dw), _ptr(db), _ptr(ds),
            M, D, stream]
    assert f(*args) == 0
    torch.cuda.synchronize()
    a0 = torch.cuda.memory_allocated()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert f(*args) == 0
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == a0
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_noalloc_rejects_oversize_and_bad_args():
    """Argument checks, all returned before any CUDA call (runs without a GPU)."""
    lib, f = _lib()
    z = ctypes.c_void_p(0)
    rc = f(z, z, z, z, z, z, z, z, z, z, 16, (HDR_MAX_D // 8 + 1) * 8, z)
    assert rc == -2 and b"exceeds" in lib.scirs_noalloc_last_error()
    rc = f(z, z, z, z, z, z, z, z, z, z, 16, 12, z)
    assert rc == -1 and b"multiple of 8" in lib.scirs_noalloc_last_error()
    rc = f(z, z, z, z, z, z, z, z, z, z, (1 << 31), 64, z)
    assert rc == -1 and b"INT_MAX" in lib.scirs_noalloc_last_error()
    rc = f(z, z, z, z, z, z, z, z, z, z, 16, 64, z)
    assert rc == -3 and b"null" in lib.scirs_noalloc_last_error()
    # pointers are never dereferenced on the host; odd addresses fail the check
    p16, odd, f4 = ctypes.c_void_p(0x1000), ctypes.c_void_p(0x1001), ctypes.c_void_p(0x2002)
    rc = f(odd, p16, p16, p16, p16, z, p16, p16, p16, z, 16, 64, z)
    assert rc == -5 and b"bf16" in lib.scirs_noalloc_last_error()
    rc = f(p16, p16, p16, f4, p16, z, p16, p16, p16, z, 16, 64, z)
    assert rc == -5 and b"fp32" in lib.scirs_noalloc_last_error()
