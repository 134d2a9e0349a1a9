"""GEMM head-to-head: the tcgen05 GEMM against cuBLAS (torch.matmul) on every
training GEMM of the three benchmark models, forward, input gradient and
weight gradient, same inputs, same event timing.

    python -m scirs_b200.bench.gemm [--models gpt2,vit,tp8] [--iters 20] [--out gemm.jsonl]

Shapes (M tokens per GPU, weights stored [out, in]):

  gpt2  GPT-2 small, 64 x 1024 tokens: QKV 768->2304, proj 768->768,
        FC1 768->3072 (+bias+GELU), FC2 3072->768 (+bias+residual),
        LM head 768->50304
  gpt2dp8  the same products at 8 x 1024 tokens (one of 8 data-parallel
        ranks at global batch 64)
  vit   ViT-B/16, 32 images x 197 tokens per GPU (global batch 256 over 8):
        the same block shapes at M = 6304
  tp8   1.3B decoder, one tensor-parallel rank of 8, 32 x 2048 tokens:
        QKV 2048->768, proj 256->2048, FC1 2048->1024, FC2 1024->2048

Per product three rows:

  fwd    out[M,N] = x[M,K] @ W[N,K]^T with the engine's epilogue (bias, GELU
         with its second output, residual) against torch.addmm (+ the same
         elementwise work for GELU / residual, which cuBLAS cannot fuse)
  dgrad  dx[M,K] = dy[M,N] @ W[N,K] (with gelu'(h) fused for FC1's input
         gradient) against torch.mm (+ the gelu' multiply)
  wgrad  dW[N,K] += dy^T @ x, fp32 accumulate (split-K when the engine picks
         it) against torch.mm with fp32 output (out_dtype) added into dW

Every operand set is larger than L2 at the GPT-2 and 1.3B shapes; times are
the mean of `iters` back-to-back launches after warm-up.
"""
from __future__ import annotations

import argparse
import json

import torch

from ..ops import kernels as K


def _time(fn, iters, warmup=5):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


# (name, M, N_out, K_in, epilogue of the forward)
def shapes(model: str):
    if model == "gpt2":
        M = 64 * 1024
        return [("qkv", M, 2304, 768, "bias"), ("proj", M, 768, 768, "resid"), ("fc1", M, 3072, 768, "gelu"),
                ("fc2", M, 768, 3072, "resid"), ("lm_head", M, 50304, 768, "none")]
    if model == "gpt2dp8":
        M = 8 * 1024
        return [("qkv", M, 2304, 768, "bias"), ("proj", M, 768, 768, "resid"), ("fc1", M, 3072, 768, "gelu"),
                ("fc2", M, 768, 3072, "resid"), ("lm_head", M, 50304, 768, "none")]
    if model == "vit":
        M = 32 * 197
        return [("qkv", M, 2304, 768, "bias"), ("proj", M, 768, 768, "resid"), ("fc1", M, 3072, 768, "gelu"),
                ("fc2", M, 768, 3072, "resid"), ("patch_embed", 32 * 196, 768, 768, "bias")]
    if model == "tp8":
        M = 32 * 2048
        return [("qkv", M, 768, 2048, "bias"), ("proj", M, 2048, 256, "resid"), ("fc1", M, 1024, 2048, "gelu"),
                ("fc2", M, 2048, 1024, "resid")]
    raise ValueError(model)


def bench_product(model, name, M, N, Kd, epi, iters, peak, dev):
    bf = torch.bfloat16
    x = torch.randn(M, Kd, device=dev, dtype=bf)
    w = torch.randn(N, Kd, device=dev, dtype=bf) * Kd**-0.5
    bias = torch.randn(N, device=dev, dtype=bf)
    y = torch.empty(M, N, device=dev, dtype=bf)
    dy = torch.randn(M, N, device=dev, dtype=bf)
    flops = 2.0 * M * N * Kd
    rows = []

    # forward
    if epi == "gelu":
        pre = torch.empty_like(y)
        ours = lambda: K.gemm(x, w, y, epi=K.EPI_BIAS_GELU, bias=bias, out2=pre)

        def ref():
            h = torch.addmm(bias, x, w.t())
            return torch.nn.functional.gelu(h, approximate="tanh")
    elif epi == "resid":
        res = torch.randn(M, N, device=dev, dtype=bf)
        ours = lambda: K.gemm(x, w, y, epi=K.EPI_RESID, bias=bias, aux=res)
        ref = lambda: torch.addmm(bias, x, w.t()).add_(res)
    elif epi == "bias":
        ours = lambda: K.gemm(x, w, y, bias=bias)
        ref = lambda: torch.addmm(bias, x, w.t())
    else:
        ours = lambda: K.gemm(x, w, y)
        ref = lambda: torch.mm(x, w.t())
    rows.append(("fwd", ours, ref))

    # input gradient dx[M,K] = dy @ W (FC1: times gelu'(pre-activation of the layer below))
    dx = torch.empty(M, Kd, device=dev, dtype=bf)
    if name == "fc2":
        # FC2's input gradient carries gelu'(h) of FC1's pre-activation [M, Kd]
        h = torch.randn(M, Kd, device=dev, dtype=bf)
        ours_d = lambda: K.gemm(dy, w, dx, b_mn=True, epi=K.EPI_DGELU, aux=h)

        def ref_d():
            g = torch.mm(dy, w)
            return g * K.gelu_tanh_grad(h.float()).to(bf)
    else:
        ours_d = lambda: K.gemm(dy, w, dx, b_mn=True)
        ref_d = lambda: torch.mm(dy, w)
    rows.append(("dgrad", ours_d, ref_d))

    # weight gradient dW[N,K] += dy^T x (fp32)
    dw = torch.zeros(N, Kd, device=dev)
    ours_w = lambda: K.gemm(dy, x, dw, a_mn=True, b_mn=True, epi=K.EPI_F32, accumulate=True)
    try:
        torch.mm(dy[:128].t(), x[:128], out_dtype=torch.float32)
        ref_w = lambda: dw.add_(torch.mm(dy.t(), x, out_dtype=torch.float32))
        wref = "torch.mm(out_dtype=fp32) + add"
    except (TypeError, RuntimeError):
        ref_w = lambda: dw.add_(torch.mm(dy.t(), x).float())
        wref = "torch.mm (bf16 out) + add"
    rows.append(("wgrad", ours_w, ref_w))

    out = []
    for kind, o, r in rows:
        t_o = _time(o, iters)
        t_r = _time(r, iters)
        out.append({"model": model, "gemm": name, "pass": kind, "M": M, "N": N if kind != "dgrad" else Kd,
                    "K": Kd if kind == "fwd" else (N if kind == "dgrad" else M),
                    "epilogue": epi if kind == "fwd" else ("dgelu" if (kind == "dgrad" and name == "fc2") else
                                                           ("f32_acc" if kind == "wgrad" else "none")),
                    "ours_ms": round(t_o, 4), "cublas_ms": round(t_r, 4),
                    "ours_tflops": round(flops / t_o / 1e9, 1), "cublas_tflops": round(flops / t_r / 1e9, 1),
                    "speedup": round(t_r / t_o, 3), "ours_frac_of_measured": round(flops / t_o / 1e9 / peak, 3),
                    "cublas_ref": wref if kind == "wgrad" else "torch.addmm/mm (+ unfused elementwise)"})
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--models", default="gpt2,gpt2dp8,vit,tp8")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    from ..utils.tracing import measured_peaks

    peak = measured_peaks().get("bf16_tflops", 1590.0)
    dev = torch.device("cuda", 0)
    outf = open(args.out, "a") if args.out else None
    for model in args.models.split(","):
        for name, M, N, Kd, epi in shapes(model):
            for rec in bench_product(model, name, M, N, Kd, epi, args.iters, peak, dev):
                line = json.dumps(rec)
                print(line, flush=True)
                if outf:
                    outf.write(line + "\n")
                    outf.flush()
            torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
