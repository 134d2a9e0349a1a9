"""Fused tensor-parallel GEMMs at the 1.3B decoder's shapes, against their
roofline and against the NCCL-collective + separate-GEMM schedule.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        -m scirs_b200.bench.tp_gemm [--tokens 16384] [--iters 20]

Cases (M tokens over the group, d = 2048, MLP 8192, per-rank slices of the
split dimension):
  ag_qkv   all-gather(LN1 rows) -> GEMM with the column-parallel QKV weights
  ag_fc1   all-gather(LN2 rows) -> GEMM + bias + GELU with the FC1 slice
  rs_proj  attention output slice x row-parallel proj -> reduce-scatter (+ bias + residual)
  rs_fc2   GELU slice x row-parallel FC2 -> reduce-scatter (+ bias + residual)

Roofline of a fused case = max(FLOPs / measured bf16 peak, bytes that must
cross NVLink into / out of one GPU / 770 GB/s); `roofline_frac` = roofline
time / measured time. Times are CUDA-event device times of one fused step
(gather or push, GEMM, signal, reduction), max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

from .. import _ext
from ..ops import kernels as K
from ..parallel import dist as sdist
from ..parallel.tensor_parallel import TPContext

LINK_GBS = 770.0


def _peak_tflops():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    try:
        return float(json.load(open(p)).get("bf16_tflops", 1590.0))
    except Exception:
        return 1590.0


def _time(fn, iters, warmup=3):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return sdist.max_over_ranks(e0.elapsed_time(e1) / iters)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    rank, world, local = sdist.init(timeout_s=120)
    dev = torch.device("cuda", local)
    M, D, F = args.tokens, 2048, 8192
    Mr = M // world
    peak = _peak_tflops()
    g = torch.Generator().manual_seed(rank)
    r = lambda *s: (torch.randn(*s, generator=g) * 0.02).to(dev, torch.bfloat16)  # noqa: E731
    w_qkv, w_fc1 = r(3 * D // world, D), r(F // world, D)
    w_proj, w_fc2 = r(D, D // world), r(D, F // world)
    b_fc1, b_d = r(F // world), r(D)
    results = []
    for mode in ("fused", "nccl"):
        heap = 2 * M * D * 2 + 2 * world * Mr * D * 2 + (8 << 20)
        ctx = TPContext(heap, mode=mode, timeout_s=10.0)
        full = ctx.alloc((M, D))
        seg = ctx.segment(full)
        seg.copy_(r(Mr, D))
        qkv = torch.empty(M, 3 * D // world, device=dev, dtype=torch.bfloat16)
        h = torch.empty(M, F // world, device=dev, dtype=torch.bfloat16)
        gl = torch.empty_like(h)
        att, gel = r(M, D // world), r(M, F // world)
        out = torch.empty(Mr, D, device=dev, dtype=torch.bfloat16)
        resid = r(Mr, D)
        partial = torch.empty(M, D, device=dev, dtype=torch.bfloat16) if mode == "nccl" else None

        def ag_qkv():
            ctx.begin_step()
            s = ctx.gather(full)
            ctx.ag_gemm(full, s, w_qkv, qkv)
            ctx.finish()

        def ag_fc1():
            ctx.begin_step()
            s = ctx.gather(full)
            ctx.ag_gemm(full, s, w_fc1, gl, epi=K.EPI_BIAS_GELU, bias=b_fc1, out2=h)
            ctx.finish()

        def rs(a, w):
            def fn():
                ctx.begin_step()
                recv, s = ctx.gemm_rs(a, w, Mr, partial=partial)
                ctx.reduce(recv, s, out, bias=b_d, resid=resid)
                ctx.finish()
            return fn

        cases = {"ag_qkv": (ag_qkv, 2 * M * D * (3 * D // world), (world - 1) / world * M * D * 2),
                 "ag_fc1": (ag_fc1, 2 * M * D * (F // world), (world - 1) / world * M * D * 2),
                 "rs_proj": (rs(att, w_proj), 2 * M * (D // world) * D, (world - 1) / world * M * D * 2),
                 "rs_fc2": (rs(gel, w_fc2), 2 * M * (F // world) * D, (world - 1) / world * M * D * 2)}
        for name, (fn, flops, link_bytes) in cases.items():
            ms = _time(fn, args.iters)
            roof_ms = max(flops / (peak * 1e12), link_bytes / (LINK_GBS * 1e9)) * 1e3
            results.append({"case": name, "mode": mode, "n_gpus": world, "tokens": M, "ms": round(ms, 4),
                            "tflops": round(flops / (ms * 1e-3) / 1e12, 1), "roofline_ms": round(roof_ms, 4),
                            "roofline_frac": round(roof_ms / ms, 3)})
        _ext.check_status(local)
        ctx.close()
        torch.cuda.synchronize()
        dist.barrier()
    if rank == 0:
        for rr in results:
            print(json.dumps(rr), flush=True)
    sdist.shutdown()


if __name__ == "__main__":
    main()
