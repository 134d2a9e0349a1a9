"""Attention kernel sweep: flash-attention forward + backward, bf16,
head_dim 64/128, seq 512..16384, causal, against PyTorch SDPA.

    python -m scirs_b200.bench.attention [--quick]

Device time from CUDA events after warm-up; inputs larger than L2 at the
long sequences. TFLOP/s counts the causal half (fwd 2 GEMMs, bwd 5 GEMMs
of 2*S*S*D/2 each); fraction of the measured bf16 peak from MEASURED_PEAKS.json.
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.nn.functional as F

from ..ops import kernels as K


def _time(fn, iters=10, warmup=3):
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--quick", action="store_true")
    args = ap.parse_args()
    peak = 1647.7
    try:
        here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        peak = json.load(open(os.path.join(here, "MEASURED_PEAKS.json")))["bf16_tflops"]
    except Exception:
        pass
    dev = torch.device("cuda", 0)
    seqs = [1024, 4096] if args.quick else [512, 1024, 2048, 4096, 8192, 16384]
    for hd in (64, 128):
        for S in seqs:
            H = 16 if hd == 64 else 8
            B = max(1, (1 << 16) // S)
            qkv = torch.randn(B, S, 3, H, hd, device=dev, dtype=torch.bfloat16)
            q, k, v = qkv.unbind(2)
            o = torch.empty(B, S, H, hd, device=dev, dtype=torch.bfloat16)
            lse = torch.empty(B, H, S, device=dev)
            do = torch.randn_like(o)
            dqkv = torch.empty_like(qkv)
            dq, dk, dv = dqkv.unbind(2)
            dq_acc = torch.empty(B * S * H * hd, device=dev)
            delta = torch.empty(B * H * S, device=dev)
            t_f = _time(lambda: K.flash_attn_fwd(q, k, v, o, lse, True))
            t_b = _time(lambda: K.flash_attn_bwd(do, q, k, v, o, lse, dq, dk, dv, dq_acc, delta, True))
            qt, kt, vt = (t.transpose(1, 2).contiguous() for t in (q, k, v))
            t_sf = _time(lambda: F.scaled_dot_product_attention(qt, kt, vt, is_causal=True))
            qr, kr, vr = (t.detach().requires_grad_(True) for t in (qt, kt, vt))
            out = F.scaled_dot_product_attention(qr, kr, vr, is_causal=True)
            g = torch.randn_like(out)
            t_sb = _time(lambda: torch.autograd.grad(out, (qr, kr, vr), g, retain_graph=True))
            fl = 4 * B * H * S * S * hd / 2  # causal forward FLOPs
            print(json.dumps({
                "head_dim": hd, "seq": S, "heads": H, "batch": B,
                "fwd_ms": round(t_f, 4), "bwd_ms": round(t_b, 4),
                "fwd_tflops": round(fl / t_f / 1e9, 1), "bwd_tflops": round(2.5 * fl / t_b / 1e9, 1),
                "sdpa_fwd_ms": round(t_sf, 4), "sdpa_bwd_ms": round(t_sb, 4),
                "fwd_frac_of_measured_peak": round(fl / t_f / 1e9 / peak, 3),
            }), flush=True)


if __name__ == "__main__":
    main()
