"""Attention kernel sweep: flash-attention forward + backward, bf16,
head_dim 64/128, seq 512..16384, 8-32 heads, causal, against PyTorch SDPA
(same inputs, same event timing); plus a sliding-window row per head_dim
(the sparse kernels with a 256-token window against the dense kernel).

    python -m scirs_b200.bench.attention [--quick] [--heads 8,16,32] [--out sweep.jsonl]
    python -m scirs_b200.bench.attention --window-only --seq 4096 --hd 64   (one window row)

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
    ap.add_argument("--heads", default="8,16,32")
    ap.add_argument("--tokens", type=int, default=1 << 16, help="batch * seq per call")
    ap.add_argument("--out", default=None, help="also append the JSON lines to this file")
    ap.add_argument("--window-only", action="store_true", help="only the sliding-window row(s)")
    ap.add_argument("--seq", type=int, default=0, help="sequence length of the window row (default: longest)")
    ap.add_argument("--hd", default="64,128", help="head dims of the window row")
    args = ap.parse_args()
    outf = open(args.out, "a") if args.out else None

    def emit(rec):
        line = json.dumps(rec)
        print(line, flush=True)
        if outf:
            outf.write(line + "\n")
            outf.flush()

    peak = 1647.7
    try:
        here = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        peak = json.load(open(os.path.join(here, "MEASURED_PEAKS.json")))["bf16_tflops"]
    except Exception:
        pass
    dev = torch.device("cuda", 0)
    seqs = [1024, 4096] if args.quick else [512, 1024, 2048, 4096, 8192, 16384]
    heads = [int(h) for h in args.heads.split(",")]
    sweep = [] if args.window_only else [(hd, S, H) for hd in (64, 128) for S in seqs for H in heads]
    for hd, S, H in sweep:
        B = max(1, args.tokens // S)
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
        emit({
            "head_dim": hd, "seq": S, "heads": H, "batch": B,
            "fwd_ms": round(t_f, 4), "bwd_ms": round(t_b, 4),
            "fwd_tflops": round(fl / t_f / 1e9, 1), "bwd_tflops": round(2.5 * fl / t_b / 1e9, 1),
            "sdpa_fwd_ms": round(t_sf, 4), "sdpa_bwd_ms": round(t_sb, 4),
            "fwd_speedup_vs_sdpa": round(t_sf / t_f, 3), "bwd_speedup_vs_sdpa": round(t_sb / t_b, 3),
            "fwd_frac_of_measured_peak": round(fl / t_f / 1e9 / peak, 3),
        })
        del qkv, q, k, v, o, do, dqkv, dq, dk, dv, dq_acc, delta, qt, kt, vt, qr, kr, vr, out, g
        torch.cuda.empty_cache()
    # sliding window (no dense mask): 256-token window at the longest sequence
    from ..ops.sparse_attention import sliding_window

    S = args.seq or seqs[-1]
    for hd in (int(h) for h in args.hd.split(",")):
        H, B = 8, max(1, args.tokens // S)
        q, k, v = (torch.randn(B, S, H, hd, device=dev, dtype=torch.bfloat16) for _ in range(3))
        o = torch.empty_like(q)
        lse = torch.empty(B, H, S, device=dev)
        plan = sliding_window(256).plan(S, S, hd, dev)
        t_d = _time(lambda: K.flash_attn_fwd(q, k, v, o, lse, False))
        t_w = _time(lambda: K.flash_attn_fwd(q, k, v, o, lse, False, plan=plan))
        emit({"head_dim": hd, "seq": S, "heads": H, "batch": B, "pattern": "window256", "dense_fwd_ms": round(t_d, 4),
              "window_fwd_ms": round(t_w, 4), "speedup": round(t_d / t_w, 2), "blocks_visited": round(plan.density, 4)})


if __name__ == "__main__":
    main()
