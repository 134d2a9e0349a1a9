"""Runs each hot kernel of the GPT-2-small training step on its real shape,
a fixed number of times, for profiling (one GPU).

    python -m scirs_b200.bench.kernel_profile [--rounds 2] [--ops gemm_fc1,attn_fwd,...]

Every round launches each selected op exactly once, in the order given, so a
profiler can skip the first round(s) and capture one launch per op, e.g.

    ncu --set full --clock-control none \
        -k regex:'gemm_tc_kernel|fa_fwd_tc_kernel|fa_bwd_tc_kernel' -s 3 -c 3 \
        -o prof python -m scirs_b200.bench.kernel_profile --rounds 2 \
        --ops gemm_fc1,attn_fwd,attn_bwd

Shapes: M = 16384 tokens (16 sequences of 1024; a quarter of the 1-GPU
step), d=768, MLP 3072, 12 heads of 64, vocabulary 50304 (padded) over 4096
rows, AdamW over a 32M-element flat buffer. Each op's working set is
larger than the 126 MB L2.

Without a profiler it prints one line per op with the CUDA-event time of the
last round (averaged over --iters back-to-back launches), the achieved TFLOP/s or GB/s, and the fraction of the measured
peaks (MEASURED_PEAKS.json at the repository root, if present).
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from .. import _ext
from ..ops import kernels as K

M, D, F, H, HD, S = 16384, 768, 3072, 12, 64, 1024
NOPT = 32 << 20  # optimizer elements (a quarter of GPT-2 small; 640 MB of state)
PB, PL = 32, 4096  # paged decode: sequences x tokens (K + V pages: 537 MB)
B = M // S


def _peaks():
    p = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                     "MEASURED_PEAKS.json")
    try:
        return json.load(open(p))
    except Exception:
        return {}


def build(dev):
    bf, f32 = torch.bfloat16, torch.float32
    g = torch.Generator(device="cpu").manual_seed(0)
    r = lambda *s: torch.randn(*s, generator=g).to(dev, bf)  # noqa: E731
    t = {}
    t["x"] = r(M, D)
    t["w_fc"] = r(F, D) * 0.02
    t["b_fc"] = torch.zeros(F, device=dev, dtype=bf)
    t["h"] = torch.empty(M, F, device=dev, dtype=bf)
    t["gout"] = torch.empty(M, F, device=dev, dtype=bf)
    t["dres"] = r(M, D)
    t["wgrad"] = torch.zeros(D, F, device=dev, dtype=f32)
    t["qkv"] = r(M, 3 * D)
    t["att"] = torch.empty(M, D, device=dev, dtype=bf)
    t["lse"] = torch.empty(B, H, S, device=dev, dtype=f32)
    t["lse128"] = torch.empty(B, H // 2, S, device=dev, dtype=f32)
    t["datt"] = r(M, D)
    t["dqkv"] = torch.empty(M, 3 * D, device=dev, dtype=bf)
    t["dq_acc"] = torch.empty(M * D, device=dev, dtype=f32)
    t["delta"] = torch.empty(B * H * S, device=dev, dtype=f32)
    t["ln_w"] = torch.ones(D, device=dev, dtype=bf)
    t["ln_b"] = torch.zeros(D, device=dev, dtype=bf)
    t["mu"] = torch.empty(M, device=dev, dtype=f32)
    t["rs"] = torch.empty(M, device=dev, dtype=f32)
    t["ln_y"] = torch.empty(M, D, device=dev, dtype=bf)
    t["ln_dx"] = torch.empty(M, D, device=dev, dtype=bf)
    t["ln_dw"] = torch.zeros(D, device=dev, dtype=f32)
    t["ln_db"] = torch.zeros(D, device=dev, dtype=f32)
    t["ln_part"] = K.ln_partials(M, D, dev)
    V = 50304
    t["logits"] = r(M // 4, V)  # 4096 rows x 50304 = 412 MB
    t["tgt"] = torch.randint(0, 50257, (M // 4,), device=dev)
    t["losses"] = torch.empty(M // 4, device=dev, dtype=f32)
    n = NOPT
    t["p"] = torch.randn(n, device=dev) * 0.02
    t["m1"] = torch.zeros(n, device=dev)
    t["m2"] = torch.zeros(n, device=dev)
    t["g"] = torch.randn(n, device=dev) * 1e-3
    t["p16"] = torch.empty(n, device=dev, dtype=bf)
    t["hp"] = torch.tensor([6e-4, 0.9, 0.95, 1e-8, 0.1, 1.0, 1.0, 1.0, 1.0, 0.0, 1.0] + [0.0] * 5, device=dev)
    t["part"] = torch.zeros(1024, device=dev)
    t["mask"] = torch.ones((n + 63) // 64, device=dev, dtype=torch.uint8)
    # embedding: GPT-2 vocabulary, M tokens
    t["tok"] = torch.randint(0, 50257, (M,), device=dev)
    t["wte"] = r(V, D)
    t["wpe"] = r(S, D)
    t["emb"] = torch.empty(M, D, device=dev, dtype=bf)
    t["dwte"] = torch.zeros(V, D, device=dev, dtype=f32)
    t["dwpe"] = torch.zeros(S, D, device=dev, dtype=f32)
    # paged decode: PB sequences of PL tokens, 32 query heads over 8 KV heads, head_dim 128, 16-token pages
    pages = PB * PL // 16
    t["pk"] = r(pages, 16, 8, 128)
    t["pv"] = r(pages, 16, 8, 128)
    t["pq"] = r(PB, 32, 128)
    t["pbt"] = torch.randperm(pages, generator=g).to(torch.int32).view(PB, PL // 16).to(dev)
    t["plen"] = torch.full((PB,), PL, dtype=torch.int32, device=dev)
    t["pout"] = torch.empty(PB, 32, 128, device=dev, dtype=bf)
    t["ppo"] = torch.empty(PB, 32, PL // 512, 128, device=dev, dtype=f32)
    t["ppml"] = torch.empty(PB, 32, PL // 512, 2, device=dev, dtype=f32)
    return t


def _attn_views(t):
    q, k, v = t["qkv"].view(B, S, 3, H, HD).unbind(2)
    return q, k, v


def op_gemm_fc1(t):
    K.gemm(t["x"], t["w_fc"], t["gout"], epi=K.EPI_BIAS_GELU, bias=t["b_fc"], out2=t["h"])


def op_gemm_fc1_plain(t):
    # same shape as fc1, no epilogue math (isolates the epilogue's cost)
    K.gemm(t["x"], t["w_fc"], t["gout"])


def op_gemm_fc2(t):
    # FC2 forward: [M, 3072] x [768, 3072]^T + bias + residual (K = 3072)
    K.gemm(t["gout"], t["w_fc"].view(D, F), t["att"], epi=K.EPI_RESID, bias=t["ln_b"], aux=t["dres"])


def op_gemm_wgrad(t):
    K.gemm(t["dres"], t["gout"], t["wgrad"], a_mn=True, b_mn=True, epi=K.EPI_F32, accumulate=True)


def op_gemm_dgelu(t):
    # dh = (dY @ W) * gelu'(h) with W [F, D] read as the [N, K] operand
    K.gemm(t["dres"], t["w_fc"], t["gout"], epi=K.EPI_DGELU, aux=t["h"])


def op_attn_fwd(t):
    q, k, v = _attn_views(t)
    K.flash_attn_fwd(q, k, v, t["att"].view(B, S, H, HD), t["lse"], causal=True)


def op_attn_fwd_pp(t):
    q, k, v = _attn_views(t)
    K.flash_attn_fwd_impl("pingpong", q, k, v, t["att"].view(B, S, H, HD), t["lse"], causal=True)


def op_attn_fwd_pp_poly(t):
    q, k, v = _attn_views(t)
    K.flash_attn_fwd_impl("pingpong_poly", q, k, v, t["att"].view(B, S, H, HD), t["lse"], causal=True)


def op_attn_fwd_pp_x2(t):
    q, k, v = _attn_views(t)
    K.flash_attn_fwd_impl("pingpong_x2", q, k, v, t["att"].view(B, S, H, HD), t["lse"], causal=True)


def op_attn_fwd_pp_x2_hd128(t):
    q, k, v = t["qkv"].view(B, S, 3, H // 2, 2 * HD).unbind(2)
    K.flash_attn_fwd_impl("pingpong_x2", q, k, v, t["att"].view(B, S, H // 2, 2 * HD), t["lse128"], causal=True)


def op_attn_fwd_pp_poly_hd128(t):
    q, k, v = t["qkv"].view(B, S, 3, H // 2, 2 * HD).unbind(2)
    K.flash_attn_fwd_impl("pingpong_poly", q, k, v, t["att"].view(B, S, H // 2, 2 * HD), t["lse128"], causal=True)


def attn_fwd_pp_trace(t, hd=64):
    """Per-phase clock64 cycles of the ping-pong forward's softmax threads
    (one per tile per CTA), averaged over CTAs and per key block."""
    from .. import _ext

    if hd == 64:
        q, k, v = _attn_views(t)
        att, lse = t["att"].view(B, S, H, HD), t["lse"]
    else:
        q, k, v = t["qkv"].view(B, S, 3, H // 2, 2 * HD).unbind(2)
        att, lse = t["att"].view(B, S, H // 2, 2 * HD), t["lse128"]
    nh = q.shape[2]
    grid = ((S + 255) // 256) * B * nh
    tr = torch.zeros(grid * 2 * 5, dtype=torch.int64, device=q.device)
    _ext.kernels().flash_attn_fwd_pp(q, k, v, att, lse, True, float(q.shape[-1]) ** -0.5, False, tr)
    torch.cuda.synchronize()
    ph = tr.view(grid, 2, 5).double()
    nq = (S + 255) // 256
    avg_blocks = sum(2 * qp + 1 + tt for qp in range(nq) for tt in (0, 1)) / (2 * nq)  # causal key blocks per tile
    per_tile = ph.sum(0).sum(0) / (grid * 2)
    names = ["wait_S", "tmem_load", "max_rescale", "exp_store_P", "signal"]
    return {n: round(float(x) / avg_blocks, 1) for n, x in zip(names, per_tile)}


def op_attn_fwd_hd128(t):
    q, k, v = t["qkv"].view(B, S, 3, H // 2, 2 * HD).unbind(2)
    K.flash_attn_fwd_impl("tcgen05", q, k, v, t["att"].view(B, S, H // 2, 2 * HD), t["lse128"], causal=True)


def op_attn_fwd_pp_hd128(t):
    q, k, v = t["qkv"].view(B, S, 3, H // 2, 2 * HD).unbind(2)
    K.flash_attn_fwd_impl("pingpong", q, k, v, t["att"].view(B, S, H // 2, 2 * HD), t["lse128"], causal=True)


def op_attn_bwd(t):
    q, k, v = _attn_views(t)
    dq, dk, dv = t["dqkv"].view(B, S, 3, H, HD).unbind(2)
    K.flash_attn_bwd(t["datt"].view(B, S, H, HD), q, k, v, t["att"].view(B, S, H, HD), t["lse"], dq, dk, dv,
                     t["dq_acc"], t["delta"], causal=True)


def op_attn_bwd_hd128(t):
    q, k, v = t["qkv"].view(B, S, 3, H // 2, 2 * HD).unbind(2)
    dq, dk, dv = t["dqkv"].view(B, S, 3, H // 2, 2 * HD).unbind(2)
    K.flash_attn_bwd(t["datt"].view(B, S, H // 2, 2 * HD), q, k, v, t["att"].view(B, S, H // 2, 2 * HD),
                     t["lse128"], dq, dk, dv, t["dq_acc"], t["delta"], causal=True)


def op_ln_fwd(t):
    K.layernorm_fwd(t["x"], t["ln_w"], t["ln_b"], t["ln_y"], t["mu"], t["rs"], 1e-5)


def op_ln_bwd(t):
    K.layernorm_bwd(t["dres"], t["x"], t["ln_w"], t["mu"], t["rs"], t["ln_dx"], t["ln_dw"], t["ln_db"],
                    t["ln_part"], dresid=t["datt"])


def op_xent(t):
    K.xent_fwd_bwd(t["logits"], t["tgt"], t["losses"], 50257, 1.0 / (M // 4))


def op_embed_fwd(t):
    K.embedding_fwd(t["tok"], t["wte"], t["wpe"], t["emb"], S)


def op_embed_bwd(t):
    K.embedding_bwd(t["tok"], t["datt"], t["dwte"], t["dwpe"], S)


def op_paged_decode(t):
    _ext.kernels().paged_attention_decode(t["pq"], t["pk"], t["pv"], t["pbt"], t["plen"], t["pout"], t["ppo"],
                                          t["ppml"], 512, 128 ** -0.5)


def op_adamw(t):
    K.optim_step("adamw", t["p"], t["m1"], t["m2"], t["g"], t["p16"], t["p"].numel(), t["hp"], part=t["part"],
                 decay_mask=t["mask"])


# name -> (fn, FLOPs, algorithmic bytes)
OPS = {
    "gemm_fc1": (op_gemm_fc1, 2 * M * D * F, (M * D + F * D + 2 * M * F) * 2),
    "gemm_fc1_plain": (op_gemm_fc1_plain, 2 * M * D * F, (M * D + F * D + M * F) * 2),
    "gemm_fc2": (op_gemm_fc2, 2 * M * D * F, (M * F + F * D + 2 * M * D) * 2),
    "gemm_wgrad": (op_gemm_wgrad, 2 * M * D * F, (M * D + M * F) * 2 + 2 * D * F * 4),
    "gemm_dgelu": (op_gemm_dgelu, 2 * M * D * F, (M * D + F * D + 2 * M * F) * 2),
    "attn_fwd": (op_attn_fwd, 4 * B * H * S * S * HD // 2, (4 * M * D) * 2),
    "attn_fwd_pp": (op_attn_fwd_pp, 4 * B * H * S * S * HD // 2, (4 * M * D) * 2),
    "attn_fwd_pp_x2": (op_attn_fwd_pp_x2, 4 * B * H * S * S * HD // 2, (4 * M * D) * 2),
    "attn_fwd_pp_x2_hd128": (op_attn_fwd_pp_x2_hd128, 4 * B * H * S * S * HD // 2, (4 * M * D) * 2),
    "attn_fwd_pp_poly": (op_attn_fwd_pp_poly, 4 * B * H * S * S * HD // 2, (4 * M * D) * 2),
    "attn_fwd_pp_poly_hd128": (op_attn_fwd_pp_poly_hd128, 4 * B * H * S * S * HD // 2, (4 * M * D) * 2),
    "attn_fwd_hd128": (op_attn_fwd_hd128, 4 * B * H * S * S * HD // 2, (4 * M * D) * 2),
    "attn_fwd_pp_hd128": (op_attn_fwd_pp_hd128, 4 * B * H * S * S * HD // 2, (4 * M * D) * 2),
    "attn_bwd": (op_attn_bwd, 10 * B * H * S * S * HD // 2, (8 * M * D) * 2),
    "attn_bwd_hd128": (op_attn_bwd_hd128, 10 * B * H * S * S * HD // 2, (8 * M * D) * 2),
    "ln_fwd": (op_ln_fwd, 0, 2 * M * D * 2),
    "ln_bwd": (op_ln_bwd, 0, 4 * M * D * 2),
    "xent": (op_xent, 0, 2 * (M // 4) * 50304 * 2),
    "adamw": (op_adamw, 0, NOPT * (4 * 2 + 8 * 2 + 4 + 2) + NOPT * 4),
    "embed_fwd": (op_embed_fwd, 0, M * D * 2 * 3),
    "embed_bwd": (op_embed_bwd, 0, M * D * 2 + 2 * M * D * 4),
    "paged_decode": (op_paged_decode, 4 * PB * 32 * PL * 128, 2 * PB * PL * 8 * 128 * 2),
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rounds", type=int, default=3)
    ap.add_argument("--iters", type=int, default=1, help="back-to-back launches timed per op per round")
    ap.add_argument("--ops", default=",".join(OPS))
    ap.add_argument("--trace-attn", action="store_true",
                    help="print the ping-pong forward's per-phase cycles per key block (head_dim 64 and 128)")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    t = build(dev)
    names = [n for n in args.ops.split(",") if n]
    peaks = _peaks()
    tf_peak = peaks.get("bf16_tflops", 1590.0)
    bw_peak = peaks.get("hbm_gbs", 6650.0)
    ms = {}
    if args.trace_attn:
        for hd in (64, 128):
            attn_fwd_pp_trace(t, hd)  # warm-up
            print(json.dumps({"trace": f"attn_fwd_pp_hd{hd}", "cycles_per_key_block": attn_fwd_pp_trace(t, hd)}),
                  flush=True)
    for _ in range(args.rounds):
        for n in names:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record()
            for _ in range(args.iters):
                OPS[n][0](t)
            e1.record()
            torch.cuda.synchronize()
            ms[n] = e0.elapsed_time(e1) / args.iters
    _ext.check_status(0)
    for n in names:
        _, fl, by = OPS[n]
        s = ms[n] / 1e3
        line = {"op": n, "ms": round(ms[n], 4)}
        if fl:
            line["tflops"] = round(fl / s / 1e12, 1)
            line["frac_of_measured_bf16"] = round(fl / s / 1e12 / tf_peak, 3)
        line["gbs"] = round(by / s / 1e9, 1)
        line["frac_of_measured_hbm"] = round(by / s / 1e9 / bw_peak, 3)
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
