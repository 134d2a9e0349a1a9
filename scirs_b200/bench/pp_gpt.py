"""Pipeline-parallel GPT training step on the fused kernels.

    python -m torch.distributed.run --nproc-per-node P --master-addr 127.0.0.1 \
        -m scirs_b200.bench.pp_gpt [--layers 12] [--batch 64] [--micro 16] [--schedule 1f1b]

GPT-2-small widths (d 768, 12 heads, vocab 50257, seq 1024), synthetic tokens,
random-init weights, fused AdamW; one line with the device time of a step
(CUDA events, max over ranks) and tokens/s of the whole pipeline.
"""
from __future__ import annotations

import argparse
import json

import torch

from .. import _ext
from ..models.gpt import GPTConfig
from ..models.gpt_pipeline import GPTPipelineStage
from ..parallel import dist as sdist


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=12)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--micro", type=int, default=16)
    ap.add_argument("--schedule", default="1f1b", choices=["1f1b", "gpipe"])
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--no-graph", action="store_true", help="run each stage's step eagerly (no CUDA graph)")
    args = ap.parse_args()
    rank, world, local = sdist.init(timeout_s=120)
    dev = torch.device("cuda", local)
    cfg = GPTConfig.gpt2_small()
    cfg.num_hidden_layers = args.layers
    S = cfg.max_position_embeddings
    st = GPTPipelineStage(cfg, stage=rank, num_stages=world, num_micro=args.micro, device=dev,
                          schedule=args.schedule)
    st.configure_adamw(lr=6e-4)
    if not args.no_graph:
        st.enable_cuda_graph()
    g = torch.Generator().manual_seed(0)
    tok = torch.randint(0, cfg.vocab_size, (args.batch, S + 1), generator=g)
    x, y = tok[:, :-1].contiguous().to(dev), tok[:, 1:].contiguous().to(dev)
    for _ in range(args.warmup):
        st.train_step(x, y)
    torch.cuda.synchronize()
    sdist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    loss = None
    for _ in range(args.steps):
        loss = st.train_step(x, y)
    e1.record()
    torch.cuda.synchronize()
    ms = sdist.max_over_ranks(e0.elapsed_time(e1) / args.steps)
    _ext.check_status(local)
    st.release_cuda_graph()
    lv = float(loss) if loss is not None else None
    vals = [lv]
    if world > 1:
        vals = [None] * world
        torch.distributed.all_gather_object(vals, lv)
    if rank == 0:
        print(json.dumps({"model": f"gpt2-small-{args.layers}L", "pp": world, "schedule": args.schedule,
                          "cuda_graph": not args.no_graph,
                          "global_batch": args.batch, "micro_batches": args.micro, "seq_len": S,
                          "ms_per_step": round(ms, 3), "tokens_per_s": round(args.batch * S / (ms * 1e-3)),
                          "loss": vals[-1]}), flush=True)
    sdist.shutdown()


if __name__ == "__main__":
    main()
