"""Expert-parallel MoE layer, forward + backward, on the peer-memory dispatch /
combine kernels against the NCCL all-to-all transport.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        -m scirs_b200.bench.moe_ep [--tokens 8192] [--d 1024] [--ff 4096] [--experts-per-rank 2]

bf16 parameters and activations, top-2 routing, capacity factor 1.25. Each
line: device time of one forward + backward of the layer (CUDA events, max
over ranks) and the bytes every rank moves across NVLink per step
(dispatch + combine, forward and backward: 4 x (W-1)/W x E x C x d x 2).
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from .. import _ext
from ..nn.moe import ExpertParallelMoE, MoEConfig
from ..parallel import dist as sdist


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192, help="tokens per rank")
    ap.add_argument("--d", type=int, default=1024)
    ap.add_argument("--ff", type=int, default=4096)
    ap.add_argument("--experts-per-rank", type=int, default=2)
    ap.add_argument("--iters", type=int, default=10)
    args = ap.parse_args()
    rank, world, local = sdist.init(timeout_s=120)
    dev = torch.device("cuda", local)
    E = args.experts_per_rank * world
    cfg = MoEConfig(num_experts=E, expert_dim=args.ff, top_k=2, capacity_factor=1.25)
    g = torch.Generator().manual_seed(rank)
    x = torch.randn(args.tokens, args.d, generator=g).to(dev, torch.bfloat16).requires_grad_(True)
    out = []
    for transport in ("peer", "nccl"):
        m = ExpertParallelMoE(args.d, cfg, seed=1, transport=transport).to(dev, torch.bfloat16)

        def step():
            y = m(x)
            y.float().square().mean().backward()

        for _ in range(3):
            step()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            step()
        e1.record()
        torch.cuda.synchronize()
        ms = sdist.max_over_ranks(e0.elapsed_time(e1) / args.iters)
        C = -(-args.tokens * 5 // (4 * E))
        nvl = 4 * (world - 1) / world * E * C * args.d * 2
        out.append({"transport": transport, "n_gpus": world, "tokens_per_rank": args.tokens, "d": args.d,
                    "ff": args.ff, "experts": E, "capacity": C, "ms_fwd_bwd": round(ms, 4),
                    "tokens_per_s": round(world * args.tokens / (ms * 1e-3)), "nvlink_bytes_per_rank": int(nvl)})
        _ext.check_status(local)
        if transport == "peer":
            m.close()
        dist.barrier()
    if rank == 0:
        for r in out:
            print(json.dumps(r), flush=True)
    sdist.shutdown()


if __name__ == "__main__":
    main()
