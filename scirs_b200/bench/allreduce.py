"""Fused gradient all-reduce sweep: in-kernel NVLink all-reduce vs NCCL.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        -m scirs_b200.bench.allreduce [--min-bytes 1024] [--max-bytes 1073741824] [--iters 20] [--zero]

Payload sizes are bf16 bytes on the wire (fp32 gradients in, fp32 out; the
push kernel scales by 1/N and casts to bf16 when publishing). NCCL runs
all_reduce(AVG) on a bf16 tensor of the same element count, i.e. the same
bytes. Where the GPUs support NVLink multicast, the NVLS kernel runs in
place on a bf16 buffer of the same size (reduction inside the NVSwitch,
fp32 accumulation); its roofline moves (N+1)/N payloads per GPU per
direction (every byte to the switch once, the reduced 1/N back, the
multicast store's 1/N out and every byte back in). Every number is device
time from CUDA events, max over ranks.
Bus bandwidth = 2 (N-1)/N * bytes / time; roofline = the time to move
2 (N-1)/N * bytes per rank over NVLink at the measured 770 GB/s per
direction. Rank 0 prints one JSON line per size.
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from .. import _ext
from ..parallel import dist as sdist
from ..parallel.nvlink import NVLinkComm

LINK_GBS = 770.0


def _time(fn, iters, warmup=5):
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
    ap.add_argument("--min-bytes", type=int, default=1024)
    ap.add_argument("--max-bytes", type=int, default=1 << 30)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--zero", action="store_true",
                    help="also time the ZeRO collectives: NVLS reduce-scatter (fp32) and all-gather (bf16) vs NCCL")
    args = ap.parse_args()
    rank, world, local = sdist.init(timeout_s=120)
    dev = torch.device("cuda", local)
    comm = NVLinkComm(area_bytes=max(args.max_bytes, 1 << 20) + (1 << 20), timeout_s=10.0)
    nvls = comm.nvls_supported()
    nbuf = comm.nvls_buffer(max(args.max_bytes // 2, 1 << 20), torch.bfloat16) if nvls else None
    zbuf32 = comm.nvls_buffer(max(args.max_bytes // 4, 1 << 20), torch.float32) if (nvls and args.zero) else None
    zbuf16 = comm.nvls_buffer(max(args.max_bytes // 2, 1 << 20), torch.bfloat16) if (nvls and args.zero) else None
    size = args.min_bytes
    while size <= args.max_bytes:
        n = max(8 * world, (size // 2) // (8 * world) * (8 * world))
        x = torch.randn(n, device=dev)
        y = torch.empty_like(x)
        xb = x.to(torch.bfloat16)
        t_ours = _time(lambda: comm.allreduce(x, y, 1.0 / world), args.iters)
        t_nccl = _time(lambda: dist.all_reduce(xb, op=dist.ReduceOp.AVG), args.iters)
        t_nvls = None
        if nvls:
            v = nbuf[:n]
            v.copy_(xb)
            t_nvls = _time(lambda: comm.allreduce_nvls_(v, 1.0 / world), args.iters)
        nbytes = 2 * n
        bus = lambda t: 2 * (world - 1) / world * nbytes / (t * 1e-3) / 1e9  # noqa: E731
        roof_ms = 2 * (world - 1) / world * nbytes / (LINK_GBS * 1e9) * 1e3
        if rank == 0:
            print(json.dumps({
                "bytes": nbytes, "n_gpus": world, "ours_ms": round(t_ours, 4), "nccl_ms": round(t_nccl, 4),
                "ours_busbw_GBs": round(bus(t_ours), 1), "nccl_busbw_GBs": round(bus(t_nccl), 1),
                "speedup_vs_nccl": round(t_nccl / t_ours, 3), "roofline_frac": round(roof_ms / t_ours, 3),
                **({} if t_nvls is None else {
                    "nvls_ms": round(t_nvls, 4), "nvls_busbw_GBs": round(bus(t_nvls), 1),
                    "nvls_speedup_vs_nccl": round(t_nccl / t_nvls, 3),
                    "nvls_roofline_frac": round((world + 1) / world * nbytes / (LINK_GBS * 1e9) * 1e3 / t_nvls, 3)}),
            }), flush=True)
        if zbuf32 is not None:
            # ZeRO collectives on `size` payload bytes: reduce-scatter of fp32
            # gradients, all-gather of bf16 weights; roofline (N-1)/N of the
            # payload into each GPU over NVLink
            nf = max(64 * world, (size // 4) // (64 * world) * (64 * world))
            full = zbuf32[:nf]
            full.normal_()
            shard = torch.empty(nf // world, device=dev)
            t_rs = _time(lambda: comm.reduce_scatter_nvls(full, shard, 1.0 / world), args.iters)
            src = full.clone()
            t_rs_nccl = _time(lambda: dist.reduce_scatter_tensor(shard, src, op=dist.ReduceOp.AVG), args.iters)
            nh = max(64 * world, (size // 2) // (64 * world) * (64 * world))
            fullh = zbuf16[:nh]
            shardh = torch.randn(nh // world, device=dev).to(torch.bfloat16)
            t_ag = _time(lambda: comm.all_gather_nvls(shardh, fullh), args.iters)
            outh = torch.empty(nh, device=dev, dtype=torch.bfloat16)
            t_ag_nccl = _time(lambda: dist.all_gather_into_tensor(outh, shardh), args.iters)
            if rank == 0:
                for op, nb, t_o, t_n in (("reduce_scatter_fp32", 4 * nf, t_rs, t_rs_nccl),
                                         ("all_gather_bf16", 2 * nh, t_ag, t_ag_nccl)):
                    roof = (world - 1) / world * nb / (LINK_GBS * 1e9) * 1e3
                    print(json.dumps({"op": op, "bytes": nb, "n_gpus": world, "nvls_ms": round(t_o, 4),
                                      "nccl_ms": round(t_n, 4), "nvls_speedup_vs_nccl": round(t_n / t_o, 3),
                                      "nvls_roofline_frac": round(roof / t_o, 3),
                                      "nccl_roofline_frac": round(roof / t_n, 3)}), flush=True)
        size *= 4
    _ext.check_status(local)
    comm.close()
    sdist.shutdown()


if __name__ == "__main__":
    main()
