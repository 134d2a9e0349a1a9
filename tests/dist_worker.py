"""Worker for the multi-GPU tests (run under torchrun, one rank per GPU).

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        tests/dist_worker.py <case> <out_json>

Each case checks the in-kernel NVLink collectives against NCCL / a local
reference and rank 0 writes a JSON verdict.
"""
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from scirs_b200 import _ext  # noqa: E402
from scirs_b200.parallel import dist as sdist  # noqa: E402


def case_collectives():
    from scirs_b200.parallel.nvlink import NVLinkComm

    rank, world = dist.get_rank(), dist.get_world_size()
    comm = NVLinkComm(area_bytes=64 << 20, timeout_s=10.0)
    dev = torch.device("cuda", torch.cuda.current_device())
    res = {}
    for n in [8 * world, 4096, 1 << 20, 3 * (1 << 20) + 64 * world]:
        g = torch.Generator(device="cpu").manual_seed(100 + rank)
        x = torch.randn(n, generator=g).to(dev)
        ref = x.to(torch.bfloat16).float() / world  # each rank's bf16-rounded scaled contribution
        ref_sum = ref.clone()
        dist.all_reduce(ref_sum)
        for algo in (1, 2):  # one-shot and two-shot
            out = torch.empty_like(x)
            for _ in range(3):  # repeated calls exercise the epoch and buffer-set protocol
                comm.allreduce(x, out, 1.0 / world, algo=algo)
            torch.cuda.synchronize()
            err = float((out - ref_sum).abs().max() / ref_sum.abs().max())
            # identical on all ranks
            o0 = out.clone()
            dist.broadcast(o0, 0)
            same = bool(torch.equal(o0, out))
            res[f"allreduce{algo}_{n}"] = {"max_err": err, "identical": same}
        # reduce-scatter
        if n % (8 * world) == 0:
            shard = torch.empty(n // world, device=dev)
            comm.reduce_scatter(x, shard, 1.0 / world)
            torch.cuda.synchronize()
            want = ref_sum[rank * (n // world) : (rank + 1) * (n // world)]
            res[f"reduce_scatter_{n}"] = {"max_err": float((shard - want).abs().max() / want.abs().max())}
            # all-gather (bf16)
            full = torch.empty(n, device=dev, dtype=torch.bfloat16)
            comm.all_gather(shard.to(torch.bfloat16), full)
            ag_ref = [torch.empty(n // world, device=dev, dtype=torch.bfloat16) for _ in range(world)]
            dist.all_gather(ag_ref, shard.to(torch.bfloat16))
            torch.cuda.synchronize()
            res[f"allgather_{n}"] = {"equal": bool(torch.equal(full, torch.cat(ag_ref)))}
    _ext.check_status()
    comm.close()
    return res


def case_nvls():
    from scirs_b200.parallel.nvlink import NVLinkComm

    rank, world = dist.get_rank(), dist.get_world_size()
    comm = NVLinkComm(area_bytes=16 << 20, timeout_s=10.0)
    if not comm.nvls_supported():
        return {"skipped": "no NVLink multicast support"}
    dev = torch.device("cuda", torch.cuda.current_device())
    res = {}
    for dtype in (torch.float32, torch.bfloat16):
        buf = comm.nvls_buffer(1 << 22, dtype)
        for off, n in [(0, 8 * world), (64, 4096 + 8), (1024, 1 << 20), (0, 1 << 22)]:
            view = buf[off:off + n]
            for rep in range(3):  # repeated calls exercise the epoch protocol
                g = torch.Generator().manual_seed(1000 * rep + rank)
                x = torch.randn(n, generator=g).to(dev).to(dtype)
                view.copy_(x)
                ref = x.float()
                dist.all_reduce(ref)
                ref /= world
                comm.allreduce_nvls_(view, 1.0 / world)
            torch.cuda.synchronize()
            got = view.float()
            err = float((got - ref).abs().max() / ref.abs().max())
            o0 = got.clone()
            dist.broadcast(o0, 0)
            res[f"nvls_{str(dtype)[6:]}_{off}_{n}"] = {"max_err": err, "identical": bool(torch.equal(o0, got))}
    # reduce-scatter (fp32) and all-gather (bf16) through the multicast mapping
    n = 1 << 20
    full = comm.nvls_buffer(n, torch.float32)
    full16 = comm.nvls_buffer(n, torch.bfloat16)
    for rep in range(3):
        g = torch.Generator().manual_seed(77 + 10 * rep + rank)
        x = torch.randn(n, generator=g).to(dev)
        full.copy_(x)
        shard = torch.empty(n // world, device=dev)
        comm.reduce_scatter_nvls(full, shard, 1.0 / world)
        want = torch.empty(n // world, device=dev)
        dist.reduce_scatter_tensor(want, x, op=dist.ReduceOp.SUM)
        want /= world
        mine = x[rank * (n // world):(rank + 1) * (n // world)].to(torch.bfloat16)
        comm.all_gather_nvls(mine, full16)
        ag = torch.empty(n, device=dev, dtype=torch.bfloat16)
        dist.all_gather_into_tensor(ag, mine)
        torch.cuda.synchronize()
    res["nvls_reduce_scatter"] = {"max_err": float((shard - want).abs().max() / want.abs().max()), "identical": True}
    res["nvls_all_gather"] = {"max_err": 0.0 if torch.equal(full16, ag) else 1.0, "identical": True}
    _ext.check_status()
    comm.close()
    return res


def case_ring_attn():
    from scirs_b200.ops import kernels as K
    from scirs_b200.parallel.context_parallel import ring_attention

    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    B, Sc, H, D = 2, 256, 4, 64
    g = torch.Generator().manual_seed(5)
    q, k, v, do = (torch.randn(B, world * Sc, H, D, generator=g).to(dev, torch.bfloat16) for _ in range(4))
    sl = slice(rank * Sc, (rank + 1) * Sc)
    res = {}
    for causal in (True, False):
        ql, kl, vl = (t[:, sl].contiguous().requires_grad_(True) for t in (q, k, v))
        o, lse = ring_attention(ql, kl, vl, causal=causal)
        o.backward(do[:, sl].contiguous())
        qf, kf, vf = (t.float().requires_grad_(True) for t in (q, k, v))
        o_ref, lse_ref = K.attention_reference(qf, kf, vf, causal, D ** -0.5)
        o_ref.backward(do.float())
        rel = lambda a, b: float((a.float() - b).norm() / (b.norm() + 1e-12))  # noqa: E731
        res[f"ring_causal{int(causal)}"] = {
            "o": rel(o, o_ref[:, sl].detach()), "lse": float((lse - lse_ref[:, :, sl]).abs().max()),
            "dq": rel(ql.grad, qf.grad[:, sl]), "dk": rel(kl.grad, kf.grad[:, sl]), "dv": rel(vl.grad, vf.grad[:, sl])}
    _ext.check_status()
    return res


def case_dp_gpt():
    """DP training with the fused all-reduce == single-process training on the
    concatenated global batch (same weights, same data)."""
    from scirs_b200.models.gpt import GPTConfig, GPTModel
    from scirs_b200.parallel.data_parallel import data_parallel

    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = GPTConfig.tiny(vocab=1024, seq=128)
    g = torch.Generator().manual_seed(7)
    tok = torch.randint(0, cfg.vocab_size, (4 * world, 129), generator=g)
    x, y = tok[:, :-1].contiguous(), tok[:, 1:].contiguous()
    lb = 4
    res = {}
    for mode in ("fused", "nccl"):
        m = GPTModel(cfg, device=dev, seed=3)
        m.configure_adamw(lr=1e-3, weight_decay=0.0, max_grad_norm=0.0)
        data_parallel(m, mode=mode)
        losses = []
        for _ in range(3):
            l = m.train_step(x[rank * lb : (rank + 1) * lb].to(dev), y[rank * lb : (rank + 1) * lb].to(dev))
            lt = l.detach().clone()
            dist.all_reduce(lt)
            losses.append(float(lt) / world)
        torch.cuda.synchronize()
        # replicas must stay identical
        w = m.fp.master.clone()
        w0 = w.clone()
        dist.broadcast(w0, 0)
        res[mode] = {"losses": losses, "replica_max_diff": float((w - w0).abs().max())}
        if m.grad_sync is not None and m.grad_sync.comm is not None:
            m.grad_sync.comm.close()
    # single-process reference on the full batch
    if rank == 0:
        m = GPTModel(cfg, device=dev, seed=3)
        m.configure_adamw(lr=1e-3, weight_decay=0.0, max_grad_norm=0.0)
        ref = [float(m.train_step(x.to(dev), y.to(dev))) for _ in range(3)]
        res["single"] = {"losses": ref}
    _ext.check_status()
    return res


def case_zero_gpt():
    """GPT with the sharded optimizer (ZeRO-1): fused (NVLS or push
    collectives, early LM-head wte reduce-scatter, lookup-gradient rows routed
    to their owners by the peer kernels) and the NCCL schedule == single-
    process training on the concatenated batch; the gathered bf16 weights are
    identical on every rank."""
    from scirs_b200.models.gpt import GPTConfig, GPTModel
    from scirs_b200.parallel.zero import zero_data_parallel

    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = GPTConfig.tiny(vocab=1000, seq=128)
    g = torch.Generator().manual_seed(7)
    lb = 4
    tok = torch.randint(0, cfg.vocab_size, (lb * world, 129), generator=g)
    x, y = tok[:, :-1].contiguous(), tok[:, 1:].contiguous()
    hp = dict(lr=1e-3, weight_decay=0.1, max_grad_norm=1.0)
    res = {}
    for mode in ("fused", "nccl"):
        m = GPTModel(cfg, device=dev, seed=3, bucket_align=64 * world)
        zero_data_parallel(m, mode=mode, **hp)
        m.enable_cuda_graph()
        losses = []
        for _ in range(4):  # eager, capture + replay, replays
            l = m.train_step(x[rank * lb : (rank + 1) * lb].to(dev), y[rank * lb : (rank + 1) * lb].to(dev))
            lt = l.detach().clone()
            dist.all_reduce(lt)
            losses.append(float(lt) / world)
        torch.cuda.synchronize()
        m.param_sync.begin_forward()  # gather the last update
        m.param_sync.finish()
        torch.cuda.synchronize()
        w = m.fp.p16.float()
        w0 = w.clone()
        dist.broadcast(w0, 0)
        res[mode] = {"losses": losses, "replica_max_diff": float((w - w0).abs().max()),
                     "early_vocab": bool(m.param_sync.early_vocab), "collectives": m.param_sync.mode}
        m.release_cuda_graph()
        if m.param_sync.vocab_route is not None:
            m.param_sync.vocab_route.close()
        if m.param_sync.comm is not None:
            m.param_sync.comm.close()
    if rank == 0:
        from scirs_b200.optim.fused import FusedFlatOptimizer

        m = GPTModel(cfg, device=dev, seed=3)
        m.optimizer = FusedFlatOptimizer(m.fp, "adamw", lr=1e-3, betas=(0.9, 0.999), weight_decay=0.1,
                                         max_grad_norm=1.0)
        ref = [float(m.train_step(x.to(dev), y.to(dev))) for _ in range(4)]
        res["single"] = {"losses": ref}
    _ext.check_status()
    return res


def case_zero_vit():
    """ZeRO (sharded AdamW, reduce-scatter of gradients, all-gather of bf16
    parameters) with the fused collectives and with NCCL == single-process
    training on the full batch."""
    from scirs_b200.models.vit import ViTConfig, ViTModel
    from scirs_b200.parallel.zero import zero_data_parallel

    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = ViTConfig.tiny(num_classes=10)
    g = torch.Generator().manual_seed(9)
    lb = 4
    img = torch.randn(lb * world, 3, 32, 32, generator=g)
    lab = torch.randint(0, 10, (lb * world,), generator=g)
    hp = dict(lr=1e-3, weight_decay=0.05, max_grad_norm=1.0)
    res = {}
    for mode in ("fused", "nccl"):
        m = ViTModel(cfg, device=dev, seed=3, bucket_align=64 * world)
        zero_data_parallel(m, mode=mode, **hp)
        losses = []
        sl = slice(rank * lb, (rank + 1) * lb)
        for it in range(4):
            if it == 2:
                m.enable_cuda_graph()
            l = m.train_step(img[sl].to(dev), lab[sl].to(dev))
            lt = l.detach().clone()
            dist.all_reduce(lt)
            losses.append(float(lt) / world)
        torch.cuda.synchronize()
        m.release_cuda_graph()
        full = m.param_sync.consolidated_master()
        res[mode] = {"losses": losses, "master_sum": float(full.double().sum())}
        if mode == "fused":
            m.param_sync.comm.close()
    if rank == 0:
        m = ViTModel(cfg, device=dev, seed=3, bucket_align=64 * world)
        m.configure_adamw(betas=(0.9, 0.999), **hp)
        ref = [float(m.train_step(img.to(dev), lab.to(dev))) for _ in range(4)]
        res["single"] = {"losses": ref, "master_sum": float(m.fp.master.double().sum())}
    _ext.check_status()
    return res


def case_tp_decoder():
    """Tensor-parallel decoder (fused AG->GEMM / GEMM->RS, and the NCCL
    baseline schedule) == the same model on one GPU (TP=1)."""
    from scirs_b200.models.tp_gpt import DecoderConfig, TPDecoder
    from scirs_b200.parallel.tensor_parallel import TPContext

    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = DecoderConfig.tiny(vocab=1024, seq=256)
    if world > 2:  # heads split over the ranks: 8 heads of 64
        cfg.hidden_size, cfg.num_attention_heads, cfg.intermediate_size = 512, 8, 2048
    B, S = 4, 256
    g = torch.Generator().manual_seed(21)
    toks = [torch.randint(0, cfg.vocab_size, (B, S + 1), generator=g) for _ in range(4)]
    hp = dict(lr=1e-3, weight_decay=0.0, max_grad_norm=1.0)

    def run(ctx, graph_from=2):
        m = TPDecoder(cfg, ctx, batch=B, seq=S, seed=3)
        m.configure_adamw(**hp)
        out = []
        for i, t in enumerate(toks):
            if i == graph_from:
                m.enable_cuda_graph()
            t = t.to(dev)
            out.append(float(m.train_step(t[:, :-1].contiguous(), t[:, 1:].contiguous())))
        torch.cuda.synchronize()
        m.close()
        return out

    res = {}
    for mode in ("fused", "nccl"):
        ctx = TPContext(TPDecoder.heap_bytes(cfg, B, S, world), mode=mode, timeout_s=10.0)
        res[mode] = {"losses": run(ctx)}
        ctx.close()
    sub = dist.new_group([0])
    if rank == 0:
        ctx = TPContext(TPDecoder.heap_bytes(cfg, B, S, 1), mode="fused", group=sub)
        res["single"] = {"losses": run(ctx, graph_from=99)}
        ctx.close()
    _ext.check_status()
    return res


def case_ep_moe():
    """Expert parallel MoE on the peer-memory dispatch / combine kernels
    against the NCCL all-to-all path (fp32), three steps (buffer reuse)."""
    from scirs_b200.nn.moe import ExpertParallelMoE, MoEConfig

    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = MoEConfig(num_experts=2 * world, expert_dim=256, top_k=2, capacity_factor=1.0)
    peer = ExpertParallelMoE(128, cfg, seed=3, transport="peer", timeout_s=10.0).to(dev)
    ref = ExpertParallelMoE(128, cfg, seed=3, transport="nccl").to(dev)
    res = {}
    for it in range(3):
        g = torch.Generator().manual_seed(100 * it + rank)
        x = torch.randn(384, 128, generator=g).to(dev)
        xp, xr = x.clone().requires_grad_(True), x.clone().requires_grad_(True)
        for m in (peer, ref):
            m.zero_grad(set_to_none=True)
        yp, yr = peer(xp), ref(xr)
        yp.square().sum().backward()
        yr.square().sum().backward()
        rel = lambda a, b: float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))  # noqa: E731
        res[f"it{it}"] = {"y": rel(yp, yr), "dx": rel(xp.grad, xr.grad),
                          "gate": rel(peer.gate.weight.grad, ref.gate.weight.grad),
                          "w1": rel(peer.experts.w1.grad, ref.experts.w1.grad),
                          "w2": rel(peer.experts.w2.grad, ref.experts.w2.grad)}
    # bf16 parameters: the expert GEMMs read the received rows without a cast
    pb = ExpertParallelMoE(128, cfg, seed=3, transport="peer", timeout_s=10.0).to(dev, torch.bfloat16)
    xb = torch.randn(384, 128, generator=torch.Generator().manual_seed(rank)).to(dev, torch.bfloat16)
    for _ in range(2):
        xb.grad = None
        pb(xb.requires_grad_(True)).float().square().sum().backward()
    res["bf16_finite"] = {"dx": 0.0 if bool(torch.isfinite(xb.grad).all()) else 1.0}
    torch.cuda.synchronize()
    _ext.check_status()
    peer.close()
    pb.close()
    return res


def case_pp_gpt():
    """Pipeline-parallel GPT (1F1B and GPipe, 4 micro-batches) == single-
    process training on the whole batch; the tied embedding copies on the
    first and last stage stay identical."""
    from scirs_b200.models.gpt import GPTConfig, GPTModel
    from scirs_b200.models.gpt_pipeline import GPTPipelineStage

    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = GPTConfig.tiny(vocab=1024, seq=128)
    cfg.num_hidden_layers = 2 * world
    g = torch.Generator().manual_seed(11)
    tok = torch.randint(0, cfg.vocab_size, (8, 129), generator=g)
    x, y = tok[:, :-1].contiguous().to(dev), tok[:, 1:].contiguous().to(dev)
    res = {}
    for sched in ("1f1b", "gpipe", "1f1b_graph"):
        st = GPTPipelineStage(cfg, stage=rank, num_stages=world, num_micro=4, device=dev, seed=5,
                              schedule=sched.split("_")[0])
        st.configure_adamw(lr=1e-3, weight_decay=0.1, max_grad_norm=0.5)
        if sched.endswith("graph"):
            st.enable_cuda_graph()
        losses = []
        for _ in range(4 if sched.endswith("graph") else 3):  # graph: eager, capture + replay, replays
            l = st.train_step(x if st.first else None, y if st.last else None, shape=(8, 128))
            v = torch.tensor([float(l) if l is not None else 0.0], device=dev)
            dist.all_reduce(v)
            losses.append(float(v))
        torch.cuda.synchronize()
        st.release_cuda_graph()
        wsum = float(st.fp.m("wte").double().abs().sum()) if (st.first or st.last) else 0.0
        sums = [None] * world
        dist.all_gather_object(sums, wsum)
        res[sched] = {"losses": losses, "tied_diff": abs(sums[0] - sums[-1])}
    if rank == 0:
        m = GPTModel(cfg, device=dev, seed=5)
        m.configure_adamw(lr=1e-3, weight_decay=0.1, max_grad_norm=0.5)
        res["single"] = {"losses": [float(m.train_step(x, y)) for _ in range(4)]}
    _ext.check_status()
    return res


def main():
    case, out = sys.argv[1], sys.argv[2]
    sdist.init(timeout_s=60)
    res = {"collectives": case_collectives, "nvls": case_nvls, "ring_attn": case_ring_attn, "dp_gpt": case_dp_gpt, "zero_gpt": case_zero_gpt, "zero_vit": case_zero_vit,
           "tp_decoder": case_tp_decoder, "ep_moe": case_ep_moe, "pp_gpt": case_pp_gpt}[case]()
    if dist.get_rank() == 0:
        json.dump(res, open(out, "w"))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
