"""Mixture of experts: routing/capacity/aux-loss semantics against a
per-token restatement, gradients, and expert parallelism over gloo ranks
against the single-device layer."""
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from scirs_b200.nn.moe import ExpertParallelMoE, MixtureOfExperts, MoEConfig


def _loop_reference(m: MixtureOfExperts, x2: torch.Tensor):
    cfg = m.config
    T, E, k = x2.shape[0], cfg.num_experts, cfg.top_k
    probs = torch.softmax(m.gate(x2).double(), -1)
    cap = max(1, math.ceil(T * cfg.capacity_factor / E))
    count = [0] * E
    out = torch.zeros(T, x2.shape[1], dtype=torch.float64)
    assigned = [0] * E
    for t in range(T):
        order = sorted(range(E), key=lambda e: -float(probs[t, e].detach()))[:k]
        ws = probs[t, order]
        ws = ws / ws.sum()
        for e, w in zip(order, ws):
            assigned[e] += 1
            if count[e] >= cap:
                continue
            count[e] += 1
            ex = m.experts
            h = torch.relu(x2[t].double() @ ex.w1[e].double() + ex.b1[e].double())
            out[t] += w * (h @ ex.w2[e].double() + ex.b2[e].double())
    f = torch.tensor(assigned, dtype=torch.float64) / T
    aux = cfg.load_balance_coeff * E * float((f * probs.mean(0)).sum())
    return out, aux


@pytest.mark.parametrize("k,cf", [(2, 1.25), (2, 0.5), (1, 1.0)])
def test_moe_matches_per_token_reference(k, cf):
    torch.manual_seed(0)
    cfg = MoEConfig(num_experts=4, expert_dim=16, top_k=k, capacity_factor=cf)
    m = MixtureOfExperts(8, cfg, seed=3)
    x = torch.randn(2, 5, 8)
    y = m(x)
    ref, aux = _loop_reference(m, x.reshape(-1, 8))
    torch.testing.assert_close(y.reshape(-1, 8).double(), ref, rtol=1e-5, atol=1e-5)
    assert abs(float(m.last_aux_loss()) - aux) < 1e-6
    if cf < 1:
        assert (m.last_routing.slot < 0).any()  # some assignments were dropped


def test_moe_gradients_flow():
    torch.manual_seed(0)
    m = MixtureOfExperts(8, MoEConfig(num_experts=4, expert_dim=16, top_k=2))
    x = torch.randn(12, 8, requires_grad=True)
    (m(x).square().mean() + m.last_aux_loss()).backward()
    for n, p in m.named_parameters():
        assert p.grad is not None and float(p.grad.abs().sum()) > 0, n
    assert float(x.grad.abs().sum()) > 0
    assert MoEConfig(gating_type="switch").top_k == 1


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ep_worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = MoEConfig(num_experts=4, expert_dim=16, top_k=2, capacity_factor=1.0)
        ep = ExpertParallelMoE(8, cfg, seed=7)
        ref = MixtureOfExperts(8, cfg, seed=7)
        g = torch.Generator().manual_seed(100 + rank)
        x = torch.randn(10, 8, generator=g)
        xe, xr = x.clone().requires_grad_(True), x.clone().requires_grad_(True)
        ye, yr = ep(xe), ref(xr)
        ye.square().sum().backward()
        yr.square().sum().backward()
        lo = rank * 2
        res = {
            "y": (ye - yr).abs().max().item(),
            "dx": (xe.grad - xr.grad).abs().max().item(),
            "gate": (ep.gate.weight.grad - ref.gate.weight.grad).abs().max().item(),
        }
        # expert gradients: this rank's experts see every rank's tokens, so
        # they equal the sum over ranks of the single-device gradients
        gsum = ref.experts.w1.grad.clone()
        dist.all_reduce(gsum)
        res["w1"] = (ep.experts.w1.grad - gsum[lo:lo + 2]).abs().max().item()
        torch.save(res, f"{out}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_expert_parallel_matches_single_device(tmp_path):
    out = str(tmp_path / "ep")
    mp.start_processes(_ep_worker, args=(2, _free_port(), out), nprocs=2, start_method="spawn")
    for r in range(2):
        res = torch.load(f"{out}.{r}")
        for k, v in res.items():
            assert v < 1e-5, (r, k, v)
