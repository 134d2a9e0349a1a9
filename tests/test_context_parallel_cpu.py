"""Ring attention over gloo ranks equals full attention on the concatenated
sequence, forward and gradients, causal and not."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _data(world, B=2, Sc=8, H=2, D=16):
    g = torch.Generator().manual_seed(3)
    q, k, v, do = (torch.randn(B, world * Sc, H, D, generator=g, dtype=torch.float64) for _ in range(4))
    return q, k, v, do


def _worker(rank, world, port, out, causal):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from scirs_b200.parallel.context_parallel import ring_attention

        q, k, v, do = _data(world)
        Sc = q.shape[1] // world
        sl = slice(rank * Sc, (rank + 1) * Sc)
        ql, kl, vl = (t[:, sl].clone().requires_grad_(True) for t in (q, k, v))
        o, lse = ring_attention(ql, kl, vl, causal=causal)
        o.backward(do[:, sl])
        torch.save({"o": o.detach(), "lse": lse.detach(), "dq": ql.grad, "dk": kl.grad, "dv": vl.grad},
                   f"{out}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(180)
@pytest.mark.parametrize("world,causal", [(2, True), (3, True), (3, False)])
def test_ring_attention_matches_full(tmp_path, world, causal):
    out = str(tmp_path / "ring")
    mp.start_processes(_worker, args=(world, _free_port(), out, causal), nprocs=world, start_method="spawn")
    q, k, v, do = _data(world)
    qf, kf, vf = (t.clone().requires_grad_(True) for t in (q, k, v))
    scale = q.shape[-1] ** -0.5
    s = torch.einsum("bqhd,bkhd->bhqk", qf, kf) * scale
    if causal:
        S = s.shape[-1]
        s = s.masked_fill(torch.ones(S, S, dtype=torch.bool).triu(1), float("-inf"))
    lse = torch.logsumexp(s, -1)
    o = torch.einsum("bhqk,bkhd->bqhd", torch.softmax(s, -1), vf)
    o.backward(do)
    Sc = q.shape[1] // world
    for r in range(world):
        res = torch.load(f"{out}.{r}")
        sl = slice(r * Sc, (r + 1) * Sc)
        # the per-chunk math runs in fp32
        torch.testing.assert_close(res["o"].double(), o[:, sl].detach(), rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(res["lse"].double(), lse[:, :, sl].detach(), rtol=1e-4, atol=1e-5)
        for name, ref in (("dq", qf.grad), ("dk", kf.grad), ("dv", vf.grad)):
            torch.testing.assert_close(res[name].double(), ref[:, sl], rtol=1e-4, atol=1e-5)
