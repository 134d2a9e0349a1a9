"""ZeRO sharding logic on gloo ranks (CPU): two ranks with half the batch
each must reach the same parameters as one process on the full batch."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from scirs_b200.models.vit import ViTConfig, ViTModel
from scirs_b200.optim.fused import FusedFlatOptimizer


def _cfg():
    c = ViTConfig.tiny(num_classes=10)
    c.embed_dim, c.num_heads, c.mlp_dim, c.num_layers = 128, 2, 256, 2
    return c


def _data(steps=3, B=4):
    g = torch.Generator().manual_seed(11)
    return [(torch.randn(B, 3, 32, 32, generator=g), torch.randint(0, 10, (B,), generator=g)) for _ in range(steps)]


HP = dict(lr=3e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, max_grad_norm=0.5)


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from scirs_b200.parallel.zero import zero_data_parallel

        torch.manual_seed(0)
        m = ViTModel(_cfg(), device="cpu", seed=5, bucket_align=64 * world)
        zero_data_parallel(m, **HP)
        per = 4 // world
        losses = []
        for img, lab in _data():
            sl = slice(rank * per, (rank + 1) * per)
            losses.append(float(m.train_step(img[sl], lab[sl])))
        full = m.param_sync.consolidated_master()
        if rank == 0:
            torch.save({"master": full, "losses": losses}, out)
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.timeout(300)
def test_zero_matches_single_process(tmp_path):
    world = 2
    out = str(tmp_path / "zero.pt")
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, start_method="spawn")
    res = torch.load(out)
    m = ViTModel(_cfg(), device="cpu", seed=5, bucket_align=64 * world)
    m.optimizer = FusedFlatOptimizer(m.fp, "adamw", **HP)
    for img, lab in _data():
        m.train_step(img, lab)
    d = (res["master"] - m.fp.master).abs()
    for name in m.fp.order:
        sl = m.fp.slots[name]
        e = float(d[sl.offset : sl.offset + sl.numel].max())
        # the key bias has an exactly-zero gradient (softmax is invariant to
        # it), so Adam amplifies rounding noise there into +-lr steps
        tol = 3.1 * HP["lr"] if name.endswith("c_attn.bias") else 1e-3
        assert e < tol, (name, e)
