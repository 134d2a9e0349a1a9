"""ZeRO sharding logic on gloo ranks (CPU): two ranks with half the batch
each must reach the same parameters as one process on the full batch (ViT
encoder and the GPT decoder with its separate wte / wpe buckets)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from scirs_b200.models.gpt import GPTConfig, GPTModel
from scirs_b200.models.vit import ViTConfig, ViTModel
from scirs_b200.optim.fused import FusedFlatOptimizer


def _cfg():
    c = ViTConfig.tiny(num_classes=10)
    c.embed_dim, c.num_heads, c.mlp_dim, c.num_layers = 128, 2, 256, 2
    return c


def _data(kind, steps=3, B=4):
    g = torch.Generator().manual_seed(11)
    if kind == "gpt":
        out = []
        for _ in range(steps):
            t = torch.randint(0, 256, (B, 33), generator=g)
            out.append((t[:, :-1].contiguous(), t[:, 1:].contiguous()))
        return out
    return [(torch.randn(B, 3, 32, 32, generator=g), torch.randint(0, 10, (B,), generator=g)) for _ in range(steps)]


def _model(kind, world):
    if kind == "gpt":
        return GPTModel(GPTConfig.tiny(vocab=256, seq=32), device="cpu", seed=5, bucket_align=64 * world)
    return ViTModel(_cfg(), device="cpu", seed=5, bucket_align=64 * world)


HP = dict(lr=3e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, max_grad_norm=0.5)


def _worker(rank, world, port, out, kind):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from scirs_b200.parallel.zero import zero_data_parallel

        torch.manual_seed(0)
        m = _model(kind, world)
        zero_data_parallel(m, **HP)
        per = 4 // world
        losses = []
        for img, lab in _data(kind):
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
@pytest.mark.parametrize("kind", ["vit", "gpt"])
def test_zero_matches_single_process(tmp_path, kind):
    world = 2
    out = str(tmp_path / "zero.pt")
    mp.start_processes(_worker, args=(world, _free_port(), out, kind), nprocs=world, start_method="spawn")
    res = torch.load(out)
    m = _model(kind, world)
    m.optimizer = FusedFlatOptimizer(m.fp, "adamw", **HP)
    for img, lab in _data(kind):
        m.train_step(img, lab)
    d = (res["master"] - m.fp.master).abs()
    for name in m.fp.order:
        sl = m.fp.slots[name]
        err = d[sl.offset : sl.offset + sl.numel]
        e = float(err.max())
        if kind == "gpt" and not name.endswith("c_attn.bias"):
            # bf16 activations of half batches differ from the full batch by
            # rounding; AdamW turns that into up to +-lr per step on the few
            # elements whose gradient is near zero. A layout error would move
            # most elements.
            assert e < 3.1 * HP["lr"], (name, e)
            assert float((err > 1e-4).float().mean()) < 0.01, (name, float((err > 1e-4).float().mean()))
            continue
        # the key bias has an exactly-zero gradient (softmax is invariant to
        # it), so Adam amplifies rounding noise there into +-lr steps
        tol = 3.1 * HP["lr"] if name.endswith("c_attn.bias") else 1e-3
        assert e < tol, (name, e)
