"""Pipeline parallelism (GPipe and 1F1B) on gloo ranks: gradients equal the
single-process gradients of the whole model."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn as nn

from scirs_b200.parallel.pipeline import (PipelineParallel, PipelineSchedule, PipelineStage, generate_1f1b_schedule,
                                          split_micro_batches)


def _model():
    torch.manual_seed(0)
    return nn.Sequential(nn.Linear(8, 16), nn.Tanh(), nn.Linear(16, 16), nn.Tanh(), nn.Linear(16, 16), nn.Tanh(),
                         nn.Linear(16, 3))


def _data():
    g = torch.Generator().manual_seed(1)
    return torch.randn(24, 8, generator=g), torch.randint(0, 3, (24,), generator=g)


CUTS = {2: [0, 4, 7], 3: [0, 2, 4, 7]}


def _worker(rank, world, port, sched, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        full = _model()
        a, b = CUTS[world][rank], CUTS[world][rank + 1]
        mod = nn.Sequential(*list(full.children())[a:b])
        stage = PipelineStage(mod, rank, world, act_shape=(6, 16))
        pp = PipelineParallel(stage, PipelineSchedule(sched))
        x, y = _data()
        loss = pp.run_schedule(split_micro_batches(x, y, 4), nn.functional.cross_entropy)
        grads = {f"{a + int(n.split('.')[0])}.{n.split('.', 1)[1]}": p.grad for n, p in mod.named_parameters()}
        torch.save({"grads": grads, "loss": loss, "stash": pp.max_stash}, f"{out}.{rank}")
    finally:
        dist.destroy_process_group()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_1f1b_schedule_shape():
    acts = generate_1f1b_schedule(4, 8, 0)
    assert acts[:4] == [("F", 0), ("F", 1), ("F", 2), ("F", 3)] and acts[4] == ("B", 0)
    assert sorted(acts) == sorted([("F", i) for i in range(8)] + [("B", i) for i in range(8)])
    assert generate_1f1b_schedule(4, 8, 3)[:2] == [("F", 0), ("B", 0)]


@pytest.mark.timeout(300)
@pytest.mark.parametrize("world,sched", [(2, "1f1b"), (3, "1f1b"), (2, "gpipe")])
def test_pipeline_gradients_match(tmp_path, world, sched):
    out = str(tmp_path / "pp")
    mp.start_processes(_worker, args=(world, _port(), sched, out), nprocs=world, start_method="spawn")
    full = _model()
    x, y = _data()
    nn.functional.cross_entropy(full(x), y).backward()
    ref = {n: p.grad for n, p in full.named_parameters()}
    got = {}
    for r in range(world):
        d = torch.load(f"{out}.{r}")
        got.update(d["grads"])
        if r == world - 1:
            assert d["loss"] is not None
        if sched == "1f1b":
            assert d["stash"] <= world - r
    assert set(got) == set(ref)
    for n in ref:
        assert torch.allclose(got[n], ref[n], atol=1e-5), n
