"""Parameter server consistency models, fault tolerance, vector clocks and
gossip averaging (in process and across gloo ranks)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from scirs_b200.parallel import param_server as P


def _ps(consistency, n=3, **kw):
    ps = P.ParameterServer(P.ParamServerConfig(num_workers=n, consistency=consistency, **kw))
    for _ in range(n):
        ps.register_worker()
    ps.init_parameter("w", torch.zeros(4))
    return ps


def test_bsp_barrier_and_aggregation():
    ps = _ps(P.ConsistencyModel.BSP)
    for wid in range(2):
        ps.push(P.ParameterUpdate("w", torch.full((4,), float(wid + 1)), wid, 1))
    with pytest.raises(RuntimeError, match="has not pushed"):
        ps.barrier_sync()
    ps.push(P.ParameterUpdate("w", torch.full((4,), 6.0), 2, 1))
    ps.barrier_sync()
    v, ver = ps.pull("w", 0)
    assert torch.equal(v, torch.full((4,), 3.0)) and ver == 1 and ps.global_version == 1
    us = [P.ParameterUpdate("w", torch.full((2,), float(i)), i, 0) for i in range(3)]
    assert torch.equal(P.aggregate_updates(us, P.AggregationMethod.sum()), torch.full((2,), 3.0))
    wm = P.aggregate_updates(us, P.AggregationMethod.weighted_mean([0.0, 1.0, 3.0]))
    assert torch.allclose(wm, torch.full((2,), 7.0 / 4.0))


def test_asp_and_ssp():
    ps = _ps(P.ConsistencyModel.ASP)
    ps.push(P.ParameterUpdate("w", torch.ones(4), 1, 5))
    assert torch.equal(ps.pull("w", 0)[0], torch.ones(4))
    ssp = _ps(P.ConsistencyModel.SSP, max_staleness=2)
    ssp.push(P.ParameterUpdate("w", torch.ones(4), 0, 2))  # others at 0: staleness 2 -> applied
    assert torch.equal(ssp.pull("w", 0)[0], torch.ones(4))
    ssp.push(P.ParameterUpdate("w", torch.full((4,), 9.0), 0, 3))  # staleness 3 -> buffered
    assert torch.equal(ssp.pull("w", 0)[0], torch.ones(4))
    assert len(ssp.update_buffer["w"]) == 1


def test_fault_tolerant_ps_and_checkpoints():
    ft = P.FaultTolerantPS(P.ParamServerConfig(num_workers=3, checkpoint_interval=10))
    for _ in range(3):
        ft.server.register_worker()
    ft.server.init_parameter("w", torch.zeros(2))
    for w in range(3):
        ft.heartbeat(w, 100)
    ft.heartbeat(0, 200)
    ft.heartbeat(1, 200)
    assert ft.check_workers(250, 100) == [2]
    ft.handle_worker_failure(2)
    with pytest.raises(RuntimeError):
        ft.handle_worker_failure(2)
    # the dead worker no longer blocks the BSP barrier
    for w in range(2):
        ft.server.push(P.ParameterUpdate("w", torch.full((2,), float(w)), w, 1))
    ft.server.barrier_sync()
    assert ft.checkpoint_if_needed(5) is None
    cp = ft.checkpoint_if_needed(10)
    assert cp is not None and cp.version == 1
    ft2 = P.FaultTolerantPS.recover_from_checkpoint(cp, ft.server.config)
    assert torch.equal(ft2.server.pull("w", 0)[0], torch.full((2,), 0.5))
    assert not ft2.server.workers[2].is_alive


def test_vector_clock():
    a, b = P.VectorClock(3), P.VectorClock(3)
    a.increment(0)
    b.merge(a)
    b.increment(1)
    assert a.happens_before(b) and not b.happens_before(a)
    a.increment(2)
    assert a.is_concurrent(b)


@pytest.mark.parametrize("topo", ["ring", "random", "exponential"])
def test_gossip_converges_to_mean(topo):
    vals = [torch.tensor([float(i), 2.0 * i]) for i in range(6)]
    g = P.GossipAllReduce(topo, num_rounds=400, num_nodes=6, seed=1)
    g.init_values(vals)
    n = g.run_to_convergence(1e-6)
    assert n < 400
    for i in range(6):
        assert torch.allclose(g.get_estimate(i), torch.tensor([2.5, 5.0], dtype=torch.float64), atol=1e-5)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = P.PSGroup()
        g.init_parameter("w", torch.zeros(3))
        agg = g.step("w", torch.full((3,), float(rank)), version=1)
        est = P.gossip_allreduce(torch.tensor([float(rank), 10.0 * rank]), rounds=60)
        torch.save({"agg": agg, "est": est}, f"{out}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_ps_group_and_gossip_across_ranks(tmp_path):
    out = str(tmp_path / "ps")
    mp.start_processes(_worker, args=(3, _free_port(), out), nprocs=3, start_method="spawn")
    for r in range(3):
        res = torch.load(f"{out}.{r}")
        assert torch.equal(res["agg"], torch.ones(3))
        assert torch.allclose(res["est"], torch.tensor([1.0, 10.0]), atol=1e-4)
