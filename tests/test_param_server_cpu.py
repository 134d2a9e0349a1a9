"""Parameter server (synchronous, bounded-staleness and asynchronous modes,
leases, snapshots), vector clocks and push-sum gossip, in process and across
gloo ranks."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from scirs_b200.parallel import param_server as P


def _ps(staleness, n=3, **kw):
    ps = P.ParameterServer(P.PSConfig(num_workers=n, staleness=staleness, **kw))
    ids = [ps.join(now=0.0) for _ in range(n)]
    ps.create("w", torch.zeros(4))
    return ps, ids


def test_synchronous_round_combines_after_every_worker_advanced():
    ps, ids = _ps(0)
    assert ps.config.mode is P.Consistency.SYNC
    for w, v in zip(ids, (1.0, 2.0, 6.0)):
        assert ps.push(w, "w", torch.full((4,), v), now=0.0) is False
    ps.advance(0, now=0.0)
    ps.advance(1, now=0.0)
    assert ps.waiting_on(0, now=0.0) == [2]
    assert torch.equal(ps.pull("w")[0], torch.zeros(4))  # round not committed yet
    ps.advance(2, now=0.0)
    v, ver = ps.pull("w")
    assert torch.equal(v, torch.full((4,), 3.0)) and ver == 1 and ps.pending() == 0


def test_combine_rules():
    vals = [torch.full((2,), float(i)) for i in range(3)]
    assert torch.equal(P.combine_sum(vals, [0, 1, 2]), torch.full((2,), 3.0))
    wm = P.combine_weighted([0.0, 1.0, 3.0])(vals, [0, 1, 2])
    assert torch.allclose(wm, torch.full((2,), 7.0 / 4.0))
    ps, ids = _ps(0, combine="sum", apply="sgd", lr=0.5)
    for w in ids:
        ps.push(w, "w", torch.ones(4), now=0.0)
        ps.advance(w, now=0.0)
    assert torch.equal(ps.pull("w")[0], torch.full((4,), -1.5))


def test_asynchronous_and_bounded_staleness():
    ps, _ = _ps(None)
    assert ps.config.mode is P.Consistency.ASYNC
    assert ps.push(1, "w", torch.ones(4), clock=5, now=0.0)
    assert torch.equal(ps.pull("w")[0], torch.ones(4))
    ssp, ids = _ps(2)
    assert ssp.push(0, "w", torch.ones(4), clock=2, now=0.0)  # floor 0 + bound 2: admitted
    assert not ssp.push(0, "w", torch.full((4,), 9.0), clock=3, now=0.0)  # too far ahead: held
    assert torch.equal(ssp.pull("w")[0], torch.ones(4)) and ssp.pending() == 1
    for w in ids:  # floor -> 1: clock 3 becomes admissible
        ssp.advance(w, now=0.0)
    assert torch.equal(ssp.pull("w")[0], torch.full((4,), 9.0)) and ssp.pending() == 0


def test_lapsed_lease_releases_synchronous_round_and_snapshots():
    ps, ids = _ps(0, lease_s=10.0, snapshot_every=1)
    for w in (0, 1):
        ps.push(w, "w", torch.full((4,), float(w)), now=1.0)
        ps.advance(w, now=1.0)
    assert ps.waiting_on(0, now=1.0) == [2]
    ps.heartbeat(0, now=8.0)
    ps.heartbeat(1, now=8.0)
    assert ps.reap(now=12.0) == [2]  # worker 2's lease (joined at 0) lapsed
    assert torch.equal(ps.pull("w")[0], torch.full((4,), 0.5))
    with pytest.raises(RuntimeError):
        ps.fail(2)
    with pytest.raises(RuntimeError):
        ps.push(2, "w", torch.ones(4), now=12.0)
    snap = ps.snapshots[-1]
    assert snap.version == 1
    ps2 = P.ParameterServer.from_snapshot(snap, ps.config, now=12.0)
    assert torch.equal(ps2.pull("w")[0], torch.full((4,), 0.5))
    assert ps2.live_workers(now=12.0) == [0, 1]


def test_vector_clock():
    a, b = P.VectorClock(3), P.VectorClock(3)
    a.tick(0)
    b.observe(a).tick(1)
    assert a.happens_before(b) and not b.happens_before(a)
    assert b.compare(a) is P.Order.AFTER and a.copy().compare(a) is P.Order.EQUAL
    a.tick(2)
    assert a.concurrent(b)


@pytest.mark.parametrize("topo", ["ring", "random", "exponential"])
def test_push_sum_converges_to_mean(topo):
    vals = [torch.tensor([float(i), 2.0 * i]) for i in range(6)]
    g = P.PushSum(vals, topology=topo, seed=1)
    P_0 = g.mixing_matrix(0)
    assert torch.allclose(P_0.sum(0), torch.ones(6, dtype=torch.float64))  # column stochastic
    n = g.run(1e-6, max_rounds=400)
    assert n < 400
    for i in range(6):
        assert torch.allclose(g.estimate(i), torch.tensor([2.5, 5.0], dtype=torch.float64), atol=1e-5)


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
        ps = P.ShardedParameterServer(apply="sgd", lr=0.5)
        for k in ("a", "b", "c", "d"):
            ps.create(k, torch.zeros(3))
        new = ps.step({k: torch.full((3,), float(rank)) for k in ("a", "b", "c", "d")})
        ring = P.push_sum_allreduce(torch.tensor([float(rank), 10.0 * rank]), rounds=60)
        expo = P.push_sum_allreduce(torch.tensor([float(rank)]), rounds=60, topology="exponential")
        torch.save({"new": new, "ring": ring, "expo": expo, "owned": ps.owned()}, f"{out}.{rank}")
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_sharded_server_and_gossip_across_ranks(tmp_path):
    out = str(tmp_path / "ps")
    mp.start_processes(_worker, args=(3, _free_port(), out), nprocs=3, start_method="spawn")
    owned = []
    for r in range(3):
        res = torch.load(f"{out}.{r}")
        for k in "abcd":
            assert torch.equal(res["new"][k], torch.full((3,), -0.5))  # 0 - 0.5 * mean(0, 1, 2)
        assert torch.allclose(res["ring"], torch.tensor([1.0, 10.0]), atol=1e-4)
        assert torch.allclose(res["expo"], torch.tensor([1.0]), atol=1e-4)
        owned += res["owned"]
    assert sorted(owned) == list("abcd")
