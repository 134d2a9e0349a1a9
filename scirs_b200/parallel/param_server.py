"""Parameter server, gossip averaging and vector clocks.

`ParameterServer` keeps named parameter tensors (any device) and applies the
workers' pushed values under a consistency model
(scirs2-core/src/distributed/param_server/server.rs:27-300, types.rs:5-140):
  BSP  updates are buffered; `barrier_sync` (all live workers pushed) sets
       every key to the aggregate (mean / sum / weighted mean by worker id)
       of its buffered values and bumps the global version
  ASP  a push replaces the value immediately
  SSP  a push whose version is within `max_staleness` of the slowest live
       worker is applied immediately; a staler one waits in the buffer for
       the next barrier
`FaultTolerantPS` adds heartbeats, dead-worker handling (a dead worker no
longer blocks the BSP barrier) and periodic checkpoints
(fault_tolerance.rs:136-250); `VectorClock` orders events causally
(fault_tolerance.rs:257-340).

`PSGroup` runs the BSP protocol across processes: rank `server` owns the
store; each step every rank's pushed tensor is gathered to the server
(torch.distributed gather; NCCL on GPUs), aggregated there, and the new
value is broadcast back (pull).

Gossip: `GossipAllReduce` is the push-sum protocol (gossip.rs:59-330): in a
round every node keeps (1 - f) of its (value, weight) and sends f to a peer
(ring: r + 1; random; exponential: r + 2^j); estimates are value / weight
and converge to the average. `gossip_allreduce` runs the ring variant across
processes with point-to-point send/recv.
"""
from __future__ import annotations

import copy
import enum
import random
import threading
from dataclasses import dataclass, field

import torch
import torch.distributed as dist


class ConsistencyModel(enum.Enum):
    BSP = "bsp"
    ASP = "asp"
    SSP = "ssp"


@dataclass
class AggregationMethod:
    kind: str = "mean"  # "mean" | "sum" | "weighted_mean"
    weights: list[float] | None = None

    @staticmethod
    def mean():
        return AggregationMethod("mean")

    @staticmethod
    def sum():
        return AggregationMethod("sum")

    @staticmethod
    def weighted_mean(weights):
        return AggregationMethod("weighted_mean", list(weights))


@dataclass
class ParamServerConfig:
    num_workers: int = 4
    consistency: ConsistencyModel = ConsistencyModel.BSP
    max_staleness: int = 0
    aggregation: AggregationMethod = field(default_factory=AggregationMethod)
    checkpoint_interval: int = 100
    replication_factor: int = 1


@dataclass
class ParameterUpdate:
    key: str
    values: torch.Tensor
    worker_id: int
    version: int


@dataclass
class WorkerState:
    worker_id: int
    version: int = 0
    is_alive: bool = True
    last_heartbeat: int = 0


@dataclass
class ServerCheckpoint:
    parameters: dict
    version: int
    worker_states: list


def aggregate_updates(updates: list[ParameterUpdate], method: AggregationMethod) -> torch.Tensor | None:
    if not updates:
        return None
    vals = torch.stack([u.values for u in updates])
    if method.kind == "sum":
        return vals.sum(0)
    if method.kind == "weighted_mean":
        w = torch.tensor([(method.weights or [])[u.worker_id] if u.worker_id < len(method.weights or []) else 1.0
                          for u in updates], dtype=vals.dtype, device=vals.device)
        tot = float(w.sum())
        s = (vals * w.view(-1, *([1] * (vals.dim() - 1)))).sum(0)
        return s if abs(tot) < 1e-300 else s / tot
    return vals.mean(0)


class ParameterServer:
    def __init__(self, config: ParamServerConfig | None = None):
        self.config = config or ParamServerConfig()
        self.parameters: dict[str, tuple[torch.Tensor, int]] = {}
        self.workers: list[WorkerState] = []
        self.global_version = 0
        self.update_buffer: dict[str, list[ParameterUpdate]] = {}
        self.bsp_pushed: list[bool] = []
        self._lock = threading.RLock()

    def register_worker(self) -> int:
        with self._lock:
            wid = len(self.workers)
            self.workers.append(WorkerState(wid))
            self.bsp_pushed.append(False)
            return wid

    def init_parameter(self, key: str, values: torch.Tensor):
        with self._lock:
            self.parameters[key] = (values.detach().clone(), 0)

    def _check_worker(self, wid: int):
        if wid >= len(self.workers):
            raise ValueError(f"unknown worker id {wid}")

    def push(self, update: ParameterUpdate):
        with self._lock:
            self._check_worker(update.worker_id)
            w = self.workers[update.worker_id]
            if not w.is_alive:
                raise RuntimeError(f"worker {update.worker_id} is not alive")
            w.version = update.version
            c = self.config.consistency
            if c == ConsistencyModel.BSP:
                self.update_buffer.setdefault(update.key, []).append(update)
                self.bsp_pushed[update.worker_id] = True
            elif c == ConsistencyModel.ASP:
                self._apply(update)
            else:
                slowest = min((x.version for x in self.workers if x.is_alive), default=0)
                if update.version - slowest <= self.config.max_staleness:
                    self._apply(update)
                else:
                    self.update_buffer.setdefault(update.key, []).append(update)

    def _apply(self, u: ParameterUpdate):
        self.parameters[u.key] = (u.values.detach().clone(), u.version)

    def pull(self, key: str, worker_id: int) -> tuple[torch.Tensor, int]:
        with self._lock:
            self._check_worker(worker_id)
            if key not in self.parameters:
                raise KeyError(f"unknown key {key}")
            v, ver = self.parameters[key]
            return v.clone(), ver

    def ready(self) -> bool:
        return all(self.bsp_pushed[w.worker_id] for w in self.workers if w.is_alive)

    def barrier_sync(self):
        with self._lock:
            for w in self.workers:
                if w.is_alive and not self.bsp_pushed[w.worker_id]:
                    raise RuntimeError(f"BSP barrier: worker {w.worker_id} has not pushed yet")
            for key, ups in self.update_buffer.items():
                agg = aggregate_updates(ups, self.config.aggregation)
                if agg is not None:
                    self.parameters[key] = (agg, self.global_version + 1)
            self.update_buffer.clear()
            self.bsp_pushed = [False] * len(self.workers)
            self.global_version += 1

    def checkpoint(self) -> ServerCheckpoint:
        with self._lock:
            return ServerCheckpoint({k: (v.clone(), ver) for k, (v, ver) in self.parameters.items()},
                                    self.global_version, copy.deepcopy(self.workers))

    @classmethod
    def restore(cls, cp: ServerCheckpoint, config: ParamServerConfig) -> "ParameterServer":
        ps = cls(config)
        ps.parameters = {k: (v.clone(), ver) for k, (v, ver) in cp.parameters.items()}
        ps.workers = copy.deepcopy(cp.worker_states)
        ps.global_version = cp.version
        ps.bsp_pushed = [False] * len(ps.workers)
        return ps

    def num_workers(self) -> int:
        return len(self.workers)


class FaultTolerantPS:
    def __init__(self, config: ParamServerConfig | None = None, server: ParameterServer | None = None):
        self.server = server or ParameterServer(config)
        self.last_checkpoint: ServerCheckpoint | None = None
        self.last_checkpoint_step = 0

    def heartbeat(self, worker_id: int, timestamp: int):
        self.server._check_worker(worker_id)
        w = self.server.workers[worker_id]
        w.last_heartbeat = timestamp
        w.is_alive = True

    def check_workers(self, current_time: int, timeout: int) -> list[int]:
        return [w.worker_id for w in self.server.workers
                if w.is_alive and current_time - w.last_heartbeat > timeout]

    def handle_worker_failure(self, worker_id: int):
        self.server._check_worker(worker_id)
        w = self.server.workers[worker_id]
        if not w.is_alive:
            raise RuntimeError(f"worker {worker_id} is already marked as dead")
        w.is_alive = False

    def checkpoint_if_needed(self, step: int) -> ServerCheckpoint | None:
        iv = self.server.config.checkpoint_interval
        if iv and step > 0 and step % iv == 0 and step > self.last_checkpoint_step:
            self.last_checkpoint = self.server.checkpoint()
            self.last_checkpoint_step = step
            return self.last_checkpoint
        return None

    @classmethod
    def recover_from_checkpoint(cls, cp: ServerCheckpoint, config: ParamServerConfig) -> "FaultTolerantPS":
        ft = cls(server=ParameterServer.restore(cp, config))
        ft.last_checkpoint = cp
        return ft


class VectorClock:
    def __init__(self, num_workers: int):
        self.clocks = [0] * num_workers

    def increment(self, worker_id: int):
        if worker_id >= len(self.clocks):
            raise ValueError("worker id out of range")
        self.clocks[worker_id] += 1

    def merge(self, other: "VectorClock"):
        if len(other.clocks) != len(self.clocks):
            raise ValueError("vector clock size mismatch")
        self.clocks = [max(a, b) for a, b in zip(self.clocks, other.clocks)]

    def happens_before(self, other: "VectorClock") -> bool:
        return all(a <= b for a, b in zip(self.clocks, other.clocks)) and self.clocks != other.clocks

    def is_concurrent(self, other: "VectorClock") -> bool:
        return not self.happens_before(other) and not other.happens_before(self) and self.clocks != other.clocks


# ----------------------------------------------------------------- across processes
class PSGroup:
    """BSP parameter server across the ranks of a process group."""

    def __init__(self, config: ParamServerConfig | None = None, server: int = 0, group=None):
        self.group, self.server_rank = group, server
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        cfg = config or ParamServerConfig(num_workers=self.world)
        self.ps = ParameterServer(cfg) if self.rank == server else None
        if self.ps is not None:
            for _ in range(self.world):
                self.ps.register_worker()

    def init_parameter(self, key: str, values: torch.Tensor):
        if self.ps is not None:
            self.ps.init_parameter(key, values)

    def step(self, key: str, values: torch.Tensor, version: int) -> torch.Tensor:
        """Push this rank's values, run the barrier on the server, pull the
        aggregate (returned on every rank)."""
        gathered = [torch.empty_like(values) for _ in range(self.world)] if self.ps is not None else None
        dist.gather(values.contiguous(), gathered, dst=self.server_rank, group=self.group)
        out = torch.empty_like(values)
        if self.ps is not None:
            for wid, v in enumerate(gathered):
                self.ps.push(ParameterUpdate(key, v, wid, version))
            self.ps.barrier_sync()
            out.copy_(self.ps.pull(key, self.rank)[0])
        dist.broadcast(out, src=self.server_rank, group=self.group)
        return out


class GossipAllReduce:
    def __init__(self, topology: str = "ring", num_rounds: int = 10, push_fraction: float = 0.5, num_nodes: int = 0,
                 seed: int = 0):
        assert topology in ("ring", "random", "exponential")
        self.topology, self.num_rounds, self.push_fraction = topology, num_rounds, push_fraction
        self.num_nodes = num_nodes
        self.rng = random.Random(seed)
        self.values: list[torch.Tensor] = []
        self.weights: list[float] = []
        self.rounds_completed = 0

    def init_values(self, node_values):
        if len(node_values) != self.num_nodes:
            raise ValueError("one value per node")
        self.values = [torch.as_tensor(v, dtype=torch.float64).clone() for v in node_values]
        self.weights = [1.0] * self.num_nodes

    def select_peer(self, sender: int) -> int:
        n = self.num_nodes
        if n <= 1:
            return 0
        if self.topology == "ring":
            return (sender + 1) % n
        if self.topology == "random":
            while True:
                p = self.rng.randrange(n)
                if p != sender:
                    return p
        j = self.rng.randrange(max(1, (n - 1).bit_length()))
        return (sender + (1 << j)) % n

    def run_round(self):
        f = self.push_fraction
        msgs = []
        for s in range(self.num_nodes):
            r = self.select_peer(s)
            msgs.append((r, self.values[s] * f, self.weights[s] * f))
            self.values[s] = self.values[s] * (1 - f)
            self.weights[s] *= 1 - f
        for r, v, w in msgs:
            self.values[r] = self.values[r] + v
            self.weights[r] += w
        self.rounds_completed += 1

    def get_estimate(self, node: int) -> torch.Tensor:
        w = self.weights[node]
        return self.values[node].clone() if abs(w) < 1e-300 else self.values[node] / w

    def is_converged(self, tol: float) -> bool:
        if self.num_nodes <= 1:
            return True
        est = torch.stack([self.get_estimate(i) for i in range(self.num_nodes)])
        return bool(((est - est.mean(0)).abs() <= tol).all())

    def run_to_convergence(self, tolerance: float) -> int:
        for i in range(self.num_rounds):
            self.run_round()
            if self.is_converged(tolerance):
                return i + 1
        return self.num_rounds


def gossip_allreduce_simulate(node_values, config: GossipAllReduce) -> list[torch.Tensor]:
    config.num_nodes = len(node_values)
    config.init_values(node_values)
    for _ in range(config.num_rounds):
        config.run_round()
    return [config.get_estimate(i) for i in range(config.num_nodes)]


def gossip_allreduce(t: torch.Tensor, rounds: int = 10, push_fraction: float = 0.5, group=None) -> torch.Tensor:
    """Ring push-sum across ranks: returns this rank's estimate of the mean
    of `t` over ranks after `rounds` rounds (exact for push_fraction 0.5 and
    rounds -> inf; every rank's (value, weight) mass is conserved)."""
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    if world == 1:
        return t.clone()
    val = torch.cat([t.reshape(-1).double(), torch.ones(1, dtype=torch.float64, device=t.device)])
    dst, src = (rank + 1) % world, (rank - 1) % world
    gdst = dist.get_global_rank(group, dst) if group is not None else dst
    gsrc = dist.get_global_rank(group, src) if group is not None else src
    for _ in range(rounds):
        send = val * push_fraction
        val = val * (1 - push_fraction)
        recv = torch.empty_like(val)
        reqs = dist.batch_isend_irecv([dist.P2POp(dist.isend, send, gdst, group),
                                       dist.P2POp(dist.irecv, recv, gsrc, group)])
        for r in reqs:
            r.wait()
        val = val + recv
    return (val[:-1] / val[-1]).to(t.dtype).view_as(t)
