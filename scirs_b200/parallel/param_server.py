"""Parameter server with a staleness-bounded clock table, rank-sharded
server over a process group, push-sum gossip averaging and vector clocks.

Design
------
One rule covers every consistency model: each worker carries a logical clock
(the number of iterations it has finished) and the server admits an update
made at clock ``c`` once ``c <= floor + bound``, where ``floor`` is the
smallest clock of the live workers and ``bound`` the configured staleness:

  * ``bound = 0``   synchronous rounds: updates of clock ``c`` wait until
                     every live worker has finished ``c`` (``floor > c``) and
                     are then combined into one new value per key
  * ``bound = k``   bounded staleness: an update is applied when it is made
                     unless its worker runs more than ``k`` clocks ahead of
                     the slowest live worker; held updates are released as
                     the floor advances
  * ``bound = None`` asynchronous: every update is applied when it arrives

Updates are kept in a table keyed by clock, so releasing work after a clock
advance is a scan of the admissible clocks only. Liveness is a lease table
(each worker renews a lease; an expired lease removes the worker from the
floor and from synchronous rounds, so a dead worker never blocks the
others). Snapshots of the parameters and the clock table are taken every
``snapshot_every`` versions into a bounded ring and can be restored.

``ShardedParameterServer`` runs the synchronous mode across processes: every
key has an owner rank (stable hash of the key), pushes are reduced to the
owner (``torch.distributed.reduce``), the owner applies the combined update
and broadcasts the new value. Keys are visited in sorted order so every rank
issues the same collectives.

Gossip (``PushSum``) is written as a product of column-stochastic mixing
matrices: in round ``t`` node ``i`` keeps a fraction ``1 - f`` of its
(value, weight) pair and sends ``f`` to ``peer_t(i)``. The estimate
value / weight of every node converges to the average. ``push_sum_allreduce``
runs the shift topologies (ring, exponential) across ranks with
point-to-point send/recv.

The reference has the same features as in-process structures
(scirs2-core/src/distributed/param_server/server.rs:45-260 BSP/ASP/SSP
server, fault_tolerance.rs:34-320 heartbeats, checkpoints and vector clocks,
gossip.rs:59-271 push-sum); this module shares their purpose, not their
structure.
"""
from __future__ import annotations

import enum
import math
import time
import zlib
from collections import defaultdict, deque
from dataclasses import dataclass, field
from typing import Callable

import torch
import torch.distributed as dist

# --------------------------------------------------------------------- combine


def combine_mean(values: list[torch.Tensor], workers: list[int]) -> torch.Tensor:
    return torch.stack(values).mean(0)


def combine_sum(values: list[torch.Tensor], workers: list[int]) -> torch.Tensor:
    return torch.stack(values).sum(0)


def combine_weighted(weights: dict[int, float] | list[float]) -> Callable:
    """Weighted mean by worker id (missing ids weigh 1)."""
    table = dict(enumerate(weights)) if isinstance(weights, (list, tuple)) else dict(weights)

    def fn(values, workers):
        w = torch.tensor([float(table.get(k, 1.0)) for k in workers], dtype=values[0].dtype)
        s = sum(v * wi for v, wi in zip(values, w.to(values[0].device)))
        tot = float(w.sum())
        return s if tot == 0.0 else s / tot

    return fn


_COMBINE = {"mean": combine_mean, "sum": combine_sum}


class Consistency(enum.Enum):
    """Named staleness bounds (the reference's BSP / SSP / ASP)."""

    SYNC = "sync"
    BOUNDED = "bounded"
    ASYNC = "async"


@dataclass
class PSConfig:
    num_workers: int = 4
    staleness: int | None = 0  # 0 synchronous, k bounded, None asynchronous
    combine: str | Callable = "mean"
    apply: str = "replace"  # "replace": key <- combined push; "sgd": key <- key - lr * combined push
    lr: float = 1.0
    lease_s: float = 30.0
    snapshot_every: int = 0  # 0: no automatic snapshots
    snapshot_keep: int = 4

    @property
    def mode(self) -> Consistency:
        if self.staleness is None:
            return Consistency.ASYNC
        return Consistency.SYNC if self.staleness == 0 else Consistency.BOUNDED


# ----------------------------------------------------------------- liveness


class LeaseTable:
    """Worker leases: a worker is live while now < its expiry time."""

    def __init__(self, lease_s: float):
        self.lease_s = float(lease_s)
        self.expiry: dict[int, float] = {}
        self.revoked: set[int] = set()

    def renew(self, worker: int, now: float | None = None):
        if worker in self.revoked:
            raise RuntimeError(f"worker {worker} was declared failed and cannot renew its lease")
        self.expiry[worker] = (time.monotonic() if now is None else now) + self.lease_s

    def revoke(self, worker: int):
        self.revoked.add(worker)
        self.expiry.pop(worker, None)

    def live(self, now: float | None = None) -> set[int]:
        t = time.monotonic() if now is None else now
        return {w for w, e in self.expiry.items() if e > t}

    def lapsed(self, now: float | None = None) -> list[int]:
        t = time.monotonic() if now is None else now
        return sorted(w for w, e in self.expiry.items() if e <= t)


# -------------------------------------------------------------------- server


@dataclass
class _Pending:
    worker: int
    value: torch.Tensor


@dataclass
class Snapshot:
    version: int
    params: dict[str, torch.Tensor]
    clocks: dict[int, int]
    failed: set[int] = field(default_factory=set)


class ParameterServer:
    """Staleness-bounded parameter server (see the module docstring).

    Typical synchronous use::

        ps = ParameterServer(PSConfig(num_workers=3))
        ids = [ps.join() for _ in range(3)]
        ps.create("w", torch.zeros(4))
        for w in ids:
            ps.push(w, "w", value)      # at the worker's current clock
            ps.advance(w)               # worker w finished this clock
        value, version = ps.pull("w")
    """

    def __init__(self, config: PSConfig | None = None):
        self.config = config or PSConfig()
        c = self.config.combine
        self._combine = _COMBINE[c] if isinstance(c, str) else c
        self.params: dict[str, torch.Tensor] = {}
        self.key_version: dict[str, int] = {}
        self.clock: dict[int, int] = {}  # worker -> finished iterations
        self.leases = LeaseTable(self.config.lease_s)
        self.table: dict[int, dict[str, list[_Pending]]] = defaultdict(lambda: defaultdict(list))
        self.version = 0  # bumped once per applied combine / async apply
        self.snapshots: deque[Snapshot] = deque(maxlen=max(1, self.config.snapshot_keep))
        self._sync_done = -1  # last clock whose synchronous round was committed

    # ------------------------------------------------------------ membership
    def join(self, now: float | None = None) -> int:
        if len(self.clock) >= self.config.num_workers:
            raise RuntimeError(f"all {self.config.num_workers} worker slots are taken")
        w = len(self.clock)
        self.clock[w] = 0
        self.leases.renew(w, now)
        return w

    def heartbeat(self, worker: int, now: float | None = None):
        self._known(worker)
        self.leases.renew(worker, now)

    def fail(self, worker: int):
        """Declare a worker failed: it leaves the floor and synchronous rounds
        at once (its pending updates of uncommitted clocks still count)."""
        self._known(worker)
        if worker in self.leases.revoked:
            raise RuntimeError(f"worker {worker} is already marked failed")
        self.leases.revoke(worker)
        self._release()

    def reap(self, now: float | None = None) -> list[int]:
        """Fail every worker whose lease has lapsed; returns their ids."""
        gone = self.leases.lapsed(now)
        for w in gone:
            self.leases.revoke(w)
        if gone:
            self._release(now)
        return gone

    def live_workers(self, now: float | None = None) -> list[int]:
        return sorted(self.leases.live(now))

    def _known(self, worker: int):
        if worker not in self.clock:
            raise KeyError(f"worker {worker} never joined")

    # ------------------------------------------------------------------ data
    def create(self, key: str, value: torch.Tensor):
        self.params[key] = value.detach().clone()
        self.key_version[key] = 0

    def pull(self, key: str) -> tuple[torch.Tensor, int]:
        return self.params[key].clone(), self.key_version[key]

    def floor(self, now: float | None = None) -> int | None:
        live = self.leases.live(now)
        return min((self.clock[w] for w in live), default=None)

    def admissible(self, clock: int, now: float | None = None) -> bool:
        b = self.config.staleness
        if b is None:
            return True
        f = self.floor(now)
        if f is None:
            return True
        return clock < f if b == 0 else clock <= f + b

    def push(self, worker: int, key: str, value: torch.Tensor, clock: int | None = None,
             now: float | None = None) -> bool:
        """Record worker's update of `key` made at `clock` (default: the
        worker's current clock). Returns True if it was applied now."""
        self._known(worker)
        if worker in self.leases.revoked:
            raise RuntimeError(f"worker {worker} was declared failed")
        if key not in self.params:
            raise KeyError(f"unknown key {key!r}")
        c = self.clock[worker] if clock is None else int(clock)
        self.leases.renew(worker, now)
        entry = _Pending(worker, value.detach().clone())
        if self.config.staleness != 0 and self.admissible(c, now):
            self._apply(key, [entry])
            return True
        self.table[c][key].append(entry)
        return False

    def advance(self, worker: int, now: float | None = None):
        """Worker finished its current clock; commit what became admissible."""
        self._known(worker)
        self.clock[worker] += 1
        self.leases.renew(worker, now)
        self._release(now)

    def _apply(self, key: str, entries: list[_Pending]):
        upd = self._combine([e.value for e in entries], [e.worker for e in entries])
        if self.config.apply == "sgd":
            self.params[key] = self.params[key] - self.config.lr * upd.to(self.params[key].dtype)
        else:
            self.params[key] = upd.to(self.params[key].dtype)
        self.key_version[key] += 1
        self.version += 1
        n = self.config.snapshot_every
        if n and self.version % n == 0:
            self.snapshots.append(self.snapshot())

    def _release(self, now: float | None = None):
        for c in sorted(self.table):
            if not self.admissible(c, now):
                break
            for key in sorted(self.table[c]):
                ents = self.table[c][key]
                if self.config.staleness == 0:
                    self._apply(key, ents)  # one combined value per key per round
                else:
                    for e in ents:
                        self._apply(key, [e])
            del self.table[c]
            self._sync_done = max(self._sync_done, c)

    def waiting_on(self, clock: int, now: float | None = None) -> list[int]:
        """Live workers that have not finished `clock` yet."""
        return sorted(w for w in self.leases.live(now) if self.clock[w] <= clock)

    def pending(self) -> int:
        return sum(len(v) for d in self.table.values() for v in d.values())

    # ------------------------------------------------------------- snapshots
    def snapshot(self) -> Snapshot:
        return Snapshot(self.version, {k: v.clone() for k, v in self.params.items()}, dict(self.clock),
                        set(self.leases.revoked))

    @classmethod
    def from_snapshot(cls, snap: Snapshot, config: PSConfig, now: float | None = None) -> "ParameterServer":
        ps = cls(config)
        for k, v in snap.params.items():
            ps.create(k, v)
        ps.version = snap.version
        ps.clock = dict(snap.clocks)
        for w in ps.clock:
            if w in snap.failed:
                ps.leases.revoke(w)
            else:
                ps.leases.renew(w, now)
        return ps


# ---------------------------------------------------------- across processes


def owner_of(key: str, world: int) -> int:
    return zlib.crc32(key.encode()) % world


class ShardedParameterServer:
    """Synchronous parameter server whose keys are spread over the ranks of a
    process group. Every rank is a worker and hosts the keys it owns.

    ``step(updates)`` with one tensor per key (same keys on every rank):
    each key's updates are summed onto its owner, the owner combines them
    (mean over ranks) and applies them (replace or SGD), then broadcasts the
    new value, which ``step`` returns for every key.
    """

    def __init__(self, apply: str = "replace", lr: float = 1.0, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.apply = apply
        self.lr = lr
        self.values: dict[str, torch.Tensor] = {}
        self.version = 0

    def create(self, key: str, value: torch.Tensor):
        """Collective: all ranks register the same keys (owner's value wins)."""
        t = value.detach().clone()
        dist.broadcast(t, src=self._global(owner_of(key, self.world)), group=self.group)
        self.values[key] = t

    def _global(self, r: int) -> int:
        return dist.get_global_rank(self.group, r) if self.group is not None else r

    def owned(self) -> list[str]:
        return sorted(k for k in self.values if owner_of(k, self.world) == self.rank)

    def step(self, updates: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
        out = {}
        for key in sorted(updates):
            own = owner_of(key, self.world)
            buf = updates[key].detach().to(self.values[key].dtype).clone()
            dist.reduce(buf, dst=self._global(own), op=dist.ReduceOp.SUM, group=self.group)
            if self.rank == own:
                buf /= self.world
                self.values[key] = self.values[key] - self.lr * buf if self.apply == "sgd" else buf
            v = self.values[key]
            dist.broadcast(v, src=self._global(own), group=self.group)
            out[key] = v
        self.version += 1
        return out


# --------------------------------------------------------------------- gossip


def peer_ring(i: int, t: int, n: int) -> int:
    return (i + 1) % n


def peer_exponential(i: int, t: int, n: int) -> int:
    hops = max(1, math.ceil(math.log2(n)))
    return (i + (1 << (t % hops))) % n


def make_peer_random(seed: int) -> Callable[[int, int, int], int]:
    """A different non-self peer per (node, round), reproducible from seed."""

    def fn(i, t, n):
        g = torch.Generator().manual_seed(seed * 1_000_003 + t * 7919 + i)
        return (i + 1 + int(torch.randint(0, n - 1, (1,), generator=g))) % n

    return fn


TOPOLOGIES = {"ring": peer_ring, "exponential": peer_exponential}


class PushSum:
    """Push-sum averaging of n node vectors as repeated mixing-matrix
    products: X <- P_t X, w <- P_t w with P_t[i, i] = 1 - f and
    P_t[peer_t(i), i] += f (columns sum to 1, so the total mass is kept)."""

    def __init__(self, values: list[torch.Tensor] | torch.Tensor, topology: str | Callable = "ring",
                 fraction: float = 0.5, seed: int = 0):
        x = torch.stack([torch.as_tensor(v, dtype=torch.float64).reshape(-1) for v in values]) \
            if not torch.is_tensor(values) else values.to(torch.float64).reshape(values.shape[0], -1)
        self.n = x.shape[0]
        self.shape = torch.as_tensor(values[0]).shape
        self.x = x.clone()
        self.w = torch.ones(self.n, dtype=torch.float64)
        if callable(topology):
            self.peer = topology
        elif topology == "random":
            self.peer = make_peer_random(seed)
        else:
            self.peer = TOPOLOGIES[topology]
        self.f = float(fraction)
        self.t = 0
        self.target = self.x.mean(0)

    def mixing_matrix(self, t: int) -> torch.Tensor:
        P = torch.eye(self.n, dtype=torch.float64) * (1.0 - self.f)
        for i in range(self.n):
            P[self.peer(i, t, self.n), i] += self.f
        return P

    def round(self):
        P = self.mixing_matrix(self.t)
        self.x = P @ self.x
        self.w = P @ self.w
        self.t += 1

    def estimates(self) -> torch.Tensor:
        return self.x / self.w[:, None]

    def estimate(self, i: int) -> torch.Tensor:
        return self.estimates()[i].reshape(self.shape)

    def spread(self) -> float:
        """Largest deviation of any estimate from the true average."""
        return float((self.estimates() - self.target).abs().max())

    def run(self, tol: float, max_rounds: int = 10_000) -> int:
        while self.spread() > tol and self.t < max_rounds:
            self.round()
        return self.t


def push_sum_allreduce(t: torch.Tensor, rounds: int = 30, topology: str = "ring", fraction: float = 0.5,
                       group=None) -> torch.Tensor:
    """Approximate average of `t` over the ranks by push-sum gossip with
    point-to-point messages. Shift topologies only: in round k every rank
    sends to (r + s_k) and receives from (r - s_k), so each exchange pairs
    one send with one receive."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if world == 1:
        return t.clone()
    peer = TOPOLOGIES[topology]
    gr = (lambda r: dist.get_global_rank(group, r)) if group is not None else (lambda r: r)
    x = torch.cat([t.detach().reshape(-1).to(torch.float64), torch.ones(1, dtype=torch.float64)])
    if t.is_cuda:
        x = x.to(t.device)
    for k in range(rounds):
        dst = peer(rank, k, world)
        shift = (dst - rank) % world
        src = (rank - shift) % world
        out = x * fraction
        inc = torch.empty_like(x)
        reqs = [dist.isend(out, gr(dst), group=group), dist.irecv(inc, gr(src), group=group)]
        for r in reqs:
            r.wait()
        x = x * (1.0 - fraction) + inc
    return (x[:-1] / x[-1]).to(t.dtype).reshape(t.shape)


# --------------------------------------------------------------- vector clock


class Order(enum.Enum):
    BEFORE = "before"
    AFTER = "after"
    EQUAL = "equal"
    CONCURRENT = "concurrent"


class VectorClock:
    """Vector clock over a fixed set of processes."""

    def __init__(self, n: int, counts=None):
        self.c = list(counts) if counts is not None else [0] * n

    def tick(self, i: int) -> "VectorClock":
        self.c[i] += 1
        return self

    def observe(self, other: "VectorClock") -> "VectorClock":
        """Merge a received clock (element-wise max)."""
        self.c = [max(a, b) for a, b in zip(self.c, other.c)]
        return self

    def compare(self, other: "VectorClock") -> Order:
        le = all(a <= b for a, b in zip(self.c, other.c))
        ge = all(a >= b for a, b in zip(self.c, other.c))
        if le and ge:
            return Order.EQUAL
        if le:
            return Order.BEFORE
        if ge:
            return Order.AFTER
        return Order.CONCURRENT

    def happens_before(self, other: "VectorClock") -> bool:
        return self.compare(other) is Order.BEFORE

    def concurrent(self, other: "VectorClock") -> bool:
        return self.compare(other) is Order.CONCURRENT

    def copy(self) -> "VectorClock":
        return VectorClock(len(self.c), self.c)

    def __repr__(self):
        return f"VectorClock({self.c})"
