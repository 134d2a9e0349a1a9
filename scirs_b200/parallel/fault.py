"""Failure detection, resilience and elastic restart on the host.

Pieces:
  NodeHealth / NodeInfo / FaultToleranceManager
      per-node health states and timeout-based failure detection
      (scirs2-core/src/distributed/fault_tolerance.rs:14-356).
  CircuitBreaker / RetryPolicy / RetryExecutor / ResilientExecutor
      closed -> open after `failure_threshold` failures, open -> half-open
      after `timeout`, half-open -> closed after `success_threshold`
      successes (a failure in half-open re-opens); retries with exponential
      back-off; a process-wide breaker registry
      (scirs2-core/src/error/circuitbreaker.rs:10-310).
  Heartbeat / HeartbeatMonitor
      every rank's background thread writes a beat counter and timestamp to
      the process group's key-value store; `check()` (call it between
      steps, before the next collective) marks ranks whose beat is older
      than the timeout as failed and raises RankFailure, so the surviving
      ranks learn of a dead peer on the host instead of blocking in a
      collective.
  FaultInjector
      host-side injection for tests: at a chosen step a rank raises, exits,
      stops beating or stalls. Nothing here touches a GPU.
  elastic_restart
      rebuilds a smaller (or larger) process group and reloads a
      world-size-independent ZeRO checkpoint into it.

Device side, every spin-wait in the fused collectives is bounded by a
timeout after which the kernel records an error in a status word and
returns; `scirs_b200._ext.check_status()` turns that into an exception.
"""
from __future__ import annotations

import enum
import os
import threading
import time
from dataclasses import dataclass, field

import torch.distributed as dist


# ----------------------------------------------------------------- health
class NodeHealth(enum.Enum):
    HEALTHY = "healthy"
    DEGRADED = "degraded"
    UNRESPONSIVE = "unresponsive"
    FAILED = "failed"
    RECOVERING = "recovering"


class RecoveryStrategy(enum.Enum):
    RESTART = "restart"
    MIGRATE = "migrate"
    REPLACE = "replace"
    MANUAL = "manual"


@dataclass
class NodeInfo:
    node_id: str
    address: str = ""
    health: NodeHealth = NodeHealth.HEALTHY
    last_seen: float = field(default_factory=time.monotonic)
    failure_count: int = 0
    recovery_strategy: RecoveryStrategy = RecoveryStrategy.RESTART

    def update_health(self, health: NodeHealth):
        if health == NodeHealth.FAILED and self.health != NodeHealth.FAILED:
            self.failure_count += 1
        self.health = health
        self.last_seen = time.monotonic()

    def is_healthy(self) -> bool:
        return self.health in (NodeHealth.HEALTHY, NodeHealth.DEGRADED)

    def has_failed(self) -> bool:
        return self.health == NodeHealth.FAILED


@dataclass
class ClusterHealthSummary:
    total_nodes: int
    healthy_nodes: int
    failed_nodes: int
    degraded_nodes: int

    def health_percentage(self) -> float:
        return 100.0 * self.healthy_nodes / self.total_nodes if self.total_nodes else 0.0

    def is_healthy(self) -> bool:
        return self.failed_nodes == 0 and self.health_percentage() >= 50.0


class FaultToleranceManager:
    def __init__(self, timeout_s: float = 30.0, max_failures: int = 3):
        self.timeout_s = timeout_s
        self.max_failures = max_failures
        self.nodes: dict[str, NodeInfo] = {}
        self._lock = threading.Lock()

    def register_node(self, node: NodeInfo):
        with self._lock:
            self.nodes[node.node_id] = node

    def update_node_health(self, node_id: str, health: NodeHealth):
        with self._lock:
            self.nodes[node_id].update_health(health)

    def seen(self, node_id: str, when: float | None = None):
        with self._lock:
            n = self.nodes[node_id]
            n.last_seen = time.monotonic() if when is None else when
            if n.health in (NodeHealth.UNRESPONSIVE, NodeHealth.RECOVERING):
                n.health = NodeHealth.HEALTHY

    def detect_failures(self, now: float | None = None) -> list[str]:
        """Nodes still marked healthy whose last sign of life is older than
        the timeout."""
        now = time.monotonic() if now is None else now
        with self._lock:
            return [k for k, n in self.nodes.items() if n.is_healthy() and now - n.last_seen > self.timeout_s]

    def get_healthy_nodes(self) -> list[NodeInfo]:
        return [n for n in self.nodes.values() if n.is_healthy()]

    def get_failed_nodes(self) -> list[NodeInfo]:
        return [n for n in self.nodes.values() if n.has_failed()]

    def is_cluster_healthy(self) -> bool:
        return self.get_cluster_health_summary().is_healthy()

    def get_cluster_health_summary(self) -> ClusterHealthSummary:
        ns = list(self.nodes.values())
        return ClusterHealthSummary(len(ns), sum(n.health == NodeHealth.HEALTHY for n in ns),
                                    sum(n.has_failed() for n in ns), sum(n.health == NodeHealth.DEGRADED for n in ns))

    def should_give_up(self, node_id: str) -> bool:
        return self.nodes[node_id].failure_count >= self.max_failures


# ----------------------------------------------------------------- circuit breaker
class CircuitState(enum.Enum):
    CLOSED = "closed"
    OPEN = "open"
    HALF_OPEN = "half_open"


class CircuitOpenError(RuntimeError):
    pass


@dataclass
class CircuitBreakerConfig:
    failure_threshold: int = 5
    success_threshold: int = 3
    timeout_s: float = 30.0


@dataclass
class CircuitBreakerStatus:
    state: CircuitState
    failure_count: int
    success_count: int
    last_state_change: float


class CircuitBreaker:
    def __init__(self, config: CircuitBreakerConfig | None = None, clock=time.monotonic):
        self.config = config or CircuitBreakerConfig()
        self._clock = clock
        self._state = CircuitState.CLOSED
        self.failure_count = 0
        self.success_count = 0
        self.last_state_change = clock()
        self._lock = threading.Lock()

    def _set(self, st: CircuitState):
        self._state = st
        self.last_state_change = self._clock()
        self.success_count = 0
        if st == CircuitState.CLOSED:
            self.failure_count = 0

    def check_state(self):
        with self._lock:
            if self._state == CircuitState.OPEN and self._clock() - self.last_state_change >= self.config.timeout_s:
                self._set(CircuitState.HALF_OPEN)

    @property
    def state(self) -> CircuitState:
        self.check_state()
        return self._state

    def record_success(self):
        with self._lock:
            if self._state == CircuitState.HALF_OPEN:
                self.success_count += 1
                if self.success_count >= self.config.success_threshold:
                    self._set(CircuitState.CLOSED)
            elif self._state == CircuitState.CLOSED:
                self.failure_count = 0

    def record_failure(self):
        with self._lock:
            if self._state == CircuitState.HALF_OPEN:
                self._set(CircuitState.OPEN)
                return
            self.failure_count += 1
            if self._state == CircuitState.CLOSED and self.failure_count >= self.config.failure_threshold:
                self._set(CircuitState.OPEN)

    def is_allowed(self) -> bool:
        return self.state != CircuitState.OPEN

    def status(self) -> CircuitBreakerStatus:
        return CircuitBreakerStatus(self.state, self.failure_count, self.success_count, self.last_state_change)

    def execute(self, fn, *args, **kw):
        if not self.is_allowed():
            raise CircuitOpenError("circuit breaker is open")
        try:
            out = fn(*args, **kw)
        except Exception:
            self.record_failure()
            raise
        self.record_success()
        return out


@dataclass
class RetryPolicy:
    max_retries: int = 3
    initial_delay_s: float = 0.1
    max_delay_s: float = 10.0
    exponential_base: float = 2.0

    def delay(self, attempt: int) -> float:
        return min(self.initial_delay_s * self.exponential_base ** attempt, self.max_delay_s)


class RetryExecutor:
    def __init__(self, policy: RetryPolicy | None = None, sleep=time.sleep, retry_on=(Exception,)):
        self.policy = policy or RetryPolicy()
        self._sleep = sleep
        self.retry_on = retry_on
        self.attempts = 0

    def execute(self, fn, *args, **kw):
        for attempt in range(self.policy.max_retries + 1):
            self.attempts = attempt + 1
            try:
                return fn(*args, **kw)
            except self.retry_on:
                if attempt == self.policy.max_retries:
                    raise
                self._sleep(self.policy.delay(attempt))


class ResilientExecutor:
    """Circuit breaker around a retrying call, with an optional fallback
    when the circuit is open or every retry failed."""

    def __init__(self, breaker: CircuitBreaker, retry: RetryExecutor, fallback=None):
        self.breaker, self.retry, self.fallback = breaker, retry, fallback

    def execute(self, fn, *args, **kw):
        try:
            return self.breaker.execute(self.retry.execute, fn, *args, **kw)
        except Exception:
            if self.fallback is None:
                raise
            return self.fallback(*args, **kw)


_BREAKERS: dict[str, CircuitBreaker] = {}


def get_circuit_breaker(name: str, config: CircuitBreakerConfig | None = None) -> CircuitBreaker:
    if name not in _BREAKERS:
        _BREAKERS[name] = CircuitBreaker(config)
    return _BREAKERS[name]


def list_circuit_breakers() -> list[str]:
    return sorted(_BREAKERS)


# ----------------------------------------------------------------- heartbeats
class RankFailure(RuntimeError):
    def __init__(self, ranks):
        self.ranks = sorted(ranks)
        super().__init__(f"ranks {self.ranks} stopped heart-beating")


class Heartbeat:
    """Background thread: writes `<prefix>/<rank>` = "<counter>" to the store
    every `interval_s` seconds. `stop()` ends it (a dead rank's beat simply
    stops arriving)."""

    def __init__(self, store, rank: int, interval_s: float = 0.2, prefix: str = "scirs_hb"):
        self.store, self.rank, self.interval_s, self.prefix = store, rank, interval_s, prefix
        self.count = 0
        self._stop = threading.Event()
        self._beat()
        self._thread = threading.Thread(target=self._run, daemon=True, name=f"heartbeat-{rank}")
        self._thread.start()

    def _beat(self):
        self.count += 1
        self.store.set(f"{self.prefix}/{self.rank}", str(self.count))

    def _run(self):
        while not self._stop.wait(self.interval_s):
            try:
                self._beat()
            except Exception:  # store gone: the job is shutting down
                return

    def stop(self):
        self._stop.set()
        self._thread.join(timeout=5)


class HeartbeatMonitor:
    """Watches the other members' beat counters. A member whose counter has
    not advanced for `timeout_s` seconds (host clock of the observer, so no
    clock agreement between hosts is needed) is declared failed.

    Members are identified by their heartbeat id (the rank they had when the
    job started); after an elastic restart :meth:`shrink` gives the monitor
    of the surviving members."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 2.0, prefix: str = "scirs_hb",
                 members: list[int] | None = None, generation: int = 0):
        self.store, self.rank, self.prefix = store, rank, prefix
        self.members = list(range(world)) if members is None else list(members)
        self.world = len(self.members)
        self.generation = generation
        self.timeout_s = timeout_s
        self.manager = FaultToleranceManager(timeout_s=timeout_s)
        self._last: dict[int, str] = {}
        for r in self.members:
            self.manager.register_node(NodeInfo(str(r)))

    def shrink(self, failed) -> "HeartbeatMonitor":
        alive = [m for m in self.members if m not in set(failed)]
        return HeartbeatMonitor(self.store, self.rank, len(alive), self.timeout_s, self.prefix, alive,
                                self.generation + 1)

    def poll(self) -> list[int]:
        now = time.monotonic()
        for r in self.members:
            if r == self.rank:
                self.manager.seen(str(r), now)
                continue
            key = f"{self.prefix}/{r}"
            v = self.store.get(key).decode() if self.store.check([key]) else None
            if v is not None and v != self._last.get(r):
                self._last[r] = v
                self.manager.seen(str(r), now)
        for d in self.manager.detect_failures(now):
            self.manager.update_node_health(d, NodeHealth.FAILED)
        return sorted(int(n.node_id) for n in self.manager.get_failed_nodes())

    def barrier(self, tag: str, poll_s: float = 0.02):
        """Host barrier through the store that cannot hang on a dead peer:
        returns when every member has arrived at `tag`, raises RankFailure as
        soon as a member that has not arrived stops beating."""
        base = f"{self.prefix}_bar{self.generation}/{tag}"
        self.store.set(f"{base}/{self.rank}", "1")
        keys = [f"{base}/{r}" for r in self.members]
        while True:
            if self.store.check(keys):
                return
            failed = self.poll()
            if failed:
                raise RankFailure(failed)
            time.sleep(poll_s)

    def check(self):
        """Raise RankFailure if any peer is (or was) declared failed."""
        failed = self.poll()
        if failed:
            raise RankFailure(failed)

    def alive(self) -> list[int]:
        return sorted(int(n.node_id) for n in self.manager.get_healthy_nodes())


# ----------------------------------------------------------------- fault injection
class FaultInjector:
    """Host-side faults for tests: at step `at_step` the rank performs
    `mode` = "raise" | "exit" | "stop_heartbeat" | "stall" (sleeps
    `stall_s` seconds between steps, holding no collective)."""

    def __init__(self, mode: str | None = None, at_step: int = -1, rank: int = -1, stall_s: float = 5.0,
                 exit_code: int = 17):
        assert mode in (None, "raise", "exit", "stop_heartbeat", "stall")
        self.mode, self.at_step, self.rank, self.stall_s = mode, at_step, rank, stall_s
        self.exit_code = exit_code

    @classmethod
    def from_env(cls, rank: int) -> "FaultInjector":
        spec = os.environ.get("SCIRS_FAULT", "")  # "<mode>:<rank>:<step>"
        if not spec:
            return cls()
        mode, r, s = spec.split(":")
        return cls(mode, int(s), int(r))

    def maybe_fail(self, step: int, rank: int, heartbeat: Heartbeat | None = None):
        ranks = self.rank if isinstance(self.rank, (list, tuple)) else [self.rank]
        if self.mode is None or rank not in ranks or step != self.at_step:
            return
        if self.mode == "raise":
            raise RuntimeError(f"injected failure on rank {rank} at step {step}")
        if self.mode == "exit":
            if heartbeat is not None:
                heartbeat.stop()
            os._exit(self.exit_code)
        if self.mode == "stop_heartbeat" and heartbeat is not None:
            heartbeat.stop()
        if self.mode == "stall":
            time.sleep(self.stall_s)


# ----------------------------------------------------------------- elastic restart
def elastic_restart(survivors: list[int], old_rank: int, store, backend: str = "gloo", timeout_s: float = 30.0,
                    generation: int = 1):
    """Re-form a process group over the surviving ranks (renumbered 0..n-1
    in order) through a fresh store prefix. The old default group must have
    been destroyed (or abandoned) by the caller. Returns (new_rank, world)."""
    import datetime

    new_rank = survivors.index(old_rank)
    world = len(survivors)
    # every survivor must have left the old group before anyone connects
    # (a peer still inside its failure detection would refuse connections)
    store.set(f"scirs_elastic_{generation}_arrive/{old_rank}", "1")
    store.wait([f"scirs_elastic_{generation}_arrive/{r}" for r in survivors], datetime.timedelta(seconds=timeout_s))
    pstore = dist.PrefixStore(f"scirs_elastic_{generation}", store)
    dist.init_process_group(backend, store=pstore, rank=new_rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return new_rank, world
