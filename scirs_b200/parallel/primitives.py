"""Host-parallel primitives: task graphs, work queues, worker pools, parallel
map / filter / fold / sort, scans and lock-free structures.

The scheduling and the numeric kernels are native (module `scirs_b200._data`,
source `csrc/host_runtime.cpp`):

* `TaskGraph` runs on a dataflow scheduler: a task starts as soon as its last
  dependency finishes, on a pool of native threads that take the interpreter
  lock only around each task body. Task bodies that release it (tensor
  operations, file and network I/O, `time.sleep`) run concurrently.
* `par_map` and the other element-wise helpers hand indices to native threads
  through one atomic counter.
* Scans and `par_sort` on host tensors run entirely in native code without the
  interpreter lock (blocked three-phase scan; stable chunk sort + parallel
  pairwise merges). Python sequences are converted to tensors when their
  elements are numbers and the operator is one of +, *, min, max; any other
  operator runs the same blocked algorithm with Python calls.
* `MpmcRing` is a bounded lock-free multi-producer / multi-consumer queue of
  int64 values for native producers and consumers; `LockFreeCounter` is an
  atomic 64-bit counter. `LockFreeQueue` / `LockFreeStack` hold Python objects
  in a `collections.deque`, whose append and pop are atomic operations under
  the interpreter lock, so they take no lock of their own.

Reference parity: scirs2-core/src/distributed/primitives.rs:94-722
(WorkQueue / WorkReceiver, WorkerPool, distributed_map, distributed_map_reduce,
chunked_parallel_process, ResourceMonitor), task_graph.rs:70-613,
par_iter.rs:72-475, parallel_scan.rs:50-427, lock_free.rs:55-496. One
difference: a task body receives the results of all of its transitive
dependencies (the reference's level-by-level executor passes every result
finished so far, which with a dataflow scheduler would depend on timing).
"""
from __future__ import annotations

import collections
import functools
import math
import os
import threading
import time
from typing import Any, Callable, Iterable, Sequence

import torch

from .. import _ext


class DistributedError(RuntimeError):
    """Raised by the primitives (closed queues, failed tasks, timeouts)."""


class TaskGraphError(DistributedError):
    def __init__(self, task: str, cause: BaseException | None):
        super().__init__(f"task '{task}' failed: {cause!r}")
        self.task, self.cause = task, cause


def _native():
    return _ext.data()


def _default_workers(n_workers: int | None) -> int:
    return max(1, n_workers if n_workers else (os.cpu_count() or 1))


# ----------------------------------------------------------------------------- work queue / worker pool


_NOTHING = object()


class WorkQueue:
    """Bounded FIFO of tasks; `WorkQueue.new(capacity)` returns the sending side and its `WorkReceiver`."""

    def __init__(self, capacity: int):
        if capacity < 1:
            raise DistributedError("WorkQueue capacity must be at least 1")
        self._cap = capacity
        self._items: collections.deque = collections.deque()
        self._cv = threading.Condition()
        self._closed = False

    @classmethod
    def new(cls, capacity: int):
        q = cls(capacity)
        return q, WorkReceiver(q)

    def push(self, task, timeout: float | None = None) -> None:
        """Blocks while the queue is full (up to `timeout` seconds)."""
        with self._cv:
            if not self._cv.wait_for(lambda: self._closed or len(self._items) < self._cap, timeout):
                raise DistributedError("WorkQueue.push timed out")
            if self._closed:
                raise DistributedError("WorkQueue is closed")
            self._items.append(task)
            self._cv.notify_all()

    def try_push(self, task) -> bool:
        with self._cv:
            if self._closed:
                raise DistributedError("WorkQueue is closed")
            if len(self._items) >= self._cap:
                return False
            self._items.append(task)
            self._cv.notify_all()
            return True

    def close(self) -> None:
        """No more pushes; receivers drain what is queued, then get None."""
        with self._cv:
            self._closed = True
            self._cv.notify_all()

    def __len__(self):
        with self._cv:
            return len(self._items)

    def is_empty(self) -> bool:
        return len(self) == 0

    def capacity(self) -> int:
        return self._cap

    def _pop(self, timeout: float | None, block: bool):
        with self._cv:
            if block:
                self._cv.wait_for(lambda: self._closed or self._items, timeout)
            if not self._items:
                return _NOTHING
            item = self._items.popleft()
            self._cv.notify_all()
            return item


class WorkReceiver:
    def __init__(self, q: WorkQueue):
        self._q = q

    def recv(self):
        """Next task; None once the queue is closed and drained."""
        return self._some(self._q._pop(None, True))

    def recv_timeout(self, timeout: float):
        return self._some(self._q._pop(timeout, True))

    def try_recv(self):
        return self._some(self._q._pop(None, False))

    @staticmethod
    def _some(x):
        return None if x is _NOTHING else x


class WorkerPool:
    """`n_workers` threads apply `worker_fn` to submitted tasks; results come back in completion order.
    A task that raises yields a `DistributedError` result (with the exception as its cause)."""

    def __init__(self, n_workers: int, worker_fn: Callable[[Any], Any], queue_capacity: int = 1024):
        if n_workers < 1:
            raise DistributedError("WorkerPool needs at least one worker")
        self._fn = worker_fn
        self._q, self._rx = WorkQueue.new(queue_capacity)
        self._results: collections.deque = collections.deque()
        self._rcv = threading.Condition()
        self._threads = [threading.Thread(target=self._run, daemon=True) for _ in range(n_workers)]
        for t in self._threads:
            t.start()

    def _run(self):
        while True:
            task = self._q._pop(None, True)
            if task is _NOTHING:  # closed and drained
                return
            try:
                r = self._fn(task)
            except Exception as e:  # noqa: BLE001 - reported through the result
                r = DistributedError(f"worker task failed: {e!r}")
                r.__cause__ = e
            with self._rcv:
                self._results.append(r)
                self._rcv.notify_all()

    @property
    def n_workers(self) -> int:
        return len(self._threads)

    def submit(self, task) -> None:
        self._q.push(task)

    def collect_result(self, timeout: float | None = None):
        with self._rcv:
            if not self._rcv.wait_for(lambda: self._results, timeout):
                return None
            return self._results.popleft()

    def collect_all(self, expected: int, timeout: float) -> list:
        deadline = time.monotonic() + timeout
        out = []
        while len(out) < expected:
            r = self.collect_result(max(0.0, deadline - time.monotonic()))
            if r is None:
                break
            out.append(r)
        return out

    def shutdown(self, timeout: float | None = 10.0) -> None:
        self._q.close()
        for t in self._threads:
            t.join(timeout)


# ----------------------------------------------------------------------------- map / reduce


def _run_indexed(fn: Callable[[int], None], n: int, n_workers: int | None) -> None:
    """fn(i) for i < n on native threads; the first exception is re-raised here."""
    err: list[BaseException] = []

    def call(i):
        if err:
            return
        try:
            fn(i)
        except BaseException as e:  # noqa: BLE001 - re-raised below
            err.append(e)

    _native().parallel_for(call, n, _default_workers(n_workers))
    if err:
        raise err[0]


def distributed_map(data: Iterable, map_fn: Callable, n_workers: int = 0) -> list:
    """[map_fn(x) for x in data], computed on `n_workers` native threads, in input order."""
    items = list(data)
    out = [None] * len(items)

    def one(i):
        out[i] = map_fn(items[i])

    _run_indexed(one, len(items), n_workers)
    return out


def distributed_map_reduce(data: Iterable, map_fn: Callable, reduce_fn: Callable, initial, n_workers: int = 0):
    """reduce_fn folded over the mapped values in input order, starting from `initial`."""
    return functools.reduce(reduce_fn, distributed_map(data, map_fn, n_workers), initial)


def chunked_parallel_process(data: Sequence, process_fn: Callable[[Sequence], list], chunk_size: int,
                             n_workers: int = 0) -> list:
    """process_fn on consecutive slices of `chunk_size` items; the returned lists are concatenated in order."""
    cs = max(1, chunk_size)
    chunks = [data[i:i + cs] for i in range(0, len(data), cs)]
    parts = distributed_map(chunks, process_fn, max(1, n_workers))
    return [x for p in parts for x in p]


class ResourceMonitor:
    """Worker and chunk-size recommendations from the logical CPU count and a CPU share; `can_submit`
    compares the host's available memory with `memory_threshold` bytes."""

    def __init__(self, cpu_threshold: float = 1.0, memory_threshold: int = 0):
        self.cpu_threshold = min(1.0, max(0.0, float(cpu_threshold)))
        self.memory_threshold = int(memory_threshold)
        self._cpus = os.cpu_count() or 1

    def logical_cpu_count(self) -> int:
        return self._cpus

    def available_workers(self) -> int:
        return max(1, math.floor(self.cpu_threshold * self._cpus))

    def recommended_chunk_size(self, total_work: int) -> int:
        if total_work <= 0:
            return 64
        return max(64, total_work // max(1, self.available_workers() * 4))

    def can_submit(self) -> bool:
        if self.memory_threshold <= 0:
            return True
        try:
            import psutil
        except ImportError:  # pragma: no cover - psutil is in the image
            return True
        return psutil.virtual_memory().available >= self.memory_threshold


# ----------------------------------------------------------------------------- parallel iterators


def _chunks(n: int, workers: int) -> list[tuple[int, int]]:
    t = max(1, min(workers, n))
    return [(n * c // t, n * (c + 1) // t) for c in range(t)]


def par_map(data: Sequence, f: Callable, num_workers: int | None = None) -> list:
    return distributed_map(data, f, _default_workers(num_workers))


def par_for_each(data: Sequence, f: Callable, num_workers: int | None = None) -> None:
    _run_indexed(lambda i: f(data[i]), len(data), num_workers)


def par_filter(data: Sequence, predicate: Callable, num_workers: int | None = None) -> list:
    keep = par_map(data, predicate, num_workers)
    return [x for x, k in zip(data, keep) if k]


def par_filter_map(data: Sequence, f: Callable, num_workers: int | None = None) -> list:
    """f returns None to drop an element."""
    return [y for y in par_map(data, f, num_workers) if y is not None]


def par_fold(data: Sequence, init, fold_op: Callable, combine_op: Callable, num_workers: int | None = None):
    """Each chunk folded from `init`, the chunk results combined left to right (init must be the identity)."""
    n = len(data)
    if n == 0:
        return init
    spans = _chunks(n, _default_workers(num_workers))
    parts = [None] * len(spans)

    def one(c):
        lo, hi = spans[c]
        acc = init
        for i in range(lo, hi):
            acc = fold_op(acc, data[i])
        parts[c] = acc

    _run_indexed(one, len(spans), len(spans))
    return functools.reduce(combine_op, parts)


def par_any(data: Sequence, predicate: Callable, num_workers: int | None = None) -> bool:
    return any(par_map(data, predicate, num_workers))


def par_all(data: Sequence, predicate: Callable, num_workers: int | None = None) -> bool:
    return all(par_map(data, predicate, num_workers))


def _as_tensor(data):
    if isinstance(data, torch.Tensor):
        return data
    if len(data) and all(isinstance(x, (int, float)) and not isinstance(x, bool) for x in data):
        dt = torch.float64 if any(isinstance(x, float) for x in data) else torch.int64
        return torch.tensor(list(data), dtype=dt)
    return None


def _back(t: torch.Tensor, like):
    return t if isinstance(like, torch.Tensor) else t.tolist()


def par_sort(data, num_workers: int | None = None, descending: bool = False, return_indices: bool = False):
    """Stable sort. Host tensors and lists of numbers sort natively (NaN above every number);
    other sequences use Python's sort."""
    t = _as_tensor(data)
    if t is not None and t.dim() == 1 and t.device.type == "cpu":
        v, i = _native().parallel_sort(t, descending, _default_workers(num_workers))
        v = _back(v, data)
        return (v, _back(i, data)) if return_indices else v
    idx = sorted(range(len(data)), key=lambda k: data[k], reverse=descending)
    v = [data[k] for k in idx]
    return (v, idx) if return_indices else v


def par_sort_by(data: Sequence, key: Callable, num_workers: int | None = None, descending: bool = False) -> list:
    """Stable sort by key(x); the keys are computed in parallel."""
    keys = par_map(data, key, num_workers)
    kt = _as_tensor(keys)
    if kt is not None:
        _, idx = _native().parallel_sort(kt, descending, _default_workers(num_workers))
        return [data[k] for k in idx.tolist()]
    order = sorted(range(len(data)), key=lambda k: keys[k], reverse=descending)
    return [data[k] for k in order]


# ----------------------------------------------------------------------------- scans

_NATIVE_OPS = {"sum": 0, "prod": 1, "min": 2, "max": 3}
_PY_OPS = {"sum": lambda a, b: a + b, "prod": lambda a, b: a * b, "min": min, "max": max}


def _scan(data, op, identity, exclusive: bool, n_workers: int | None):
    if isinstance(op, str) and op in _NATIVE_OPS:
        t = _as_tensor(data)
        if t is not None and t.dim() == 1 and t.device.type == "cpu":
            return _back(_native().scan(t, _NATIVE_OPS[op], exclusive, _default_workers(n_workers)), data)
        if identity is None:
            raise ValueError("a non-numeric scan needs an identity element")
        op = _PY_OPS[op]
    items = list(data)
    n = len(items)
    spans = _chunks(n, _default_workers(n_workers)) if n else []
    out = [None] * n
    totals = [identity] * len(spans)

    def local(c):
        lo, hi = spans[c]
        acc = identity
        for i in range(lo, hi):
            acc = op(acc, items[i])
            out[i] = acc
        totals[c] = acc

    _run_indexed(local, len(spans), len(spans))
    carry = [identity] * len(spans)
    for c in range(1, len(spans)):
        carry[c] = op(carry[c - 1], totals[c - 1])

    def fix(c):
        lo, hi = spans[c]
        for i in range(lo, hi):
            out[i] = op(carry[c], out[i])

    if len(spans) > 1:
        _run_indexed(fix, len(spans), len(spans))
    if exclusive and n:
        out = [identity] + out[:-1]
    return out


def parallel_scan(data, identity, op: Callable | str, n_workers: int | None = None):
    """Inclusive scan: out[i] = op(... op(op(identity, x0), x1) ..., xi); op must be associative."""
    return _scan(data, op, identity, False, n_workers)


def parallel_scan_exclusive(data, identity, op: Callable | str, n_workers: int | None = None):
    """out[0] = identity, out[i] = inclusive scan at i - 1."""
    return _scan(data, op, identity, True, n_workers)


def parallel_prefix_sum(data, n_workers: int | None = None):
    return _scan(data, "sum", 0, False, n_workers)


def parallel_prefix_sum_exclusive(data, n_workers: int | None = None):
    return _scan(data, "sum", 0, True, n_workers)


def parallel_prefix_min(data, n_workers: int | None = None):
    return _scan(data, "min", None, False, n_workers)


def parallel_prefix_max(data, n_workers: int | None = None):
    return _scan(data, "max", None, False, n_workers)


def segmented_prefix_sum(data, flags, n_workers: int | None = None):
    """Running sum that restarts wherever flags[i] is true (a segment starts at element i)."""
    t = _as_tensor(data)
    if t is None:
        raise ValueError("segmented_prefix_sum wants numbers")
    f = torch.as_tensor(flags, dtype=torch.bool)
    return _back(_native().segmented_scan_sum(t, f, _default_workers(n_workers)), data)


# ----------------------------------------------------------------------------- task graph


class TaskGraph:
    """Named tasks with dependencies, executed with maximal concurrency.

        g = TaskGraph()
        g.add_task("load", [], lambda r: 42)
        g.add_task("double", ["load"], lambda r: r["load"] * 2)
        g.execute()  # {"load": 42, "double": 84}

    A task body gets a dict of the results of its transitive dependencies. Dependencies must be
    added first (so the graph is acyclic by construction); `add_dependency` adds an edge later and
    rejects one that would close a cycle."""

    def __init__(self, n_threads: int = 0):
        self._core = _native().TaskGraphCore()
        self._fns: list[Callable] = []
        self._n_threads = n_threads

    def add_task(self, name: str, deps: Sequence[str], func: Callable[[dict], Any]) -> None:
        try:
            self._core.add_task(name, list(deps))
        except RuntimeError as e:
            raise ValueError(str(e).splitlines()[0]) from None
        self._fns.append(func)

    def add_dependency(self, task: str, dep: str) -> None:
        try:
            self._core.add_dependency(task, dep)
        except RuntimeError as e:
            raise ValueError(str(e).splitlines()[0]) from None

    def __len__(self):
        return self._core.size()

    def is_empty(self) -> bool:
        return len(self) == 0

    def contains_task(self, name: str) -> bool:
        return name in self._core.names()

    def dependencies(self, name: str) -> list[str] | None:
        names = self._core.names()
        if name not in names:
            return None
        return [names[i] for i in self._core.dependencies(name)]

    def execution_order(self) -> list[str]:
        return self._core.order()

    def execution_levels(self) -> list[list[str]]:
        return self._core.levels()

    def _ancestors(self) -> list[list[int]]:
        names = self._core.names()
        anc: list[set[int]] = [set() for _ in names]
        pos = {n: i for i, n in enumerate(names)}
        for n in self._core.order():
            i = pos[n]
            for d in self._core.dependencies(n):
                anc[i].add(d)
                anc[i] |= anc[d]
        return [sorted(a) for a in anc]

    def _run(self, partial: bool):
        names = self._core.names()
        anc = self._ancestors()
        results: dict[str, Any] = {}
        errors: dict[str, BaseException] = {}

        def call(i: int) -> bool:
            try:
                results[names[i]] = self._fns[i]({names[a]: results[names[a]] for a in anc[i]})
                return True
            except BaseException as e:  # noqa: BLE001 - reported by execute()
                errors[names[i]] = e
                return False

        status = self._core.run(call, self._n_threads, partial)
        self.last_status = {names[i]: ("pending", "ok", "failed", "skipped", "not_run")[s] for i, s in enumerate(status)}
        return results, errors

    def execute(self) -> dict:
        """All results by task name; raises TaskGraphError for the first failed task (no task is started
        after a failure)."""
        results, errors = self._run(partial=False)
        if errors:
            name = next(iter(errors))
            raise TaskGraphError(name, errors[name])
        return results

    def execute_partial(self) -> dict:
        """Results of the tasks that succeeded; a failure skips only the tasks that depend on it."""
        results, _ = self._run(partial=True)
        return results


# ----------------------------------------------------------------------------- lock-free structures


class LockFreeCounter:
    """Atomic 64-bit counter (native std::atomic)."""

    def __init__(self, initial: int = 0):
        self._c = _native().AtomicCounter(initial)

    def increment(self) -> int:
        return self._c.increment()

    def decrement(self) -> int:
        return self._c.decrement()

    def add(self, n: int) -> int:
        return self._c.add(n)

    def get(self) -> int:
        return self._c.get()

    def compare_and_swap(self, expected: int, new: int) -> tuple[bool, int]:
        """(True, expected) if swapped, else (False, current value)."""
        return tuple(self._c.compare_and_swap(expected, new))

    def reset(self) -> int:
        """Sets 0 and returns the previous value."""
        return self._c.reset()


class LockFreeQueue:
    def __init__(self):
        self._d = collections.deque()

    def enqueue(self, value) -> None:
        self._d.append(value)

    def dequeue(self):
        try:
            return self._d.popleft()
        except IndexError:
            return None

    def is_empty(self) -> bool:
        return not self._d

    def __len__(self):
        return len(self._d)


class LockFreeStack:
    def __init__(self):
        self._d = collections.deque()

    def push(self, value) -> None:
        self._d.append(value)

    def pop(self):
        try:
            return self._d.pop()
        except IndexError:
            return None

    def is_empty(self) -> bool:
        return not self._d

    def __len__(self):
        return len(self._d)


def MpmcRing(capacity: int):  # noqa: N802 - constructor of the native class
    """Bounded lock-free MPMC queue of int64 values (capacity a power of two): try_push(v) -> bool,
    pop() -> int | None, size(), capacity()."""
    return _native().MpmcRing(capacity)


def ring_stress(capacity: int, producers: int, consumers: int, per_producer: int, timeout_s: float = 30.0) -> dict:
    """Moves producers * per_producer values through one MpmcRing from native threads; every value must
    arrive exactly once."""
    r, dup, miss, to = _native().ring_stress(capacity, producers, consumers, per_producer, timeout_s)
    return {"received": r, "duplicates": dup, "missing": miss, "timed_out": bool(to)}
