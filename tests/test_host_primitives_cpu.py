"""Host-parallel primitives on the native runtime: task graph scheduling and failure
propagation, work queue / worker pool, parallel map / fold / sort, scans (against
torch / serial oracles) and the lock-free ring under native producer / consumer
threads."""
import threading
import time

import pytest
import torch

from scirs_b200.parallel import primitives as P


def test_task_graph_results_order_levels():
    g = P.TaskGraph()
    g.add_task("load", [], lambda r: 42)
    g.add_task("process", ["load"], lambda r: r["load"] * 2)
    g.add_task("side", ["load"], lambda r: r["load"] + 1)
    g.add_task("save", ["process", "side"], lambda r: r["process"] + r["side"] + r["load"])
    assert len(g) == 4 and g.contains_task("side") and not g.contains_task("x")
    assert g.dependencies("save") == ["process", "side"] and g.dependencies("nope") is None
    assert g.execution_order() == ["load", "process", "side", "save"]
    assert g.execution_levels() == [["load"], ["process", "side"], ["save"]]
    assert g.execute() == {"load": 42, "process": 84, "side": 43, "save": 169}
    assert P.TaskGraph().execute() == {}


def test_task_graph_rejects_duplicates_missing_and_cycles():
    g = P.TaskGraph()
    g.add_task("a", [], lambda r: 1)
    g.add_task("b", ["a"], lambda r: 2)
    with pytest.raises(ValueError, match="already exists"):
        g.add_task("a", [], lambda r: 0)
    with pytest.raises(ValueError, match="does not exist"):
        g.add_task("c", ["zzz"], lambda r: 0)
    with pytest.raises(ValueError, match="cycle"):
        g.add_dependency("a", "b")
    g.add_task("c", [], lambda r: 3)
    g.add_dependency("c", "b")
    assert g.execution_order() == ["a", "b", "c"]


def test_task_graph_failure_strict_and_partial():
    def boom(r):
        raise KeyError("bad")

    def build():
        g = P.TaskGraph(n_threads=1)
        g.add_task("a", [], lambda r: 1)
        g.add_task("bad", ["a"], boom)
        g.add_task("after_bad", ["bad"], lambda r: 5)
        g.add_task("deep", ["after_bad"], lambda r: 6)
        g.add_task("ok", ["a"], lambda r: r["a"] + 10)
        return g

    g = build()
    with pytest.raises(P.TaskGraphError) as ei:
        g.execute()
    assert ei.value.task == "bad" and isinstance(ei.value.cause, KeyError)
    assert g.last_status["after_bad"] == "skipped" and g.last_status["deep"] == "skipped"
    g = build()
    res = g.execute_partial()
    assert res == {"a": 1, "ok": 11}
    assert g.last_status == {"a": "ok", "bad": "failed", "after_bad": "skipped", "deep": "skipped", "ok": "ok"}


def test_task_graph_runs_independent_tasks_concurrently():
    g = P.TaskGraph(n_threads=8)
    for i in range(8):
        g.add_task(f"t{i}", [], lambda r: time.sleep(0.2) or 1)  # sleep releases the interpreter lock
    g.add_task("sum", [f"t{i}" for i in range(8)], lambda r: sum(r.values()))
    t0 = time.perf_counter()
    assert g.execute()["sum"] == 8
    assert time.perf_counter() - t0 < 1.0  # serial would take 1.6 s


def test_task_graph_dataflow_starts_before_level_finishes():
    # "fast2" depends only on "fast"; it must not wait for the slow task of the same level
    events = []
    g = P.TaskGraph(n_threads=4)
    g.add_task("slow", [], lambda r: time.sleep(0.5) or events.append("slow"))
    g.add_task("fast", [], lambda r: events.append("fast"))
    g.add_task("fast2", ["fast"], lambda r: events.append("fast2"))
    g.execute()
    assert events.index("fast2") < events.index("slow")


def test_work_queue_and_receiver():
    q, rx = P.WorkQueue.new(2)
    assert q.capacity() == 2 and q.is_empty()
    q.push(1)
    assert q.try_push(2) and not q.try_push(3)
    with pytest.raises(P.DistributedError):
        q.push(3, timeout=0.05)
    assert rx.recv() == 1 and rx.try_recv() == 2 and rx.try_recv() is None
    assert rx.recv_timeout(0.05) is None
    q.push(None)  # None is a valid task
    q.close()
    assert len(q) == 1 and rx.recv() is None and rx.recv() is None
    with pytest.raises(P.DistributedError):
        q.try_push(4)


def test_worker_pool_collects_results_and_errors():
    pool = P.WorkerPool(3, lambda x: 10 // x)
    assert pool.n_workers == 3
    for x in (1, 2, 5, 0):
        pool.submit(x)
    res = pool.collect_all(4, timeout=5.0)
    pool.shutdown()
    assert sorted(r for r in res if not isinstance(r, Exception)) == [2, 5, 10]
    errs = [r for r in res if isinstance(r, P.DistributedError)]
    assert len(errs) == 1 and isinstance(errs[0].__cause__, ZeroDivisionError)
    assert pool.collect_result(timeout=0.01) is None


def test_map_reduce_and_chunked():
    assert P.distributed_map(range(1, 9), lambda x: x * x, 4) == [1, 4, 9, 16, 25, 36, 49, 64]
    assert P.distributed_map_reduce(range(1, 101), lambda x: x, lambda a, b: a + b, 0, 4) == 5050
    assert P.chunked_parallel_process(list(range(1, 13)), lambda c: [x * 2 for x in c], 5, 3) == \
        [2 * x for x in range(1, 13)]
    assert P.distributed_map([], lambda x: x) == []
    with pytest.raises(ZeroDivisionError):
        P.distributed_map([1, 0, 2], lambda x: 1 // x, 2)


def test_resource_monitor():
    m = P.ResourceMonitor(0.5, 0)
    assert m.available_workers() == max(1, m.logical_cpu_count() // 2)
    assert m.recommended_chunk_size(0) == 64 and m.recommended_chunk_size(10) == 64
    assert m.recommended_chunk_size(10**7) == 10**7 // (m.available_workers() * 4)
    assert m.can_submit() and not P.ResourceMonitor(1.0, 1 << 62).can_submit()
    assert P.ResourceMonitor(7.0).cpu_threshold == 1.0


def test_par_iterators():
    data = list(range(1000))
    assert P.par_map(data, lambda x: x + 1, 4) == [x + 1 for x in data]
    assert P.par_filter(data, lambda x: x % 7 == 0, 4) == [x for x in data if x % 7 == 0]
    assert P.par_filter_map(data, lambda x: x * 2 if x % 3 == 0 else None) == [x * 2 for x in data if x % 3 == 0]
    assert P.par_fold(data, 0, lambda a, x: a + x, lambda a, b: a + b, 8) == sum(data)
    assert P.par_fold([], 5, lambda a, x: a + x, lambda a, b: a + b) == 5
    assert P.par_any(data, lambda x: x == 999) and not P.par_any(data, lambda x: x < 0)
    assert P.par_all(data, lambda x: x >= 0) and not P.par_all(data, lambda x: x < 999)
    seen = []
    lock = threading.Lock()

    def rec(x):
        with lock:
            seen.append(x)

    P.par_for_each(data, rec, 4)
    assert sorted(seen) == data


def test_par_sort_matches_torch_stable():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(200_000, generator=g)
    x[::997] = float("nan")
    for desc in (False, True):
        v, i = P.par_sort(x, 8, descending=desc, return_indices=True)
        tv, ti = torch.sort(x, descending=desc, stable=True)
        assert torch.equal(i, ti) and torch.allclose(v, tv, equal_nan=True)
    xi = torch.randint(0, 20, (100_000,), generator=g)
    assert torch.equal(P.par_sort(xi, 6, return_indices=True)[1], torch.sort(xi, stable=True)[1])
    assert P.par_sort([3, 1, 2]) == [1, 2, 3]
    assert P.par_sort(["b", "a", "c"], descending=True) == ["c", "b", "a"]
    words = ["ccc", "a", "bb", "dd", "e"]
    assert P.par_sort_by(words, len) == ["a", "e", "bb", "dd", "ccc"]  # stable on equal keys


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32, torch.int64, torch.int32])
def test_scans_against_torch(dtype):
    g = torch.Generator().manual_seed(1)
    n = 300_001
    x = (torch.randn(n, generator=g) * 10).to(dtype)
    tol = dict(rtol=1e-9, atol=1e-7) if dtype == torch.float64 else dict(rtol=1e-4, atol=1e-1)
    assert torch.allclose(P.parallel_prefix_sum(x, 8).double(), x.double().cumsum(0), **tol)
    ex = P.parallel_prefix_sum_exclusive(x, 8)
    assert ex[0] == 0 and torch.allclose(ex[1:].double(), x.double().cumsum(0)[:-1], **tol)
    assert torch.equal(P.parallel_prefix_min(x, 8), x.cummin(0).values)
    assert torch.equal(P.parallel_prefix_max(x, 8), x.cummax(0).values)


def test_scans_on_lists_and_custom_ops():
    assert P.parallel_prefix_sum([1, 2, 3, 4]) == [1, 3, 6, 10]
    assert P.parallel_prefix_sum_exclusive([1, 2, 3, 4]) == [0, 1, 3, 6]
    assert P.parallel_scan([2, 3, 4], 1, "prod") == [2, 6, 24]
    # a non-commutative associative operator: string concatenation, chunked over 4 workers
    words = [chr(97 + i % 26) for i in range(103)]
    got = P.parallel_scan(words, "", lambda a, b: a + b, 4)
    assert got == ["".join(words[: i + 1]) for i in range(len(words))]
    assert P.parallel_scan_exclusive(words, "", lambda a, b: a + b, 4)[:3] == ["", "a", "ab"]
    assert P.parallel_scan([], 0, "sum") == []


def test_segmented_prefix_sum():
    assert P.segmented_prefix_sum([1, 2, 3, 4, 5], [True, False, True, False, False]) == [1, 3, 3, 7, 12]
    g = torch.Generator().manual_seed(2)
    n = 250_000
    x = torch.randint(-3, 4, (n,), generator=g)
    f = torch.rand(n, generator=g) < 0.0005
    got = P.segmented_prefix_sum(x, f, 8)
    seg = torch.cumsum(f.long(), 0)
    cs = torch.cumsum(x, 0)
    start = torch.zeros(int(seg.max()) + 1, dtype=torch.long)
    heads = torch.nonzero(f).flatten()
    start[seg[heads]] = cs[heads] - x[heads]
    assert torch.equal(got, cs - start[seg])


def test_lock_free_counter_and_containers():
    c = P.LockFreeCounter(5)
    assert c.increment() == 6 and c.decrement() == 5 and c.add(10) == 15
    assert c.compare_and_swap(15, 1) == (True, 15) and c.compare_and_swap(3, 9) == (False, 1)
    assert c.reset() == 1 and c.get() == 0
    q, s = P.LockFreeQueue(), P.LockFreeStack()
    for i in range(3):
        q.enqueue(i)
        s.push(i)
    assert [q.dequeue() for _ in range(4)] == [0, 1, 2, None]
    assert [s.pop() for _ in range(4)] == [2, 1, 0, None] and s.is_empty() and q.is_empty()


def test_counter_under_threads():
    c = P.LockFreeCounter()
    P.par_for_each(list(range(4000)), lambda _: c.increment(), 8)
    assert c.get() == 4000


def test_mpmc_ring_single_thread_and_native_stress():
    r = P.MpmcRing(4)
    assert r.capacity() == 4 and r.pop() is None
    assert all(r.try_push(i) for i in range(4)) and not r.try_push(9)
    assert [r.pop() for _ in range(5)] == [0, 1, 2, 3, None]
    with pytest.raises(RuntimeError):
        P.MpmcRing(6)
    res = P.ring_stress(64, producers=4, consumers=3, per_producer=25_000, timeout_s=60.0)
    assert res == {"received": 100_000, "duplicates": 0, "missing": 0, "timed_out": False}
