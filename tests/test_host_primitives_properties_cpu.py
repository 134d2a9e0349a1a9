"""Property-based tests of the native host runtime: scans, segmented scans and
the stable sort against serial oracles for arbitrary sizes (including 0 and
1) and thread counts, and random DAGs through the task-graph scheduler
(dependencies respected, failures skip exactly the dependents)."""
import threading

import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from scirs_b200 import _ext
from scirs_b200.parallel import primitives as P

SET = settings(max_examples=40, deadline=None)
N = _ext.data()


@SET
@given(st.integers(0, 200_000), st.integers(1, 16), st.sampled_from([0, 1, 2, 3]), st.booleans(),
       st.integers(0, 2**31 - 1))
def test_native_scan_matches_serial(n, threads, op, exclusive, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randint(-3, 4, (n,), generator=g, dtype=torch.int64)
    if op == 1:  # products: keep them small and exact
        x = torch.randint(1, 2, (n,), generator=g, dtype=torch.int64) * torch.where(
            torch.rand(n, generator=g) < 0.01, -1, 1)
    got = N.scan(x, op, exclusive, threads)
    ref = {0: lambda t: t.cumsum(0), 1: lambda t: t.cumprod(0), 2: lambda t: t.cummin(0).values,
           3: lambda t: t.cummax(0).values}[op](x) if n else x.clone()
    if exclusive and n:
        ident = {0: 0, 1: 1, 2: torch.iinfo(torch.int64).max, 3: torch.iinfo(torch.int64).min}[op]
        ref = torch.cat([torch.tensor([ident]), ref[:-1]])
    assert torch.equal(got, ref)


@SET
@given(st.integers(0, 150_000), st.integers(1, 16), st.floats(0.0, 0.05), st.integers(0, 2**31 - 1))
def test_native_segmented_scan_matches_serial(n, threads, head_rate, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randint(-5, 6, (n,), generator=g)
    f = torch.rand(n, generator=g) < head_rate
    got = N.segmented_scan_sum(x, f, threads)
    acc = 0
    xs, fs = x.tolist(), f.tolist()
    out = []
    for v, h in zip(xs, fs):
        acc = v if h else acc + v
        out.append(acc)
    assert got.tolist() == out


@SET
@given(st.integers(0, 100_000), st.integers(1, 16), st.booleans(), st.sampled_from(["f32", "f64", "i32"]),
       st.integers(0, 2**31 - 1))
def test_native_sort_is_torch_stable_sort(n, threads, desc, dt, seed):
    g = torch.Generator().manual_seed(seed)
    if dt == "i32":
        x = torch.randint(-50, 50, (n,), generator=g, dtype=torch.int32)
    else:
        x = torch.randn(n, generator=g, dtype=torch.float32 if dt == "f32" else torch.float64).round(decimals=1)
        if n:
            x[torch.rand(n, generator=g) < 0.01] = float("nan")
    v, i = N.parallel_sort(x, desc, threads)
    tv, ti = torch.sort(x, descending=desc, stable=True)
    assert torch.equal(i, ti)
    assert torch.equal(v.isnan(), tv.isnan()) and torch.equal(v[~v.isnan()], tv[~tv.isnan()])


@settings(max_examples=30, deadline=None)
@given(st.integers(1, 40), st.floats(0.0, 0.5), st.floats(0.0, 0.3), st.integers(1, 8), st.booleans(),
       st.integers(0, 2**31 - 1))
def test_random_dags(n, edge_p, fail_p, threads, partial, seed):
    g = torch.Generator().manual_seed(seed)
    deps = [[j for j in range(i) if torch.rand(1, generator=g).item() < edge_p] for i in range(n)]
    fails = {i for i in range(n) if torch.rand(1, generator=g).item() < fail_p}
    done, lock = [], threading.Lock()

    def body(i):
        def f(results):
            assert set(results) >= {f"t{d}" for d in deps[i]}  # every dependency finished first
            with lock:
                done.append(i)
            if i in fails:
                raise ValueError(i)
            return i

        return f

    tg = P.TaskGraph(threads)
    for i in range(n):
        tg.add_task(f"t{i}", [f"t{d}" for d in deps[i]], body(i))
    bad = set()  # tasks that fail or (transitively) depend on a failure
    for i in range(n):
        if i in fails or any(d in bad for d in deps[i]):
            bad.add(i)
    if partial:
        res = tg.execute_partial()
        assert set(res) == {f"t{i}" for i in range(n) if i not in bad}
        skipped = {i for i in range(n) if any(d in bad for d in deps[i])}  # a failed dependency: never run
        assert {i for i in range(n) if tg.last_status[f"t{i}"] == "skipped"} == skipped
    else:
        try:
            res = tg.execute()
            assert not fails and len(res) == n
        except P.TaskGraphError as e:
            assert int(e.task[1:]) in fails
    assert all(not any(d in bad for d in deps[i]) for i in done)  # no task after a failure ever ran
    level = {}
    for lv, names in enumerate(tg.execution_levels()):
        for nm in names:
            level[int(nm[1:])] = lv
    assert all(level[d] < level[i] for i in range(n) for d in deps[i])
