"""Graph rewriting (CSE, constant folding, simplification, fusion groups)
and scheduling / memory planning on define-then-run graphs."""
import numpy as np

from scirs_b200.autograd import graph as G
from scirs_b200.autograd import graph_opt as O


def _graph():
    g = G.Graph()
    x = g.placeholder("x", [4, 8])
    c = g.constant(2.0) * g.constant(3.0)  # foldable
    a = x * c
    b = x * c  # duplicate of a
    y = (a + b) * 1.0 + 0.0  # simplifiable
    z = G.Tensor(g, "exp", (G.Tensor(g, "neg", (y,)),))
    return g, x, y, z


def test_cse_fold_simplify_preserve_values():
    g, x, y, z = _graph()
    data = np.random.default_rng(0).standard_normal((4, 8)).astype(np.float32)
    before = z.eval({"x": data})
    n0 = len(O.reachable([z]))
    assert O.eliminate_common_subexpressions([z]) >= 1
    assert O.fold_constants([z]) >= 1
    assert O.simplify([z]) >= 2
    after = z.eval({"x": data})
    np.testing.assert_allclose(before, after, rtol=1e-6)
    assert len(O.reachable([z])) < n0
    assert any(n.op == "constant" and not n.inputs for n in O.reachable([z]))


def test_fusion_groups_chain_single_consumers():
    g = G.Graph()
    x = g.placeholder("x", [16])
    h = G.Tensor(g, "relu", (G.Tensor(g, "exp", (x * 2.0,)),))
    out = h + x
    groups = O.fusion_groups([out])
    assert groups and [n.op for n in groups[0]][:3] == ["mul", "exp", "relu"]


def test_schedules_and_memory_plan():
    g = G.Graph()
    x = g.placeholder("x", [1024])
    big = [G.Tensor(g, "exp", (x,), shape_hint=[1024]) for _ in range(4)]
    s = big[0]
    for b in big[1:]:
        s = G.Tensor(g, "add", (s, b), shape_hint=[1024])
    fwd = O.forward_schedule([s])
    assert O.validate_schedule(fwd) and O.validate_schedule(O.reverse_schedule([s]))
    mem = O.memory_optimal_schedule([s])
    assert O.validate_schedule(mem) and len(mem.order) == len(fwd.order)
    iv_mem = O.liveness(mem, [s])
    iv_fwd = O.liveness(fwd, [s])
    assert O.peak_memory(iv_mem) <= O.peak_memory(iv_fwd)
    slots = O.assign_memory_slots(iv_mem)
    ivs = {iv.node_id: iv for iv in iv_mem}
    for a in ivs.values():
        for b in ivs.values():
            if a.node_id != b.node_id and slots[a.node_id] == slots[b.node_id]:
                assert not a.overlaps(b)
    assert max(slots.values()) + 1 < len(iv_mem)
    levels = O.level_decomposition([s])
    assert len(levels[1]) == 4  # the four exps are independent
    path, cost = O.critical_path([s])
    assert path[-1] is s and cost == len(path) - 1
