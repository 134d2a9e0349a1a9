"""LR range test, curriculum learner, initialisers and activation
checkpointing plans."""
import math

import pytest
import torch

from scirs_b200.autograd import checkpointing as C
from scirs_b200.training import curriculum as CU
from scirs_b200.training import lr_finder as L
from scirs_b200.utils import initializers as I


def test_lr_schedule_and_smoothing():
    cfg = L.LRFinderConfig(min_lr=1e-4, max_lr=1.0, num_iterations=4)
    assert math.isclose(cfg.lr_at_step(2), 1e-2)
    lin = L.LRFinderConfig(min_lr=0.1, max_lr=0.5, num_iterations=4, schedule=L.LRScheduleType.LINEAR)
    assert math.isclose(lin.lr_at_step(1), 0.2)
    r = L.LRFinderResult.from_losses([2.0, 1.0], L.LRFinderConfig(smoothing_factor=0.5, num_iterations=2))
    assert math.isclose(r.points[0].smoothed_loss, 2.0)
    assert math.isclose(r.points[1].smoothed_loss, (0.25 * 2 + 0.5 * 1.0) / 0.75)
    ref = L.LRFinderResult.from_losses([2.0, 1.0], L.LRFinderConfig(smoothing_factor=0.5, num_iterations=2,
                                                                    bias_correction="reference"))
    # the reference seeds the EMA with the first loss and still divides
    assert math.isclose(ref.points[0].smoothed_loss, 4.0)
    assert math.isclose(ref.points[1].smoothed_loss, 1.5 / 0.75)


def test_lr_finder_on_quadratic_finds_useful_lr():
    torch.manual_seed(0)
    w = torch.nn.Parameter(torch.randn(20))
    opt = torch.optim.SGD([w], lr=1e-5)

    def step():
        loss = (w - 3).square().sum()
        opt.zero_grad()
        loss.backward()
        opt.step()
        return loss.item()

    def set_lr(lr):
        for g in opt.param_groups:
            g["lr"] = lr

    w0 = w.detach().clone()
    res = L.find_optimal_lr(step, set_lr, L.LRFinderConfig(min_lr=1e-5, max_lr=10, num_iterations=80),
                            state=lambda: w.detach().clone(), restore=lambda s: w.data.copy_(s))
    assert res.diverged  # lr 10 on this quadratic blows up
    s = res.suggested_lr()
    assert s is not None and 1e-4 < s < 1.0
    assert torch.equal(w.detach(), w0)
    assert "suggested lr" in res.summary()


def test_curriculum_strategies():
    d = [0.9, 0.1, 0.5, 0.3, 0.7]
    cfg = CU.CurriculumConfig(initial_competence=0.2, num_epochs=4, shuffle_within_subset=False)
    cl = CU.CurriculumLearner(cfg, d)
    assert cl.get_batch_indices(0) == [1]
    assert cl.get_batch_indices(4) == [1, 3, 2, 4, 0]
    anti = CU.CurriculumLearner(CU.CurriculumConfig(CU.CurriculumStrategy.ANTI_CURRICULUM, initial_competence=0.2,
                                                    num_epochs=4, shuffle_within_subset=False), d)
    assert anti.get_batch_indices(0) == [0]
    op = CU.CurriculumLearner(CU.CurriculumConfig(CU.CurriculumStrategy.ONE_PASS, initial_competence=0.2,
                                                  num_epochs=4, shuffle_within_subset=False), d)
    bands = [op.get_batch_indices(e) for e in range(5)]
    assert {i for b in bands for i in b} == {0, 1, 2, 3, 4}  # bands may share an edge sample
    sp = CU.CurriculumLearner(CU.CurriculumConfig(CU.CurriculumStrategy.SELF_PACED, min_samples=2,
                                                  shuffle_within_subset=False), d)
    sp.update_losses([0.1, 5.0, 0.2, 5.0, 5.0])
    assert sp.get_batch_indices(0) == [0, 2]
    assert math.isclose(sp.self_paced_threshold, 0.6)
    step = CU.CurriculumConfig(schedule=CU.CompetenceSchedule("step", 2), initial_competence=0.5, num_epochs=10)
    assert step.competence_at(3) == 0.75 and step.competence_at(10) == 1.0
    with pytest.raises(ValueError):
        CU.CurriculumConfig(initial_competence=0.0)


def test_initializers():
    g = torch.Generator().manual_seed(0)
    w = torch.empty(256, 512)
    I.xavier_uniform_(w, generator=g)
    assert float(w.abs().max()) <= math.sqrt(6 / 768) + 1e-6
    I.kaiming_normal_(w, generator=g)
    assert abs(float(w.std()) - math.sqrt(2 / 512)) < 0.003
    q = torch.empty(64, 128)
    I.orthogonal_(q, generator=g)
    torch.testing.assert_close(q @ q.t(), torch.eye(64), atol=1e-5, rtol=0)
    assert I.fans(torch.empty(8, 4, 3, 3)) == (36, 72)
    I.initialize(w, "zeros")
    assert float(w.abs().sum()) == 0


def test_checkpoint_plans():
    p = C.sqrt_checkpoint_plan(16)
    assert p.checkpoint_indices == [0, 4, 8, 12, 15]
    u = C.uniform_checkpoint_plan(10, 3)
    assert u.checkpoint_indices == [0, 3, 6, 9]
    b = C.binomial_checkpoint_plan(20, 3)
    assert b.recomputation_cost == 3 and math.comb(6, 3) >= 20 > math.comb(5, 3)
    assert 1 <= len(b.checkpoint_indices) <= 3 and b.checkpoint_indices[0] == 0
    assert C.binomial_checkpoint_plan(0, 3).checkpoint_indices == []


def test_checkpoint_sequential_matches_plain_backward():
    torch.manual_seed(0)
    layers = [torch.nn.Sequential(torch.nn.Linear(16, 16), torch.nn.GELU(), torch.nn.Dropout(0.1))
              for _ in range(9)]
    x = torch.randn(4, 16, requires_grad=True)
    torch.manual_seed(1)
    y = x
    for m in layers:
        y = m(y)
    y.square().sum().backward()
    ref = [p.grad.clone() for m in layers for p in m.parameters()]
    gx = x.grad.clone()
    for m in layers:
        m.zero_grad()
    x.grad = None
    torch.manual_seed(1)
    C.checkpoint_sequential(layers, x, C.sqrt_checkpoint_plan(9)).square().sum().backward()
    got = [p.grad for m in layers for p in m.parameters()]
    for a, b in zip(ref, got):
        torch.testing.assert_close(a, b)
    torch.testing.assert_close(gx, x.grad)
