"""Host-side pieces of the pipeline-parallel GPT: the stage split and the
canonical initialisation order shared with the unsplit model."""
import torch

from scirs_b200.models.gpt import GPTConfig, GPTModel, gpt_init_values, gpt_param_shapes
from scirs_b200.models.gpt_pipeline import stage_bounds
from scirs_b200.parallel.pipeline import generate_1f1b_schedule


def test_stage_bounds_cover_all_layers():
    for L in (1, 4, 12, 13, 48):
        for P in range(1, min(L, 8) + 1):
            spans = [stage_bounds(L, P, s) for s in range(P)]
            assert spans[0][0] == 0 and spans[-1][1] == L
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1 and min(sizes) >= 1


def test_init_values_match_unsplit_model():
    cfg = GPTConfig.tiny()
    m = GPTModel(cfg, device="cpu", seed=4)
    assert m.fp.order == [n for n, _ in gpt_param_shapes(cfg)]
    for name, t in gpt_init_values(cfg, 4):
        assert torch.equal(m.fp.m(name).cpu(), t), name


def test_1f1b_stash_bound():
    # the activation pool of stage s holds min(micro, P - s) sets
    for P in (2, 4, 8):
        for s in range(P):
            live, peak = 0, 0
            for kind, _ in generate_1f1b_schedule(P, 8, s):
                live += 1 if kind == "F" else -1
                peak = max(peak, live)
            assert peak == min(8, P - s)
