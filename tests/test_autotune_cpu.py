"""GEMM auto-tuner logic with a stand-in kernel and timer: candidate sets,
selection of the fastest configuration, skipped configurations, accumulate
restore, and the persistent cache."""
import pytest
import torch

from scirs_b200.ops import autotune as AT
from scirs_b200.ops import kernels as K


class FakeGemm:
    """Adds a @ b.T into out; 'time' depends on the configuration; bn=128 is rejected for N < 256."""

    def __init__(self):
        self.calls = []
        self.cfg = None

    def __call__(self, a, b, out, *, a_mn, b_mn, epi, accumulate, splits, bn, **kw):
        if bn == 128 and out.shape[1] < 256:
            raise RuntimeError("tile width not supported for this shape\nmore")
        self.cfg = (splits, bn)
        self.calls.append(self.cfg)
        r = a @ b.t()
        out.copy_(out + r if accumulate else r)


def fake_time(gemm):
    table = {(0, 0): 1.0, (4, 256): 0.4, (2, 0): 0.7}

    def timer(fn):
        fn()
        return table.get(gemm.cfg, 2.0)

    return timer


def test_candidates():
    assert AT.GemmAutotuner.candidates(K.EPI_BF16) == [(0, 0), (0, 128), (0, 256)]
    assert len(AT.GemmAutotuner.candidates(K.EPI_F32)) == len(AT.SPLITS_F32) * 3


def test_tune_picks_fastest_and_skips_rejected(tmp_path):
    g = FakeGemm()
    tuner = AT.GemmAutotuner(str(tmp_path / "c.json"), warmup=1, timer=fake_time(g), gemm_fn=g)
    a, b = torch.randn(16, 8), torch.randn(64, 8)
    out = torch.zeros(16, 64)
    e = tuner.tune(a, b, out, epi=K.EPI_F32)
    assert (e["splits"], e["bn"]) == (4, 256) and e["ms"] == 0.4 and e["default_ms"] == 1.0
    assert sum("error" in r for r in e["results"]) == len(AT.SPLITS_F32)  # every bn=128 candidate
    assert tuner.lookup(a, b, epi=K.EPI_F32) == (4, 256)
    # persisted and reloaded
    again = AT.GemmAutotuner(str(tmp_path / "c.json"), gemm_fn=g)
    assert again.lookup(a, b, epi=K.EPI_F32) == (4, 256)
    g.calls.clear()
    again.gemm(a, b, out, epi=K.EPI_F32)
    assert g.calls == [(4, 256)] and torch.allclose(out, a @ b.t())
    assert again.lookup(a, b, epi=K.EPI_BF16) is None


def test_accumulate_output_restored_and_untuned_default():
    g = FakeGemm()
    tuner = AT.GemmAutotuner(None, warmup=2, timer=fake_time(g), gemm_fn=g)
    a, b = torch.randn(4, 8), torch.randn(256, 8)
    out = torch.full((4, 256), 3.0)
    tuner.tune(a, b, out, epi=K.EPI_F32, accumulate=True)
    assert torch.equal(out, torch.full((4, 256), 3.0))  # tuning runs did not leak into the output
    g.calls.clear()
    tuner.gemm(a, b, torch.zeros(4, 256), epi=K.EPI_BF16, tune_missing=False)
    assert g.calls == [(0, 0)]


def test_all_rejected_raises():
    def bad(*a, **k):
        raise RuntimeError("no")

    with pytest.raises(RuntimeError, match="no GEMM configuration"):
        AT.GemmAutotuner(None, timer=lambda fn: 1.0, gemm_fn=bad).tune(torch.zeros(2, 8), torch.zeros(8, 8),
                                                                      torch.zeros(2, 8))
