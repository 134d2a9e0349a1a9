"""Phase timers, per-step JSONL metrics and the roofline calculator on a
CPU GPT engine step."""
import json

import torch

from scirs_b200.models.gpt import GPTConfig, GPTModel
from scirs_b200.utils import tracing as T


def test_phase_timer_and_step_logger(tmp_path):
    cfg = GPTConfig.tiny(vocab=256, seq=32)
    m = GPTModel(cfg, device="cpu", seed=0)
    m.configure_adamw(lr=1e-3)
    m.tracer = T.PhaseTimer()
    log = T.StepLogger(str(tmp_path / "steps.jsonl"), tokens_per_step=2 * 32, flops_per_token=cfg.flops_per_token(32),
                       model=m)
    tok = torch.randint(0, 256, (2, 33), generator=torch.Generator().manual_seed(0))
    for _ in range(3):
        log.begin()
        loss = m.train_step(tok[:, :-1], tok[:, 1:])
        log.log(loss, phases=m.tracer.collect())
    recs = [json.loads(l) for l in open(tmp_path / "steps.jsonl")]
    assert [r["step"] for r in recs] == [0, 1, 2]
    assert {"forward", "loss", "backward", "optimizer"} <= set(recs[-1]["phases_ms"])
    assert recs[-1]["tokens_per_s"] > 0 and "grad_norm" in recs[-1] and recs[-1]["comm_bytes_per_rank"] == 0
    assert set(m.tracer.summary()) == set(recs[-1]["phases_ms"])


def test_roofline():
    r = T.roofline(1.0, flops=1e12)
    assert r["bound"] == "compute" and 0.5 < r["frac_of_roofline"] < 0.8
    r = T.roofline(2.0, hbm_bytes=6e9, link_bytes=0.5e9)
    assert r["bound"] == "memory" and r["hbm_gbs"] == 3000.0
    with T.nvtx("noop"):
        pass
