"""Callback manager, function callbacks, gradient clipping, LR schedule callbacks, visualization
callback, driven through Sequential.fit (CPU)."""
import math

import torch

from scirs_b200.nn.layers import Dense
from scirs_b200.nn.sequential import Sequential
from scirs_b200.training import callbacks as C


def _lr(m):
    o = m.optimizer
    return o.get_learning_rate() if hasattr(o, "get_learning_rate") else o.param_groups[0]["lr"]


def _model():
    torch.manual_seed(0)
    m = Sequential()
    m.add(Dense(4, 8, activation="relu"))
    m.add(Dense(8, 1))
    m.compile(loss="mse", optimizer="sgd", learning_rate=0.05)
    return m


def test_fit_with_callbacks(tmp_path):
    x, y = torch.randn(32, 4), torch.randn(32, 1)
    seen = []
    fc = C.FunctionCallback(C.CallbackTiming.AFTER_EPOCH, lambda ctx: seen.append(ctx["epoch"]))
    clip = C.GradientClipping.by_global_norm(1e-3)
    sched = C.StepDecay(0.2, 0.5, 2)
    viz = C.VisualizationCallback(frequency=2, save_path=str(tmp_path))
    m = _model()
    m.fit(x, y, epochs=4, batch_size=8, callbacks=[C.CallbackManager([fc, clip, sched, viz])])
    assert seen == [0, 1, 2, 3]
    assert clip.clipping_applied and 0 < clip.clipping_ratio < 1
    assert abs(_lr(m) - 0.2 * 0.5 ** 1) < 1e-12 and sched.current_lr == _lr(m)  # epochs 0..3: last 3 // 2 = 1
    assert len(viz.rendered) == 2 and (tmp_path / "loss.svg").exists()


def test_clip_by_value_and_schedules():
    m = _model()
    x, y = torch.randn(8, 4), 100 * torch.randn(8, 1)
    clip = C.GradientClipping.by_value(0.01)
    m.fit(x, y, epochs=1, batch_size=8, callbacks=[clip])
    assert clip.clipping_applied
    cos = C.CosineAnnealingLR(1.0, 0.0, 4)
    assert [round(cos.lr_at(s), 6) for s in range(5)] == [1.0, round((1 + math.cos(math.pi / 4)) / 2, 6), 0.5,
                                                          round((1 + math.cos(3 * math.pi / 4)) / 2, 6), 1.0]
    rp = C.ReduceOnPlateau(0.1, factor=0.5, patience=2, min_lr=0.02)
    m2 = _model()
    rp.on_train_begin(m2)
    for ep, v in enumerate([1.0, 0.9, 0.95, 0.95, 0.97, 0.99, 0.99]):
        rp.on_epoch_end(ep, m2, {"val_loss": v})
    assert abs(rp.current_lr - 0.025) < 1e-12 and _lr(m2) == rp.current_lr
