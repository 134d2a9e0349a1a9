"""Hyperparameter tuner, metrics tracker, augmentation pipeline, enhanced
trainer and training profiler."""
import math

import torch

from scirs_b200.data import augmentation as A
from scirs_b200.training import hparam_tuner as HT
from scirs_b200.training.metrics_tracker import MetricGoal, MetricsTracker
from scirs_b200.training.trainer import EarlyStoppingConfig, EnhancedTrainer, EnhancedTrainingConfig, LRWarmupConfig


def _objective(cfg, resource=1):
    return (math.log10(cfg["lr"]) + 2) ** 2 + (cfg["layers"] - 3) ** 2 + (0 if cfg["act"] == "gelu" else 1) + 1 / resource


def _spaces():
    return [HT.HParamSpace.log_uniform("lr", 1e-4, 1.0), HT.HParamSpace.int_range("layers", 1, 6),
            HT.HParamSpace.choice("act", ["relu", "gelu"])]


def test_grid_random_halving_tpe_find_good_configs():
    best = HT.HParamTuner(_spaces(), HT.SearchStrategy.grid(5)).run(_objective)
    assert abs(math.log10(best.config["lr"]) + 2) < 0.6 and best.config["act"] == "gelu"
    rnd = HT.HParamTuner(_spaces(), HT.SearchStrategy.random_search(60), seed=1).run(_objective)
    assert rnd.score < 2.5
    sh = HT.HParamTuner(_spaces(), HT.SearchStrategy.successive_halving(27, 3, 27), seed=2)
    b = sh.run(_objective)
    assert b.resource == 27 and len({t.resource for t in sh.trials}) > 1
    tpe = HT.HParamTuner(_spaces(), HT.SearchStrategy.tpe(40, 8), seed=3)
    assert tpe.run(_objective).score < 2.5
    startup = [t.score for t in tpe.trials[:8]]
    guided = [t.score for t in tpe.trials[8:]]
    assert sum(guided) / len(guided) < sum(startup) / len(startup)  # the model concentrates on good regions


def test_metrics_tracker():
    mt = MetricsTracker(smoothing=0.5)
    mt.register_metric("acc", MetricGoal.MAXIMIZE)
    assert mt.record_batch("acc", 1.0) == 1.0 and mt.record_batch("acc", 0.0) == 0.5
    assert mt.end_epoch("acc", 0) == 0.0
    assert mt.record_epoch("acc", 1, 0.9) is not None
    assert mt.record_epoch("acc", 2, 0.7) is None
    assert mt.best("acc").epoch == 1 and mt.epochs_since_improvement("acc") == 1
    assert mt.stats("acc").count == 3


def test_augmentation_pipeline_shapes_and_determinism():
    x = torch.rand(4, 3, 32, 32)
    p = A.AugmentationPipeline.cifar10_train().with_seed(7)
    y = p(x)
    assert y.shape == x.shape
    q = A.AugmentationPipeline.cifar10_train().with_seed(7)
    torch.testing.assert_close(q(x), y)
    full = (A.AugmentationPipeline().add(A.RandomAffine(15, 0.1, (0.9, 1.1))).add(A.ColorJitter(0.2, 0.2, 0.2))
            .add(A.RandomErasing(1.0)).add(A.Cutout(8)).add(A.GaussianNoise(0.01)).add(A.RandomVerticalFlip(1.0)))
    assert full(x).shape == x.shape
    flip = A.AugmentationPipeline().add(A.RandomHorizontalFlip(1.0))
    torch.testing.assert_close(flip(x), x.flip(-1))
    cut = A.AugmentationPipeline().add(A.Cutout(8))(torch.ones(2, 1, 16, 16))
    assert float((cut == 0).sum()) == 2 * 64
    xm, ym = A.apply_mixup(x, torch.tensor([0, 1, 2, 3]), 4, seed=1)
    assert xm.shape == x.shape and torch.allclose(ym.sum(1), torch.ones(4))
    xc, yc = A.apply_cutmix(x, torch.tensor([0, 1, 2, 3]), 4, seed=1)
    assert xc.shape == x.shape and torch.allclose(yc.sum(1), torch.ones(4))


def test_enhanced_trainer_warmup_early_stopping_and_profiler():
    torch.manual_seed(0)
    w = torch.randn(8, 1)
    xs = torch.randn(256, 8)
    data = [(xs[i:i + 32], xs[i:i + 32] @ w) for i in range(0, 256, 32)]
    model = torch.nn.Sequential(torch.nn.Linear(8, 16), torch.nn.ReLU(), torch.nn.Linear(16, 1))
    opt = torch.optim.SGD(model.parameters(), lr=0.05)
    cfg = EnhancedTrainingConfig(epochs=40, grad_accumulation=2, max_grad_norm=5.0, log_every=0,
                                 warmup=LRWarmupConfig(warmup_steps=10),
                                 early_stopping=EarlyStoppingConfig(enabled=True, patience=3, min_delta=1e-4),
                                 profile=True)
    tr = EnhancedTrainer(model, opt, torch.nn.functional.mse_loss, cfg, log=lambda *_: None)
    st = tr.fit(data, val_data=data[:2])
    assert st.history["loss"][-1] < st.history["loss"][0] * 0.5
    assert st.global_step >= 10 and opt.param_groups[0]["lr"] == 0.05
    assert LRWarmupConfig(10).factor(5) == 0.5
    b = tr.profiler.bottlenecks()
    assert b and 0 < b[0].share <= 1 and tr.profiler.layers["0"].avg_forward() > 0
