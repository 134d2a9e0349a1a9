"""Legacy JSON model layout, serde-compatible float text, safetensors
checkpoint directories, and the MLP configuration end to end on CPU."""
import json
import math
import os
import random

import torch

from scirs_b200.models.mlp import mnist_mlp, train_mnist_mlp
from scirs_b200.nn.conv import Conv2D, MaxPool2D
from scirs_b200.nn.layers import BatchNorm, Dense, Dropout, LayerNorm
from scirs_b200.nn.sequential import Sequential
from scirs_b200.training import checkpoint as ck
from scirs_b200.training.serialization import (
    format_float,
    load_model,
    load_model_safetensors,
    save_model,
    save_model_safetensors,
    to_serde_pretty,
)


def test_format_float_serde_rules():
    cases = {1.0: "1.0", 0.5: "0.5", -2.25: "-2.25", 1e-05: "0.00001", 1.234e-06: "1.234e-6", 0.0001234: "0.0001234",
             1e16: "1e16", 1e15: "1000000000000000.0", 123.456: "123.456", 0.1: "0.1",
             1.5e300: "1.5e300", 3e-300: "3e-300", 100.0: "100.0"}
    for v, s in cases.items():
        assert format_float(v) == s, (v, format_float(v), s)
    assert format_float(0.0) == "0.0" and format_float(-0.0) == "-0.0"
    rng = random.Random(0)
    for _ in range(2000):
        v = rng.uniform(-1, 1) * 10 ** rng.randint(-30, 30)
        assert float(format_float(v)) == v


def test_serde_pretty_layout():
    s = to_serde_pretty({"name": "x", "layers": [{"type": "Dropout", "p": 0.5}], "parameters": [[]]})
    assert s == ('{\n  "name": "x",\n  "layers": [\n    {\n      "type": "Dropout",\n      "p": 0.5\n    }\n  ],\n'
                 '  "parameters": [\n    []\n  ]\n}')


def test_legacy_json_roundtrip(tmp_path):
    m = Sequential(Dense(6, 4, "relu", seed=1, dtype=torch.float64), Dropout(0.25),
                   Dense(4, 3, None, seed=2, dtype=torch.float64))
    p = tmp_path / "mnist_model.json"
    save_model(m, p)
    obj = json.load(open(p))
    assert obj["name"] == "SciRS2 Sequential Model" and obj["version"] == "0.1.0"
    assert obj["layers"][0] == {"type": "Dense", "input_dim": 6, "output_dim": 4, "activation": "relu"}
    assert obj["layers"][1] == {"type": "Dropout", "p": 0.25}
    assert len(obj["parameters"][0][0]) == 24 and len(obj["parameters"][0][1]) == 4 and obj["parameters"][1] == []
    # weights are [in, out] row-major
    assert obj["parameters"][0][0][:4] == m.layers()[0].weight[0].tolist()
    m2 = load_model(p)
    x = torch.randn(5, 6, dtype=torch.float64)
    m.eval()
    m2.eval()
    assert torch.equal(m(x), m2(x))
    # reference quirks mode writes what the reference writer writes
    save_model(m, tmp_path / "q.json", reference_quirks=True)
    q = json.load(open(tmp_path / "q.json"))
    assert q["layers"][0]["activation"] is None and q["layers"][1]["p"] == 0.5


def test_legacy_json_other_layer_kinds(tmp_path):
    m = Sequential(Conv2D(1, 2, 3, 1, 1, dtype=torch.float64), BatchNorm(2, dtype=torch.float64),
                   MaxPool2D(2), LayerNorm(7, dtype=torch.float64))
    save_model(m, tmp_path / "m.json")
    m2 = load_model(tmp_path / "m.json")
    x = torch.randn(1, 1, 14, 14, dtype=torch.float64)
    m.eval()
    m2.eval()
    assert torch.allclose(m(x), m2(x))


def test_checkpoint_directory(tmp_path):
    m = mnist_mlp(dtype=torch.float32, seed=0)
    params = {f"layers.{i}.{n}": t for i, l in enumerate(m.layers()) for n, t in l.state_dict().items()}
    for ep, vl in [(0, 2.0), (1, 1.5), (2, 1.7)]:
        md = ck.CheckpointMetadata(epoch=ep, global_step=10 * ep, learning_rate=1e-3, val_loss=vl,
                                   optimizer_state=ck.OptimizerStateMetadata(
                                       "Adam", 1, [ck.ParamGroupState.adam(1e-3, 0.9, 0.999, 1e-8)]))
        ck.save_checkpoint(tmp_path / ck.checkpoint_dir_name(ep), params, md,
                           optimizer_moments={"m": torch.zeros(3), "v": torch.ones(3)})
    d = tmp_path / "checkpoint_epoch_0001"
    assert sorted(os.listdir(d)) == ["checkpoint_meta.json", "model.safetensors", "optimizer_state.safetensors"]
    p2, md2, mom = ck.load_checkpoint(d)
    assert md2.epoch == 1 and md2.optimizer_state.param_groups[0].beta1 == 0.9
    assert torch.equal(p2["layers.0.weight"], params["layers.0.weight"]) and torch.equal(mom["v"], torch.ones(3))
    assert [e for e, _ in ck.list_checkpoints(tmp_path)] == [0, 1, 2]
    assert ck.latest_checkpoint(tmp_path).endswith("0002") and ck.best_checkpoint(tmp_path).endswith("0001")


def test_checkpoint_manager_keeps_last_and_best(tmp_path):
    mgr = ck.CheckpointManager(ck.CheckpointConfig(save_dir=str(tmp_path), keep_last=2))
    for ep, vl in enumerate([1.0, 0.5, 0.9, 0.8, 0.7]):
        mgr.save({"w": torch.full((2,), float(ep))}, ck.CheckpointMetadata(epoch=ep, val_loss=vl))
    left = sorted(os.listdir(tmp_path))
    assert "checkpoint_epoch_0001" in left and "checkpoint_epoch_0004" in left and len(left) == 3
    p, md, _ = mgr.load_best()
    assert md.epoch == 1


def test_safetensors_model_roundtrip(tmp_path):
    m = mnist_mlp(seed=3)
    save_model_safetensors(m, tmp_path / "model.safetensors", architecture="MLP")
    m2 = mnist_mlp(seed=9)
    md = load_model_safetensors(m2, tmp_path / "model.safetensors")
    assert md["architecture"] == "MLP" and md["num_parameters"] == str(784 * 128 + 128 + 128 * 10 + 10)
    x = torch.rand(4, 784)
    assert torch.equal(m(x), m2(x))


def test_mlp_config_cpu(tmp_path):
    from scirs_b200.models.mlp import numpy_reference_losses, synthetic_mnist

    init = mnist_mlp(seed=0)
    r = train_mnist_mlp(steps=100, batch=64, lr=1e-3, seed=0, checkpoint_path=str(tmp_path / "mnist_model.json"))
    L = r["losses"]
    assert abs(L[0] - math.log(10)) < 0.3 and all(math.isfinite(v) for v in L)
    x, y = synthetic_mnist(100 * 64, seed=0)
    ws = [t.detach().double().numpy() for t in
          (init.layers()[0].weight, init.layers()[0].bias, init.layers()[1].weight, init.layers()[1].bias)]
    ref = numpy_reference_losses(*ws, x.double().numpy(), y.numpy(), 100, 64, 1e-3)
    assert max(abs(a - b) for a, b in zip(L, ref)) < 2e-3
    m2 = load_model(tmp_path / "mnist_model.json", dtype=torch.float32)
    x = torch.rand(3, 784)
    r["model"].eval()
    assert torch.allclose(m2(x), r["model"](x))
