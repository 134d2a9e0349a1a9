"""Architecture-aware model files: configuration round trips in the reference's
field names, directory / safetensors / JSON layouts, architecture detection and
by-name parameter loading."""
import json

import pytest
import torch

from scirs_b200.export import model_io as M
from scirs_b200.models import architectures as A
from scirs_b200.models.gpt import GPTConfig


@pytest.mark.parametrize("cfg", [
    A.ResNetConfig.resnet50(3, 10), A.BertConfig(), A.MambaConfig(vocab_size=100),
    A.EfficientNetConfig(width=1.1, depth=1.2), A.MobileNetConfig(version=1), A.VGGConfig(),
    GPTConfig(num_hidden_layers=2),
])
def test_config_round_trip(cfg):
    env = M.envelope(cfg)
    assert env["format_version"] == "1.0"
    back = M.config_from_json(env["architecture"], json.loads(json.dumps(env["config"])))
    assert back == cfg


def test_reference_field_names():
    r = M.config_to_json(A.ResNetConfig.resnet18(3, 7))
    assert r["block"] == "Basic" and r["layers"][1] == {"blocks": 2, "channels": 128, "stride": 2}
    e = M.config_to_json(A.EfficientNetConfig(width=1.4, depth=1.8))
    assert e["width_coefficient"] == 1.4 and e["depth_coefficient"] == 1.8 and "width" not in e
    assert M.config_to_json(A.MobileNetConfig(version=2))["version"] == "V2"
    m = M.config_to_json(A.MambaConfig())
    assert {"dt_rank", "bias", "dt_min", "dt_max"} <= set(m)
    # a configuration as the reference writes it
    ref_resnet = {"block": "Bottleneck", "layers": [{"blocks": 3, "channels": 64, "stride": 1},
                                                    {"blocks": 4, "channels": 128, "stride": 2},
                                                    {"blocks": 6, "channels": 256, "stride": 2},
                                                    {"blocks": 3, "channels": 512, "stride": 2}],
                  "input_channels": 3, "num_classes": 1000, "dropout_rate": 0.0}
    assert M.config_from_json("ResNet", ref_resnet) == A.ResNetConfig.resnet50()
    with pytest.raises(M.SerializationError):
        M.config_from_json("ResNet", dict(ref_resnet, block="Weird"))
    with pytest.raises(M.SerializationError):
        M.config_from_json("MobileNet", {"version": "V3Small", "width_multiplier": 1.0, "input_channels": 3,
                                         "num_classes": 10, "dropout_rate": 0.0})
    with pytest.raises(M.SerializationError):
        M.config_from_json("Nope", {})


def _same(a, b):
    sa, sb = a.state_dict(), b.state_dict()
    return sa.keys() == sb.keys() and all(torch.equal(sa[k], sb[k]) for k in sa)


def test_directory_layout_round_trip(tmp_path):
    torch.manual_seed(0)
    cfg = A.ResNetConfig.resnet18(3, 10)
    model = cfg.build()
    M.save_model_dir(model, cfg, tmp_path / "m")
    assert (tmp_path / "m" / "config.json").exists() and (tmp_path / "m" / "weights.safetensors").exists()
    assert M.detect_architecture(tmp_path / "m") == "ResNet"
    assert M.detect_architecture(tmp_path / "m" / "weights.safetensors") == "ResNet"
    loaded, rep = M.load_model_dir(tmp_path / "m")
    assert _same(model, loaded) and rep["skipped"] == [] and rep["missing"] == []


@pytest.mark.parametrize("fmt", ["safetensors", "json"])
def test_single_file_round_trip_and_detection(tmp_path, fmt):
    torch.manual_seed(1)
    cfg = GPTConfig(vocab_size=64, max_position_embeddings=16, hidden_size=32, num_hidden_layers=1,
                    num_attention_heads=2, intermediate_size=64)
    model = M._build(cfg)
    p = tmp_path / f"gpt.{fmt}"
    M.save_model(model, cfg, p, fmt)
    assert M.detect_architecture(p) == "GPT"
    loaded, rep = M.load_model(p)
    assert _same(model, loaded) and not rep["missing"]


def test_load_ignores_unknown_and_reports_missing(tmp_path):
    cfg = A.BertConfig(vocab_size=50, hidden_size=32, num_hidden_layers=1, num_attention_heads=2,
                       intermediate_size=64, max_position_embeddings=16)
    model = cfg.build()
    p = tmp_path / "bert.json"
    M.save_model(model, cfg, p, "json")
    doc = json.loads(p.read_text())
    dropped = doc["parameters"].pop(0)["name"]
    doc["parameters"].append({"name": "extra.weight", "shape": [2], "data": [1.0, 2.0]})
    p.write_text(json.dumps(doc))
    _, rep = M.load_model(p)
    assert rep["skipped"] == ["extra.weight"] and rep["missing"] == [dropped]


def test_detection_rejects_unknown_bytes():
    with pytest.raises(M.SerializationError):
        M.detect_architecture_from_bytes(b"\x00\x01garbage")
    assert M.detect_architecture_from_bytes(json.dumps({"architecture": {"architecture": "BERT"}}).encode()) == "BERT"
