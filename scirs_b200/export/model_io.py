"""Architecture-aware model files: configuration + named weights, in the three
layouts of the reference's serializer.

* directory: `config.json` (the architecture envelope) + `weights.safetensors`
* single safetensors file: the weights, with metadata `architecture` (the
  name) and `architecture_config` (the envelope as a JSON string)
* single JSON file: `{"architecture": <envelope>, "parameters":
  [{"name", "shape", "data"}, ...]}`

The envelope is `{"architecture": name, "format_version": "1.0", "config":
{...}}`. The per-architecture `config` objects use the reference's field
names (ResNet as `block` "Basic"/"Bottleneck" + `layers` of {blocks,
channels, stride}; EfficientNet `width_coefficient` / `depth_coefficient`;
MobileNet `version` "V1"/"V2"; Mamba with `dt_rank` / `bias` / `dt_min` /
`dt_max`), so files written by either side describe the same model.
Architectures the reference does not serialise (VGG, MLP-Mixer, ConvNeXt,
U-Net, autoencoders, sequence-to-sequence, ViT) use their configuration
fields as they are. Loading builds the model from the configuration, then
restores every parameter whose name exists in the model (other names are
ignored, so files stay loadable across added or removed layers) and reports
the names it skipped and the model parameters it did not find.

Reference parity: scirs2-neural/src/serialization/architecture.rs:45-1610
(ArchitectureConfig, Serializable*Config, JSON / SafeTensors save and load,
detect_architecture / detect_architecture_from_bytes) and
model_serializer.rs:70-330 (directory layout, load by name ignoring unknown
names).
"""
from __future__ import annotations

import dataclasses
import json
import os
import struct
from pathlib import Path

import torch

from ..models import architectures as A
from ..training.serialization import load_safetensors, save_safetensors

FORMAT_VERSION = "1.0"


def _gpt_config():
    from ..models.gpt import GPTConfig

    return GPTConfig


def _vit_config():
    from ..models.vit import ViTConfig

    return ViTConfig


# name -> config class (callables for the engines imported lazily)
_ARCH = {
    "ResNet": lambda: A.ResNetConfig, "BERT": lambda: A.BertConfig, "GPT": _gpt_config,
    "Mamba": lambda: A.MambaConfig, "EfficientNet": lambda: A.EfficientNetConfig,
    "MobileNet": lambda: A.MobileNetConfig, "VGG": lambda: A.VGGConfig, "MLPMixer": lambda: A.MLPMixerConfig,
    "ConvNeXt": lambda: A.ConvNeXtConfig, "UNet": lambda: A.UNetConfig, "Autoencoder": lambda: A.AutoencoderConfig,
    "VAE": lambda: A.VAEConfig, "Seq2Seq": lambda: A.Seq2SeqConfig, "ViT": _vit_config,
}

_GPT_FIELDS = ("vocab_size", "max_position_embeddings", "hidden_size", "num_hidden_layers", "num_attention_heads",
               "intermediate_size", "hidden_act", "hidden_dropout_prob", "attention_probs_dropout_prob",
               "layer_norm_eps", "initializer_range")


class SerializationError(ValueError):
    pass


def architecture_name(cfg) -> str:
    for name, get in _ARCH.items():
        if type(cfg) is get():
            return name
    raise SerializationError(f"no serialisable architecture for {type(cfg).__name__}")


def _plain(v):
    if isinstance(v, tuple):
        return [_plain(x) for x in v]
    if isinstance(v, list):
        return [_plain(x) for x in v]
    if isinstance(v, dict):
        return {k: _plain(x) for k, x in v.items()}
    return v


def config_to_json(cfg) -> dict:
    """The architecture-specific `config` object (reference field names where it has them)."""
    arch = architecture_name(cfg)
    d = {f.name: _plain(getattr(cfg, f.name)) for f in dataclasses.fields(cfg)}
    if arch == "ResNet":
        return {"block": "Bottleneck" if cfg.bottleneck else "Basic",
                "layers": [{"blocks": n, "channels": 64 * 2 ** i, "stride": 1 if i == 0 else 2}
                           for i, n in enumerate(cfg.layers)],
                "input_channels": cfg.input_channels, "num_classes": cfg.num_classes,
                "dropout_rate": cfg.dropout_rate}
    if arch == "EfficientNet":
        d["width_coefficient"], d["depth_coefficient"] = d.pop("width"), d.pop("depth")
    elif arch == "MobileNet":
        d["version"] = f"V{cfg.version}"
        d.setdefault("resolution_multiplier", 1.0)
    elif arch == "Mamba":
        d.update({"dt_rank": None, "bias": False, "dt_min": 0.001, "dt_max": 0.1})
    elif arch == "GPT":
        d = {k: d[k] for k in _GPT_FIELDS if k in d} | {k: v for k, v in d.items() if k not in _GPT_FIELDS}
    return d


def config_from_json(arch: str, d: dict):
    if arch not in _ARCH:
        raise SerializationError(f"unknown architecture {arch!r}")
    cls = _ARCH[arch]()
    d = dict(d)
    if arch == "ResNet":
        if d.get("block") not in ("Basic", "Bottleneck"):
            raise SerializationError(f"unknown ResNet block type {d.get('block')!r}")
        for i, l in enumerate(d["layers"]):
            if l["channels"] != 64 * 2 ** i or l["stride"] != (1 if i == 0 else 2):
                raise SerializationError("ResNet stages must have the standard channels (64 * 2^i) and strides")
        d = {"layers": [l["blocks"] for l in d["layers"]], "bottleneck": d["block"] == "Bottleneck",
             "input_channels": d["input_channels"], "num_classes": d["num_classes"],
             "dropout_rate": d.get("dropout_rate", 0.0)}
    elif arch == "EfficientNet":
        d["width"], d["depth"] = d.pop("width_coefficient"), d.pop("depth_coefficient")
    elif arch == "MobileNet":
        v = str(d["version"]).upper().lstrip("V")
        if v not in ("1", "2"):
            raise SerializationError(f"MobileNet version {d['version']!r} is not built by the zoo")
        d["version"] = int(v)
    names = {f.name: f for f in dataclasses.fields(cls)}
    kw = {}
    for k, v in d.items():
        if k in names:
            default = names[k].default
            kw[k] = tuple(v) if isinstance(default, tuple) and isinstance(v, list) else v
    return cls(**kw)


def envelope(cfg) -> dict:
    return {"architecture": architecture_name(cfg), "format_version": FORMAT_VERSION, "config": config_to_json(cfg)}


def _build(cfg):
    arch = architecture_name(cfg)
    if arch == "GPT":
        from ..models.torch_gpt import TorchGPT

        return TorchGPT(cfg)
    if arch == "ViT":
        from ..models.torch_vit import TorchViT

        return TorchViT(cfg)
    return cfg.build()


def _load_params(model, params: dict) -> dict:
    sd = model.state_dict()
    loaded, skipped = [], []
    with torch.no_grad():
        for name, t in params.items():
            if name in sd and tuple(sd[name].shape) == tuple(t.shape):
                sd[name].copy_(t.to(sd[name].dtype))
                loaded.append(name)
            else:
                skipped.append(name)
    return {"loaded": loaded, "skipped": skipped, "missing": [n for n in sd if n not in params]}


# ---------------------------------------------------------------------------- directory layout


def save_model_dir(model, cfg, directory) -> None:
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    (d / "config.json").write_text(json.dumps(envelope(cfg), indent=2))
    sd = model.state_dict()
    save_safetensors(sd, d / "weights.safetensors",
                     {"architecture": architecture_name(cfg), "format_version": FORMAT_VERSION,
                      "num_parameters": str(sum(v.numel() for v in sd.values()))})


def load_model_dir(directory, model=None):
    """(model, report): builds the model from config.json unless one is given."""
    d = Path(directory)
    env = json.loads((d / "config.json").read_text())
    cfg = config_from_json(env["architecture"], env["config"])
    model = model if model is not None else _build(cfg)
    params, _ = load_safetensors(d / "weights.safetensors")
    return model, _load_params(model, params)


# ---------------------------------------------------------------------------- single files


def save_model(model, cfg, path, fmt: str = "safetensors") -> None:
    env = envelope(cfg)
    sd = model.state_dict()
    if fmt == "safetensors":
        save_safetensors(sd, path, {"architecture": env["architecture"], "architecture_config": json.dumps(env),
                                    "format_version": FORMAT_VERSION})
    elif fmt == "json":
        doc = {"architecture": env,
               "parameters": [{"name": k, "shape": list(v.shape), "data": v.detach().float().reshape(-1).tolist()}
                              for k, v in sd.items()]}
        Path(path).write_text(json.dumps(doc))
    else:
        raise SerializationError(f"unknown format {fmt!r}")


def load_model(path, model=None, fmt: str | None = None):
    """(model, report) from a single safetensors or JSON file (format from the content if not given)."""
    raw = Path(path).read_bytes()
    fmt = fmt or ("json" if raw.lstrip()[:1] == b"{" else "safetensors")
    if fmt == "safetensors":
        params, md = load_safetensors(path)
        if "architecture_config" not in md:
            raise SerializationError("missing architecture_config in the safetensors metadata")
        env = json.loads(md["architecture_config"])
    else:
        doc = json.loads(raw)
        if "architecture" not in doc:
            raise SerializationError("missing 'architecture' key in the JSON model file")
        env = doc["architecture"]
        params = {p["name"]: torch.tensor(p["data"], dtype=torch.float32).reshape(p["shape"])
                  for p in doc.get("parameters", [])}
    cfg = config_from_json(env["architecture"], env["config"])
    model = model if model is not None else _build(cfg)
    return model, _load_params(model, params)


def detect_architecture_from_bytes(data: bytes) -> str:
    """The architecture name recorded in a safetensors header or a JSON model file."""
    if len(data) >= 8:
        (n,) = struct.unpack("<Q", data[:8])
        if 0 < n <= len(data) - 8:
            try:
                header = json.loads(data[8:8 + n])
                md = header.get("__metadata__", {})
                if "architecture" in md:
                    return md["architecture"]
            except (ValueError, UnicodeDecodeError):
                pass
    try:
        doc = json.loads(data)
    except (ValueError, UnicodeDecodeError):
        doc = None
    if isinstance(doc, dict):
        arch = doc.get("architecture")
        if isinstance(arch, dict) and "architecture" in arch:
            return arch["architecture"]
        if isinstance(arch, str):
            return arch
    raise SerializationError("cannot detect the architecture: unrecognised format")


def detect_architecture(path) -> str:
    p = Path(path)
    if p.is_dir():
        return json.loads((p / "config.json").read_text())["architecture"]
    with open(os.fspath(p), "rb") as f:
        return detect_architecture_from_bytes(f.read())
