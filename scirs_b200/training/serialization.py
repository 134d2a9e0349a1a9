"""Model serialization.

Legacy JSON model file (the `mnist_model.json` layout of
scirs2-neural/src/serialization/mod.rs:100-420):

    {"name": "SciRS2 Sequential Model", "version": "0.1.0",
     "layers": [{"type": "Dense", "input_dim": I, "output_dim": O, "activation": null}, {"type": "Dropout", "p": P}, ...],
     "parameters": [[[W row-major [I, O]], [b [O]]], [], ...]}

written in serde_json's pretty style (2-space indent) with floats formatted
the way serde_json's shortest round-trip formatter does, so a file written
here is byte-identical to one the reference writes for the same values.
The reference writer always emits `"activation": null` and `"p": 0.5`
(it cannot read them back from its layers); `reference_quirks=True`
reproduces that, the default writes the real values. The loader accepts
both. Besides Dense / Dropout, the other layer kinds of the reference's
LayerConfig enum (Conv2D, LayerNorm, BatchNorm, MaxPool2D) are written and
read as well.

SafeTensors files with the reference's metadata keys (architecture,
version, framework_version, num_parameters, dtype + extras) and the
`layers.{i}.{weight,bias}` naming of scirs2-neural/src/serialization/architecture.rs:389-420.
"""
from __future__ import annotations

import json
import math
import os

import torch

from ..nn import conv as _conv
from ..nn import layers as _layers
from ..nn.sequential import Sequential

FRAMEWORK_VERSION = "0.1.0"


# ---------------------------------------------------------------------------- serde-style JSON
def format_float(x: float) -> str:
    """Shortest round-trip float text laid out like serde_json (ryu):
    integers get ".0"; plain decimal when the decimal point falls in
    (-5, 16]; otherwise d.ddde<exp> with no '+' and no zero padding."""
    x = float(x)
    if math.isnan(x) or math.isinf(x):
        return "null"
    if x == 0.0:
        return "-0.0" if math.copysign(1.0, x) < 0 else "0.0"
    sign = "-" if x < 0 else ""
    r = repr(abs(x))  # shortest round-trip digits
    if "e" in r:
        mant, e = r.split("e")
        exp10 = int(e)
    else:
        mant, exp10 = r, 0
    if "." in mant:
        ip, fp = mant.split(".")
    else:
        ip, fp = mant, ""
    digits = (ip + fp).lstrip("0")
    # value = 0.<digits> * 10^kk
    point = len(ip) + exp10  # decimal point position relative to start of ip+fp
    lead_zeros = len(ip + fp) - len((ip + fp).lstrip("0"))
    kk = point - lead_zeros
    digits = digits.rstrip("0") or "0"
    n = len(digits)
    if 0 <= kk - n and kk <= 16:  # integer value
        out = digits + "0" * (kk - n) + ".0"
    elif 0 < kk <= 16:
        out = digits[:kk] + "." + digits[kk:]
    elif -5 < kk <= 0:
        out = "0." + "0" * (-kk) + digits
    else:
        e = kk - 1
        out = digits[0] + ("." + digits[1:] if n > 1 else "") + "e" + str(e)
    return sign + out


def _dump(v, ind: int = 0) -> str:
    pad, pad2 = "  " * ind, "  " * (ind + 1)
    if v is None:
        return "null"
    if isinstance(v, bool):
        return "true" if v else "false"
    if isinstance(v, int):
        return str(v)
    if isinstance(v, float):
        return format_float(v)
    if isinstance(v, str):
        return json.dumps(v, ensure_ascii=False)
    if isinstance(v, (list, tuple)):
        if len(v) == 0:
            return "[]"
        return "[\n" + ",\n".join(pad2 + _dump(x, ind + 1) for x in v) + "\n" + pad + "]"
    if isinstance(v, dict):
        if len(v) == 0:
            return "{}"
        return "{\n" + ",\n".join(pad2 + json.dumps(k) + ": " + _dump(x, ind + 1) for k, x in v.items()) + "\n" + pad + "}"
    raise TypeError(type(v))


def to_serde_pretty(obj) -> str:
    return _dump(obj)


# ---------------------------------------------------------------------------- legacy JSON model
def _flat(t: torch.Tensor) -> list:
    return [float(x) for x in t.detach().double().reshape(-1).tolist()]


def serialize_model(model: Sequential, reference_quirks: bool = False) -> dict:
    layers, params = [], []
    for layer in model.layers():
        if isinstance(layer, _layers.Dense):
            layers.append({"type": "Dense", "input_dim": layer.input_dim(), "output_dim": layer.output_dim(),
                           "activation": None if reference_quirks else layer.activation()})
            params.append([_flat(layer.weight), _flat(layer.bias)])
        elif isinstance(layer, _layers.Dropout):
            layers.append({"type": "Dropout", "p": 0.5 if reference_quirks else float(layer.p)})
            params.append([])
        elif isinstance(layer, _conv.Conv2D):
            layers.append({"type": "Conv2D", "in_channels": layer.in_channels, "out_channels": layer.out_channels,
                           "kernel_size": layer.kernel_size, "stride": layer.stride,
                           "padding_mode": layer.padding_mode if layer.padding_mode != "explicit" else str(layer.padding)})
            params.append([_flat(layer.weight)] + ([_flat(layer.bias)] if layer.bias is not None else []))
        elif isinstance(layer, _layers.LayerNorm):
            layers.append({"type": "LayerNorm", "normalizedshape": layer.weight.numel(), "eps": float(layer.eps)})
            params.append([_flat(layer.weight), _flat(layer.bias)])
        elif isinstance(layer, _layers.BatchNorm):
            layers.append({"type": "BatchNorm", "num_features": layer.weight.numel(), "momentum": float(layer.momentum),
                           "eps": float(layer.eps)})
            params.append([_flat(layer.weight), _flat(layer.bias), _flat(layer.running_mean), _flat(layer.running_var)])
        elif isinstance(layer, _conv.MaxPool2D):
            k, s = layer.kernel_size, layer.stride
            layers.append({"type": "MaxPool2D", "kernel_size": [k, k], "stride": [s, s],
                           "padding": [layer.padding, layer.padding] if layer.padding else None})
            params.append([])
        else:
            raise ValueError(f"layer {type(layer).__name__} has no legacy JSON form; use save_safetensors")
    return {"name": "SciRS2 Sequential Model", "version": "0.1.0", "layers": layers, "parameters": params}


def save_model(model: Sequential, path, reference_quirks: bool = False) -> None:
    with open(path, "w") as f:
        f.write(to_serde_pretty(serialize_model(model, reference_quirks)))


def deserialize_model(obj: dict, dtype=torch.float64, device=None) -> Sequential:
    seq = Sequential()
    params = obj.get("parameters", [])
    for i, cfg in enumerate(obj["layers"]):
        p = params[i] if i < len(params) else []
        kind = cfg["type"]
        kw = dict(dtype=dtype, device=device)
        if kind == "Dense":
            layer = _layers.Dense(cfg["input_dim"], cfg["output_dim"], cfg.get("activation"), seed=42, **kw)
            if len(p) >= 2:
                n_in, n_out = cfg["input_dim"], cfg["output_dim"]
                if len(p[0]) != n_in * n_out:
                    raise ValueError(f"weight vector length {len(p[0])} != {n_in * n_out}")
                layer.set_params([torch.tensor(p[0]).reshape(n_in, n_out), torch.tensor(p[1])])
        elif kind == "Dropout":
            layer = _layers.Dropout(cfg["p"])
        elif kind == "Conv2D":
            pm = cfg.get("padding_mode", "valid")
            pad = int(pm) if str(pm).isdigit() else pm
            layer = _conv.Conv2D(cfg["in_channels"], cfg["out_channels"], cfg["kernel_size"], cfg["stride"], pad,
                                 bias=len(p) != 1, **kw)
            if p:
                layer.set_params([torch.tensor(x) for x in p])
        elif kind == "LayerNorm":
            layer = _layers.LayerNorm(cfg["normalizedshape"], cfg["eps"], **kw)
            if p:
                layer.set_params([torch.tensor(x) for x in p])
        elif kind == "BatchNorm":
            layer = _layers.BatchNorm(cfg["num_features"], cfg["momentum"], cfg["eps"], **kw)
            if p:
                layer.set_params([torch.tensor(p[0]), torch.tensor(p[1])])
                if len(p) >= 4:
                    layer.running_mean.copy_(torch.tensor(p[2]))
                    layer.running_var.copy_(torch.tensor(p[3]))
        elif kind == "MaxPool2D":
            ks, st, pd = cfg["kernel_size"], cfg["stride"], cfg.get("padding")
            layer = _conv.MaxPool2D(ks[0], st[0], (pd or [0, 0])[0])
        else:
            raise ValueError(f"unknown layer type {kind}")
        seq.add(layer)
    return seq


def load_model(path, dtype=torch.float64, device=None) -> Sequential:
    with open(path) as f:
        return deserialize_model(json.load(f), dtype=dtype, device=device)


# ---------------------------------------------------------------------------- safetensors
_DT = {torch.float64: "f64", torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}


def model_metadata(architecture: str, dtype: str, num_parameters: int, **extra) -> dict:
    md = {"architecture": architecture, "version": "0.1.0", "framework_version": FRAMEWORK_VERSION,
          "num_parameters": str(num_parameters), "dtype": dtype}
    md.update({k: str(v) for k, v in extra.items()})
    return md


def named_parameters(model) -> dict[str, torch.Tensor]:
    """`layers.{i}.{name}` for Sequential models (reference naming), the
    model's own state_dict keys otherwise."""
    if isinstance(model, Sequential):
        out = {}
        for i, layer in enumerate(model.layers()):
            for n, t in layer.state_dict().items():
                out[f"layers.{i}.{n}"] = t
        return out
    return dict(model.state_dict())


def save_safetensors(tensors: dict, path, metadata: dict | None = None) -> None:
    from safetensors.torch import save_file

    save_file({k: v.detach().contiguous().cpu() for k, v in tensors.items()}, str(path), metadata=metadata or {})


def load_safetensors(path) -> tuple[dict, dict]:
    from safetensors import safe_open

    out = {}
    with safe_open(str(path), framework="pt") as f:
        md = f.metadata() or {}
        for k in f.keys():
            out[k] = f.get_tensor(k)
    return out, md


def save_model_safetensors(model, path, architecture: str = "Sequential") -> None:
    t = named_parameters(model)
    dt = _DT.get(next(iter(t.values())).dtype, "f32") if t else "f32"
    save_safetensors(t, path, model_metadata(architecture, dt, sum(v.numel() for v in t.values())))


def load_model_safetensors(model, path, strict: bool = True) -> dict:
    t, md = load_safetensors(path)
    if isinstance(model, Sequential):
        for i, layer in enumerate(model.layers()):
            sd = {n[len(f"layers.{i}.") :]: v for n, v in t.items() if n.startswith(f"layers.{i}.")}
            if sd:
                layer.load_state_dict({k: v.to(layer.state_dict()[k].dtype) for k, v in sd.items()}, strict=strict)
    else:
        model.load_state_dict(t, strict=strict)
    return md
