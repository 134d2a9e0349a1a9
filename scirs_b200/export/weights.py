"""Named weight stores: a name -> float64 tensor map with string metadata,
renaming between PyTorch and SciRS2 parameter names, shape validation and
three on-disk formats.

  Json         {"metadata": {...}, "tensors": {name: {"shape": [...], "data": [...]}}}
               (the reference's JSON layout, so files move both ways)
  SafeTensors  a real safetensors file (float64 tensors, metadata in the header);
               the reference writes its own binary encoding under this name,
               which only it can read, so this one is the interoperable choice
  NpzLike      numpy .npz archive plus a `<path>.idx.json` sidecar of shapes

Name mapping: `.weight` <-> `.kernel`, `.running_mean` <-> `.mean`,
`.running_var` <-> `.var`; `num_batches_tracked` maps to "" (no
counterpart; filter it out).

Reference parity: scirs2-neural/src/export/weights.rs:94-400.
"""
from __future__ import annotations

import json
from enum import Enum

import numpy as np
import torch


class WeightFormat(Enum):
    SAFETENSORS = "safetensors"
    NPZ_LIKE = "npz"
    JSON = "json"


class WeightStore:
    def __init__(self):
        self.weights: dict[str, torch.Tensor] = {}
        self.metadata: dict[str, str] = {}

    def insert(self, name: str, tensor):
        self.weights[str(name)] = torch.as_tensor(tensor).detach().to(torch.float64).cpu()

    def get(self, name: str):
        return self.weights.get(name)

    def remove(self, name: str):
        return self.weights.pop(name, None)

    def names(self) -> list:
        return sorted(self.weights)

    def __len__(self):
        return len(self.weights)

    def is_empty(self) -> bool:
        return not self.weights

    def set_metadata(self, key: str, value: str):
        self.metadata[str(key)] = str(value)

    def get_metadata(self, key: str):
        return self.metadata.get(key)

    def upcast_f32(self) -> "WeightStore":
        """Every value rounded through float32 (a store loaded from f32 weights compares exactly)."""
        s = WeightStore()
        s.weights = {k: v.to(torch.float32).to(torch.float64) for k, v in self.weights.items()}
        s.metadata = dict(self.metadata)
        return s

    def rename_with(self, fn) -> "WeightStore":
        s = WeightStore()
        s.weights = {fn(k): v for k, v in self.weights.items()}
        s.metadata = dict(self.metadata)
        return s

    def validate_shapes(self, expected: dict):
        for name, shape in expected.items():
            t = self.weights.get(name)
            if t is None:
                raise KeyError(f"Weight '{name}' not found in store (available: {self.names()})")
            if list(t.shape) != list(shape):
                raise ValueError(f"Weight '{name}': expected shape {list(shape)}, got {list(t.shape)}")

    @staticmethod
    def from_module(module: torch.nn.Module, rename=None) -> "WeightStore":
        s = WeightStore()
        for k, v in module.state_dict().items():
            name = rename(k) if rename else k
            if name:
                s.insert(name, v.float() if v.is_floating_point() else v)
        return s

    def save(self, path: str, fmt: WeightFormat = WeightFormat.JSON):
        if fmt is WeightFormat.JSON:
            payload = {"metadata": self.metadata,
                       "tensors": {k: {"shape": list(v.shape), "data": v.reshape(-1).tolist()}
                                   for k, v in self.weights.items()}}
            with open(path, "w") as f:
                json.dump(payload, f, indent=2)
        elif fmt is WeightFormat.SAFETENSORS:
            from ..training.serialization import save_safetensors

            save_safetensors({k: v.contiguous() for k, v in self.weights.items()}, path, self.metadata)
        elif fmt is WeightFormat.NPZ_LIKE:
            with open(path, "wb") as f:
                np.savez(f, **{k: v.numpy() for k, v in self.weights.items()},
                         __metadata__=np.array(json.dumps(self.metadata)))
            with open(f"{path}.idx.json", "w") as f:
                json.dump({k: list(v.shape) for k, v in self.weights.items()}, f, indent=2)
        else:
            raise ValueError(f"unknown format {fmt}")

    @staticmethod
    def load(path: str, fmt: WeightFormat = WeightFormat.JSON) -> "WeightStore":
        s = WeightStore()
        if fmt is WeightFormat.JSON:
            with open(path) as f:
                payload = json.load(f)
            s.metadata = {str(k): str(v) for k, v in payload.get("metadata", {}).items()}
            for name, e in payload["tensors"].items():
                n = 1
                for d in e["shape"]:
                    n *= int(d)
                if len(e["data"]) != n:
                    raise ValueError(f"tensor {name}: shape {e['shape']} expects {n} elements, "
                                     f"data has {len(e['data'])}")
                s.weights[name] = torch.tensor(e["data"], dtype=torch.float64).reshape(e["shape"])
        elif fmt is WeightFormat.SAFETENSORS:
            from ..training.serialization import load_safetensors

            tensors, meta = load_safetensors(path)
            s.weights = {k: v.to(torch.float64) for k, v in tensors.items()}
            s.metadata = {str(k): str(v) for k, v in (meta or {}).items()}
        elif fmt is WeightFormat.NPZ_LIKE:
            with np.load(path, allow_pickle=False) as z:
                for k in z.files:
                    if k == "__metadata__":
                        s.metadata = json.loads(str(z[k]))
                    else:
                        s.weights[k] = torch.from_numpy(np.array(z[k], dtype=np.float64))
        else:
            raise ValueError(f"unknown format {fmt}")
        return s


def pytorch_to_scirs2_names(name: str) -> str:
    if name == "num_batches_tracked" or name.endswith(".num_batches_tracked"):
        return ""
    if name.endswith(".weight"):
        name = name[: -len(".weight")] + ".kernel"
    return name.replace(".running_mean", ".mean").replace(".running_var", ".var")


def scirs2_to_pytorch_names(name: str) -> str:
    if name.endswith(".kernel"):
        name = name[: -len(".kernel")] + ".weight"
    if name.endswith(".mean"):
        name = name[: -len(".mean")] + ".running_mean"
    if name.endswith(".var"):
        name = name[: -len(".var")] + ".running_var"
    return name
