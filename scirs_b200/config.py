"""Run configuration: parallel layout, model / data / optimizer settings,
config files and `SCIRS_*` environment overrides.

`RunConfig` bundles everything one training run needs:

    model      "mlp" | "gpt2" | "vit" | "gpt1.3b" | "attention_sweep" and the
               model's own dataclass (GPTConfig, ViTConfig, DecoderConfig)
               overrides as a dict
    data       global batch, sequence length, seed
    optim      AdamW / Adam / SGD hyperparameters, global-norm clip
    parallel   ParallelConfig{dp, tp, pp, cp, zero, dp_mode, tp_mode}
    runtime    cuda_graph, steps, warmup

Files are YAML or JSON (`load_config(path)`); `configs/` next to this
package holds one file per benchmark configuration. Environment variables
override file values (`apply_env`):

    SCIRS_KERNELS      custom | torch     layer-API ops on the framework's kernels
                                          (default) or on PyTorch
    SCIRS_COMM         fused | nccl       data-parallel / ZeRO / TP collectives
    SCIRS_WAIT_TIMEOUT_S  seconds         bound of every cross-GPU wait
    SCIRS_PRECISION    bf16 | fp32        compute dtype of the layer API on CUDA
    SCIRS_THREADS      n                  host threads (torch.set_num_threads)
    SCIRS_ATTN_FWD / SCIRS_ATTN_BWD       attention kernel variant
    SCIRS_ATTN_FWD_PERSIST  0 | 1         attention forward on one CTA per SM
    SCIRS_ATTN_BWD_TRACE    1             phase trace of the pipelined attention
                                          backward (profiling; kernels.attn_bwd_trace())
    SCIRS_<SECTION>_<FIELD>               any field, e.g. SCIRS_PARALLEL_DP=8,
                                          SCIRS_DATA_GLOBAL_BATCH=64

Reference parity: scirs2-core/src/config.rs:30-312 (Config with the SCIRS_
prefix), config/unified.rs:29-32,240-246 (SCIRS2_THREADS / PRECISION /
MEMORY_LIMIT / POOL_SIZE), config/production.rs:284-305,
scirs2-neural/src/models/trainer.rs:33-60 (TrainingConfig),
scirs2-autograd/src/distributed/mod.rs (ParallelStrategy
{DataParallel, ModelParallel, PipelineParallel, Hybrid}).
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field

HERE = os.path.dirname(os.path.abspath(__file__))
CONFIG_DIR = os.path.join(HERE, "configs")


@dataclass
class ParallelConfig:
    """How a run is laid out over `dp * tp * pp * cp` GPUs of one node."""

    dp: int = 1
    tp: int = 1
    pp: int = 1
    cp: int = 1  # context (sequence) parallel ranks (ring attention)
    zero: int = 1  # 0: replicated optimizer, 1: sharded optimizer state (ZeRO-1)
    dp_mode: str = "fused"  # fused | push | nvls | nccl
    tp_mode: str = "fused"  # fused | nccl
    pp_schedule: str = "1f1b"  # 1f1b | gpipe
    micro_batches: int = 1

    @property
    def world_size(self) -> int:
        return self.dp * self.tp * self.pp * self.cp

    def validate(self, world: int | None = None):
        for k in ("dp", "tp", "pp", "cp", "micro_batches"):
            if getattr(self, k) < 1:
                raise ValueError(f"parallel.{k} must be >= 1")
        if self.dp_mode not in ("fused", "push", "nvls", "nccl"):
            raise ValueError(f"unknown dp_mode {self.dp_mode}")
        if self.tp_mode not in ("fused", "nccl"):
            raise ValueError(f"unknown tp_mode {self.tp_mode}")
        if self.pp_schedule not in ("1f1b", "gpipe"):
            raise ValueError(f"unknown pp_schedule {self.pp_schedule}")
        if world is not None and world != self.world_size:
            raise ValueError(f"dp*tp*pp*cp = {self.world_size} but the job has {world} ranks")
        if self.pp > 1 and self.micro_batches < self.pp:
            raise ValueError("pipeline parallelism needs at least pp micro-batches")
        return self

    def describe(self) -> str:
        parts = [f"{k}{getattr(self, k)}" for k in ("dp", "tp", "pp", "cp") if getattr(self, k) > 1]
        return "+".join(parts) or "dp1"


@dataclass
class DataConfig:
    global_batch: int = 64
    seq_len: int = 1024
    seed: int = 1234
    synthetic: bool = True


@dataclass
class OptimConfig:
    name: str = "adamw"
    lr: float = 6e-4
    betas: tuple = (0.9, 0.95)
    eps: float = 1e-8
    weight_decay: float = 0.1
    max_grad_norm: float = 1.0


@dataclass
class RuntimeConfig:
    cuda_graph: bool = True
    steps: int = 10
    warmup: int = 3
    kernels: str = "custom"  # custom | torch
    comm: str = "fused"  # fused | nccl
    wait_timeout_s: float = 5.0
    precision: str = "bf16"
    threads: int = 0


@dataclass
class RunConfig:
    model: str = "gpt2"
    model_overrides: dict = field(default_factory=dict)
    data: DataConfig = field(default_factory=DataConfig)
    optim: OptimConfig = field(default_factory=OptimConfig)
    parallel: ParallelConfig = field(default_factory=ParallelConfig)
    runtime: RuntimeConfig = field(default_factory=RuntimeConfig)
    name: str = ""

    # -------------------------------------------------------------- models
    def model_config(self):
        """The model's own config dataclass with the overrides applied."""
        if self.model == "gpt2":
            from .models.gpt import GPTConfig

            c = GPTConfig.gpt2_small()
        elif self.model == "vit":
            from .models.vit import ViTConfig

            c = ViTConfig.vit_base()
        elif self.model == "gpt1.3b":
            from .models.tp_gpt import DecoderConfig

            c = DecoderConfig.decoder_1_3b()
        else:
            return dict(self.model_overrides)
        for k, v in self.model_overrides.items():
            if not hasattr(c, k):
                raise KeyError(f"{type(c).__name__} has no field {k!r}")
            setattr(c, k, v)
        return c

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)


_SECTIONS = {"data": DataConfig, "optim": OptimConfig, "parallel": ParallelConfig, "runtime": RuntimeConfig}


def from_dict(d: dict) -> RunConfig:
    d = dict(d)
    kw = {}
    for sec, cls in _SECTIONS.items():
        vals = dict(d.pop(sec, {}) or {})
        names = {f.name for f in dataclasses.fields(cls)}
        bad = set(vals) - names
        if bad:
            raise KeyError(f"unknown {sec} fields: {sorted(bad)}")
        if "betas" in vals:
            vals["betas"] = tuple(vals["betas"])
        kw[sec] = cls(**vals)
    overrides = d.pop("model_overrides", d.pop("model_config", {})) or {}
    cfg = RunConfig(model=d.pop("model", "gpt2"), model_overrides=dict(overrides), name=d.pop("name", ""), **kw)
    if d:
        raise KeyError(f"unknown top-level config keys: {sorted(d)}")
    return cfg


def _coerce(old, text: str):
    if isinstance(old, bool):
        return text.lower() in ("1", "true", "yes", "on")
    if isinstance(old, int):
        return int(text)
    if isinstance(old, float):
        return float(text)
    if isinstance(old, tuple):
        return tuple(float(x) for x in text.split(","))
    return text


def apply_env(cfg: RunConfig, env=None) -> RunConfig:
    """Apply SCIRS_* overrides (see the module docstring) in place."""
    env = os.environ if env is None else env
    short = {"SCIRS_KERNELS": ("runtime", "kernels"), "SCIRS_COMM": ("runtime", "comm"),
             "SCIRS_WAIT_TIMEOUT_S": ("runtime", "wait_timeout_s"), "SCIRS_PRECISION": ("runtime", "precision"),
             "SCIRS_THREADS": ("runtime", "threads")}
    for key, text in env.items():
        if not key.startswith("SCIRS_"):
            continue
        if key in short:
            sec, name = short[key]
        else:
            rest = key[len("SCIRS_"):].lower()
            sec = next((s for s in _SECTIONS if rest.startswith(s + "_")), None)
            if sec is None:
                continue
            name = rest[len(sec) + 1:]
        obj = getattr(cfg, sec)
        if not hasattr(obj, name):
            continue
        setattr(obj, name, _coerce(getattr(obj, name), text))
    if cfg.runtime.comm == "nccl":
        cfg.parallel.dp_mode = cfg.parallel.tp_mode = "nccl"
    return cfg


def load_config(path: str, env=None, apply_environment: bool = True) -> RunConfig:
    """Read a YAML or JSON run configuration (a bare name is looked up in the
    package's configs/ directory)."""
    if not os.path.exists(path):
        for ext in ("", ".yaml", ".yml", ".json"):
            cand = os.path.join(CONFIG_DIR, path + ext)
            if os.path.exists(cand):
                path = cand
                break
    with open(path) as f:
        text = f.read()
    if path.endswith(".json"):
        d = json.loads(text)
    else:
        import yaml

        d = yaml.safe_load(text)
    cfg = from_dict(d)
    if not cfg.name:
        cfg.name = os.path.splitext(os.path.basename(path))[0]
    return apply_env(cfg, env) if apply_environment else cfg


def list_configs() -> list[str]:
    if not os.path.isdir(CONFIG_DIR):
        return []
    return sorted(os.path.splitext(f)[0] for f in os.listdir(CONFIG_DIR) if f.endswith((".yaml", ".yml", ".json")))


def runtime_settings(env=None) -> RuntimeConfig:
    """The runtime section from the environment alone (what the library's
    ops consult when no RunConfig is in play)."""
    return apply_env(RunConfig(), env).runtime
