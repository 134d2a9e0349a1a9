"""Step tracing: NVTX ranges, CUDA-event phase timers, roofline figures and
per-step JSONL metrics.

* `nvtx(name)` marks a host range that shows up in Nsight timelines
  (torch.cuda.nvtx; a no-op unless enabled with `enable_nvtx` or
  SCIRS_NVTX=1, and on CPU).
* `PhaseTimer` records a CUDA event at every phase boundary on the current
  stream (`with timer.phase("backward"): ...`) and, at `collect()`, turns
  them into device milliseconds per phase with one synchronisation. Phases
  of a step replayed from a CUDA graph are not separated; time eager steps
  (enable_cuda_graph(False)) when a breakdown is wanted.
* `roofline(...)` relates a measured time to the measured peaks (bf16 GEMM
  rate and copy bandwidth from MEASURED_PEAKS.json when present, else an
  earlier B200 measurement: 6.65 TB/s, 1.59 PFLOP/s) and to NVLink for
  collectives.
* `StepLogger` appends one JSON line per step: loss, device step time
  (maximum over ranks), tokens/s, gradient norm, bytes the step's
  collectives moved per rank, model-FLOP utilisation and the phase times.

Reference parity: scirs2-core/src/profiling/timer.rs:7-112 and
profiler.rs:12-290 (hierarchical host timers), scirs2-neural/src/training/
profiler.rs:45-972 (per-layer timing, bottleneck detection, FLOP and memory
estimates), scirs2-autograd/src/tracing.rs:17-43 (ExecutionTracer),
scirs2-neural/src/callbacks (metric logging). Here the timers are device
events, not host clocks.
"""
from __future__ import annotations

import contextlib
import json
import os
import time

import torch

_NVTX = os.environ.get("SCIRS_NVTX", "0") == "1"


def enable_nvtx(on: bool = True):
    global _NVTX
    _NVTX = bool(on)


@contextlib.contextmanager
def nvtx(name: str):
    if _NVTX and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


class PhaseTimer:
    """Device time per named phase of a step (CUDA events on the current
    stream; host wall clock on the CPU)."""

    def __init__(self, enabled: bool = True):
        self.enabled = enabled
        self._marks: list[tuple[str, object, object]] = []
        self.totals: dict[str, float] = {}
        self.counts: dict[str, int] = {}

    @contextlib.contextmanager
    def phase(self, name: str):
        if not self.enabled:
            yield
            return
        with nvtx(name):
            if torch.cuda.is_available() and torch.cuda.is_initialized():
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                try:
                    yield
                finally:
                    b.record()
                self._marks.append((name, a, b))
            else:
                t0 = time.perf_counter()
                try:
                    yield
                finally:
                    self._marks.append((name, t0, time.perf_counter()))

    def collect(self) -> dict[str, float]:
        """Milliseconds per phase since the last collect (sums repeated phases)."""
        out: dict[str, float] = {}
        if self._marks and isinstance(self._marks[0][1], torch.cuda.Event):
            torch.cuda.synchronize()
        for name, a, b in self._marks:
            ms = a.elapsed_time(b) if isinstance(a, torch.cuda.Event) else (b - a) * 1e3
            out[name] = out.get(name, 0.0) + ms
            self.totals[name] = self.totals.get(name, 0.0) + ms
            self.counts[name] = self.counts.get(name, 0) + 1
        self._marks.clear()
        return out

    def summary(self) -> dict[str, float]:
        """Mean milliseconds per phase over everything collected."""
        return {k: self.totals[k] / self.counts[k] for k in self.totals}


# ------------------------------------------------------------------ roofline
_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
NVLINK_GBS = 770.0  # measured peer copy per direction per GPU on this hardware class


def measured_peaks() -> dict:
    """MEASURED_PEAKS.json next to the package when present (with a
    `source` key saying which), else an earlier B200 measurement."""
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                        "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        d["source"] = "measured"
        return d
    except (OSError, ValueError):
        return dict(_FALLBACK, source="fallback")


def roofline(ms: float, flops: float = 0.0, hbm_bytes: float = 0.0, link_bytes: float = 0.0,
             sustained: bool = False) -> dict:
    """Achieved rates and the fraction of the roofline time for one kernel or
    step: target = max(flops / GEMM peak, HBM bytes / copy bandwidth, NVLink
    bytes / link bandwidth); frac = target / measured time."""
    pk = measured_peaks()
    tf = pk.get("bf16_tflops_sustained" if sustained else "bf16_tflops", 1400.0)
    t_flop = flops / (tf * 1e12) * 1e3
    t_hbm = hbm_bytes / (pk.get("hbm_gbs", 6650.0) * 1e9) * 1e3
    t_link = link_bytes / (NVLINK_GBS * 1e9) * 1e3
    target = max(t_flop, t_hbm, t_link)
    bound = ("compute", "memory", "nvlink")[[t_flop, t_hbm, t_link].index(target)] if target > 0 else None
    return {"ms": ms, "tflops": flops / ms / 1e9 if ms else 0.0, "hbm_gbs": hbm_bytes / ms / 1e6 if ms else 0.0,
            "link_gbs": link_bytes / ms / 1e6 if ms else 0.0, "target_ms": target, "bound": bound,
            "frac_of_roofline": target / ms if ms else 0.0, "peaks": pk.get("source")}


# ------------------------------------------------------------------- logger
def collective_bytes(model) -> int:
    """Payload bytes this rank's gradient / parameter collectives carry per
    step (all-reduce: the fp32 gradient once; ZeRO: reduce-scatter of the
    fp32 gradient plus all-gather of the bf16 weights)."""
    gs = getattr(model, "grad_sync", None)
    if gs is None:
        return 0
    fp = model.fp
    if getattr(model, "param_sync", None) is gs:  # ZeRO
        return fp.total * 4 + fp.total * 2
    return fp.total * 4


class StepLogger:
    """Appends one JSON line per training step to `path` (rank 0 writes;
    every rank must call `log` because the step time is reduced with MAX)."""

    def __init__(self, path: str, tokens_per_step: int, flops_per_token: float = 0.0, model=None):
        self.path = path
        self.tokens = tokens_per_step
        self.flops_tok = flops_per_token
        self.model = model
        self.step = 0
        self._ev = None
        d = os.path.dirname(path)
        if d:
            os.makedirs(d, exist_ok=True)

    def begin(self):
        if torch.cuda.is_available() and torch.cuda.is_initialized():
            self._ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            self._ev[0].record()
        else:
            self._ev = (time.perf_counter(), None)

    def log(self, loss, phases: dict | None = None, grad_norm=None, extra: dict | None = None) -> dict:
        if isinstance(self._ev[0], torch.cuda.Event):
            self._ev[1].record()
            self._ev[1].synchronize()
            ms = self._ev[0].elapsed_time(self._ev[1])
        else:
            ms = (time.perf_counter() - self._ev[0]) * 1e3
        world, rank = 1, 0
        if torch.distributed.is_available() and torch.distributed.is_initialized():
            world, rank = torch.distributed.get_world_size(), torch.distributed.get_rank()
            dev = "cuda" if torch.cuda.is_available() and torch.cuda.is_initialized() else "cpu"
            t = torch.tensor([ms], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            ms = float(t)
        rec = {"step": self.step, "loss": float(loss), "ms": round(ms, 4),
               "tokens_per_s": round(self.tokens / (ms / 1e3), 1) if ms > 0 else None, "world": world}
        if grad_norm is None and self.model is not None:
            opt = getattr(self.model, "optimizer", None)
            gn = getattr(opt, "grad_norm", None)
            if isinstance(gn, torch.Tensor) and gn.numel():
                grad_norm = float(gn.reshape(-1)[0])
        if grad_norm is not None:
            rec["grad_norm"] = float(grad_norm)
        if self.model is not None:
            rec["comm_bytes_per_rank"] = collective_bytes(self.model)
        if self.flops_tok and ms > 0:
            pk = measured_peaks()
            rec["mfu"] = round(self.tokens * self.flops_tok / (ms / 1e3) /
                               (pk.get("bf16_tflops_sustained", 1400.0) * 1e12 * world), 4)
        if phases:
            rec["phases_ms"] = {k: round(v, 4) for k, v in phases.items()}
        if extra:
            rec.update(extra)
        if rank == 0:
            with open(self.path, "a") as f:
                f.write(json.dumps(rec) + "\n")
        self.step += 1
        return rec
