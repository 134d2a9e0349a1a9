"""GEMM auto-tuning with a persistent cache.

The tcgen05 GEMM picks its tile width (128 or 256 columns) and split-K factor
by a wave-count heuristic. `GemmAutotuner` measures the alternatives for a
given problem instead: every candidate (tile width auto / 128 / 256; split-K
auto / 1 / 2 / 4 / 8 / 16 for fp32-output GEMMs, which is where the kernel
honours a forced split) runs `warmup` times, then `iters` timed launches, each
bracketed by its own CUDA events with an L2 flush (a write larger than the
126 MB L2) between them; the fastest median wins. Candidates the kernel
rejects (its argument checks raise) are skipped. Results are keyed by device
name, problem shape, operand layouts and epilogue, and persist as JSON, so a
serving or training process tunes each shape once.

Reference parity: scirs2-core/src/advanced_tensor_cores/*.rs and
gpu/auto_tuning.rs (tensor-core kernel configuration search with a cache of
tuned configurations); there models without kernels, here measurements of
the framework's GEMM.
"""
from __future__ import annotations

import json
import os
import statistics
from typing import Callable

import torch

from . import kernels as K

SPLITS_F32 = (0, 1, 2, 4, 8, 16)
WIDTHS = (0, 128, 256)


class GemmAutotuner:
    def __init__(self, cache_path: str | None = None, warmup: int = 3, iters: int = 10, flush_l2: bool = True,
                 timer: Callable[[Callable[[], None]], float] | None = None,
                 gemm_fn: Callable | None = None):
        """`timer(fn) -> ms` and `gemm_fn` replace the CUDA-event timing and the kernel (host tests)."""
        self.cache_path, self.warmup, self.iters, self.flush_l2 = cache_path, warmup, iters, flush_l2
        self._timer, self._gemm = timer, gemm_fn or K.gemm
        self.cache: dict[str, dict] = {}
        self._flush_buf: torch.Tensor | None = None
        if cache_path and os.path.exists(cache_path):
            with open(cache_path) as f:
                self.cache = json.load(f)

    @staticmethod
    def _device_name(t: torch.Tensor) -> str:
        return torch.cuda.get_device_name(t.device) if t.is_cuda else "cpu"

    def key(self, a: torch.Tensor, b: torch.Tensor, a_mn: bool, b_mn: bool, epi: int, accumulate: bool) -> str:
        M = a.shape[1] if a_mn else a.shape[0]
        Kd = a.shape[0] if a_mn else a.shape[1]
        N = b.shape[1] if b_mn else b.shape[0]
        return f"{self._device_name(a)}|M{M}|N{N}|K{Kd}|amn{int(a_mn)}|bmn{int(b_mn)}|epi{epi}|acc{int(accumulate)}"

    @staticmethod
    def candidates(epi: int) -> list[tuple[int, int]]:
        splits = SPLITS_F32 if epi == K.EPI_F32 else (0,)
        return [(s, w) for s in splits for w in WIDTHS]

    def _flush(self, dev):
        if self._flush_buf is None or self._flush_buf.device != dev:
            self._flush_buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
        self._flush_buf.zero_()

    def _measure(self, fn: Callable[[], None], dev) -> float:
        if self._timer is not None:
            return self._timer(fn)
        times = []
        for _ in range(self.iters):
            if self.flush_l2:
                self._flush(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize(dev)
            times.append(e0.elapsed_time(e1))
        return statistics.median(times)

    def tune(self, a, b, out, *, a_mn: bool = False, b_mn: bool = False, epi: int = K.EPI_BF16,
             accumulate: bool = False, **kw) -> dict:
        """Measures every candidate on these operands (`out` is overwritten; with accumulate, a copy is
        restored after tuning) and records the fastest."""
        key = self.key(a, b, a_mn, b_mn, epi, accumulate)
        saved = out.clone() if accumulate else None
        results = []
        for splits, bn in self.candidates(epi):
            def run(s=splits, w=bn):
                self._gemm(a, b, out, a_mn=a_mn, b_mn=b_mn, epi=epi, accumulate=accumulate, splits=s, bn=w, **kw)

            try:
                for _ in range(self.warmup):
                    run()
                ms = self._measure(run, out.device)
            except RuntimeError as e:  # a configuration the kernel does not take for this shape
                results.append({"splits": splits, "bn": bn, "error": str(e).splitlines()[0]})
                continue
            results.append({"splits": splits, "bn": bn, "ms": ms})
        if saved is not None:
            out.copy_(saved)
        ok = [r for r in results if "ms" in r]
        if not ok:
            raise RuntimeError(f"no GEMM configuration ran for {key}")
        best = min(ok, key=lambda r: r["ms"])
        default = next((r for r in ok if r["splits"] == 0 and r["bn"] == 0), None)
        entry = {"splits": best["splits"], "bn": best["bn"], "ms": best["ms"],
                 "default_ms": default["ms"] if default else None, "results": results}
        self.cache[key] = entry
        self.save()
        return entry

    def lookup(self, a, b, *, a_mn: bool = False, b_mn: bool = False, epi: int = K.EPI_BF16,
               accumulate: bool = False) -> tuple[int, int] | None:
        e = self.cache.get(self.key(a, b, a_mn, b_mn, epi, accumulate))
        return (e["splits"], e["bn"]) if e else None

    def gemm(self, a, b, out, *, a_mn: bool = False, b_mn: bool = False, epi: int = K.EPI_BF16,
             accumulate: bool = False, tune_missing: bool = True, **kw):
        """The GEMM with the tuned configuration (tuning this shape first if it is not cached and
        `tune_missing`; otherwise the kernel's own choice)."""
        cfg = self.lookup(a, b, a_mn=a_mn, b_mn=b_mn, epi=epi, accumulate=accumulate)
        if cfg is None and tune_missing:
            e = self.tune(a, b, out, a_mn=a_mn, b_mn=b_mn, epi=epi, accumulate=accumulate, **kw)
            cfg = (e["splits"], e["bn"])
        splits, bn = cfg or (0, 0)
        return self._gemm(a, b, out, a_mn=a_mn, b_mn=b_mn, epi=epi, accumulate=accumulate, splits=splits, bn=bn,
                          **kw)

    def save(self) -> None:
        if self.cache_path:
            tmp = self.cache_path + ".tmp"
            with open(tmp, "w") as f:
                json.dump(self.cache, f, indent=1, sort_keys=True)
            os.replace(tmp, self.cache_path)


def main(argv=None) -> None:
    """python -m scirs_b200.ops.autotune --shape 8192x768x3072 [--shape ...] [--f32] --cache tuned.json"""
    import argparse

    ap = argparse.ArgumentParser(description="tune the tcgen05 GEMM for the given M x N x K shapes")
    ap.add_argument("--shape", action="append", required=True, help="MxNxK (out[M, N] = a[M, K] @ b[N, K]^T)")
    ap.add_argument("--f32", action="store_true", help="fp32 output (the weight-gradient form; split-K applies)")
    ap.add_argument("--cache", default="gemm_tuning.json")
    args = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("GEMM tuning needs a CUDA device")
    tuner = GemmAutotuner(args.cache)
    for s in args.shape:
        M, N, Kd = (int(x) for x in s.lower().split("x"))
        a = torch.randn(M, Kd, device="cuda", dtype=torch.bfloat16)
        b = torch.randn(N, Kd, device="cuda", dtype=torch.bfloat16)
        out = torch.empty(M, N, device="cuda", dtype=torch.float32 if args.f32 else torch.bfloat16)
        e = tuner.tune(a, b, out, epi=K.EPI_F32 if args.f32 else K.EPI_BF16)
        tflops = 2 * M * N * Kd / (e["ms"] * 1e-3) / 1e12
        print(f"{s}: splits={e['splits']} bn={e['bn']} {e['ms']:.4f} ms ({tflops:.0f} TFLOP/s), "
              f"kernel default {e['default_ms']:.4f} ms")


if __name__ == "__main__":
    main()
