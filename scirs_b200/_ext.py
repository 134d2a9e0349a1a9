"""Loader for the compiled sm_100a extensions.

CUDA tensors always go through the native kernels; if the extension cannot be
imported while a GPU is present, the import error is raised (there is no
silent PyTorch fallback on the device). CPU tensors use the pure-PyTorch
reference paths in :mod:`scirs_b200.ops`, which are also the numerical
oracles of the tests.
"""
from __future__ import annotations

import importlib

import torch

_C = None
_COMM = None
_ERR: dict[str, BaseException] = {}


def _load(name: str):
    try:
        return importlib.import_module(f"scirs_b200.{name}")
    except ImportError as e:  # pragma: no cover - depends on the build
        _ERR[name] = e
        return None


def kernels():
    """The `_C` module (GEMM, attention, norm, loss, optimizer kernels)."""
    global _C
    if _C is None:
        _C = _load("_C")
        if _C is None:
            raise RuntimeError(
                "scirs_b200._C is not built; run `python setup.py build_ext --inplace` "
                f"(import error: {_ERR.get('_C')})"
            )
    return _C


def comm():
    """The `_comm` module (in-kernel NVLink collectives)."""
    global _COMM
    if _COMM is None:
        _COMM = _load("_comm")
        if _COMM is None:
            raise RuntimeError(
                "scirs_b200._comm is not built; run `python setup.py build_ext --inplace` "
                f"(import error: {_ERR.get('_comm')})"
            )
    return _COMM


def data():
    """The `_data` module (native host batch prefetcher)."""
    mod = _load("_data")
    if mod is None:
        raise RuntimeError(
            "scirs_b200._data is not built; run `python setup.py build_ext --inplace` "
            f"(import error: {_ERR.get('_data')})"
        )
    return mod


def available() -> bool:
    try:
        kernels()
        return True
    except RuntimeError:
        return False


def check_status(device: int | None = None) -> None:
    """Raise if any native kernel recorded an error in its device status word."""
    if device is None:
        device = torch.cuda.current_device()
    codes = {1: "mbarrier wait timed out", 2: "peer wait timed out", 3: "bounds check failed", 4: "bad argument"}
    for mod in (kernels(),) + ((_COMM,) if _COMM is not None else ()):
        code, where, block, info = mod.status_read_and_clear(device)
        if code != 0:
            raise RuntimeError(
                f"native kernel error on cuda:{device}: {codes.get(code, code)} (site {where}, block {block}, info {info})"
            )
