"""Kernel-level operations (sm_100a kernels with CPU reference paths)."""
from . import kernels  # noqa: F401
