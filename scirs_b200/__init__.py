"""scirs_b200: a Blackwell-native (sm_100a) training framework with the ML
capabilities of SciRS2 (autograd, neural-network layers, optimizers,
training loop, serialization and distributed gradient primitives).

PyTorch is the framework layer; the hot paths are hand-written sm_100a
kernels (scirs_b200/csrc) and in-kernel NVLink collectives.
"""
__version__ = "0.1.0"

from . import _ext  # noqa: F401
