"""Device layer: backend detection, device inventory, a context with buffers,
transfers and basic array operations, the registry of the framework's native
kernels, and a runtime compiler for user CUDA kernels.

* `GpuBackend.preferred()` is CUDA when a device is visible, else CPU; the
  framework targets one device generation (B200, compute capability 10.0),
  `DeviceInfo.is_sm100` says whether a device is one.
* `detect_devices()` reads the device inventory through NVML (read-only
  queries: name, UUID, memory, compute capability, driver version, maximum
  SM clock, power limit, active NVLink links) and adds the SM count from the
  CUDA runtime when a device is visible. Nothing is ever set through NVML.
* `GpuContext` owns a device and a stream: `create_buffer`,
  host <-> device transfers (pinned staging for the asynchronous forms),
  reductions, GEMM (bf16 on the framework's tcgen05 kernel, other dtypes on
  the library GEMM), activations and their gradients.
* `kernel_registry()` lists the native entry points of the compiled
  extensions with the source file of each.
* `GpuCompiler` compiles CUDA C++ source with NVRTC for sm_100a straight to a
  cubin (never to PTX text), and `GpuKernelHandle` binds arguments by the
  parameter names of the kernel's signature and launches it on the current
  stream through the driver API.

Reference parity: scirs2-core/src/gpu/mod.rs:21-1010 (GpuBackend preferred /
is_available, GpuDevice, GpuBuffer copy_from_host / copy_to_host / to_vec,
GpuKernelHandle set_buffer / set_u32 / set_i32 / set_f32 / set_f64 /
dispatch, GpuCompiler, GpuContext create_buffer / execute / get_kernel /
memory queries / transfers / reductions / gemm / activations and backward),
gpu/backends/mod.rs:62-560 (backend detection), gpu/kernels/mod.rs:221-330
(kernel registry). The reference's CUDA launch is commented out; here the
registry names kernels that run, and user kernels are launched for real.
"""
from __future__ import annotations

import contextlib
import ctypes
import dataclasses
import enum
import hashlib
import os
import re
from typing import Any, Callable

import numpy as np
import torch

from . import _ext


class GpuError(RuntimeError):
    pass


class GpuBackend(enum.Enum):
    CUDA = "cuda"
    CPU = "cpu"

    @classmethod
    def preferred(cls) -> "GpuBackend":
        return cls.CUDA if torch.cuda.is_available() else cls.CPU

    def is_available(self) -> bool:
        return self is GpuBackend.CPU or torch.cuda.is_available()


# ----------------------------------------------------------------------------- detection


@dataclasses.dataclass
class DeviceInfo:
    index: int
    name: str
    uuid: str | None = None
    compute_capability: tuple[int, int] | None = None
    total_memory: int | None = None
    free_memory: int | None = None
    driver_version: str | None = None
    max_sm_clock_mhz: int | None = None
    power_limit_w: float | None = None
    nvlink_active_links: int = 0
    sm_count: int | None = None

    @property
    def is_sm100(self) -> bool:
        return self.compute_capability == (10, 0)


def _s(x):
    return x.decode() if isinstance(x, bytes) else x


def detect_devices(nvml: Any = None, max_links: int = 18) -> list[DeviceInfo]:
    """Device inventory from NVML (module `pynvml` unless another object with the same functions is
    given); an empty list when NVML cannot be initialised. Only read queries are issued."""
    if nvml is None:
        try:
            import pynvml as nvml  # nvidia-ml-py
        except ImportError:
            return []
    try:
        nvml.nvmlInit()
    except Exception:  # noqa: BLE001 - no driver on this host
        return []
    out = []
    try:
        driver = _s(nvml.nvmlSystemGetDriverVersion())
        for i in range(nvml.nvmlDeviceGetCount()):
            h = nvml.nvmlDeviceGetHandleByIndex(i)
            info = DeviceInfo(i, _s(nvml.nvmlDeviceGetName(h)), driver_version=driver)

            def q(fn, *a):
                try:
                    return fn(h, *a)
                except Exception:  # noqa: BLE001 - query not supported on this device
                    return None

            info.uuid = _s(q(nvml.nvmlDeviceGetUUID))
            mem = q(nvml.nvmlDeviceGetMemoryInfo)
            if mem is not None:
                info.total_memory, info.free_memory = int(mem.total), int(mem.free)
            cc = q(nvml.nvmlDeviceGetCudaComputeCapability)
            info.compute_capability = tuple(cc) if cc is not None else None
            info.max_sm_clock_mhz = q(nvml.nvmlDeviceGetMaxClockInfo, getattr(nvml, "NVML_CLOCK_SM", 1))
            pl = q(nvml.nvmlDeviceGetPowerManagementLimit)
            info.power_limit_w = pl / 1000.0 if pl is not None else None
            links = 0
            for link in range(max_links):
                st = q(nvml.nvmlDeviceGetNvLinkState, link)
                if st is None:
                    continue
                links += int(bool(st))
            info.nvlink_active_links = links
            if torch.cuda.is_available() and i < torch.cuda.device_count():
                info.sm_count = torch.cuda.get_device_properties(i).multi_processor_count
            out.append(info)
    finally:
        try:
            nvml.nvmlShutdown()
        except Exception:  # noqa: BLE001
            pass
    return out


# ----------------------------------------------------------------------------- buffers and context


class GpuBuffer:
    """A 1-D array on the context's device (a torch tensor underneath: `.tensor`)."""

    def __init__(self, tensor: torch.Tensor, ctx: "GpuContext"):
        self.tensor, self._ctx = tensor, ctx

    def __len__(self):
        return self.tensor.numel()

    def is_empty(self) -> bool:
        return len(self) == 0

    @property
    def dtype(self):
        return self.tensor.dtype

    def copy_from_host(self, data) -> None:
        src = torch.as_tensor(np.asarray(data)).reshape(-1)
        if src.numel() != len(self):
            raise GpuError(f"size mismatch: buffer {len(self)}, host data {src.numel()}")
        with self._ctx._stream_ctx():
            self.tensor.copy_(src.to(self.tensor.dtype))

    def copy_to_host(self, out: np.ndarray | None = None) -> np.ndarray:
        with self._ctx._stream_ctx():
            host = self.tensor.detach().to("cpu")
        arr = host.float().numpy() if host.dtype == torch.bfloat16 else host.numpy()
        if out is not None:
            out[...] = arr.reshape(out.shape)
            return out
        return arr

    def to_vec(self) -> list:
        return self.copy_to_host().tolist()

    @property
    def ptr(self) -> int:
        return self.tensor.data_ptr()


class GpuContext:
    def __init__(self, backend: GpuBackend | None = None, device: int = 0):
        self.backend = backend or GpuBackend.preferred()
        if not self.backend.is_available():
            raise GpuError(f"backend {self.backend.value} is not available")
        if self.backend is GpuBackend.CUDA:
            self.device = torch.device("cuda", device)
            self.stream = torch.cuda.Stream(self.device)
        else:
            self.device, self.stream = torch.device("cpu"), None
        self._compiler: GpuCompiler | None = None

    @property
    def backend_name(self) -> str:
        return "CUDA (sm_100a)" if self.backend is GpuBackend.CUDA else "CPU"

    def _stream_ctx(self):
        return torch.cuda.stream(self.stream) if self.stream is not None else contextlib.nullcontext()

    # buffers and transfers
    def create_buffer(self, size: int, dtype=torch.float32) -> GpuBuffer:
        return GpuBuffer(torch.zeros(size, dtype=dtype, device=self.device), self)

    def create_buffer_from_slice(self, data, dtype=None) -> GpuBuffer:
        t = torch.as_tensor(np.asarray(data)).reshape(-1)
        return self.transfer_host_to_device(t.to(dtype) if dtype is not None else t)

    def transfer_host_to_device(self, data, non_blocking: bool = False) -> GpuBuffer:
        t = torch.as_tensor(np.asarray(data) if not isinstance(data, torch.Tensor) else data).reshape(-1)
        if self.backend is GpuBackend.CPU:
            return GpuBuffer(t.clone(), self)
        if non_blocking and not t.is_pinned():
            t = t.pin_memory()
        with self._stream_ctx():
            return GpuBuffer(t.to(self.device, non_blocking=non_blocking), self)

    def transfer_device_to_host(self, buf: GpuBuffer, non_blocking: bool = False) -> torch.Tensor:
        if self.backend is GpuBackend.CPU:
            return buf.tensor.clone()
        out = torch.empty(buf.tensor.shape, dtype=buf.dtype, pin_memory=non_blocking)
        with self._stream_ctx():
            out.copy_(buf.tensor, non_blocking=non_blocking)
        return out

    def read_buffer(self, buf: GpuBuffer) -> np.ndarray:
        return buf.copy_to_host()

    def synchronize(self) -> None:
        if self.stream is not None:
            self.stream.synchronize()

    def execute(self, fn: Callable[["GpuContext"], Any]):
        """Runs fn(ctx) with the context's stream current."""
        with self._stream_ctx():
            return fn(self)

    def get_available_memory(self) -> int | None:
        return torch.cuda.mem_get_info(self.device)[0] if self.backend is GpuBackend.CUDA else None

    def get_total_memory(self) -> int | None:
        return torch.cuda.mem_get_info(self.device)[1] if self.backend is GpuBackend.CUDA else None

    # array operations (results are new buffers)
    def _wrap(self, t: torch.Tensor) -> GpuBuffer:
        return GpuBuffer(t.reshape(-1) if t.dim() != 1 else t, self)

    def _run(self, fn):
        with self._stream_ctx():
            return self._wrap(fn())

    def sum_all(self, b: GpuBuffer) -> GpuBuffer:
        return self._run(lambda: b.tensor.sum().reshape(1))

    def mean_all(self, b: GpuBuffer) -> GpuBuffer:
        return self._run(lambda: b.tensor.float().mean().reshape(1).to(b.dtype))

    def max_all(self, b: GpuBuffer) -> GpuBuffer:
        return self._run(lambda: b.tensor.max().reshape(1))

    def min_all(self, b: GpuBuffer) -> GpuBuffer:
        return self._run(lambda: b.tensor.min().reshape(1))

    def _axis(self, b, shape, axis, op):
        return self._run(lambda: op(b.tensor.reshape(shape), axis))

    def sum_axis(self, b: GpuBuffer, shape, axis: int) -> GpuBuffer:
        return self._axis(b, shape, axis, lambda t, a: t.sum(a))

    def mean_axis(self, b: GpuBuffer, shape, axis: int) -> GpuBuffer:
        return self._axis(b, shape, axis, lambda t, a: t.float().mean(a).to(t.dtype))

    def max_axis(self, b: GpuBuffer, shape, axis: int) -> GpuBuffer:
        return self._axis(b, shape, axis, lambda t, a: t.amax(a))

    def min_axis(self, b: GpuBuffer, shape, axis: int) -> GpuBuffer:
        return self._axis(b, shape, axis, lambda t, a: t.amin(a))

    def broadcast(self, b: GpuBuffer, from_shape, to_shape) -> GpuBuffer:
        return self._run(lambda: b.tensor.reshape(from_shape).expand(to_shape).contiguous())

    def scale(self, b: GpuBuffer, alpha: float) -> GpuBuffer:
        return self._run(lambda: b.tensor * alpha)

    def gemm(self, a: GpuBuffer, b: GpuBuffer, m: int, k: int, n: int, transpose_a: bool = False,
             transpose_b: bool = False) -> GpuBuffer:
        """C[m, n] = op(A) op(B) with A stored [m, k] (or [k, m] when transposed) and B stored [k, n]
        (or [n, k]). bf16 operands on a device run the framework's tcgen05 GEMM."""
        A = a.tensor.reshape(k, m).t() if transpose_a else a.tensor.reshape(m, k)
        Bkn = b.tensor.reshape(n, k).t() if transpose_b else b.tensor.reshape(k, n)

        def go():
            if A.is_cuda and A.dtype == torch.bfloat16 and Bkn.dtype == torch.bfloat16:
                from .ops import functional as F

                return F.linear(A.contiguous(), Bkn)
            return A @ Bkn

        return self._run(go)

    def gemm_transpose_a(self, a, b, m, k, n) -> GpuBuffer:
        return self.gemm(a, b, m, k, n, transpose_a=True)

    def gemm_transpose_b(self, a, b, m, k, n) -> GpuBuffer:
        return self.gemm(a, b, m, k, n, transpose_b=True)

    def relu(self, x: GpuBuffer) -> GpuBuffer:
        return self._run(lambda: torch.relu(x.tensor))

    def relu_backward(self, grad: GpuBuffer, x: GpuBuffer) -> GpuBuffer:
        return self._run(lambda: grad.tensor * (x.tensor > 0).to(grad.dtype))

    def sigmoid(self, x: GpuBuffer) -> GpuBuffer:
        return self._run(lambda: torch.sigmoid(x.tensor))

    def sigmoid_backward(self, grad: GpuBuffer, y: GpuBuffer) -> GpuBuffer:
        """Gradient through y = sigmoid(x), given y."""
        return self._run(lambda: grad.tensor * y.tensor * (1 - y.tensor))

    def tanh(self, x: GpuBuffer) -> GpuBuffer:
        return self._run(lambda: torch.tanh(x.tensor))

    def tanh_backward(self, grad: GpuBuffer, y: GpuBuffer) -> GpuBuffer:
        """Gradient through y = tanh(x), given y."""
        return self._run(lambda: grad.tensor * (1 - y.tensor * y.tensor))

    def gelu(self, x: GpuBuffer) -> GpuBuffer:
        return self._run(lambda: torch.nn.functional.gelu(x.tensor, approximate="tanh"))

    def gelu_backward(self, grad: GpuBuffer, x: GpuBuffer) -> GpuBuffer:
        """Gradient of the tanh-form GELU; bf16 device buffers use the framework's fused kernel."""
        g, xt = grad.tensor, x.tensor
        if g.is_cuda and g.dtype == torch.bfloat16 and xt.dtype == torch.bfloat16 and g.numel() % 8 == 0:
            def fused():
                out = torch.empty_like(g)
                _ext.kernels().dgelu_mul(g.contiguous(), xt.contiguous(), out)
                return out

            return self._run(fused)

        def ref():
            ct = torch.float64 if xt.dtype == torch.float64 else torch.float32
            xf = xt.to(ct)
            k0, k1 = 0.7978845608028654, 0.044715
            t = torch.tanh(k0 * (xf + k1 * xf ** 3))
            d = 0.5 * (1 + t) + 0.5 * xf * (1 - t * t) * k0 * (1 + 3 * k1 * xf * xf)
            return (g.to(ct) * d).to(g.dtype)

        return self._run(ref)

    # kernels
    def get_kernel(self, name: str):
        """A native kernel entry point of the framework by name (see kernel_registry())."""
        reg = kernel_registry()
        if name not in reg:
            raise GpuError(f"no kernel named {name!r}")
        return getattr(_ext.kernels() if reg[name]["module"] == "_C" else _ext.comm(), name)

    def compiler(self) -> "GpuCompiler":
        if self._compiler is None:
            self._compiler = GpuCompiler()
        return self._compiler


# ----------------------------------------------------------------------------- native kernel registry

_SOURCES = {
    "gemm": "gemm_sm100.cu", "gemm_tp": "gemm_sm100.cu", "layernorm_fwd": "norm_loss.cu",
    "layernorm_bwd": "norm_loss.cu", "xent_fwd_bwd": "norm_loss.cu", "xent_fwd": "norm_loss.cu",
    "embedding_fwd": "norm_loss.cu", "embedding_bwd": "norm_loss.cu", "bias_grad": "norm_loss.cu",
    "optim_step": "optim.cu", "grad_sumsq": "optim.cu", "conv_im2col": "conv.cu", "conv_col2im": "conv.cu",
    "conv_rows_nchw": "conv.cu", "pool2d_fwd": "conv.cu", "pool2d_bwd": "conv.cu", "dgelu_mul": "elementwise.cu",
    "scale_by": "elementwise.cu", "lstm_cell_fwd": "rnn.cu", "lstm_cell_bwd": "rnn.cu", "gru_cell_fwd": "rnn.cu",
    "gru_cell_bwd": "rnn.cu", "rnn_cell_fwd": "rnn.cu", "rnn_cell_bwd": "rnn.cu", "flash_attn_fwd": "attention.cu",
    "flash_attn_bwd": "attention.cu", "flash_attn_fwd_pp": "attention_fwd_sm100.cu",
    "flash_attn_fwd_tc": "attention_sm100.cu", "paged_kv_append": "paged_attention.cu",
    "paged_attention_decode": "paged_attention.cu", "rope_apply": "tp.cu", "tp_reduce": "tp.cu",
    "ep_dispatch": "tp.cu", "ep_combine": "tp.cu", "ep_grad_w": "tp.cu", "patchify": "vision.cu",
    "vit_embed_fwd": "vision.cu", "vit_embed_bwd": "vision.cu",
}


def kernel_registry() -> dict[str, dict]:
    """Native entry points of the compiled extensions: name -> {module, source, doc}."""
    reg = {}
    for modname, loader in (("_C", _ext.kernels), ("_comm", _ext.comm)):
        try:
            mod = loader()
        except RuntimeError:
            continue
        for name in dir(mod):
            fn = getattr(mod, name)
            if name.startswith("_") or not callable(fn) or isinstance(fn, type):
                continue
            src = _SOURCES.get(name, "comm.cu" if modname == "_comm" else None)
            doc_lines = (fn.__doc__ or "").strip().splitlines()
            reg[name] = {"module": modname, "source": src, "doc": doc_lines[-1] if doc_lines else ""}
    return reg


# ----------------------------------------------------------------------------- runtime compilation

_CTYPES = {
    "float": ctypes.c_float, "double": ctypes.c_double, "int": ctypes.c_int, "int32_t": ctypes.c_int32,
    "unsigned": ctypes.c_uint, "unsigned int": ctypes.c_uint, "uint32_t": ctypes.c_uint32,
    "long": ctypes.c_long, "long long": ctypes.c_longlong, "int64_t": ctypes.c_int64,
    "unsigned long": ctypes.c_ulong, "unsigned long long": ctypes.c_ulonglong, "uint64_t": ctypes.c_uint64,
    "size_t": ctypes.c_size_t, "bool": ctypes.c_bool, "char": ctypes.c_char,
}

_LB = r"(?:__launch_bounds__\s*\([^)]*\)\s*)?"
_SIG = re.compile(r"__global__\s+" + _LB + r"void\s+" + _LB + r"(\w+)\s*\(([^)]*)\)", re.S)


def parse_kernel_params(source: str, name: str | None = None) -> tuple[str, list[tuple[str, Any]]]:
    """(kernel name, [(parameter name, ctypes type or 'ptr')]) of the named (or first) __global__
    function."""
    for m in _SIG.finditer(source):
        if name is None or m.group(1) == name:
            params = []
            for p in [s.strip() for s in m.group(2).split(",") if s.strip()]:
                p = re.sub(r"\b(const|__restrict__|volatile)\b", " ", p)
                pm = re.match(r"(.*?)([A-Za-z_]\w*)\s*$", p.strip(), re.S)
                if pm is None:
                    raise GpuError(f"cannot parse parameter {p!r}")
                ty, pname = " ".join(pm.group(1).split()), pm.group(2)
                if "*" in ty:
                    params.append((pname, "ptr"))
                elif ty in _CTYPES:
                    params.append((pname, _CTYPES[ty]))
                else:
                    raise GpuError(f"unsupported parameter type {ty!r} of {pname!r}")
            return m.group(1), params
    raise GpuError(f"no __global__ function {name or ''} found")


class GpuCompiler:
    """NVRTC compilation of CUDA C++ source for sm_100a to a cubin (kernels must be extern "C")."""

    def __init__(self, options: list[str] | None = None):
        home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
        self.options = ["--gpu-architecture=sm_100a", "--std=c++17", "-default-device", "-lineinfo",
                        f"--include-path={home}/include"] + list(options or [])
        self._cache: dict[str, bytes] = {}

    def compile_cubin(self, source: str) -> bytes:
        key = hashlib.sha256((source + "\0" + " ".join(self.options)).encode()).hexdigest()
        if key in self._cache:
            return self._cache[key]
        from cuda.bindings import nvrtc

        err, prog = nvrtc.nvrtcCreateProgram(source.encode(), b"user_kernel.cu", 0, [], [])
        self._check(nvrtc, err, prog, "create")
        opts = [o.encode() for o in self.options]
        (err,) = nvrtc.nvrtcCompileProgram(prog, len(opts), opts)
        if err != nvrtc.nvrtcResult.NVRTC_SUCCESS:
            _, n = nvrtc.nvrtcGetProgramLogSize(prog)
            log = b" " * n
            nvrtc.nvrtcGetProgramLog(prog, log)
            nvrtc.nvrtcDestroyProgram(prog)
            raise GpuError("NVRTC compilation failed:\n" + log.decode(errors="replace").rstrip("\x00 "))
        err, n = nvrtc.nvrtcGetCUBINSize(prog)
        self._check(nvrtc, err, prog, "cubin size")
        cubin = b" " * n
        (err,) = nvrtc.nvrtcGetCUBIN(prog, cubin)
        self._check(nvrtc, err, prog, "cubin")
        nvrtc.nvrtcDestroyProgram(prog)
        self._cache[key] = cubin
        return cubin

    @staticmethod
    def _check(nvrtc, err, prog, what):
        if err != nvrtc.nvrtcResult.NVRTC_SUCCESS:
            raise GpuError(f"NVRTC {what} failed: {err}")

    def compile(self, source: str, name: str | None = None) -> "GpuKernelHandle":
        kname, params = parse_kernel_params(source, name)
        return GpuKernelHandle(kname, params, self.compile_cubin(source))


class GpuKernelHandle:
    """Arguments are bound by parameter name; dispatch(grid, block) launches on the current stream."""

    def __init__(self, name: str, params: list, cubin: bytes):
        self.name, self.params, self.cubin = name, params, cubin
        self._args: dict[str, Any] = {}
        self._fn: dict[int, Any] = {}

    def _set(self, pname: str, value, kinds):
        types = dict(self.params)
        if pname not in types:
            raise GpuError(f"kernel {self.name} has no parameter {pname!r}")
        if types[pname] not in kinds:
            raise GpuError(f"parameter {pname!r} of {self.name} does not take this kind of value")
        self._args[pname] = value

    def set_buffer(self, pname: str, buf: "GpuBuffer | torch.Tensor") -> None:
        t = buf.tensor if isinstance(buf, GpuBuffer) else buf
        if not t.is_cuda:
            raise GpuError("kernel buffers must live on a CUDA device")
        self._set(pname, t, ("ptr",))

    def set_u32(self, pname: str, v: int) -> None:
        self._set(pname, int(v), (ctypes.c_uint, ctypes.c_uint32, ctypes.c_ulong, ctypes.c_ulonglong,
                                  ctypes.c_uint64, ctypes.c_size_t))

    def set_i32(self, pname: str, v: int) -> None:
        self._set(pname, int(v), (ctypes.c_int, ctypes.c_int32, ctypes.c_long, ctypes.c_longlong, ctypes.c_int64))

    def set_f32(self, pname: str, v: float) -> None:
        self._set(pname, float(v), (ctypes.c_float,))

    def set_f64(self, pname: str, v: float) -> None:
        self._set(pname, float(v), (ctypes.c_double,))

    def _packed(self):
        missing = [p for p, _ in self.params if p not in self._args]
        if missing:
            raise GpuError(f"kernel {self.name}: unset parameters {missing}")
        vals = []
        for p, ty in self.params:
            a = self._args[p]
            vals.append(ctypes.c_void_p(a.data_ptr()) if ty == "ptr" else ty(a))
        arr = (ctypes.c_void_p * len(vals))(*[ctypes.addressof(v) for v in vals])
        return vals, arr

    def dispatch(self, grid, block=(256, 1, 1), shared_mem: int = 0) -> None:
        if not torch.cuda.is_available():
            raise GpuError("no CUDA device: user kernels cannot be launched")
        from cuda.bindings import driver

        dev = torch.cuda.current_device()
        torch.cuda.init()
        if dev not in self._fn:
            err, mod = driver.cuModuleLoadData(self.cubin)
            if err != driver.CUresult.CUDA_SUCCESS:
                raise GpuError(f"cuModuleLoadData failed: {err}")
            err, fn = driver.cuModuleGetFunction(mod, self.name.encode())
            if err != driver.CUresult.CUDA_SUCCESS:
                raise GpuError(f"cuModuleGetFunction failed: {err}")
            self._fn[dev] = (mod, fn)
        g = tuple(grid) + (1,) * (3 - len(tuple(grid)))
        b = tuple(block) + (1,) * (3 - len(tuple(block)))
        vals, arr = self._packed()
        stream = driver.CUstream(torch.cuda.current_stream().cuda_stream)
        (err,) = driver.cuLaunchKernel(self._fn[dev][1], *g, *b, shared_mem, stream, ctypes.addressof(arr), 0)
        if err != driver.CUresult.CUDA_SUCCESS:
            raise GpuError(f"cuLaunchKernel failed: {err}")
        del vals  # the launch copied the parameter values
