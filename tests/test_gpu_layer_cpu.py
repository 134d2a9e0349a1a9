"""Device layer on the host: NVML inventory against a fake NVML (read-only
queries), the CPU context's array operations against numpy, the native
kernel registry, NVRTC compilation for sm_100a and kernel argument binding."""
import ctypes
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from scirs_b200 import gpu as G


class FakeNvml:
    NVML_CLOCK_SM = 1

    def __init__(self, n=2, fail_init=False):
        self.n, self.fail_init, self.calls = n, fail_init, []
        self.shutdown = False

    def nvmlInit(self):
        if self.fail_init:
            raise RuntimeError("no driver")

    def nvmlShutdown(self):
        self.shutdown = True

    def nvmlSystemGetDriverVersion(self):
        return b"580.159"

    def nvmlDeviceGetCount(self):
        return self.n

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetName(self, h):
        return b"NVIDIA B200"

    def nvmlDeviceGetUUID(self, h):
        return f"GPU-{h:04d}"

    def nvmlDeviceGetMemoryInfo(self, h):
        return SimpleNamespace(total=183_359 * 2**20, free=180_000 * 2**20)

    def nvmlDeviceGetCudaComputeCapability(self, h):
        return (10, 0)

    def nvmlDeviceGetMaxClockInfo(self, h, kind):
        assert kind == self.NVML_CLOCK_SM
        return 1965

    def nvmlDeviceGetPowerManagementLimit(self, h):
        if h == 1:
            raise RuntimeError("not supported")
        return 1_000_000

    def nvmlDeviceGetNvLinkState(self, h, link):
        if link >= 18:
            raise RuntimeError("invalid link")
        return 1 if link < 18 - 2 * h else 0

    def __getattr__(self, name):  # any setter would land here: none may be called
        if name.startswith("nvmlDeviceSet") or name.startswith("nvmlDeviceReset"):
            raise AssertionError(f"{name} must never be called")
        raise AttributeError(name)


def test_detect_devices_with_fake_nvml():
    nv = FakeNvml()
    devs = G.detect_devices(nv)
    assert nv.shutdown and len(devs) == 2
    d0, d1 = devs
    assert d0.name == "NVIDIA B200" and d0.uuid == "GPU-0000" and d0.is_sm100
    assert d0.total_memory == 183_359 * 2**20 and d0.driver_version == "580.159"
    assert d0.max_sm_clock_mhz == 1965 and d0.power_limit_w == 1000.0 and d0.nvlink_active_links == 18
    assert d1.power_limit_w is None and d1.nvlink_active_links == 16
    assert G.detect_devices(FakeNvml(fail_init=True)) == []


def test_backend_selection_on_this_host():
    be = G.GpuBackend.preferred()
    assert be is (G.GpuBackend.CUDA if torch.cuda.is_available() else G.GpuBackend.CPU)
    assert G.GpuBackend.CPU.is_available()


def test_cpu_context_operations_match_numpy():
    ctx = G.GpuContext(G.GpuBackend.CPU)
    assert ctx.backend_name == "CPU" and ctx.get_total_memory() is None
    rng = np.random.default_rng(0)
    a_np, b_np = rng.standard_normal((5, 7)), rng.standard_normal((7, 3))
    a = ctx.create_buffer_from_slice(a_np.ravel(), torch.float64)
    b = ctx.create_buffer_from_slice(b_np.ravel(), torch.float64)
    np.testing.assert_allclose(ctx.gemm(a, b, 5, 7, 3).copy_to_host().reshape(5, 3), a_np @ b_np)
    at = ctx.create_buffer_from_slice(a_np.T.ravel(), torch.float64)
    bt = ctx.create_buffer_from_slice(b_np.T.ravel(), torch.float64)
    np.testing.assert_allclose(ctx.gemm_transpose_a(at, b, 5, 7, 3).to_vec(), (a_np @ b_np).ravel())
    np.testing.assert_allclose(ctx.gemm_transpose_b(a, bt, 5, 7, 3).to_vec(), (a_np @ b_np).ravel())
    x = ctx.create_buffer_from_slice(a_np.ravel())
    assert ctx.sum_all(x).to_vec()[0] == pytest.approx(a_np.sum())
    assert ctx.mean_all(x).to_vec()[0] == pytest.approx(a_np.mean())
    assert ctx.max_all(x).to_vec()[0] == a_np.max() and ctx.min_all(x).to_vec()[0] == a_np.min()
    np.testing.assert_allclose(ctx.sum_axis(x, (5, 7), 0).copy_to_host(), a_np.sum(0))
    np.testing.assert_allclose(ctx.max_axis(x, (5, 7), 1).copy_to_host(), a_np.max(1))
    np.testing.assert_allclose(ctx.broadcast(ctx.create_buffer_from_slice([1.0, 2.0]), (1, 2), (3, 2)).to_vec(),
                               [1, 2] * 3)
    np.testing.assert_allclose(ctx.scale(x, 2.0).copy_to_host(), 2 * a_np.ravel())
    np.testing.assert_allclose(ctx.relu(x).copy_to_host(), np.maximum(a_np.ravel(), 0))
    g = ctx.create_buffer_from_slice(np.ones(35))
    np.testing.assert_allclose(ctx.relu_backward(g, x).copy_to_host(), (a_np.ravel() > 0).astype(float))
    y = ctx.tanh(x)
    np.testing.assert_allclose(ctx.tanh_backward(g, y).copy_to_host(), 1 - np.tanh(a_np.ravel()) ** 2)
    s = ctx.sigmoid(x)
    sig = 1 / (1 + np.exp(-a_np.ravel()))
    np.testing.assert_allclose(ctx.sigmoid_backward(g, s).copy_to_host(), sig * (1 - sig))
    xt = torch.tensor(a_np.ravel(), requires_grad=True)
    torch.nn.functional.gelu(xt, approximate="tanh").sum().backward()
    np.testing.assert_allclose(ctx.gelu_backward(g, x).copy_to_host(), xt.grad.numpy(), rtol=1e-6)
    buf = ctx.create_buffer(4)
    buf.copy_from_host([1, 2, 3, 4])
    out = np.zeros(4, np.float32)
    assert buf.copy_to_host(out) is out and out.tolist() == [1, 2, 3, 4]
    with pytest.raises(G.GpuError):
        buf.copy_from_host([1, 2])
    assert ctx.execute(lambda c: c is ctx)


def test_kernel_registry_lists_native_entry_points():
    reg = G.kernel_registry()
    for name in ("gemm", "flash_attn_fwd", "flash_attn_bwd", "layernorm_fwd", "optim_step", "lstm_cell_fwd"):
        assert name in reg and reg[name]["module"] == "_C" and reg[name]["source"].endswith(".cu")
    assert G.GpuContext(G.GpuBackend.CPU).get_kernel("gemm") is not None
    with pytest.raises(G.GpuError):
        G.GpuContext(G.GpuBackend.CPU).get_kernel("nope")


SRC = r'''
#include <cuda_bf16.h>
extern "C" __global__ void __launch_bounds__(256)
scaled_add(float a, const float* __restrict__ x, float* y, unsigned int n, long long tag, double unused) {
  unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] += a * x[i];
}
'''


def test_parse_kernel_params():
    name, params = G.parse_kernel_params(SRC)
    assert name == "scaled_add"
    assert params == [("a", ctypes.c_float), ("x", "ptr"), ("y", "ptr"), ("n", ctypes.c_uint),
                      ("tag", ctypes.c_longlong), ("unused", ctypes.c_double)]
    with pytest.raises(G.GpuError):
        G.parse_kernel_params("__global__ void k(MyStruct s) {}")
    with pytest.raises(G.GpuError):
        G.parse_kernel_params(SRC, "other")


def test_nvrtc_compiles_for_sm100a_and_reports_errors():
    comp = G.GpuCompiler()
    h = comp.compile(SRC)
    assert h.name == "scaled_add" and len(h.cubin) > 1000
    assert comp.compile_cubin(SRC) is h.cubin  # cached
    with pytest.raises(G.GpuError, match="undefined"):
        comp.compile('extern "C" __global__ void k(float* x) { x[0] = undefined_name; }')


def test_kernel_argument_binding_checks():
    h = G.GpuCompiler().compile(SRC)
    h.set_f32("a", 2.0)
    h.set_u32("n", 10)
    h.set_i32("tag", -1)
    h.set_f64("unused", 0.5)
    with pytest.raises(G.GpuError, match="no parameter"):
        h.set_f32("zzz", 1.0)
    with pytest.raises(G.GpuError, match="does not take"):
        h.set_f32("n", 1.0)
    with pytest.raises(G.GpuError, match="CUDA device"):
        h.set_buffer("x", torch.zeros(4))
    with pytest.raises(G.GpuError, match="unset parameters"):
        h._packed()
    if not torch.cuda.is_available():
        with pytest.raises(G.GpuError, match="no CUDA device"):
            h.dispatch((1,))
