// Small elementwise kernels for the layer API's backward passes.
//
//   dgelu_mul:   out = gy * gelu'(pre)  (tanh-form GELU, fp32 math, bf16 I/O);
//                the gradient of y = gelu(pre) for a Dense layer whose forward
//                ran the GEMM's bias+GELU epilogue
//   scale_by:    out = x * (g[0] / count[0]) with both scalars read on the
//                device (no host synchronisation): the cross-entropy
//                backward's upstream-gradient / valid-token scaling
//
// Reference parity: scirs2-neural/src/activations_minimal.rs:57-68 (GELU,
// tanh form) and losses/crossentropy.rs:54-143 (mean reduction).
#include "host_common.h"

namespace scirs {
namespace ew {

__device__ __forceinline__ float gelu_tanh_grad(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  const float u = k0 * (x + k1 * x * x * x);
  const float t = tanhf(u);
  return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * k0 * (1.f + 3.f * k1 * x * x);
}

__global__ void __launch_bounds__(256) dgelu_mul_kernel(const __nv_bfloat16* __restrict__ gy,
                                                        const __nv_bfloat16* __restrict__ pre,
                                                        __nv_bfloat16* __restrict__ out, long n) {
  const long nv = n / 8;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (long)gridDim.x * blockDim.x) {
    const uint4 a = reinterpret_cast<const uint4*>(gy)[i];
    const uint4 b = reinterpret_cast<const uint4*>(pre)[i];
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
      o[e] = pack_bf16x2(bf16_lo(aw[e]) * gelu_tanh_grad(bf16_lo(bw[e])),
                         bf16_hi(aw[e]) * gelu_tanh_grad(bf16_hi(bw[e])));
    reinterpret_cast<uint4*>(out)[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  for (long i = nv * 8 + (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    out[i] = __float2bfloat16(__bfloat162float(gy[i]) * gelu_tanh_grad(__bfloat162float(pre[i])));
}

__global__ void __launch_bounds__(256) scale_by_kernel(const __nv_bfloat16* __restrict__ x, const float* g,
                                                       const float* count, __nv_bfloat16* __restrict__ out, long n) {
  const float s = g[0] / fmaxf(count[0], 1.f);
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    out[i] = __float2bfloat16(__bfloat162float(x[i]) * s);
}

static int grid_for(long work, int dev) {
  return (int)std::max<long>(1, std::min<long>((work + 255) / 256, 16L * num_sms(dev)));
}

}  // namespace ew

void dgelu_mul(torch::Tensor gy, torch::Tensor pre, torch::Tensor out) {
  for (auto* t : {&gy, &pre, &out}) {
    CHECK_DTYPE((*t), at::kBFloat16);
    CHECK_CONTIG((*t));
  }
  TORCH_CHECK(gy.numel() == pre.numel() && gy.numel() == out.numel(), "dgelu_mul: size mismatch");
  const bool vec = ((reinterpret_cast<uintptr_t>(gy.data_ptr()) | reinterpret_cast<uintptr_t>(pre.data_ptr()) |
                     reinterpret_cast<uintptr_t>(out.data_ptr())) & 15) == 0;
  TORCH_CHECK(vec, "dgelu_mul: operands must be 16-byte aligned");
  const int dev = gy.get_device();
  c10::cuda::CUDAGuard guard(dev);
  ew::dgelu_mul_kernel<<<ew::grid_for(gy.numel() / 8 + 1, dev), 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(gy.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(pre.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), gy.numel());
  SCIRS_CHECK_LAUNCH();
}

void scale_by(torch::Tensor x, torch::Tensor g, torch::Tensor count, torch::Tensor out) {
  CHECK_DTYPE(x, at::kBFloat16);
  CHECK_CONTIG(x);
  CHECK_DTYPE(out, at::kBFloat16);
  CHECK_CONTIG(out);
  CHECK_DTYPE(g, at::kFloat);
  CHECK_DTYPE(count, at::kFloat);
  TORCH_CHECK(x.numel() == out.numel(), "scale_by: size mismatch");
  const int dev = x.get_device();
  c10::cuda::CUDAGuard guard(dev);
  ew::scale_by_kernel<<<ew::grid_for(x.numel(), dev), 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), g.data_ptr<float>(), count.data_ptr<float>(),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), x.numel());
  SCIRS_CHECK_LAUNCH();
}

}  // namespace scirs
