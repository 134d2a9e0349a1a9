// Fused optimizer steps over flat fp32 buffers (one launch updates every
// parameter of a model), with optional global-norm gradient clipping, grad
// unscaling (mixed-precision loss scale), non-finite skip and a bf16 copy of
// the updated parameters for the tensor-core kernels.
//
// Step-dependent scalars (lr, bias corrections, grad scale) are read from a
// small device buffer, so a captured CUDA graph replays correctly across
// steps; the host refreshes that buffer before each replay.
//
// Update rules follow the reference optimizers:
//   Adam    scirs2-neural/src/optimizers/adam.rs:163-215   (L2 wd added to the gradient)
//   AdamW   scirs2-neural/src/optimizers/adamw.rs:149-196  (decoupled p *= 1 - lr*wd)
//   SGD     scirs2-neural/src/optimizers/sgd.rs:95-130     (v = mu v + lr g; p -= v)
//   RMSprop scirs2-neural/src/optimizers/rmsprop.rs:123-161
//   Adagrad scirs2-neural/src/optimizers/adagrad.rs:100-130
// and the reference's CUDA sources scirs2-core/src/gpu/kernels/adam_optimizer.cu:28-340
// (whose fused-clip variant needs a cooperative grid.sync; here the norm is a
// separate partial-sum launch instead).
#include "host_common.h"

namespace scirs {

enum OptMode : int { OPT_ADAM = 0, OPT_ADAMW = 1, OPT_SGD = 2, OPT_RMSPROP = 3, OPT_ADAGRAD = 4 };

// hp layout (fp32, device):
//  0 lr, 1 beta1 | momentum | rho, 2 beta2, 3 eps, 4 weight_decay,
//  5 bias_correction1, 6 bias_correction2, 7 grad multiplier, 8 max_norm (<=0: off),
//  9 step counter, 10 device-managed bias correction flag. When the flag is
//  set, the norm kernel increments the step counter and the update kernel
//  derives the bias corrections from it, so a captured step replays without
//  any host writes.
struct HP {
  float lr, b1, b2, eps, wd, bc1, bc2, gmul, max_norm, step, dev_step;
};

template <typename G>
__device__ __forceinline__ float gload(const G* g, long i);
template <>
__device__ __forceinline__ float gload<float>(const float* g, long i) {
  return g[i];
}
template <>
__device__ __forceinline__ float gload<__nv_bfloat16>(const __nv_bfloat16* g, long i) {
  return __bfloat162float(g[i]);
}

template <typename G>
__global__ void __launch_bounds__(256) sumsq_kernel(const G* __restrict__ g, long n, float* __restrict__ part,
                                                    float* __restrict__ hp_dev) {
  if (blockIdx.x == 0 && threadIdx.x == 0 && hp_dev[10] != 0.f) hp_dev[9] += 1.f;
  float s = 0.f;
  for (long i = blockIdx.x * 256L + threadIdx.x; i < n; i += (long)gridDim.x * 256) {
    float x = gload(g, i);
    s += x * x;
  }
  s = warp_sum(s);
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int k = 0; k < 8; ++k) t += red[k];
    part[blockIdx.x] = t;
  }
}

__device__ __forceinline__ float block_total(const float* part, int nparts) {
  __shared__ float red[8];
  __shared__ float tot;
  float s = 0.f;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) s += part[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) t += red[k];
    tot = t;
  }
  __syncthreads();
  return tot;
}

template <int MODE, typename G>
__global__ void __launch_bounds__(256)
    optim_kernel(float* __restrict__ p, float* __restrict__ s1, float* __restrict__ s2, const G* __restrict__ g,
                 __nv_bfloat16* __restrict__ p16, long n, long n_decay, const uint8_t* __restrict__ decay_mask,
                 const float* __restrict__ hp_dev, const float* __restrict__ part, int nparts,
                 float* __restrict__ norm_out) {
  HP h = *reinterpret_cast<const HP*>(hp_dev);
  if (h.dev_step != 0.f) {
    h.bc1 = 1.f - powf(h.b1, h.step);
    h.bc2 = 1.f - powf(h.b2, h.step);
  }
  float gmul = h.gmul;
  if (part != nullptr) {
    // global gradient norm (of the unscaled gradient)
    const float tot = block_total(part, nparts);
    const float norm = sqrtf(tot) * fabsf(h.gmul);
    if (blockIdx.x == 0 && threadIdx.x == 0 && norm_out != nullptr) norm_out[0] = norm;
    if (!isfinite(norm)) return;  // overflow: skip the step (GradScaler semantics)
    if (h.max_norm > 0.f && norm > h.max_norm) gmul *= h.max_norm / (norm + 1e-6f);
  }
  for (long i = blockIdx.x * 256L + threadIdx.x; i < n; i += (long)gridDim.x * 256) {
    float x = p[i];
    float gr = gload(g, i) * gmul;
    const bool dec = decay_mask ? (decay_mask[i >> 6] != 0) : (i < n_decay);
    const float wd = dec ? h.wd : 0.f;
    if (MODE == OPT_ADAM || MODE == OPT_ADAMW) {
      if (MODE == OPT_ADAM) gr += wd * x;
      float m = s1[i] * h.b1 + (1.f - h.b1) * gr;
      float v = s2[i] * h.b2 + (1.f - h.b2) * gr * gr;
      s1[i] = m;
      s2[i] = v;
      const float mh = m / h.bc1, vh = v / h.bc2;
      if (MODE == OPT_ADAMW) x *= (1.f - h.lr * wd);
      x -= h.lr * mh / (sqrtf(vh) + h.eps);
    } else if (MODE == OPT_SGD) {
      gr += wd * x;
      float v = (h.b1 > 0.f) ? (s1[i] * h.b1 + h.lr * gr) : h.lr * gr;
      if (h.b1 > 0.f) s1[i] = v;
      x -= v;
    } else if (MODE == OPT_RMSPROP) {
      gr += wd * x;
      float v = s1[i] * h.b1 + (1.f - h.b1) * gr * gr;
      s1[i] = v;
      x -= h.lr * gr / (sqrtf(v) + h.eps);
    } else {  // ADAGRAD
      gr += wd * x;
      float acc = s1[i] + gr * gr;
      s1[i] = acc;
      x -= h.lr * gr / (sqrtf(acc) + h.eps);
    }
    p[i] = x;
    if (p16 != nullptr) p16[i] = __float2bfloat16(x);
  }
}

template <int MODE, typename G>
static void launch_optim(float* p, float* s1, float* s2, const G* g, __nv_bfloat16* p16, long n, long n_decay,
                         const uint8_t* mask, const float* hp, const float* part, int nparts, float* norm_out,
                         int grid, cudaStream_t st) {
  optim_kernel<MODE, G><<<grid, 256, 0, st>>>(p, s1, s2, g, p16, n, n_decay, mask, hp, part, nparts, norm_out);
  SCIRS_CHECK_LAUNCH();
}

// params fp32 [n]; state1/state2 fp32 [n] (unused ones may be empty);
// grads fp32 or bf16 [n]; params16 optional bf16 [n];
// hp fp32 device [9]; part fp32 scratch [>= nparts] when clipping or
// non-finite detection is wanted; norm_out fp32 [1] optional.
void optim_step(int64_t mode, torch::Tensor params, torch::Tensor state1, torch::Tensor state2, torch::Tensor grads,
                c10::optional<torch::Tensor> params16, int64_t n_decay, c10::optional<torch::Tensor> decay_mask,
                torch::Tensor hp, c10::optional<torch::Tensor> part, c10::optional<torch::Tensor> norm_out,
                int64_t parts_ready) {
  CHECK_DTYPE(params, at::kFloat);
  CHECK_CONTIG(params);
  CHECK_CONTIG(grads);
  CHECK_DTYPE(hp, at::kFloat);
  TORCH_CHECK(hp.numel() >= 11 && hp.is_cuda(), "hp must be a device fp32 tensor with 11 entries");
  const long n = params.numel();
  TORCH_CHECK(grads.numel() == n, "grads size mismatch");
  c10::cuda::CUDAGuard guard(params.get_device());
  cudaStream_t st = cur_stream();
  const int sms = num_sms(params.get_device());
  const int grid = (int)std::max<long>(1, std::min<long>((n + 255) / 256, 8L * sms));
  float* pp = params.data_ptr<float>();
  float* s1 = state1.numel() ? state1.data_ptr<float>() : nullptr;
  float* s2 = state2.numel() ? state2.data_ptr<float>() : nullptr;
  if (mode != OPT_SGD || true) {
    if ((mode == OPT_ADAM || mode == OPT_ADAMW) && (s1 == nullptr || s2 == nullptr))
      TORCH_CHECK(false, "Adam needs two state buffers");
    if ((mode == OPT_RMSPROP || mode == OPT_ADAGRAD) && s1 == nullptr) TORCH_CHECK(false, "state1 required");
  }
  __nv_bfloat16* p16 = nullptr;
  if (params16.has_value() && params16->defined()) {
    CHECK_DTYPE((*params16), at::kBFloat16);
    TORCH_CHECK(params16->numel() == n, "params16 size mismatch");
    p16 = reinterpret_cast<__nv_bfloat16*>(params16->data_ptr());
  }
  float* partp = nullptr;
  int nparts = 0;
  const bool bf = grads.scalar_type() == at::kBFloat16;
  if (part.has_value() && part->defined() && parts_ready > 0) {
    // partial sums of squares already in `part` (e.g. summed over the ranks
    // that each hold one shard of the gradient)
    TORCH_CHECK(parts_ready <= part->numel(), "parts_ready exceeds part");
    nparts = (int)parts_ready;
    partp = part->data_ptr<float>();
  } else if (part.has_value() && part->defined()) {
    nparts = (int)std::min<long>(part->numel(), 2L * sms);
    partp = part->data_ptr<float>();
    if (bf)
      sumsq_kernel<__nv_bfloat16><<<nparts, 256, 0, st>>>(
          reinterpret_cast<const __nv_bfloat16*>(grads.data_ptr()), n, partp, hp.data_ptr<float>());
    else
      sumsq_kernel<float><<<nparts, 256, 0, st>>>(grads.data_ptr<float>(), n, partp, hp.data_ptr<float>());
    SCIRS_CHECK_LAUNCH();
  }
  const uint8_t* mk = nullptr;
  if (decay_mask.has_value() && decay_mask->defined()) {
    CHECK_DTYPE((*decay_mask), at::kByte);
    TORCH_CHECK(decay_mask->numel() >= (n + 63) / 64, "decay_mask needs one byte per 64 elements");
    mk = decay_mask->data_ptr<uint8_t>();
  }
  float* no = (norm_out.has_value() && norm_out->defined()) ? norm_out->data_ptr<float>() : nullptr;
  const float* hpp = hp.data_ptr<float>();
#define SCIRS_OPT_CASE(M)                                                                                   \
  case M:                                                                                                   \
    if (bf)                                                                                                 \
      launch_optim<M, __nv_bfloat16>(pp, s1, s2, reinterpret_cast<const __nv_bfloat16*>(grads.data_ptr()), \
                                     p16, n, n_decay, mk, hpp, partp, nparts, no, grid, st);                    \
    else                                                                                                    \
      launch_optim<M, float>(pp, s1, s2, grads.data_ptr<float>(), p16, n, n_decay, mk, hpp, partp, nparts, no, \
                             grid, st);                                                                     \
    break;
  switch (mode) {
    SCIRS_OPT_CASE(OPT_ADAM)
    SCIRS_OPT_CASE(OPT_ADAMW)
    SCIRS_OPT_CASE(OPT_SGD)
    SCIRS_OPT_CASE(OPT_RMSPROP)
    SCIRS_OPT_CASE(OPT_ADAGRAD)
    default: TORCH_CHECK(false, "unknown optimizer mode ", mode);
  }
#undef SCIRS_OPT_CASE
}

// Partial sums of squares of `grads` into part[0 .. nparts) (and the device
// step counter update of the optimizer). Returns nparts. Used when the global
// gradient norm needs a reduction across ranks before the update.
int64_t grad_sumsq(torch::Tensor grads, torch::Tensor part, torch::Tensor hp) {
  CHECK_CONTIG(grads);
  CHECK_DTYPE(part, at::kFloat);
  CHECK_DTYPE(hp, at::kFloat);
  TORCH_CHECK(hp.numel() >= 11 && hp.is_cuda(), "hp must be a device fp32 tensor with 11 entries");
  c10::cuda::CUDAGuard guard(grads.get_device());
  cudaStream_t st = cur_stream();
  const int nparts = (int)std::min<long>(part.numel(), 2L * num_sms(grads.get_device()));
  if (grads.scalar_type() == at::kBFloat16)
    sumsq_kernel<__nv_bfloat16><<<nparts, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(grads.data_ptr()),
                                                        grads.numel(), part.data_ptr<float>(), hp.data_ptr<float>());
  else
    sumsq_kernel<float><<<nparts, 256, 0, st>>>(grads.data_ptr<float>(), grads.numel(), part.data_ptr<float>(),
                                                hp.data_ptr<float>());
  SCIRS_CHECK_LAUNCH();
  return nparts;
}

}  // namespace scirs
