// Recurrent-cell kernels for sm_100a: the pointwise part of one time step of
// LSTM / GRU / Elman RNN, forward and backward (bf16 activations, fp32 cell
// state and math). The matrix products around them run on the tcgen05 GEMM:
// the input projection of all time steps is one GEMM before the loop, each
// step adds one [B, H] x [H, G*H] GEMM for the recurrent projection, and the
// backward pass batches dX, dW_ih and dW_hh into three GEMMs after the loop.
//
// Gate layouts (PyTorch's and the reference's order):
//   LSTM  [i, f, g, o] (4H): i, f, o = sigmoid, g = tanh;
//         c' = f * c + i * g, h' = o * tanh(c')
//   GRU   [r, z, n] (3H): r, z = sigmoid(gx + gh), n = tanh(gx_n + r * gh_n);
//         h' = (1 - z) * n + z * h
//   RNN   h' = tanh(gx + gh)
// gx / gh are the input / recurrent projections with their biases.
//
// Reference parity: scirs2-neural/src/layers/recurrent/lstm.rs:20-560,
// gru.rs, rnn.rs, cells.rs (per-step CPU loops there).
#include "host_common.h"

namespace scirs {
namespace rnn {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + __expf(-x)); }
__device__ __forceinline__ float ld(const bf16* p, long i) { return __bfloat162float(p[i]); }

// acts [B, 4H] <- (i, f, g, o) after their nonlinearities; c [B, H] fp32
// (in: c_prev, out: c'); h [B, H] bf16.
__global__ void __launch_bounds__(256) lstm_fwd_kernel(const bf16* __restrict__ gx, const bf16* __restrict__ gh,
                                                       const float* __restrict__ c_prev, float* __restrict__ c_out,
                                                       bf16* __restrict__ h_out, bf16* __restrict__ acts, int B,
                                                       int H) {
  const long n = (long)B * H;
  for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long)gridDim.x * blockDim.x) {
    const long b = e / H;
    const int j = (int)(e - b * H);
    const long base = b * 4L * H;
    float gv[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) gv[q] = ld(gx, base + q * H + j) + (gh ? ld(gh, base + q * H + j) : 0.f);
    const float i = sigm(gv[0]), f = sigm(gv[1]), g = tanhf(gv[2]), o = sigm(gv[3]);
    const float c = f * (c_prev ? c_prev[e] : 0.f) + i * g;
    c_out[e] = c;
    h_out[e] = __float2bfloat16(o * tanhf(c));
    acts[base + j] = __float2bfloat16(i);
    acts[base + H + j] = __float2bfloat16(f);
    acts[base + 2 * H + j] = __float2bfloat16(g);
    acts[base + 3 * H + j] = __float2bfloat16(o);
  }
}

// dh: gradient w.r.t. h' (bf16), dc: in = gradient w.r.t. c' (fp32, may be
// null for zero), out = gradient w.r.t. c_prev; dgates [B, 4H] bf16 =
// gradient w.r.t. the pre-activations.
__global__ void __launch_bounds__(256) lstm_bwd_kernel(const bf16* __restrict__ dh, const float* __restrict__ dc_in,
                                                       const bf16* __restrict__ acts, const float* __restrict__ c_prev,
                                                       const float* __restrict__ c, float* __restrict__ dc_out,
                                                       bf16* __restrict__ dgates, int B, int H) {
  const long n = (long)B * H;
  for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long)gridDim.x * blockDim.x) {
    const long b = e / H;
    const int j = (int)(e - b * H);
    const long base = b * 4L * H;
    const float i = ld(acts, base + j), f = ld(acts, base + H + j), g = ld(acts, base + 2 * H + j),
                o = ld(acts, base + 3 * H + j);
    const float tc = tanhf(c[e]);
    const float gh = ld(dh, e);
    const float dct = (dc_in ? dc_in[e] : 0.f) + gh * o * (1.f - tc * tc);
    const float cp = c_prev ? c_prev[e] : 0.f;
    dgates[base + j] = __float2bfloat16(dct * g * i * (1.f - i));
    dgates[base + H + j] = __float2bfloat16(dct * cp * f * (1.f - f));
    dgates[base + 2 * H + j] = __float2bfloat16(dct * i * (1.f - g * g));
    dgates[base + 3 * H + j] = __float2bfloat16(gh * tc * o * (1.f - o));
    dc_out[e] = dct * f;
  }
}

// GRU: acts [B, 4H] <- (r, z, n, gh_n) (gh_n = the recurrent projection of
// the n gate, needed by the backward); h_prev may be null (zeros).
__global__ void __launch_bounds__(256) gru_fwd_kernel(const bf16* __restrict__ gx, const bf16* __restrict__ gh,
                                                      const bf16* __restrict__ h_prev, bf16* __restrict__ h_out,
                                                      bf16* __restrict__ acts, int B, int H) {
  const long n = (long)B * H;
  for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long)gridDim.x * blockDim.x) {
    const long b = e / H;
    const int j = (int)(e - b * H);
    const long g3 = b * 3L * H;
    const float hr = gh ? ld(gh, g3 + j) : 0.f, hz = gh ? ld(gh, g3 + H + j) : 0.f,
                hn = gh ? ld(gh, g3 + 2 * H + j) : 0.f;
    const float r = sigm(ld(gx, g3 + j) + hr), z = sigm(ld(gx, g3 + H + j) + hz);
    const float nn = tanhf(ld(gx, g3 + 2 * H + j) + r * hn);
    const float hp = h_prev ? ld(h_prev, e) : 0.f;
    h_out[e] = __float2bfloat16((1.f - z) * nn + z * hp);
    const long a4 = b * 4L * H;
    acts[a4 + j] = __float2bfloat16(r);
    acts[a4 + H + j] = __float2bfloat16(z);
    acts[a4 + 2 * H + j] = __float2bfloat16(nn);
    acts[a4 + 3 * H + j] = __float2bfloat16(hn);
  }
}

// dgx [B, 3H] (pre-activation grads of the input projection), dgh [B, 3H]
// (of the recurrent projection: r and z equal dgx, n gets r * dn), dh_prev
// [B, H] fp32 (direct path z * dh only; the caller adds dgh @ W_hh).
__global__ void __launch_bounds__(256) gru_bwd_kernel(const bf16* __restrict__ dh, const bf16* __restrict__ acts,
                                                      const bf16* __restrict__ h_prev, bf16* __restrict__ dgx,
                                                      bf16* __restrict__ dgh, float* __restrict__ dh_prev, int B,
                                                      int H) {
  const long n = (long)B * H;
  for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long)gridDim.x * blockDim.x) {
    const long b = e / H;
    const int j = (int)(e - b * H);
    const long a4 = b * 4L * H, g3 = b * 3L * H;
    const float r = ld(acts, a4 + j), z = ld(acts, a4 + H + j), nn = ld(acts, a4 + 2 * H + j),
                hn = ld(acts, a4 + 3 * H + j);
    const float g = ld(dh, e);
    const float hp = h_prev ? ld(h_prev, e) : 0.f;
    const float dn = g * (1.f - z) * (1.f - nn * nn);
    const float dz = g * (hp - nn) * z * (1.f - z);
    const float dr = dn * hn * r * (1.f - r);
    dgx[g3 + j] = __float2bfloat16(dr);
    dgx[g3 + H + j] = __float2bfloat16(dz);
    dgx[g3 + 2 * H + j] = __float2bfloat16(dn);
    dgh[g3 + j] = __float2bfloat16(dr);
    dgh[g3 + H + j] = __float2bfloat16(dz);
    dgh[g3 + 2 * H + j] = __float2bfloat16(dn * r);
    dh_prev[e] = g * z;
  }
}

__global__ void __launch_bounds__(256) rnn_fwd_kernel(const bf16* __restrict__ gx, const bf16* __restrict__ gh,
                                                      bf16* __restrict__ h_out, long n) {
  for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long)gridDim.x * blockDim.x)
    h_out[e] = __float2bfloat16(tanhf(ld(gx, e) + (gh ? ld(gh, e) : 0.f)));
}

__global__ void __launch_bounds__(256) rnn_bwd_kernel(const bf16* __restrict__ dh, const bf16* __restrict__ h,
                                                      bf16* __restrict__ dg, long n) {
  for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long)gridDim.x * blockDim.x) {
    const float y = ld(h, e);
    dg[e] = __float2bfloat16(ld(dh, e) * (1.f - y * y));
  }
}

// out (bf16) = a (bf16) + b (fp32): the recurrent gradient dh_t = dy_t +
// dh_from_next (the sum feeds the next cell backward)
__global__ void __launch_bounds__(256) add_bf16_f32_kernel(const bf16* __restrict__ a, const float* __restrict__ b,
                                                           bf16* __restrict__ out, long n) {
  for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (long)gridDim.x * blockDim.x)
    out[e] = __float2bfloat16(ld(a, e) + (b ? b[e] : 0.f));
}

static int grid_for(long work, int dev) {
  return (int)std::max<long>(1, std::min<long>((work + 255) / 256, 8L * num_sms(dev)));
}

template <typename T>
static T* opt_ptr(const c10::optional<torch::Tensor>& t) {
  return (t.has_value() && t->defined()) ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

}  // namespace rnn

#define RNN_BF16(t) reinterpret_cast<__nv_bfloat16*>((t).data_ptr())
#define RNN_CBF16(t) reinterpret_cast<const __nv_bfloat16*>((t).data_ptr())

void lstm_cell_fwd(torch::Tensor gx, c10::optional<torch::Tensor> gh, c10::optional<torch::Tensor> c_prev,
                   torch::Tensor c_out, torch::Tensor h_out, torch::Tensor acts) {
  const int B = (int)h_out.size(0), H = (int)h_out.size(1);
  TORCH_CHECK(gx.numel() == 4L * B * H && acts.numel() == 4L * B * H && c_out.numel() == (long)B * H, "lstm shapes");
  CHECK_DTYPE(c_out, at::kFloat);
  const int dev = gx.get_device();
  c10::cuda::CUDAGuard guard(dev);
  rnn::lstm_fwd_kernel<<<rnn::grid_for((long)B * H, dev), 256, 0, cur_stream()>>>(
      RNN_CBF16(gx), rnn::opt_ptr<const __nv_bfloat16>(gh), rnn::opt_ptr<const float>(c_prev), c_out.data_ptr<float>(),
      RNN_BF16(h_out), RNN_BF16(acts), B, H);
  SCIRS_CHECK_LAUNCH();
}

void lstm_cell_bwd(torch::Tensor dh, c10::optional<torch::Tensor> dc_in, torch::Tensor acts,
                   c10::optional<torch::Tensor> c_prev, torch::Tensor c, torch::Tensor dc_out, torch::Tensor dgates) {
  const int B = (int)dh.size(0), H = (int)dh.size(1);
  TORCH_CHECK(acts.numel() == 4L * B * H && dgates.numel() == 4L * B * H, "lstm shapes");
  const int dev = dh.get_device();
  c10::cuda::CUDAGuard guard(dev);
  rnn::lstm_bwd_kernel<<<rnn::grid_for((long)B * H, dev), 256, 0, cur_stream()>>>(
      RNN_CBF16(dh), rnn::opt_ptr<const float>(dc_in), RNN_CBF16(acts), rnn::opt_ptr<const float>(c_prev),
      c.data_ptr<float>(), dc_out.data_ptr<float>(), RNN_BF16(dgates), B, H);
  SCIRS_CHECK_LAUNCH();
}

void gru_cell_fwd(torch::Tensor gx, c10::optional<torch::Tensor> gh, c10::optional<torch::Tensor> h_prev,
                  torch::Tensor h_out, torch::Tensor acts) {
  const int B = (int)h_out.size(0), H = (int)h_out.size(1);
  TORCH_CHECK(gx.numel() == 3L * B * H && acts.numel() == 4L * B * H, "gru shapes");
  const int dev = gx.get_device();
  c10::cuda::CUDAGuard guard(dev);
  rnn::gru_fwd_kernel<<<rnn::grid_for((long)B * H, dev), 256, 0, cur_stream()>>>(
      RNN_CBF16(gx), rnn::opt_ptr<const __nv_bfloat16>(gh), rnn::opt_ptr<const __nv_bfloat16>(h_prev),
      RNN_BF16(h_out), RNN_BF16(acts), B, H);
  SCIRS_CHECK_LAUNCH();
}

void gru_cell_bwd(torch::Tensor dh, torch::Tensor acts, c10::optional<torch::Tensor> h_prev, torch::Tensor dgx,
                  torch::Tensor dgh, torch::Tensor dh_prev) {
  const int B = (int)dh.size(0), H = (int)dh.size(1);
  TORCH_CHECK(dgx.numel() == 3L * B * H && dgh.numel() == 3L * B * H && dh_prev.numel() == (long)B * H, "gru shapes");
  const int dev = dh.get_device();
  c10::cuda::CUDAGuard guard(dev);
  rnn::gru_bwd_kernel<<<rnn::grid_for((long)B * H, dev), 256, 0, cur_stream()>>>(
      RNN_CBF16(dh), RNN_CBF16(acts), rnn::opt_ptr<const __nv_bfloat16>(h_prev), RNN_BF16(dgx), RNN_BF16(dgh),
      dh_prev.data_ptr<float>(), B, H);
  SCIRS_CHECK_LAUNCH();
}

void rnn_cell_fwd(torch::Tensor gx, c10::optional<torch::Tensor> gh, torch::Tensor h_out) {
  const int dev = gx.get_device();
  c10::cuda::CUDAGuard guard(dev);
  rnn::rnn_fwd_kernel<<<rnn::grid_for(h_out.numel(), dev), 256, 0, cur_stream()>>>(
      RNN_CBF16(gx), rnn::opt_ptr<const __nv_bfloat16>(gh), RNN_BF16(h_out), h_out.numel());
  SCIRS_CHECK_LAUNCH();
}

void rnn_cell_bwd(torch::Tensor dh, torch::Tensor h, torch::Tensor dg) {
  const int dev = dh.get_device();
  c10::cuda::CUDAGuard guard(dev);
  rnn::rnn_bwd_kernel<<<rnn::grid_for(dh.numel(), dev), 256, 0, cur_stream()>>>(RNN_CBF16(dh), RNN_CBF16(h),
                                                                                  RNN_BF16(dg), dh.numel());
  SCIRS_CHECK_LAUNCH();
}

void add_bf16_f32(torch::Tensor a, c10::optional<torch::Tensor> b, torch::Tensor out) {
  const int dev = a.get_device();
  c10::cuda::CUDAGuard guard(dev);
  rnn::add_bf16_f32_kernel<<<rnn::grid_for(a.numel(), dev), 256, 0, cur_stream()>>>(
      RNN_CBF16(a), rnn::opt_ptr<const float>(b), RNN_BF16(out), a.numel());
  SCIRS_CHECK_LAUNCH();
}

#undef RNN_BF16
#undef RNN_CBF16

}  // namespace scirs
