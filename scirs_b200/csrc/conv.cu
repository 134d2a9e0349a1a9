// Convolution and pooling kernels for sm_100a (NCHW, bf16 data).
//
// Conv2D runs as an implicit-GEMM pipeline around the framework's tcgen05
// GEMM (gemm_sm100.cu):
//   forward   im2col_kernel: x [N, C, H, W] -> cols [N*OH*OW, Kp] (column
//             k = (c * KH + kh) * KW + kw, zero for padding taps and for the
//             pad columns K <= k < Kp, Kp = K rounded up to 8 so TMA rows are
//             16-byte multiples); y_rows = cols @ W^T (+bias) on tensor cores
//   backward  dcols = dy_rows @ W (GEMM), col2im_kernel gathers every input
//             pixel's taps from dcols in a fixed order (deterministic, no
//             atomics); dW = dy_rows^T @ cols (GEMM, fp32); dbias = column sums
// Pooling: max / average 2-D pooling forward (max records the argmax) and
// backward (max scatters through the recorded argmax, which is unique per
// output so writes never collide; average gathers like col2im).
//
// Reference parity: scirs2-neural/src/layers/conv/conv2d.rs:284-400
// (im2col + GEMM forward), :608-624 (backward), layers/conv/pooling.rs
// (max / average pooling), scirs2-core/src/gpu/kernels/ml/pooling (CUDA
// source strings, never launched there).
#include "host_common.h"

namespace scirs {
namespace conv {

using bf16 = __nv_bfloat16;

struct Geom {
  int N, C, H, W, KH, KW, OH, OW, sh, sw, ph, pw, dh, dw;
  long K, Kp;
};

// One thread writes 8 consecutive columns (16 bytes) of one cols row.
__global__ void __launch_bounds__(256) im2col_kernel(const bf16* __restrict__ x, bf16* __restrict__ cols, Geom g,
                                                     long rows) {
  const long vec_per_row = g.Kp / 8;
  const long total = rows * vec_per_row;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long r = i / vec_per_row;
    const int k0 = (int)(i - r * vec_per_row) * 8;
    const int ow = (int)(r % g.OW);
    const long t = r / g.OW;
    const int oh = (int)(t % g.OH);
    const int n = (int)(t / g.OH);
    __align__(16) bf16 v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int k = k0 + e;
      float val = 0.f;
      if (k < g.K) {
        const int kw = k % g.KW;
        const int kh = (k / g.KW) % g.KH;
        const int c = k / (g.KW * g.KH);
        const int h = oh * g.sh - g.ph + kh * g.dh;
        const int w = ow * g.sw - g.pw + kw * g.dw;
        if (h >= 0 && h < g.H && w >= 0 && w < g.W)
          val = __bfloat162float(x[(((long)n * g.C + c) * g.H + h) * g.W + w]);
      }
      v[e] = __float2bfloat16(val);
    }
    *reinterpret_cast<uint4*>(cols + r * g.Kp + k0) = *reinterpret_cast<const uint4*>(v);
  }
}

// dx[n, c, h, w] = sum over taps (kh, kw) whose output position lies on the
// stride grid and inside the output of dcols[(n, oh, ow), (c, kh, kw)].
__global__ void __launch_bounds__(256) col2im_kernel(const bf16* __restrict__ dcols, bf16* __restrict__ dx, Geom g) {
  const long total = (long)g.N * g.C * g.H * g.W;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int w = (int)(i % g.W);
    const int h = (int)((i / g.W) % g.H);
    const int c = (int)((i / ((long)g.W * g.H)) % g.C);
    const int n = (int)(i / ((long)g.W * g.H * g.C));
    float acc = 0.f;
    for (int kh = 0; kh < g.KH; ++kh) {
      const int hh = h + g.ph - kh * g.dh;
      if (hh < 0 || hh % g.sh) continue;
      const int oh = hh / g.sh;
      if (oh >= g.OH) continue;
      for (int kw = 0; kw < g.KW; ++kw) {
        const int ww = w + g.pw - kw * g.dw;
        if (ww < 0 || ww % g.sw) continue;
        const int ow = ww / g.sw;
        if (ow >= g.OW) continue;
        const long r = ((long)n * g.OH + oh) * g.OW + ow;
        acc += __bfloat162float(dcols[r * g.Kp + ((long)c * g.KH + kh) * g.KW + kw]);
      }
    }
    dx[i] = __float2bfloat16(acc);
  }
}

// rows [N*OH*OW, ldr] (NHWC order, first C columns used) <-> NCHW
__global__ void __launch_bounds__(256) rows_to_nchw_kernel(const bf16* __restrict__ rows, long ldr,
                                                           bf16* __restrict__ y, int N, int C, int HW) {
  const long total = (long)N * C * HW;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int p = (int)(i % HW);
    const int c = (int)((i / HW) % C);
    const long n = i / ((long)HW * C);
    y[i] = rows[(n * HW + p) * ldr + c];
  }
}

__global__ void __launch_bounds__(256) nchw_to_rows_kernel(const bf16* __restrict__ y, bf16* __restrict__ rows,
                                                           long ldr, int N, int C, int HW) {
  const long total = (long)N * HW * ldr;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int c = (int)(i % ldr);
    const long r = i / ldr;
    const int p = (int)(r % HW);
    const long n = r / HW;
    rows[i] = c < C ? y[(n * C + c) * HW + p] : __float2bfloat16(0.f);
  }
}

// ------------------------------------------------------------------ pooling
__global__ void __launch_bounds__(256) pool_fwd_kernel(const bf16* __restrict__ x, bf16* __restrict__ y,
                                                       int* __restrict__ arg, Geom g, int is_max, int count_pad) {
  const long total = (long)g.N * g.C * g.OH * g.OW;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int ow = (int)(i % g.OW);
    const int oh = (int)((i / g.OW) % g.OH);
    const long nc = i / ((long)g.OW * g.OH);
    const bf16* xp = x + nc * g.H * g.W;
    float best = -INFINITY, sum = 0.f;
    int bi = -1, cnt = 0;
    for (int kh = 0; kh < g.KH; ++kh) {
      const int h = oh * g.sh - g.ph + kh;
      for (int kw = 0; kw < g.KW; ++kw) {
        const int w = ow * g.sw - g.pw + kw;
        if (h < 0 || h >= g.H || w < 0 || w >= g.W) continue;
        const float v = __bfloat162float(xp[h * g.W + w]);
        ++cnt;
        sum += v;
        if (v > best || bi < 0) best = v, bi = h * g.W + w;
      }
    }
    if (is_max) {
      y[i] = __float2bfloat16(best);
      arg[i] = bi;
    } else {
      const int div = count_pad ? g.KH * g.KW : max(cnt, 1);
      y[i] = __float2bfloat16(sum / (float)div);
    }
  }
}

// Max: each output owns one input position (its argmax); zero the input
// gradient first, then add. Windows may overlap, so one input can be the
// argmax of several outputs: fp32 atomics into a zeroed fp32 buffer.
__global__ void __launch_bounds__(256) maxpool_bwd_kernel(const bf16* __restrict__ dy, const int* __restrict__ arg,
                                                          float* __restrict__ dx, Geom g) {
  const long total = (long)g.N * g.C * g.OH * g.OW;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long nc = i / ((long)g.OW * g.OH);
    const int a = arg[i];
    if (a >= 0) atomicAdd(dx + nc * g.H * g.W + a, __bfloat162float(dy[i]));
  }
}

__global__ void __launch_bounds__(256) avgpool_bwd_kernel(const bf16* __restrict__ dy, bf16* __restrict__ dx, Geom g,
                                                          int count_pad) {
  const long total = (long)g.N * g.C * g.H * g.W;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int w = (int)(i % g.W);
    const int h = (int)((i / g.W) % g.H);
    const long nc = i / ((long)g.W * g.H);
    float acc = 0.f;
    for (int kh = 0; kh < g.KH; ++kh) {
      const int hh = h + g.ph - kh;
      if (hh < 0 || hh % g.sh) continue;
      const int oh = hh / g.sh;
      if (oh >= g.OH) continue;
      for (int kw = 0; kw < g.KW; ++kw) {
        const int ww = w + g.pw - kw;
        if (ww < 0 || ww % g.sw) continue;
        const int ow = ww / g.sw;
        if (ow >= g.OW) continue;
        int div = g.KH * g.KW;
        if (!count_pad) {
          const int h0 = oh * g.sh - g.ph, w0 = ow * g.sw - g.pw;
          const int hs = max(h0, 0), he = min(h0 + g.KH, g.H), ws = max(w0, 0), we = min(w0 + g.KW, g.W);
          div = max((he - hs) * (we - ws), 1);
        }
        acc += __bfloat162float(dy[(nc * g.OH + oh) * g.OW + ow]) / (float)div;
      }
    }
    dx[i] = __float2bfloat16(acc);
  }
}

static int grid_for(long work, int dev) {
  return (int)std::max<long>(1, std::min<long>((work + 255) / 256, 16L * num_sms(dev)));
}

static Geom geom(const torch::Tensor& x, int64_t KH, int64_t KW, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                 int64_t dh, int64_t dw) {
  TORCH_CHECK(x.dim() == 4, "input must be NCHW");
  Geom g{};
  g.N = (int)x.size(0), g.C = (int)x.size(1), g.H = (int)x.size(2), g.W = (int)x.size(3);
  g.KH = (int)KH, g.KW = (int)KW, g.sh = (int)sh, g.sw = (int)sw, g.ph = (int)ph, g.pw = (int)pw;
  g.dh = (int)dh, g.dw = (int)dw;
  TORCH_CHECK(g.sh > 0 && g.sw > 0 && g.dh > 0 && g.dw > 0 && g.KH > 0 && g.KW > 0, "bad conv geometry");
  g.OH = (g.H + 2 * g.ph - g.dh * (g.KH - 1) - 1) / g.sh + 1;
  g.OW = (g.W + 2 * g.pw - g.dw * (g.KW - 1) - 1) / g.sw + 1;
  TORCH_CHECK(g.OH > 0 && g.OW > 0, "empty conv output");
  g.K = (long)g.C * g.KH * g.KW;
  g.Kp = (g.K + 7) / 8 * 8;
  return g;
}

}  // namespace conv

// cols [N*OH*OW, Kp] bf16 from x [N, C, H, W] bf16
void conv_im2col(torch::Tensor x, torch::Tensor cols, int64_t KH, int64_t KW, int64_t sh, int64_t sw, int64_t ph,
                 int64_t pw, int64_t dh, int64_t dw) {
  CHECK_DTYPE(x, at::kBFloat16);
  CHECK_CONTIG(x);
  CHECK_DTYPE(cols, at::kBFloat16);
  CHECK_CONTIG(cols);
  conv::Geom g = conv::geom(x, KH, KW, sh, sw, ph, pw, dh, dw);
  const long rows = (long)g.N * g.OH * g.OW;
  TORCH_CHECK(cols.dim() == 2 && cols.size(0) == rows && cols.size(1) == g.Kp, "cols must be [N*OH*OW, Kp]");
  const int dev = x.get_device();
  c10::cuda::CUDAGuard guard(dev);
  conv::im2col_kernel<<<conv::grid_for(rows * (g.Kp / 8), dev), 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<__nv_bfloat16*>(cols.data_ptr()), g,
      rows);
  SCIRS_CHECK_LAUNCH();
}

// dx [N, C, H, W] bf16 from dcols [N*OH*OW, Kp] bf16 (x gives the geometry)
void conv_col2im(torch::Tensor dcols, torch::Tensor dx, int64_t KH, int64_t KW, int64_t sh, int64_t sw, int64_t ph,
                 int64_t pw, int64_t dh, int64_t dw) {
  CHECK_DTYPE(dcols, at::kBFloat16);
  CHECK_CONTIG(dcols);
  CHECK_DTYPE(dx, at::kBFloat16);
  CHECK_CONTIG(dx);
  conv::Geom g = conv::geom(dx, KH, KW, sh, sw, ph, pw, dh, dw);
  TORCH_CHECK(dcols.dim() == 2 && dcols.size(0) == (long)g.N * g.OH * g.OW && dcols.size(1) == g.Kp,
              "dcols must be [N*OH*OW, Kp]");
  const int dev = dx.get_device();
  c10::cuda::CUDAGuard guard(dev);
  conv::col2im_kernel<<<conv::grid_for(dx.numel(), dev), 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dcols.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), g);
  SCIRS_CHECK_LAUNCH();
}

// y [N, C, H*W] NCHW <- rows [N*H*W, ldr] (first C columns), or the reverse
void conv_rows_nchw(torch::Tensor rows, torch::Tensor y, bool to_nchw) {
  CHECK_DTYPE(rows, at::kBFloat16);
  CHECK_DTYPE(y, at::kBFloat16);
  CHECK_CONTIG(y);
  TORCH_CHECK(rows.dim() == 2 && rows.stride(1) == 1 && y.dim() == 4, "rows [N*H*W, ld], y [N, C, H, W]");
  const int N = (int)y.size(0), C = (int)y.size(1), HW = (int)(y.size(2) * y.size(3));
  TORCH_CHECK(rows.size(0) == (long)N * HW && rows.size(1) >= C, "rows shape mismatch");
  const int dev = y.get_device();
  c10::cuda::CUDAGuard guard(dev);
  if (to_nchw) {
    conv::rows_to_nchw_kernel<<<conv::grid_for(y.numel(), dev), 256, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(rows.data_ptr()), rows.stride(0),
        reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), N, C, HW);
  } else {
    TORCH_CHECK(rows.is_contiguous(), "rows must be contiguous");
    conv::nchw_to_rows_kernel<<<conv::grid_for(rows.numel(), dev), 256, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(y.data_ptr()), reinterpret_cast<__nv_bfloat16*>(rows.data_ptr()),
        rows.size(1), N, C, HW);
  }
  SCIRS_CHECK_LAUNCH();
}

void pool2d_fwd(torch::Tensor x, torch::Tensor y, c10::optional<torch::Tensor> arg, int64_t KH, int64_t KW,
                int64_t sh, int64_t sw, int64_t ph, int64_t pw, bool is_max, bool count_pad) {
  CHECK_DTYPE(x, at::kBFloat16);
  CHECK_CONTIG(x);
  CHECK_DTYPE(y, at::kBFloat16);
  CHECK_CONTIG(y);
  conv::Geom g = conv::geom(x, KH, KW, sh, sw, ph, pw, 1, 1);
  TORCH_CHECK(y.dim() == 4 && y.size(2) == g.OH && y.size(3) == g.OW, "y must be [N, C, OH, OW]");
  int* ap = nullptr;
  if (is_max) {
    TORCH_CHECK(arg.has_value() && arg->defined() && arg->scalar_type() == at::kInt && arg->numel() == y.numel(),
                "max pooling needs an int32 argmax buffer like y");
    ap = arg->data_ptr<int>();
  }
  const int dev = x.get_device();
  c10::cuda::CUDAGuard guard(dev);
  conv::pool_fwd_kernel<<<conv::grid_for(y.numel(), dev), 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), ap, g,
      (int)is_max, (int)count_pad);
  SCIRS_CHECK_LAUNCH();
}

// dx: fp32 (max; zeroed here) or bf16 (average)
void pool2d_bwd(torch::Tensor dy, torch::Tensor dx, c10::optional<torch::Tensor> arg, int64_t KH, int64_t KW,
                int64_t sh, int64_t sw, int64_t ph, int64_t pw, bool is_max, bool count_pad) {
  CHECK_DTYPE(dy, at::kBFloat16);
  CHECK_CONTIG(dy);
  CHECK_CONTIG(dx);
  conv::Geom g = conv::geom(dx, KH, KW, sh, sw, ph, pw, 1, 1);
  TORCH_CHECK(dy.dim() == 4 && dy.size(2) == g.OH && dy.size(3) == g.OW, "dy must be [N, C, OH, OW]");
  const int dev = dy.get_device();
  c10::cuda::CUDAGuard guard(dev);
  if (is_max) {
    CHECK_DTYPE(dx, at::kFloat);
    TORCH_CHECK(arg.has_value() && arg->defined() && arg->numel() == dy.numel(), "argmax buffer required");
    SCIRS_CHECK_CUDA(cudaMemsetAsync(dx.data_ptr(), 0, dx.numel() * sizeof(float), cur_stream()));
    conv::maxpool_bwd_kernel<<<conv::grid_for(dy.numel(), dev), 256, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), arg->data_ptr<int>(), dx.data_ptr<float>(), g);
  } else {
    CHECK_DTYPE(dx, at::kBFloat16);
    conv::avgpool_bwd_kernel<<<conv::grid_for(dx.numel(), dev), 256, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dx.data_ptr()), g,
        (int)count_pad);
  }
  SCIRS_CHECK_LAUNCH();
}

}  // namespace scirs
