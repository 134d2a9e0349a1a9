// Vision-transformer input kernels: patch extraction (im2col of a
// stride == kernel convolution) and the [CLS] + position-embedding assembly,
// forward and backward.
//
// The reference's ViT (scirs2-neural/src/models/architectures/vit.rs:296-470)
// is commented out pending a PatchEmbedding layer; these kernels provide the
// patch embedding as a gather into GEMM rows, so the projection itself runs
// on the tcgen05 GEMM.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include "host_common.h"

namespace scirs {
namespace vision {

// One thread moves 8 contiguous pixels of one patch row (16-byte store).
// imgs [B, C, H, W] (fp32 or bf16), out [B * (H/P) * (W/P), C * P * P] bf16;
// column index c * P * P + ky * P + kx, i.e. a conv weight [E, C, P, P]
// flattened row-major is the GEMM's B operand.
template <typename T>
__global__ void patchify_kernel(const T* __restrict__ img, __nv_bfloat16* __restrict__ out, int B, int C, int H,
                                int W, int P) {
  const int gx = W / P, gy = H / P, np = gx * gy, v8 = P / 8;
  const long total = (long)B * np * C * P * v8;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    long r = i;
    const int kv = r % v8;
    r /= v8;
    const int ky = r % P;
    r /= P;
    const int c = r % C;
    r /= C;
    const int pidx = r % np;
    const int b = (int)(r / np);
    const int py = pidx / gx, px = pidx % gx;
    const long src = (((long)b * C + c) * H + (long)py * P + ky) * W + (long)px * P + kv * 8;
    float f[8];
    if constexpr (sizeof(T) == 4) {
      const float4 a = *reinterpret_cast<const float4*>(img + src);
      const float4 bq = *reinterpret_cast<const float4*>(img + src + 4);
      f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w, f[4] = bq.x, f[5] = bq.y, f[6] = bq.z, f[7] = bq.w;
    } else {
      const uint4 u = *reinterpret_cast<const uint4*>(img + src);
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
      for (int k = 0; k < 8; ++k) f[k] = __bfloat162float(h[k]);
    }
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) oh[k] = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
    const long dst = ((long)b * np + pidx) * ((long)C * P * P) + (long)c * P * P + ky * P + kv * 8;
    *reinterpret_cast<uint4*>(out + dst) = o;
  }
}

// x[b*T + t] = (t == 0 ? cls : pe[b*np + t - 1]) + pos[t]; T = np + 1.
__global__ void embed_fwd_kernel(const __nv_bfloat16* __restrict__ pe, const __nv_bfloat16* __restrict__ cls,
                                 const __nv_bfloat16* __restrict__ pos, __nv_bfloat16* __restrict__ x, int B, int T,
                                 int D) {
  const int dv = D / 8;
  const long total = (long)B * T * dv;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int j = i % dv;
    const long row = i / dv;
    const int t = row % T, b = (int)(row / T);
    const __nv_bfloat16* src = t == 0 ? cls : pe + ((long)b * (T - 1) + t - 1) * D;
    const uint4 a = *reinterpret_cast<const uint4*>(src + j * 8);
    const uint4 p = *reinterpret_cast<const uint4*>(pos + (long)t * D + j * 8);
    const __nv_bfloat162* ah = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* ph = reinterpret_cast<const __nv_bfloat162*>(&p);
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 fa = __bfloat1622float2(ah[k]), fp = __bfloat1622float2(ph[k]);
      oh[k] = __floats2bfloat162_rn(fa.x + fp.x, fa.y + fp.y);
    }
    *reinterpret_cast<uint4*>(x + row * D + j * 8) = o;
  }
}

// Backward of embed_fwd: dpe[b*np + t-1] = dx[b*T + t] (t >= 1),
// dpos[t] += sum_b dx[b*T + t], dcls += sum_b dx[b*T]. One thread owns a
// (token, 8-column) strip and sums over the batch in a fixed order, so the
// result is deterministic (no atomics).
__global__ void embed_bwd_kernel(const __nv_bfloat16* __restrict__ dx, __nv_bfloat16* __restrict__ dpe,
                                 float* __restrict__ dpos, float* __restrict__ dcls, int B, int T, int D) {
  const int dv = D / 8;
  const long total = (long)T * dv;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int j = i % dv, t = (int)(i / dv);
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int b = 0; b < B; ++b) {
      const uint4 u = *reinterpret_cast<const uint4*>(dx + ((long)b * T + t) * D + j * 8);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(h[k]);
        s[2 * k] += f.x, s[2 * k + 1] += f.y;
      }
      if (t > 0) *reinterpret_cast<uint4*>(dpe + ((long)b * (T - 1) + t - 1) * D + j * 8) = u;
    }
    float4* dp = reinterpret_cast<float4*>(dpos + (long)t * D + j * 8);
    float4 a = dp[0], c = dp[1];
    a.x += s[0], a.y += s[1], a.z += s[2], a.w += s[3], c.x += s[4], c.y += s[5], c.z += s[6], c.w += s[7];
    dp[0] = a, dp[1] = c;
    if (t == 0) {
      float4* dc = reinterpret_cast<float4*>(dcls + j * 8);
      float4 e = dc[0], g = dc[1];
      e.x += s[0], e.y += s[1], e.z += s[2], e.w += s[3], g.x += s[4], g.y += s[5], g.z += s[6], g.w += s[7];
      dc[0] = e, dc[1] = g;
    }
  }
}

static int grid_for(long work, int dev) { return (int)std::max<long>(1, std::min<long>((work + 255) / 256, 16L * num_sms(dev))); }

}  // namespace vision

void patchify(torch::Tensor img, torch::Tensor out, int64_t patch) {
  TORCH_CHECK(img.is_cuda(), "images must be on the GPU");
  CHECK_CONTIG(img);
  CHECK_CONTIG(out);
  CHECK_DTYPE(out, at::kBFloat16);
  TORCH_CHECK(img.dim() == 4, "images must be [B, C, H, W]");
  const int B = img.size(0), C = img.size(1), H = img.size(2), W = img.size(3), P = (int)patch;
  TORCH_CHECK(P % 8 == 0 && H % P == 0 && W % P == 0, "patch must be a multiple of 8 dividing H and W");
  TORCH_CHECK(out.numel() == (long)B * (H / P) * (W / P) * C * P * P, "out has the wrong size");
  c10::cuda::CUDAGuard guard(img.get_device());
  const long work = (long)B * (H / P) * (W / P) * C * P * (P / 8);
  const int grid = vision::grid_for(work, img.get_device());
  auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (img.scalar_type() == at::kFloat)
    vision::patchify_kernel<float><<<grid, 256, 0, cur_stream()>>>(img.data_ptr<float>(), o, B, C, H, W, P);
  else if (img.scalar_type() == at::kBFloat16)
    vision::patchify_kernel<__nv_bfloat16><<<grid, 256, 0, cur_stream()>>>(
        reinterpret_cast<const __nv_bfloat16*>(img.data_ptr()), o, B, C, H, W, P);
  else
    TORCH_CHECK(false, "images must be fp32 or bf16");
  SCIRS_CHECK_LAUNCH();
}

void vit_embed_fwd(torch::Tensor pe, torch::Tensor cls, torch::Tensor pos, torch::Tensor x, int64_t B) {
  CHECK_CONTIG(pe);
  CHECK_CONTIG(cls);
  CHECK_CONTIG(pos);
  CHECK_CONTIG(x);
  CHECK_DTYPE(x, at::kBFloat16);
  const int D = x.size(-1);
  const int T = pos.size(0);
  TORCH_CHECK(D % 8 == 0, "embedding width must be a multiple of 8");
  TORCH_CHECK(x.numel() == B * T * D && pe.numel() == B * (T - 1) * D && cls.numel() == D, "shape mismatch");
  c10::cuda::CUDAGuard guard(x.get_device());
  const int grid = vision::grid_for(B * T * (D / 8), x.get_device());
  vision::embed_fwd_kernel<<<grid, 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(pe.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(cls.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(pos.data_ptr()), reinterpret_cast<__nv_bfloat16*>(x.data_ptr()), (int)B,
      T, D);
  SCIRS_CHECK_LAUNCH();
}

void vit_embed_bwd(torch::Tensor dx, torch::Tensor dpe, torch::Tensor dpos, torch::Tensor dcls, int64_t B) {
  CHECK_CONTIG(dx);
  CHECK_CONTIG(dpe);
  CHECK_CONTIG(dpos);
  CHECK_CONTIG(dcls);
  CHECK_DTYPE(dpos, at::kFloat);
  CHECK_DTYPE(dcls, at::kFloat);
  const int D = dx.size(-1);
  const int T = dpos.size(0);
  TORCH_CHECK(D % 8 == 0, "embedding width must be a multiple of 8");
  TORCH_CHECK(dx.numel() == B * T * D && dpe.numel() == B * (T - 1) * D && dcls.numel() == D, "shape mismatch");
  c10::cuda::CUDAGuard guard(dx.get_device());
  const int grid = vision::grid_for((long)T * (D / 8), dx.get_device());
  vision::embed_bwd_kernel<<<grid, 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dx.data_ptr()), reinterpret_cast<__nv_bfloat16*>(dpe.data_ptr()),
      dpos.data_ptr<float>(), dcls.data_ptr<float>(), (int)B, T, D);
  SCIRS_CHECK_LAUNCH();
}

}  // namespace scirs
