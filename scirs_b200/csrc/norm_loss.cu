// Memory-bound training kernels for sm_100a: LayerNorm forward/backward,
// fused softmax cross-entropy (forward + backward in one pass over the
// logits), token+position embedding forward/backward, bias gradient.
//
// Reference parity:
//   LayerNorm     scirs2-neural/src/layers/normalization.rs:140-260 (forward;
//                 the reference's backward is a stub, the math here is the
//                 standard one and is tested against torch fp32)
//   CrossEntropy  scirs2-neural/src/losses/crossentropy.rs:54-143 and
//                 scirs2-core/src/gpu/kernels/ml/softmax.rs:57-141 (3-pass
//                 softmax, here one online pass + one gradient pass)
//   Embedding     scirs2-neural/src/layers/embedding.rs:256-330
#include "host_common.h"
#include "scirs_noalloc.h"

#include <climits>
#include <cstdint>

namespace scirs {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ void unpack8(const uint4& q, float* f) {
  f[0] = bf16_lo(q.x); f[1] = bf16_hi(q.x);
  f[2] = bf16_lo(q.y); f[3] = bf16_hi(q.y);
  f[4] = bf16_lo(q.z); f[5] = bf16_hi(q.z);
  f[6] = bf16_lo(q.w); f[7] = bf16_hi(q.w);
}
__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 q;
  q.x = pack_bf16x2(f[0], f[1]);
  q.y = pack_bf16x2(f[2], f[3]);
  q.z = pack_bf16x2(f[4], f[5]);
  q.w = pack_bf16x2(f[6], f[7]);
  return q;
}

// ===========================================================================
// LayerNorm forward. RW warps share one row; each lane keeps NV 8-wide
// vectors in registers, so D = RW * 256 * NV. A block of 256 threads handles
// 8/RW rows per iteration.
// ===========================================================================
template <int RW>
__device__ __forceinline__ float row_sum(float v, float* red /*[8]*/, int wib) {
  v = warp_sum(v);
  if (RW == 1) return v;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[wib] = v;
  __syncthreads();
  const int g0 = (wib / RW) * RW;
  float t = 0.f;
#pragma unroll
  for (int k = 0; k < RW; ++k) t += red[g0 + k];
  return t;
}

template <int NV, int RW>
__global__ void __launch_bounds__(256) ln_fwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w,
                                                     const bf16* __restrict__ b, bf16* __restrict__ y,
                                                     float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                                     int M, float eps) {
  constexpr int D = RW * 256 * NV;
  constexpr int RPB = 8 / RW;  // rows per block
  __shared__ float red[8];
  const int wib = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int sub = (wib % RW) * 32 + lane;  // thread index within the row group
  const int row = blockIdx.x * RPB + wib / RW;
  const bool ok = row < M;
  float v[NV * 8];
  const uint4* xr = reinterpret_cast<const uint4*>(x + (long)(ok ? row : 0) * D);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if (ok) unpack8(xr[sub + 32 * RW * i], v + 8 * i);
    else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[8 * i + e] = 0.f;
    }
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV * 8; ++i) s += v[i];
  const float mu = row_sum<RW>(s, red, wib) * (1.f / D);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV * 8; ++i) {
    float d = v[i] - mu;
    ss += d * d;
  }
  const float rs = rsqrtf(row_sum<RW>(ss, red, wib) * (1.f / D) + eps);
  if (!ok) return;
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  const uint4* br = reinterpret_cast<const uint4*>(b);
  uint4* yr = reinterpret_cast<uint4*>(y + (long)row * D);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    float wf[8], bf[8], o[8];
    unpack8(__ldg(wr + sub + 32 * RW * i), wf);
    unpack8(__ldg(br + sub + 32 * RW * i), bf);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = (v[8 * i + e] - mu) * rs * wf[e] + bf[e];
    yr[sub + 32 * RW * i] = pack8(o);
  }
  if (sub == 0) {
    mean_out[row] = mu;
    rstd_out[row] = rs;
  }
}

// Generic LayerNorm forward for any D (multiple of 8): one warp per row, two
// passes over global memory.
__global__ void __launch_bounds__(256) ln_fwd_generic(const bf16* __restrict__ x, const bf16* __restrict__ w,
                                                      const bf16* __restrict__ b, bf16* __restrict__ y,
                                                      float* __restrict__ mean_out, float* __restrict__ rstd_out,
                                                      int M, int D, float eps) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const bf16* xr = x + (long)row * D;
  float s = 0.f;
  for (int j = lane; j < D; j += 32) s += __bfloat162float(xr[j]);
  const float mu = warp_sum(s) / D;
  float ss = 0.f;
  for (int j = lane; j < D; j += 32) {
    float d = __bfloat162float(xr[j]) - mu;
    ss += d * d;
  }
  const float rs = rsqrtf(warp_sum(ss) / D + eps);
  for (int j = lane; j < D; j += 32)
    y[(long)row * D + j] =
        __float2bfloat16((__bfloat162float(xr[j]) - mu) * rs * __bfloat162float(w[j]) + __bfloat162float(b[j]));
  if (lane == 0) {
    mean_out[row] = mu;
    rstd_out[row] = rs;
  }
}

// ===========================================================================
// LayerNorm backward.
//   dx = rstd * (g*dy - mean(g*dy) - xhat * mean(g*dy*xhat)) (+ dresid)
//   dgamma / dbeta: per-block partial column sums in registers, written to
//   part[block] and summed by ln_bwd_reduce.
// Persistent grid: each row group walks rows with a grid-wide stride.
// ===========================================================================
template <int NV, int RW>
__global__ void __launch_bounds__(256, 2) ln_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ x,
                                                        const bf16* __restrict__ w, const float* __restrict__ mean,
                                                        const float* __restrict__ rstd,
                                                        const bf16* __restrict__ dresid, bf16* __restrict__ dx,
                                                        float* __restrict__ part, int M) {
  constexpr int D = RW * 256 * NV;
  constexpr int RPB = 8 / RW;
  // Per row-group partial column sums (dgamma, dbeta, sum dx) live in shared
  // memory: each lane owns distinct columns of its group, so no atomics.
  // Layout [RPB][3][NV*8 slots][RW*32 threads]: consecutive lanes touch
  // consecutive words (bank-conflict free). Slot k of thread `sub` is
  // column (sub + 32*RW*(k/8))*8 + k%8.
  extern __shared__ float ps[];
  __shared__ float red[8];
  const int wib = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int sub = (wib % RW) * 32 + lane;
  const int grp = wib / RW;
  for (int i = threadIdx.x; i < RPB * 3 * D; i += 256) ps[i] = 0.f;
  __syncthreads();
  float* pg = ps + grp * 3 * D;
  float* pb = pg + D;
  float* pd = pb + D;
  const uint4* wr = reinterpret_cast<const uint4*>(w);

  for (int base = blockIdx.x * RPB; base < M; base += gridDim.x * RPB) {
    const int row = base + grp;
    const bool ok = row < M;
    const int rr = ok ? row : 0;
    const uint4* xr = reinterpret_cast<const uint4*>(x + (long)rr * D);
    const uint4* dyr = reinterpret_cast<const uint4*>(dy + (long)rr * D);
    const float mu = mean[rr], rs = rstd[rr];
    float xh[NV * 8], g[NV * 8];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      unpack8(xr[sub + 32 * RW * i], xh + 8 * i);
      unpack8(dyr[sub + 32 * RW * i], g + 8 * i);
    }
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float wf[8];
      unpack8(__ldg(wr + sub + 32 * RW * i), wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int k = 8 * i + e;
        xh[k] = (xh[k] - mu) * rs;
        if (ok) {
          pg[k * RW * 32 + sub] += g[k] * xh[k];
          pb[k * RW * 32 + sub] += g[k];
        }
        g[k] *= wf[e];
        s1 += g[k];
        s2 += g[k] * xh[k];
      }
    }
    s1 = row_sum<RW>(s1, red, wib) * (1.f / D);
    s2 = row_sum<RW>(s2, red, wib) * (1.f / D);
    if (ok) {
      uint4* dxr = reinterpret_cast<uint4*>(dx + (long)row * D);
      const uint4* drr = dresid ? reinterpret_cast<const uint4*>(dresid + (long)row * D) : nullptr;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = rs * (g[8 * i + e] - s1 - xh[8 * i + e] * s2);
        if (drr) {
          float r8[8];
          unpack8(drr[sub + 32 * RW * i], r8);
#pragma unroll
          for (int e = 0; e < 8; ++e) o[e] += r8[e];
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) pd[(8 * i + e) * RW * 32 + sub] += o[e];
        dxr[sub + 32 * RW * i] = pack8(o);
      }
    }
  }
  __syncthreads();
  float* out = part + (long)blockIdx.x * 3 * D;
  for (int c = threadIdx.x; c < 3 * D; c += 256) {
    // c = arr*D + k*(RW*32) + t  ->  column (t + 32*RW*(k/8))*8 + k%8 of array arr
    const int arr = c / D, rem = c % D, k = rem / (RW * 32), t = rem % (RW * 32);
    float a = 0.f;
#pragma unroll
    for (int j = 0; j < RPB; ++j) a += ps[j * 3 * D + c];
    out[arr * D + (t + 32 * RW * (k >> 3)) * 8 + (k & 7)] = a;
  }
}

// Generic LayerNorm backward (any D), one warp per row, per-block partials.
__global__ void __launch_bounds__(256) ln_bwd_generic(const bf16* __restrict__ dy, const bf16* __restrict__ x,
                                                      const bf16* __restrict__ w, const float* __restrict__ mean,
                                                      const float* __restrict__ rstd, const bf16* __restrict__ dresid,
                                                      bf16* __restrict__ dx, float* __restrict__ part, int M, int D) {
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int nw = gridDim.x * 8;
  float* out_g = part + (long)blockIdx.x * 3 * D;
  float* out_b = out_g + D;
  float* out_s = out_b + D;
  for (int j = threadIdx.x; j < 3 * D; j += blockDim.x) out_g[j] = 0.f;
  __syncthreads();
  for (int row = gw; row < M; row += nw) {
    const bf16* xr = x + (long)row * D;
    const bf16* dyr = dy + (long)row * D;
    const float mu = mean[row], rs = rstd[row];
    float s1 = 0.f, s2 = 0.f;
    for (int j = lane; j < D; j += 32) {
      float xh = (__bfloat162float(xr[j]) - mu) * rs;
      float g = __bfloat162float(dyr[j]);
      atomicAdd(&out_g[j], g * xh);
      atomicAdd(&out_b[j], g);
      g *= __bfloat162float(w[j]);
      s1 += g;
      s2 += g * xh;
    }
    s1 = warp_sum(s1) / D;
    s2 = warp_sum(s2) / D;
    for (int j = lane; j < D; j += 32) {
      float xh = (__bfloat162float(xr[j]) - mu) * rs;
      float g = __bfloat162float(dyr[j]) * __bfloat162float(w[j]);
      float o = rs * (g - s1 - xh * s2);
      if (dresid) o += __bfloat162float(dresid[(long)row * D + j]);
      atomicAdd(&out_s[j], o);
      dx[(long)row * D + j] = __float2bfloat16(o);
    }
  }
}

// Sum per-block partials [nb, 3, D] into fp32 gradients (accumulating):
// dgamma, dbeta and (optional) the column sum of the produced dx, which is
// the bias gradient of the projection that wrote the residual stream.
// A block covers 32 consecutive columns; its 8 warps sum interleaved subsets
// of the nb partials (four loads in flight per thread) and combine through
// shared memory, so a few thousand rows' worth of partials reduce in one wave.
__global__ void __launch_bounds__(256) ln_bwd_reduce(const float* __restrict__ part, int nb, int D,
                                                     float* __restrict__ dw, float* __restrict__ db,
                                                     float* __restrict__ dsum) {
  __shared__ float red[8][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  const bool live = c < 3 * D && (c < 2 * D || dsum != nullptr);
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (live) {
    const long st = 3L * D;
    int k = warp;
    for (; k + 24 < nb; k += 32) {
      s0 += __ldcs(part + (long)k * st + c);
      s1 += __ldcs(part + (long)(k + 8) * st + c);
      s2 += __ldcs(part + (long)(k + 16) * st + c);
      s3 += __ldcs(part + (long)(k + 24) * st + c);
    }
    for (; k < nb; k += 8) s0 += __ldcs(part + (long)k * st + c);
  }
  red[warp][lane] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (warp == 0 && live) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[w][lane];
    if (c < D) dw[c] += s;
    else if (c < 2 * D) db[c - D] += s;
    else dsum[c - 2 * D] += s;
  }
}

// ===========================================================================
// Softmax cross-entropy, forward + backward fused, one CTA per row.
// logits [M, ld] bf16 (only the first V columns are real classes; columns
// [V, Vp) are padding and get zero gradient). On exit the logits buffer holds
// d loss / d logits * grad_scale. loss_out[row] = logsumexp - logit[target].
// Rows whose target equals ignore_index get zero loss and zero gradient.
// ===========================================================================
template <int THREADS>
__global__ void __launch_bounds__(THREADS) xent_fwd_bwd_kernel(bf16* __restrict__ logits, long ld,
                                                               const int64_t* __restrict__ targets,
                                                               float* __restrict__ loss_out, int V, int Vp,
                                                               float grad_scale, int64_t ignore_index) {
  const int row = blockIdx.x;
  bf16* lr = logits + (long)row * ld;
  const int64_t tgt = targets[row];
  const int nvec = V >> 3;  // full 8-wide vectors of real classes
  const uint4* lv = reinterpret_cast<const uint4*>(lr);
  float m = -INFINITY, s = 0.f;
  for (int i = threadIdx.x; i < nvec; i += THREADS) {
    float f[8];
    unpack8(lv[i], f);
    float lm = f[0];
#pragma unroll
    for (int e = 1; e < 8; ++e) lm = fmaxf(lm, f[e]);
    if (lm > m) {
      s *= __expf(m - lm);
      m = lm;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) s += __expf(f[e] - m);
  }
  for (int j = nvec * 8 + threadIdx.x; j < V; j += THREADS) {
    float f = __bfloat162float(lr[j]);
    if (f > m) {
      s *= __expf(m - f);
      m = f;
    }
    s += __expf(f - m);
  }
  // block reduction of (m, s)
  __shared__ float sm[THREADS / 32], ss[THREADS / 32];
  __shared__ float fin_m, fin_s;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    float mm = fmaxf(m, m2);
    s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
    m = mm;
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    sm[w] = m;
    ss[w] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M_ = sm[0], S_ = ss[0];
    for (int k = 1; k < THREADS / 32; ++k) {
      float mm = fmaxf(M_, sm[k]);
      S_ = (M_ == -INFINITY ? 0.f : S_ * __expf(M_ - mm)) + (sm[k] == -INFINITY ? 0.f : ss[k] * __expf(sm[k] - mm));
      M_ = mm;
    }
    fin_m = M_;
    fin_s = S_;
  }
  __syncthreads();
  const float M_ = fin_m;
  const float inv_s = 1.f / fin_s;
  const bool ignored = (tgt == ignore_index) || tgt < 0 || tgt >= V;
  if (threadIdx.x == 0) {
    float lt = ignored ? 0.f : __bfloat162float(lr[tgt]);
    loss_out[row] = ignored ? 0.f : (logf(fin_s) + M_ - lt);
  }
  __syncthreads();  // the target logit is read before it is overwritten
  const float gs = ignored ? 0.f : grad_scale;
  uint4* lw = reinterpret_cast<uint4*>(lr);
  for (int i = threadIdx.x; i < nvec; i += THREADS) {
    float f[8];
    unpack8(lw[i], f);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float p = __expf(f[e] - M_) * inv_s;
      if (i * 8 + e == tgt) p -= 1.f;
      f[e] = p * gs;
    }
    lw[i] = pack8(f);
  }
  for (int j = nvec * 8 + threadIdx.x; j < Vp; j += THREADS) {
    float g = 0.f;
    if (j < V) {
      float p = __expf(__bfloat162float(lr[j]) - M_) * inv_s;
      if (j == tgt) p -= 1.f;
      g = p * gs;
    }
    lr[j] = __float2bfloat16(g);
  }
}

// Cross-entropy forward only (no gradient), same layout.
template <int THREADS>
__global__ void __launch_bounds__(THREADS) xent_fwd_kernel(const bf16* __restrict__ logits, long ld,
                                                           const int64_t* __restrict__ targets,
                                                           float* __restrict__ loss_out, int V,
                                                           int64_t ignore_index) {
  const int row = blockIdx.x;
  const bf16* lr = logits + (long)row * ld;
  float m = -INFINITY, s = 0.f;
  for (int j = threadIdx.x; j < V; j += THREADS) {
    float f = __bfloat162float(lr[j]);
    if (f > m) {
      s *= __expf(m - f);
      m = f;
    }
    s += __expf(f - m);
  }
  __shared__ float sm[THREADS / 32], ss[THREADS / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    float mm = fmaxf(m, m2);
    s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
    m = mm;
  }
  if ((threadIdx.x & 31) == 0) {
    sm[threadIdx.x >> 5] = m;
    ss[threadIdx.x >> 5] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M_ = sm[0], S_ = ss[0];
    for (int k = 1; k < THREADS / 32; ++k) {
      float mm = fmaxf(M_, sm[k]);
      S_ = (M_ == -INFINITY ? 0.f : S_ * __expf(M_ - mm)) + (sm[k] == -INFINITY ? 0.f : ss[k] * __expf(sm[k] - mm));
      M_ = mm;
    }
    const int64_t tgt = targets[row];
    const bool ignored = (tgt == ignore_index) || tgt < 0 || tgt >= V;
    loss_out[row] = ignored ? 0.f : (logf(S_) + M_ - __bfloat162float(lr[tgt]));
  }
}

// ===========================================================================
// Embedding: out[m] = wte[tok[m]] + wpe[m % S]  (wpe may be null)
// ===========================================================================
__global__ void embed_fwd_kernel(const int64_t* __restrict__ tok, const bf16* __restrict__ wte,
                                 const bf16* __restrict__ wpe, bf16* __restrict__ out, int M, int S, int D, long V,
                                 DevStatus* st) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const long t = tok[row];
  if (!input_in_range(t, V, st, 80)) return;  // token id outside the vocabulary
  const uint4* a = reinterpret_cast<const uint4*>(wte + t * D);
  const uint4* p = wpe ? reinterpret_cast<const uint4*>(wpe + (long)(row % S) * D) : nullptr;
  uint4* o = reinterpret_cast<uint4*>(out + (long)row * D);
  for (int i = lane; i < D / 8; i += 32) {
    float f[8];
    unpack8(__ldg(a + i), f);
    if (p) {
      float g[8];
      unpack8(__ldg(p + i), g);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] += g[e];
    }
    o[i] = pack8(f);
  }
}

// dwte[tok[m]] += dout[m]; dwpe[m % S] += dout[m]  (fp32 atomics; either
// table may be null)
__global__ void embed_bwd_kernel(const int64_t* __restrict__ tok, const bf16* __restrict__ dout,
                                 float* __restrict__ dwte, float* __restrict__ dwpe, int M, int S, int D, long V,
                                 DevStatus* st) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  float* a = nullptr;
  if (dwte != nullptr) {
    const long t = tok[row];
    if (input_in_range(t, V, st, 81)) a = dwte + t * D;
  }
  float* p = dwpe ? dwpe + (long)(row % S) * D : nullptr;
  if (a == nullptr && p == nullptr) return;
  const uint4* g = reinterpret_cast<const uint4*>(dout + (long)row * D);
  for (int i = lane; i < D / 8; i += 32) {
    float f[8];
    unpack8(g[i], f);
    if (a) {
      atomicAdd(reinterpret_cast<float4*>(a + 8 * i), make_float4(f[0], f[1], f[2], f[3]));
      atomicAdd(reinterpret_cast<float4*>(a + 8 * i + 4), make_float4(f[4], f[5], f[6], f[7]));
    }
    if (p) {
      atomicAdd(reinterpret_cast<float4*>(p + 8 * i), make_float4(f[0], f[1], f[2], f[3]));
      atomicAdd(reinterpret_cast<float4*>(p + 8 * i + 4), make_float4(f[4], f[5], f[6], f[7]));
    }
  }
}

// ===========================================================================
// Bias gradient: out[n] += sum_m dy[m, n]   (dy bf16 [M, N], out fp32)
// block = 32 x 8 threads: x covers 8-column vectors, y strides rows.
// ===========================================================================
__global__ void __launch_bounds__(256) colsum_kernel(const bf16* __restrict__ dy, long ld, int M, int N,
                                                     int rows_per_block, float* __restrict__ out) {
  const int vc = blockIdx.x * 32 + threadIdx.x;  // vector column
  const int r0 = blockIdx.y * rows_per_block;
  const int r1 = min(M, r0 + rows_per_block);
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (vc * 8 < N) {
    for (int r = r0 + threadIdx.y; r < r1; r += 8) {
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(dy + (long)r * ld + vc * 8), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += f[e];
    }
  }
  __shared__ float red[8][32][9];
#pragma unroll
  for (int e = 0; e < 8; ++e) red[threadIdx.y][threadIdx.x][e] = acc[e];
  __syncthreads();
  if (threadIdx.y == 0 && vc * 8 < N) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float s = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) s += red[k][threadIdx.x][e];
      atomicAdd(out + vc * 8 + e, s);
    }
  }
}

// ===========================================================================
// host launchers
// ===========================================================================
void layernorm_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor b, torch::Tensor y, torch::Tensor mean,
                   torch::Tensor rstd, double eps) {
  CHECK_DTYPE(x, at::kBFloat16);
  CHECK_CONTIG(x);
  CHECK_CONTIG(y);
  const int D = (int)x.size(-1);
  const int M = (int)(x.numel() / D);
  TORCH_CHECK(D % 8 == 0, "LayerNorm width must be a multiple of 8");
  c10::cuda::CUDAGuard g(x.get_device());
  auto s = cur_stream();
  dim3 grid((M + 7) / 8), block(256);
  auto xp = (const bf16*)x.data_ptr(), wp = (const bf16*)w.data_ptr(), bp = (const bf16*)b.data_ptr();
  auto yp = (bf16*)y.data_ptr();
  auto mp = mean.data_ptr<float>(), rp = rstd.data_ptr<float>();
#define LNF(NV, RW) \
  ln_fwd_kernel<NV, RW><<<(M + (8 / RW) - 1) / (8 / RW), block, 0, s>>>(xp, wp, bp, yp, mp, rp, M, (float)eps)
  switch (D) {
    case 256: LNF(1, 1); break;
    case 512: LNF(2, 1); break;
    case 768: LNF(3, 1); break;
    case 1024: LNF(4, 1); break;
    case 1536: LNF(3, 2); break;
    case 2048: LNF(4, 2); break;
    case 3072: LNF(3, 4); break;
    case 4096: LNF(4, 4); break;
    default: ln_fwd_generic<<<grid, block, 0, s>>>(xp, wp, bp, yp, mp, rp, M, D, (float)eps);
  }
#undef LNF
  SCIRS_CHECK_LAUNCH();
}

// part: scratch fp32 [nblocks, 3, D]; dw/db (and optional dsum = colsum(dx)) fp32 [D] accumulated into.
void layernorm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor mean, torch::Tensor rstd,
                   c10::optional<torch::Tensor> dresid, torch::Tensor dx, torch::Tensor dw, torch::Tensor db,
                   torch::Tensor part, c10::optional<torch::Tensor> dsum) {
  CHECK_CONTIG(dy);
  CHECK_CONTIG(x);
  CHECK_CONTIG(dx);
  const int D = (int)x.size(-1);
  const int M = (int)(x.numel() / D);
  CHECK_DTYPE(dw, at::kFloat);
  CHECK_DTYPE(db, at::kFloat);
  const int nb = (int)(part.numel() / (3 * D));
  TORCH_CHECK(nb >= 1, "part too small");
  c10::cuda::CUDAGuard g(x.get_device());
  auto s = cur_stream();
  const bf16* dr = nullptr;
  if (dresid.has_value() && dresid->defined()) {
    CHECK_CONTIG((*dresid));
    dr = (const bf16*)dresid->data_ptr();
  }
  auto dyp = (const bf16*)dy.data_ptr(), xp = (const bf16*)x.data_ptr(), wp = (const bf16*)w.data_ptr();
  auto mp = mean.data_ptr<float>(), rp = rstd.data_ptr<float>();
  auto dxp = (bf16*)dx.data_ptr();
  auto pp = part.data_ptr<float>();
#define LNB(NV, RW)                                                                                 \
  {                                                                                                 \
    const int smem_b = (8 / RW) * 3 * (RW * 256 * NV) * (int)sizeof(float);                       \
    set_max_smem((const void*)ln_bwd_kernel<NV, RW>, smem_b);    \
    ln_bwd_kernel<NV, RW><<<nb, 256, smem_b, s>>>(dyp, xp, wp, mp, rp, dr, dxp, pp, M);             \
  }
  switch (D) {
    case 256: LNB(1, 1); break;
    case 512: LNB(2, 1); break;
    case 768: LNB(3, 1); break;
    case 1024: LNB(4, 1); break;
    case 1536: LNB(3, 2); break;
    case 2048: LNB(4, 2); break;
    case 3072: LNB(3, 4); break;
    case 4096: LNB(4, 4); break;
    default: ln_bwd_generic<<<nb, 256, 0, s>>>(dyp, xp, wp, mp, rp, dr, dxp, pp, M, D);
  }
#undef LNB
  SCIRS_CHECK_LAUNCH();
  float* dsp = nullptr;
  if (dsum.has_value() && dsum->defined()) {
    CHECK_DTYPE((*dsum), at::kFloat);
    TORCH_CHECK(dsum->numel() == D, "dsum must have D entries");
    dsp = dsum->data_ptr<float>();
  }
  ln_bwd_reduce<<<(3 * D + 31) / 32, 256, 0, s>>>(pp, nb, D, dw.data_ptr<float>(), db.data_ptr<float>(), dsp);
  SCIRS_CHECK_LAUNCH();
}

void xent_fwd_bwd(torch::Tensor logits, torch::Tensor targets, torch::Tensor loss, int64_t V, double grad_scale,
                  int64_t ignore_index) {
  CHECK_DTYPE(logits, at::kBFloat16);
  CHECK_DTYPE(targets, at::kLong);
  TORCH_CHECK(logits.stride(1) == 1 && logits.stride(0) % 8 == 0, "logits rows must be 16-byte aligned");
  const int M = (int)logits.size(0);
  const int Vp = (int)logits.size(1);
  TORCH_CHECK(V <= Vp, "V > padded width");
  c10::cuda::CUDAGuard g(logits.get_device());
  xent_fwd_bwd_kernel<512><<<M, 512, 0, cur_stream()>>>((bf16*)logits.data_ptr(), logits.stride(0),
                                                         targets.data_ptr<int64_t>(), loss.data_ptr<float>(), (int)V,
                                                         Vp, (float)grad_scale, ignore_index);
  SCIRS_CHECK_LAUNCH();
}

void xent_fwd(torch::Tensor logits, torch::Tensor targets, torch::Tensor loss, int64_t V, int64_t ignore_index) {
  CHECK_DTYPE(logits, at::kBFloat16);
  TORCH_CHECK(logits.stride(1) == 1, "logits inner stride must be 1");
  const int M = (int)logits.size(0);
  c10::cuda::CUDAGuard g(logits.get_device());
  xent_fwd_kernel<512><<<M, 512, 0, cur_stream()>>>((const bf16*)logits.data_ptr(), logits.stride(0),
                                                     targets.data_ptr<int64_t>(), loss.data_ptr<float>(), (int)V,
                                                     ignore_index);
  SCIRS_CHECK_LAUNCH();
}

void embedding_fwd(torch::Tensor tok, torch::Tensor wte, c10::optional<torch::Tensor> wpe, torch::Tensor out,
                   int64_t S) {
  CHECK_DTYPE(tok, at::kLong);
  const int D = (int)wte.size(1);
  const int M = (int)tok.numel();
  TORCH_CHECK(D % 8 == 0, "embedding width must be a multiple of 8");
  c10::cuda::CUDAGuard g(tok.get_device());
  const bf16* pp = (wpe.has_value() && wpe->defined()) ? (const bf16*)wpe->data_ptr() : nullptr;
  embed_fwd_kernel<<<(M + 7) / 8, 256, 0, cur_stream()>>>(tok.data_ptr<int64_t>(), (const bf16*)wte.data_ptr(), pp,
                                                          (bf16*)out.data_ptr(), M, (int)S, D, (long)wte.size(0),
                                                          status_ptr(tok.get_device()));
  SCIRS_CHECK_LAUNCH();
}

void embedding_bwd(torch::Tensor tok, torch::Tensor dout, c10::optional<torch::Tensor> dwte,
                   c10::optional<torch::Tensor> dwpe, int64_t S) {
  const bool has_wte = dwte.has_value() && dwte->defined();
  const bool has_wpe = dwpe.has_value() && dwpe->defined();
  TORCH_CHECK(has_wte || has_wpe, "embedding_bwd needs dwte or dwpe");
  CHECK_DTYPE(tok, at::kLong);
  CHECK_CONTIG(tok);
  CHECK_DTYPE(dout, at::kBFloat16);
  CHECK_CONTIG(dout);
  const int D = (int)dout.size(-1);
  const int M = (int)tok.numel();
  TORCH_CHECK(D % 8 == 0 && dout.numel() == (long)M * D, "dout [M, D] with D % 8 == 0");
  float* wp = nullptr;
  long V = 0;
  if (has_wte) {
    CHECK_DTYPE((*dwte), at::kFloat);
    CHECK_CONTIG((*dwte));
    TORCH_CHECK(dwte->size(1) == D, "dwte [V, D]");
    wp = dwte->data_ptr<float>();
    V = (long)dwte->size(0);
  }
  float* pp = nullptr;
  if (has_wpe) {
    CHECK_DTYPE((*dwpe), at::kFloat);
    CHECK_CONTIG((*dwpe));
    TORCH_CHECK(dwpe->size(-1) == D && dwpe->size(0) >= S, "dwpe [>= S, D]");
    pp = dwpe->data_ptr<float>();
  }
  c10::cuda::CUDAGuard g(tok.get_device());
  embed_bwd_kernel<<<(M + 7) / 8, 256, 0, cur_stream()>>>(tok.data_ptr<int64_t>(), (const bf16*)dout.data_ptr(), wp,
                                                          pp, M, (int)S, D, V, status_ptr(tok.get_device()));
  SCIRS_CHECK_LAUNCH();
}

void bias_grad(torch::Tensor dy, torch::Tensor out) {
  CHECK_DTYPE(dy, at::kBFloat16);
  CHECK_DTYPE(out, at::kFloat);
  TORCH_CHECK(dy.dim() == 2 && dy.stride(1) == 1 && dy.stride(0) % 8 == 0, "dy must be 2-D with aligned rows");
  const int M = (int)dy.size(0), N = (int)dy.size(1);
  TORCH_CHECK(N % 8 == 0, "bias_grad needs N % 8 == 0");
  c10::cuda::CUDAGuard g(dy.get_device());
  const int sms = num_sms(dy.get_device());
  const int gx = (N / 8 + 31) / 32;
  int gy = std::max(1, std::min((M + 63) / 64, (4 * sms + gx - 1) / gx));
  const int rpb = (M + gy - 1) / gy;
  gy = (M + rpb - 1) / rpb;
  colsum_kernel<<<dim3(gx, gy), dim3(32, 8), 0, cur_stream()>>>((const bf16*)dy.data_ptr(), dy.stride(0), M, N, rpb,
                                                                 out.data_ptr<float>());
  SCIRS_CHECK_LAUNCH();
}



// ===========================================================================
// No-allocation entry point (C ABI, declared in scirs_noalloc.h, which also
// states the contract: size limit, first-call set-up, the shared array and
// its race). It has no counterpart in the reference. It serves callers that
// cannot allocate device memory at the point of the call: C or
// other-language hosts working inside a fixed device-memory budget with no
// allocator of their own, and code that must not call cudaMalloc where it
// runs (cudaMalloc can synchronise the device).
//
// scirs_layernorm_bwd_noalloc() computes the same LayerNorm backward as
// layernorm_bwd() with the same kernels; its per-block partial column sums
// live in the file-scope array below instead of a caller-provided scratch
// tensor. A call needs nblocks * 3 * D floats; nblocks is reduced to fit the
// array and a row width whose single block would not fit is rejected. Each
// call writes every partial it later reads, so nothing needs clearing.
// ===========================================================================
constexpr long kNoAllocScratchFloats = SCIRS_NOALLOC_SCRATCH_FLOATS;
constexpr int kNoAllocMaxD = SCIRS_NOALLOC_LN_MAX_D;
static_assert(kNoAllocMaxD == (int)(kNoAllocScratchFloats / 3), "header and implementation disagree");
static __device__ __align__(256) float g_noalloc_ln_scratch[kNoAllocScratchFloats];

namespace {
float* g_noalloc_ptr[64] = {nullptr};
std::mutex g_noalloc_mu;
thread_local std::string g_noalloc_err;

// Device address of the scratch array for `device` (looked up once, with
// `device` current on the calling thread).
cudaError_t noalloc_scratch(int device, float** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[device] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_ln_scratch);
    if (e != cudaSuccess) return e;
    g_noalloc_ptr[device] = reinterpret_cast<float*>(p);
  }
  *out = g_noalloc_ptr[device];
  return cudaSuccess;
}

inline bool aligned_to(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }
}  // namespace

extern "C" __attribute__((visibility("default"))) const char* scirs_noalloc_last_error() {
  return g_noalloc_err.c_str();
}

extern "C" __attribute__((visibility("default"))) int scirs_layernorm_bwd_noalloc(
    const void* dy, const void* x, const void* w, const float* mean, const float* rstd, const void* dresid,
    void* dx, float* dw, float* db, float* dsum, long long rows, int D, void* stream) {
  g_noalloc_err.clear();
  if (rows <= 0 || rows > (long long)INT_MAX || D <= 0 || D % 8 != 0) {
    g_noalloc_err = "rows must be in 1..INT_MAX and D a positive multiple of 8 (rows = " + std::to_string(rows) +
                    ", D = " + std::to_string(D) + ")";
    return SCIRS_NOALLOC_EARG;
  }
  if (D > kNoAllocMaxD) {
    g_noalloc_err = "D = " + std::to_string(D) + " exceeds the no-allocation scratch limit (D <= " +
                    std::to_string(kNoAllocMaxD) + ")";
    return SCIRS_NOALLOC_ETOOBIG;
  }
  if (dy == nullptr || x == nullptr || w == nullptr || mean == nullptr || rstd == nullptr || dx == nullptr ||
      dw == nullptr || db == nullptr) {
    g_noalloc_err = "null pointer argument";
    return SCIRS_NOALLOC_ENULL;
  }
  const void* bf_ptrs[] = {dy, x, w, dresid, dx};
  const void* f_ptrs[] = {mean, rstd, dw, db, dsum};
  bool vec_ok = true;  // every bf16 operand 16-byte aligned: the vectorised kernels apply
  for (const void* p : bf_ptrs) {
    if (p == nullptr) continue;
    if (!aligned_to(p, 2)) {
      g_noalloc_err = "a bf16 pointer is not 2-byte aligned";
      return SCIRS_NOALLOC_EALIGN;
    }
    vec_ok = vec_ok && aligned_to(p, 16);
  }
  for (const void* p : f_ptrs) {
    if (p != nullptr && !aligned_to(p, 4)) {
      g_noalloc_err = "an fp32 pointer is not 4-byte aligned";
      return SCIRS_NOALLOC_EALIGN;
    }
  }
  // An error left pending by earlier work is returned as is (and stays
  // pending) rather than being reported later as this call's failure.
  cudaError_t e = cudaPeekAtLastError();
  if (e != cudaSuccess) return (int)e;
  int device = 0;
  e = cudaGetDevice(&device);
  if (e != cudaSuccess) return (int)e;
  if (device < 0 || device >= 64) {
    g_noalloc_err = "device index out of range";
    return SCIRS_NOALLOC_EDEVICE;
  }
  float* part = nullptr;
  e = noalloc_scratch(device, &part);
  if (e != cudaSuccess) return (int)e;
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return (int)e;
  const int M = (int)rows;
  long nb = std::min<long>(2L * sms, (rows + 7) / 8);
  nb = std::max<long>(1, std::min<long>(nb, kNoAllocScratchFloats / (3L * D)));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  auto dyp = (const bf16*)dy, xp = (const bf16*)x, wp = (const bf16*)w, dr = (const bf16*)dresid;
  auto dxp = (bf16*)dx;
  const int inb = (int)nb;
#define NOALLOC_LNB(NV, RW)                                                                        \
  {                                                                                                \
    const int smem_b = (8 / RW) * 3 * (RW * 256 * NV) * (int)sizeof(float);                      \
    e = cudaFuncSetAttribute(ln_bwd_kernel<NV, RW>, cudaFuncAttributeMaxDynamicSharedMemorySize,   \
                             smem_b);                                                              \
    if (e != cudaSuccess) return (int)e;                                                           \
    ln_bwd_kernel<NV, RW><<<inb, 256, smem_b, s>>>(dyp, xp, wp, mean, rstd, dr, dxp, part, M);     \
  }
  switch (vec_ok ? D : -1) {
    case 256: NOALLOC_LNB(1, 1); break;
    case 512: NOALLOC_LNB(2, 1); break;
    case 768: NOALLOC_LNB(3, 1); break;
    case 1024: NOALLOC_LNB(4, 1); break;
    case 1536: NOALLOC_LNB(3, 2); break;
    case 2048: NOALLOC_LNB(4, 2); break;
    case 3072: NOALLOC_LNB(3, 4); break;
    case 4096: NOALLOC_LNB(4, 4); break;
    default: ln_bwd_generic<<<inb, 256, 0, s>>>(dyp, xp, wp, mean, rstd, dr, dxp, part, M, D);
  }
#undef NOALLOC_LNB
  e = cudaGetLastError();
  if (e != cudaSuccess) return (int)e;
  ln_bwd_reduce<<<(3 * D + 31) / 32, 256, 0, s>>>(part, inb, D, dw, db, dsum);
  return (int)cudaGetLastError();
}

}  // namespace scirs
