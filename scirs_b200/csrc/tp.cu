// Tensor-parallel helper kernels: cross-rank signals, the reduction half of
// GEMM -> reduce-scatter, rotary position embedding, and the vocabulary-
// parallel softmax cross-entropy.
//
// Synchronisation model: every rank owns a small array of 32-bit flag words
// (one per source rank) inside its symmetric buffer. A producer sets its word
// in every peer's array to `epoch * 4096 + idx` with st.release.sys once its
// data is written; a consumer waits (bounded by a globaltimer budget, then
// reports kStPeerTimeout and skips) until the word reaches the value of the
// signal it depends on, then reads. `epoch` is a device counter advanced once
// per training step (so a step captured in a CUDA graph replays correctly)
// and `idx` numbers the signals inside a step, identically on every rank.
//
// Reference parity: scirs2-neural/src/training/tensor_parallel.rs:85-385
// (ColumnParallelLinear concat, RowParallelLinear sum + bias, vocabulary-
// partitioned embedding; single-process simulation there),
// scirs2-neural/src/attention/rope.rs:53-250 (rotary embedding, half-rotation
// form), scirs2-neural/src/losses/crossentropy.rs (loss).
#include "host_common.h"

namespace scirs {
namespace tp {

constexpr unsigned kSigStride = 4096;
constexpr int kMaxPeers = 8;

struct FlagPtrs {
  unsigned* p[kMaxPeers];
};

__device__ __forceinline__ unsigned ld_acq(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_rel(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Threads 0..world-1 of the block wait for the peers' flags; false on timeout.
__device__ bool block_wait(const unsigned* flags, const unsigned* epoch, unsigned idx, int rank, int world,
                           long long timeout_ns, DevStatus* st, int site) {
  __shared__ int fail;
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  const int r = threadIdx.x;
  if (r < world && r != rank) {
    const unsigned want = *epoch * kSigStride + idx;
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while ((int)(ld_acq(flags + r) - want) < 0) {
      if ((++spins & 255u) == 0 && (long long)(globaltimer_ns() - t0) > timeout_ns) {
        report_status(st, kStPeerTimeout, site, (unsigned)r);
        fail = 1;
        break;
      }
    }
  }
  __syncthreads();
  return fail == 0;
}

// Last block to finish signals every peer (after a system-scope fence).
__device__ void last_block_signal(const FlagPtrs& sig, int world, const unsigned* epoch, unsigned idx,
                                  unsigned* done) {
  __syncthreads();
  if (threadIdx.x == 0 && sig.p[0] != nullptr) {
    __threadfence_system();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0u;
      const unsigned v = *epoch * kSigStride + idx;
      __threadfence_system();
      for (int r = 0; r < world; ++r) st_rel(sig.p[r], v);
    }
  }
}

__global__ void signal_kernel(FlagPtrs sig, int world, const unsigned* epoch, unsigned idx) {
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned v = *epoch * kSigStride + idx;
    for (int r = 0; r < world; ++r) st_rel(sig.p[r], v);
  }
}

// Advance the step epoch and (optionally) lay out this step's flag values
// vals[i] = epoch * 4096 + i, the words the copy engines write into peers'
// flag arrays to announce data they pushed.
__global__ void step_begin_kernel(unsigned* epoch, unsigned* vals, int n) {
  const unsigned e = *epoch + 1u;
  for (int i = threadIdx.x; i < n; i += blockDim.x) vals[i] = e * kSigStride + (unsigned)i;
  __syncthreads();
  if (threadIdx.x == 0) *epoch = e;
}

// out[row] = resid[row] + bias + sum_r recv[r][row]   (fixed rank order)
__global__ void __launch_bounds__(256) reduce_kernel(const __nv_bfloat16* __restrict__ recv,
                                                     __nv_bfloat16* __restrict__ out,
                                                     const __nv_bfloat16* __restrict__ bias,
                                                     const __nv_bfloat16* __restrict__ resid, long rows, int D,
                                                     int rank, int world, const unsigned* flags,
                                                     const unsigned* epoch, unsigned wait_idx, long long timeout_ns,
                                                     DevStatus* st, FlagPtrs sig, unsigned sig_idx,
                                                     unsigned* done) {
  const bool ok = flags == nullptr || block_wait(flags, epoch, wait_idx, rank, world, timeout_ns, st, 70);
  if (ok) {
    const int dv = D / 8;
    const long nvec = rows * dv;
    const long slot = rows * D;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < nvec; i += (long)gridDim.x * blockDim.x) {
      float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (resid != nullptr) {
        const uint4 q = reinterpret_cast<const uint4*>(resid)[i];
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) f[2 * e] += bf16_lo(w[e]), f[2 * e + 1] += bf16_hi(w[e]);
      }
      if (bias != nullptr) {
        const uint4 q = reinterpret_cast<const uint4*>(bias)[i % dv];
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) f[2 * e] += bf16_lo(w[e]), f[2 * e + 1] += bf16_hi(w[e]);
      }
      for (int r = 0; r < world; ++r) {
        const uint4 q = __ldcg(reinterpret_cast<const uint4*>(recv + r * slot) + i);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) f[2 * e] += bf16_lo(w[e]), f[2 * e + 1] += bf16_hi(w[e]);
      }
      reinterpret_cast<uint4*>(out)[i] = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                                     pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
    }
  }
  last_block_signal(sig, world, epoch, sig_idx, done);
}

// Rotary embedding on the q and k parts of a fused [rows, 3, H, hd] buffer,
// half-rotation form: (x1, x2) -> (x1 cos - x2 sin, x2 cos + x1 sin) with
// angle pos * theta^(-2i/hd) (table precomputed on the host). `inverse`
// applies the transpose rotation (the backward pass).
__global__ void __launch_bounds__(256) rope_kernel(__nv_bfloat16* __restrict__ qkv, const float* __restrict__ cos_t,
                                                   const float* __restrict__ sin_t, long rows, int S, int H, int hd,
                                                   int inverse) {
  const int half = hd / 2;
  const long per_row = 2L * H * half;  // q and k, one thread per rotated pair
  const long total = rows * per_row;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long row = i / per_row;
    const int rem = (int)(i % per_row);
    const int part = rem / (H * half);  // 0 = q, 1 = k
    const int h = (rem / half) % H;
    const int j = rem % half;
    const int pos = (int)(row % S);
    __nv_bfloat16* base = qkv + row * (3L * H * hd) + ((long)part * H + h) * hd;
    const float c = cos_t[pos * half + j];
    const float sn = inverse ? -sin_t[pos * half + j] : sin_t[pos * half + j];
    const float x1 = __bfloat162float(base[j]);
    const float x2 = __bfloat162float(base[j + half]);
    base[j] = __float2bfloat16(x1 * c - x2 * sn);
    base[j + half] = __float2bfloat16(x2 * c + x1 * sn);
  }
}

// Vocabulary-parallel cross-entropy, pass 1: per row of this rank's logits
// slice [rows, Vl] (valid columns [0, nvalid)): local max, sum of exp(x -
// max), and the target logit if the target falls in [v0, v0 + nvalid).
// The 4-float record is stored into every rank's stats buffer at
// [rank][row]; the last block signals.
__global__ void __launch_bounds__(256) xent_stats_kernel(const __nv_bfloat16* __restrict__ logits,
                                                         const int64_t* __restrict__ tgt, long rows, int Vl,
                                                         int nvalid, long v0, int rank, int world, FlagPtrs dst,
                                                         FlagPtrs sig, const unsigned* epoch, unsigned sig_idx,
                                                         unsigned* done) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long row = blockIdx.x * 8L + warp;
  if (row < rows) {
    const __nv_bfloat16* x = logits + row * Vl;
    float m = -INFINITY;
    for (int c = lane; c < nvalid; c += 32) m = fmaxf(m, __bfloat162float(x[c]));
    m = warp_max(m);
    float s = 0.f;
    for (int c = lane; c < nvalid; c += 32) s += ex2_fast((__bfloat162float(x[c]) - m) * 1.4426950408889634f);
    s = warp_sum(s);
    const long t = tgt[row];
    const float tl = (t >= v0 && t < v0 + nvalid) ? __bfloat162float(x[t - v0]) : 0.f;
    if (lane < world) {
      float4* d = reinterpret_cast<float4*>(dst.p[lane]) + ((long)rank * rows + row);
      *d = make_float4(m, s, tl, 0.f);
    }
  }
  last_block_signal(sig, world, epoch, sig_idx, done);
}

// Pass 2: combine the world records of every row (local reads) into the
// log-sum-exp, write the row loss and overwrite this rank's logits slice
// with d loss / d logits = (softmax - onehot) * scale (padded columns 0).
__global__ void __launch_bounds__(256) xent_finish_kernel(__nv_bfloat16* __restrict__ logits,
                                                          const int64_t* __restrict__ tgt,
                                                          const float4* __restrict__ stats, float* __restrict__ loss,
                                                          long rows, int Vl, int nvalid, long v0, int rank, int world,
                                                          float scale, const unsigned* flags, const unsigned* epoch,
                                                          unsigned wait_idx, long long timeout_ns, DevStatus* st) {
  // wait_idx 0: the statistics were exchanged by other means (nothing to wait on)
  const bool ok = wait_idx == 0 || block_wait(flags, epoch, wait_idx, rank, world, timeout_ns, st, 71);
  if (!ok) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long row = blockIdx.x * 8L + warp;
  if (row >= rows) return;
  float m = -INFINITY;
  for (int r = 0; r < world; ++r) m = fmaxf(m, __ldcg(stats + (long)r * rows + row).x);
  float s = 0.f, tl = 0.f;
  for (int r = 0; r < world; ++r) {
    const float4 q = __ldcg(stats + (long)r * rows + row);
    s += q.y * ex2_fast((q.x - m) * 1.4426950408889634f);
    tl += q.z;
  }
  const float lse = m + logf(s);
  if (lane == 0 && loss != nullptr) loss[row] = lse - tl;
  const long t = tgt[row];
  __nv_bfloat16* x = logits + row * Vl;
  for (int c = lane; c < Vl; c += 32) {
    float g = 0.f;
    if (c < nvalid) {
      g = ex2_fast((__bfloat162float(x[c]) - lse) * 1.4426950408889634f);
      if (t == v0 + c) g -= 1.f;
      g *= scale;
    }
    x[c] = __float2bfloat16(g);
  }
}

static FlagPtrs to_ptrs(const std::vector<int64_t>& v) {
  FlagPtrs f;
  memset(&f, 0, sizeof(f));
  TORCH_CHECK(v.size() <= (size_t)kMaxPeers, "too many ranks");
  for (size_t i = 0; i < v.size(); ++i) f.p[i] = reinterpret_cast<unsigned*>(v[i]);
  return f;
}

static unsigned* done_ctr(int dev) {
  static unsigned* c[64] = {nullptr};
  if (c[dev] == nullptr) {
    SCIRS_CHECK_CUDA(cudaMalloc(&c[dev], sizeof(unsigned)));
    SCIRS_CHECK_CUDA(cudaMemset(c[dev], 0, sizeof(unsigned)));
  }
  return c[dev];
}

static int grid_for(long work, int dev) {
  return (int)std::max<long>(1, std::min<long>((work + 255) / 256, 8L * num_sms(dev)));
}

}  // namespace tp

void tp_signal(std::vector<int64_t> sig_flags, torch::Tensor epoch, int64_t idx) {
  c10::cuda::CUDAGuard guard(epoch.get_device());
  tp::signal_kernel<<<1, 32, 0, cur_stream()>>>(tp::to_ptrs(sig_flags), (int)sig_flags.size(),
                                                 reinterpret_cast<const unsigned*>(epoch.data_ptr()), (unsigned)idx);
  SCIRS_CHECK_LAUNCH();
}

void tp_step_begin(torch::Tensor epoch, c10::optional<torch::Tensor> vals) {
  c10::cuda::CUDAGuard guard(epoch.get_device());
  unsigned* vp = nullptr;
  int n = 0;
  if (vals.has_value() && vals->defined()) {
    TORCH_CHECK(vals->element_size() == 4 && vals->is_contiguous() && vals->numel() <= (long)tp::kSigStride,
                "vals: contiguous 32-bit, at most 4096 entries");
    vp = reinterpret_cast<unsigned*>(vals->data_ptr());
    n = (int)vals->numel();
  }
  tp::step_begin_kernel<<<1, 256, 0, cur_stream()>>>(reinterpret_cast<unsigned*>(epoch.data_ptr()), vp, n);
  SCIRS_CHECK_LAUNCH();
}

// out = resid + bias + sum over the receive slots (after waiting for every
// peer's signal `wait_idx`); optionally signals `sig_idx` when done.
void tp_reduce(torch::Tensor recv, torch::Tensor out, c10::optional<torch::Tensor> bias,
               c10::optional<torch::Tensor> resid, int64_t rank, c10::optional<torch::Tensor> flags,
               torch::Tensor epoch, int64_t wait_idx, std::vector<int64_t> sig_flags, int64_t sig_idx,
               double timeout_s) {
  CHECK_DTYPE(recv, at::kBFloat16);
  CHECK_DTYPE(out, at::kBFloat16);
  CHECK_CONTIG(recv);
  CHECK_CONTIG(out);
  TORCH_CHECK(recv.dim() == 3 && out.dim() == 2 && recv.size(1) == out.size(0) && recv.size(2) == out.size(1),
              "recv [world, rows, D], out [rows, D]");
  const int world = recv.size(0);
  const long rows = out.size(0);
  const int D = out.size(1);
  TORCH_CHECK(D % 8 == 0, "D must be a multiple of 8");
  const __nv_bfloat16* bp = nullptr;
  const __nv_bfloat16* rp = nullptr;
  if (bias.has_value() && bias->defined()) bp = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  if (resid.has_value() && resid->defined()) {
    CHECK_CONTIG((*resid));
    rp = reinterpret_cast<const __nv_bfloat16*>(resid->data_ptr());
  }
  const int dev = out.get_device();
  c10::cuda::CUDAGuard guard(dev);
  const unsigned* fp = (flags.has_value() && flags->defined()) ? reinterpret_cast<const unsigned*>(flags->data_ptr())
                                                               : nullptr;
  const int grid = tp::grid_for(rows * (D / 8), dev);
  tp::reduce_kernel<<<grid, 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(recv.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), bp,
      rp, rows, D, (int)rank, world, fp, reinterpret_cast<const unsigned*>(epoch.data_ptr()), (unsigned)wait_idx,
      (long long)(timeout_s * 1e9), status_ptr(dev), tp::to_ptrs(sig_flags), (unsigned)sig_idx, tp::done_ctr(dev));
  SCIRS_CHECK_LAUNCH();
}

void rope_apply(torch::Tensor qkv, torch::Tensor cos_t, torch::Tensor sin_t, int64_t S, int64_t H, int64_t hd,
                bool inverse) {
  CHECK_DTYPE(qkv, at::kBFloat16);
  CHECK_DTYPE(cos_t, at::kFloat);
  CHECK_DTYPE(sin_t, at::kFloat);
  TORCH_CHECK(qkv.is_contiguous() && qkv.size(-1) == 3 * H * hd, "qkv must be contiguous [rows, 3*H*hd]");
  TORCH_CHECK(cos_t.numel() >= S * hd / 2 && sin_t.numel() >= S * hd / 2, "rope tables too small");
  const long rows = qkv.numel() / (3 * H * hd);
  const int dev = qkv.get_device();
  c10::cuda::CUDAGuard guard(dev);
  const int grid = tp::grid_for(rows * H * hd, dev);
  tp::rope_kernel<<<grid, 256, 0, cur_stream()>>>(reinterpret_cast<__nv_bfloat16*>(qkv.data_ptr()),
                                                   cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), rows, (int)S,
                                                   (int)H, (int)hd, inverse ? 1 : 0);
  SCIRS_CHECK_LAUNCH();
}

void tp_xent_stats(torch::Tensor logits, torch::Tensor targets, int64_t nvalid, int64_t v0, int64_t rank,
                   std::vector<int64_t> stats_dst, std::vector<int64_t> sig_flags, torch::Tensor epoch,
                   int64_t sig_idx) {
  CHECK_DTYPE(logits, at::kBFloat16);
  CHECK_CONTIG(logits);
  TORCH_CHECK(targets.scalar_type() == at::kLong, "targets must be int64");
  const long rows = logits.size(0);
  const int Vl = logits.size(1);
  const int dev = logits.get_device();
  c10::cuda::CUDAGuard guard(dev);
  const int grid = (int)((rows + 7) / 8);
  tp::xent_stats_kernel<<<grid, 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr()), targets.data_ptr<int64_t>(), rows, Vl, (int)nvalid,
      v0, (int)rank, (int)stats_dst.size(), tp::to_ptrs(stats_dst), tp::to_ptrs(sig_flags),
      reinterpret_cast<const unsigned*>(epoch.data_ptr()), (unsigned)sig_idx, tp::done_ctr(dev));
  SCIRS_CHECK_LAUNCH();
}

void tp_xent_finish(torch::Tensor logits, torch::Tensor targets, torch::Tensor stats, c10::optional<torch::Tensor> loss,
                    int64_t nvalid, int64_t v0, int64_t rank, double scale, torch::Tensor flags, torch::Tensor epoch,
                    int64_t wait_idx, double timeout_s) {
  CHECK_DTYPE(logits, at::kBFloat16);
  CHECK_DTYPE(stats, at::kFloat);
  const long rows = logits.size(0);
  const int Vl = logits.size(1);
  const int world = stats.size(0);
  TORCH_CHECK(stats.dim() == 3 && stats.size(1) == rows && stats.size(2) == 4, "stats [world, rows, 4]");
  const int dev = logits.get_device();
  c10::cuda::CUDAGuard guard(dev);
  float* lp = (loss.has_value() && loss->defined()) ? loss->data_ptr<float>() : nullptr;
  const int grid = (int)((rows + 7) / 8);
  tp::xent_finish_kernel<<<grid, 256, 0, cur_stream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), targets.data_ptr<int64_t>(),
      reinterpret_cast<const float4*>(stats.data_ptr()), lp, rows, Vl, (int)nvalid, v0, (int)rank, world,
      (float)scale, reinterpret_cast<const unsigned*>(flags.data_ptr()),
      reinterpret_cast<const unsigned*>(epoch.data_ptr()), (unsigned)wait_idx, (long long)(timeout_s * 1e9),
      status_ptr(dev));
  SCIRS_CHECK_LAUNCH();
}

}  // namespace scirs
