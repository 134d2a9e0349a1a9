// Tensor-parallel helper kernels: cross-rank signals, the reduction half of
// GEMM -> reduce-scatter, rotary position embedding, the vocabulary-parallel
// softmax cross-entropy, and the expert-parallel dispatch / combine.
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

// ---------------------------------------------------------------------------
// Expert parallelism: top-k mixture of experts with a per-expert capacity of C
// slots, L experts per rank, W ranks (expert e lives on rank e / L). A rank's
// assignments are numbered destination-major, send row q = (w * L + l) * C + c
// for expert e = w * L + l and slot c; every rank keeps, for each local expert,
// a receive buffer [L, W, C, D] (source-rank-major inside each expert).
//
// ep_dispatch_kernel: the permutation and the all-to-all in one pass. A warp
//   takes one send row, reads row idx[q] of `src` (zeros for an empty slot),
//   optionally scales it by scale[q], and stores it directly into rank w's
//   buffer, row l * sl + rank * sr + c, over NVLink. The last block to finish
//   signals every peer.
// ep_combine_kernel: the return all-to-all and the weighted sum in one pass.
//   After the owners' signals, a warp takes one token and reads its k expert
//   outputs straight from the owners' buffers (row ((e % L) * W + rank) * C +
//   slot), accumulating sum_j w_j * y_j in fp32.
// ep_grad_w_kernel: the routing-weight gradient <dout[t], y_j>, y_j read from
//   the owner's buffer.
//
// Reference parity: scirs2-neural/src/layers/moe.rs:120-440 (top-k gating,
// capacity, weighted combination; single device there).

struct PeerBase {
  char* p[kMaxPeers];
};

constexpr int kEpMaxK = 8;

__device__ __forceinline__ void scale_bf16x8(uint4& q, float s) {
  uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) w[e] = pack_bf16x2(bf16_lo(w[e]) * s, bf16_hi(w[e]) * s);
  q = make_uint4(w[0], w[1], w[2], w[3]);
}

__global__ void __launch_bounds__(256) ep_dispatch_kernel(const __nv_bfloat16* __restrict__ src, long nsrc,
                                                          const int* __restrict__ idx,
                                                          const float* __restrict__ scale, PeerBase dst, int L,
                                                          int C, long sl, long sr, int D, int rank, int world,
                                                          DevStatus* st, FlagPtrs sig, const unsigned* epoch,
                                                          unsigned sig_idx, unsigned* done) {
  const int lane = threadIdx.x & 31;
  const long nwarps = ((long)gridDim.x * blockDim.x) >> 5;
  const long rows = (long)world * L * C;
  const long per_rank = (long)L * C;
  const int dv = D / 8;
  for (long q = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; q < rows; q += nwarps) {
    const int w = (int)(q / per_rank);
    const long rem = q - w * per_rank;
    const int l = (int)(rem / C);
    const int c = (int)(rem - (long)l * C);
    const int t = idx[q];
    const bool have = t >= 0 && input_in_range(t, nsrc, st, 80);
    const float s = (have && scale != nullptr) ? scale[q] : 1.f;
    const uint4* sp = reinterpret_cast<const uint4*>(src + (have ? (long)t * D : 0L));
    uint4* dp = reinterpret_cast<uint4*>(dst.p[w] + ((long)l * sl + (long)rank * sr + c) * D * (long)sizeof(__nv_bfloat16));
    for (int v = lane; v < dv; v += 32) {
      uint4 x = make_uint4(0u, 0u, 0u, 0u);
      if (have) {
        x = sp[v];
        if (scale != nullptr) scale_bf16x8(x, s);
      }
      dp[v] = x;
    }
  }
  last_block_signal(sig, world, epoch, sig_idx, done);
}

// Pointers to the (at most kEpMaxK) kept expert outputs of token t; returns
// how many.
__device__ __forceinline__ int ep_rows(const PeerBase& srcp, const int* expert, const int* slot, const float* wt,
                                       long t, int k, int L, int C, int D, int rank, int world, DevStatus* st,
                                       const uint4** rows, float* wj) {
  int n = 0;
  for (int j = 0; j < k; ++j) {
    const int e = expert[t * k + j];
    const int s = slot[t * k + j];
    if (s < 0) continue;
    if (!input_in_range(e, (long)L * world, st, 82) || !input_in_range(s, C, st, 83)) continue;
    const int w = e / L;
    const int l = e - w * L;
    rows[n] = reinterpret_cast<const uint4*>(srcp.p[w] +
                                             ((((long)l * world + rank) * C + s) * D) * (long)sizeof(__nv_bfloat16));
    wj[n] = wt != nullptr ? wt[t * k + j] : 1.f;
    ++n;
  }
  return n;
}

__global__ void __launch_bounds__(256) ep_combine_kernel(PeerBase srcp, const int* __restrict__ expert,
                                                         const int* __restrict__ slot, const float* __restrict__ wt,
                                                         int k, long T, int L, int C, int D, int rank, int world,
                                                         const unsigned* flags, const unsigned* epoch,
                                                         unsigned wait_idx, long long timeout_ns, DevStatus* st,
                                                         __nv_bfloat16* __restrict__ out) {
  if (flags != nullptr && !block_wait(flags, epoch, wait_idx, rank, world, timeout_ns, st, 81)) return;
  const int lane = threadIdx.x & 31;
  const long nwarps = ((long)gridDim.x * blockDim.x) >> 5;
  const int dv = D / 8;
  for (long t = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < T; t += nwarps) {
    const uint4* rows[kEpMaxK];
    float wj[kEpMaxK];
    const int n = ep_rows(srcp, expert, slot, wt, t, k, L, C, D, rank, world, st, rows, wj);
    uint4* op = reinterpret_cast<uint4*>(out + t * D);
    for (int v = lane; v < dv; v += 32) {
      float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int j = 0; j < n; ++j) {
        const uint4 q = __ldcg(rows[j] + v);
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) f[2 * e] += wj[j] * bf16_lo(w[e]), f[2 * e + 1] += wj[j] * bf16_hi(w[e]);
      }
      op[v] = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                         pack_bf16x2(f[6], f[7]));
    }
  }
}

__global__ void __launch_bounds__(256) ep_grad_w_kernel(PeerBase srcp, const int* __restrict__ expert,
                                                        const int* __restrict__ slot,
                                                        const __nv_bfloat16* __restrict__ dout,
                                                        float* __restrict__ gw, int k, long T, int L, int C, int D,
                                                        int rank, int world, DevStatus* st) {
  const int lane = threadIdx.x & 31;
  const long nwarps = ((long)gridDim.x * blockDim.x) >> 5;
  const int dv = D / 8;
  for (long a = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; a < T * k; a += nwarps) {
    const long t = a / k;
    const int e = expert[a];
    const int s = slot[a];
    float acc = 0.f;
    if (s >= 0 && input_in_range(e, (long)L * world, st, 85) && input_in_range(s, C, st, 86)) {
      const int w = e / L;
      const int l = e - w * L;
      const uint4* yr = reinterpret_cast<const uint4*>(
          srcp.p[w] + ((((long)l * world + rank) * C + s) * D) * (long)sizeof(__nv_bfloat16));
      const uint4* dr = reinterpret_cast<const uint4*>(dout + t * D);
      for (int v = lane; v < dv; v += 32) {
        const uint4 qy = __ldcg(yr + v);
        const uint4 qd = dr[v];
        const uint32_t a4[4] = {qy.x, qy.y, qy.z, qy.w};
        const uint32_t b4[4] = {qd.x, qd.y, qd.z, qd.w};
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) acc += bf16_lo(a4[e2]) * bf16_lo(b4[e2]) + bf16_hi(a4[e2]) * bf16_hi(b4[e2]);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) gw[a] = acc;
  }
}

// ---------------------------------------------------------------------------
// Vocabulary-gradient routing for sharded data parallelism. The fp32
// gradient of a [V, D] embedding table is sharded by rows over the W ranks
// (rank o owns rows [o * R, (o + 1) * R)). The lookup part of the gradient
// (row tok[m] += dout[m] for this rank's M tokens) is sent to the owners
// instead of being reduced densely:
//
// vocab_route_kernel: a warp per token row m. Lane w < W writes the id word
//   ids_w[rank * M + m] = tok[m] - o * R on the owner o (-1 on every other
//   rank) and the warp stores the bf16 row into rows_o[rank * M + m] over
//   NVLink. The last block signals every peer.
// vocab_accum_kernel: on the owner, after every source's signal, a warp per
//   received row adds scale * row into its shard row with fp32 vector
//   atomics (local memory only).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) vocab_route_kernel(const int64_t* __restrict__ tok,
                                                          const __nv_bfloat16* __restrict__ dout, long M, int D,
                                                          long R, long V, PeerBase rows, PeerBase ids, int rank,
                                                          int world, DevStatus* st, FlagPtrs sig,
                                                          const unsigned* epoch, unsigned sig_idx, unsigned* done) {
  const int lane = threadIdx.x & 31;
  const long nwarps = ((long)gridDim.x * blockDim.x) >> 5;
  const int dv = D / 8;
  for (long m = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; m < M; m += nwarps) {
    const long t = tok[m];
    const bool valid = input_in_range(t, V, st, 87);
    const int o = valid ? (int)(t / R) : -1;
    if (lane < world) {
      int* ip = reinterpret_cast<int*>(ids.p[lane]) + (long)rank * M + m;
      *ip = (lane == o) ? (int)(t - (long)o * R) : -1;
    }
    if (!valid) continue;
    const uint4* sp = reinterpret_cast<const uint4*>(dout + m * D);
    uint4* dp = reinterpret_cast<uint4*>(rows.p[o] + ((long)rank * M + m) * D * (long)sizeof(__nv_bfloat16));
    for (int v = lane; v < dv; v += 32) dp[v] = sp[v];
  }
  last_block_signal(sig, world, epoch, sig_idx, done);
}

__global__ void __launch_bounds__(256) vocab_accum_kernel(const __nv_bfloat16* __restrict__ rows,
                                                          const int* __restrict__ ids, float* __restrict__ shard,
                                                          float scale, long M, int D, long R, int rank, int world,
                                                          const unsigned* flags, const unsigned* epoch,
                                                          unsigned wait_idx, long long timeout_ns, DevStatus* st) {
  if (!block_wait(flags, epoch, wait_idx, rank, world, timeout_ns, st, 88)) return;
  const int lane = threadIdx.x & 31;
  const long nwarps = ((long)gridDim.x * blockDim.x) >> 5;
  const int dv = D / 8;
  const long total = (long)world * M;
  for (long q = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; q < total; q += nwarps) {
    const int id = __ldcg(ids + q);
    if (id < 0) continue;
    if (!input_in_range(id, R, st, 89)) continue;
    const uint4* rp = reinterpret_cast<const uint4*>(rows + q * D);
    float* gp = shard + (long)id * D;
    for (int v = lane; v < dv; v += 32) {
      const uint4 x = __ldcg(rp + v);
      const uint32_t w[4] = {x.x, x.y, x.z, x.w};
      atomicAdd(reinterpret_cast<float4*>(gp + 8 * v),
                make_float4(scale * bf16_lo(w[0]), scale * bf16_hi(w[0]), scale * bf16_lo(w[1]), scale * bf16_hi(w[1])));
      atomicAdd(reinterpret_cast<float4*>(gp + 8 * v + 4),
                make_float4(scale * bf16_lo(w[2]), scale * bf16_hi(w[2]), scale * bf16_lo(w[3]), scale * bf16_hi(w[3])));
    }
  }
}

// A bounded wait on every peer's signal `idx`, for consumers that are not
// kernels of this file (library GEMMs on the received rows).
__global__ void wait_kernel(const unsigned* flags, const unsigned* epoch, unsigned idx, int rank, int world,
                            long long timeout_ns, DevStatus* st) {
  block_wait(flags, epoch, idx, rank, world, timeout_ns, st, 84);
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

static tp::PeerBase to_base(const std::vector<int64_t>& v) {
  tp::PeerBase b;
  memset(&b, 0, sizeof(b));
  TORCH_CHECK(!v.empty() && v.size() <= (size_t)tp::kMaxPeers, "1..8 ranks");
  for (size_t i = 0; i < v.size(); ++i) {
    TORCH_CHECK(v[i] % 16 == 0, "peer buffers must be 16-byte aligned");
    b.p[i] = reinterpret_cast<char*>(v[i]);
  }
  return b;
}

static int warp_grid(long warps, int dev) {
  return (int)std::max<long>(1, std::min<long>((warps + 7) / 8, 8L * num_sms(dev)));
}

// Expert-parallel dispatch (see ep_dispatch_kernel): `dst[w]` is rank w's
// receive buffer, `idx` [W * L * C] int32 the source row of every send row
// (-1: empty slot), `scale` an optional fp32 factor per send row.
void ep_dispatch(torch::Tensor src, torch::Tensor idx, c10::optional<torch::Tensor> scale, std::vector<int64_t> dst,
                 int64_t L, int64_t C, int64_t sl, int64_t sr, int64_t rank, std::vector<int64_t> sig_flags,
                 torch::Tensor epoch, int64_t sig_idx) {
  CHECK_DTYPE(src, at::kBFloat16);
  CHECK_CONTIG(src);
  CHECK_DTYPE(idx, at::kInt);
  CHECK_CONTIG(idx);
  TORCH_CHECK(src.dim() == 2 && src.size(1) % 8 == 0, "src [rows, D], D a multiple of 8");
  const int world = (int)dst.size();
  TORCH_CHECK(idx.numel() == world * L * C, "idx must have world * L * C entries");
  TORCH_CHECK(sig_flags.empty() || (int)sig_flags.size() == world, "one signal word per rank");
  const float* sp = nullptr;
  if (scale.has_value() && scale->defined()) {
    CHECK_DTYPE((*scale), at::kFloat);
    CHECK_CONTIG((*scale));
    TORCH_CHECK(scale->numel() == idx.numel(), "scale must match idx");
    sp = scale->data_ptr<float>();
  }
  const int dev = src.get_device();
  c10::cuda::CUDAGuard guard(dev);
  tp::ep_dispatch_kernel<<<warp_grid(idx.numel(), dev), 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(src.data_ptr()), src.size(0), idx.data_ptr<int>(), sp, to_base(dst),
      (int)L, (int)C, sl, sr, (int)src.size(1), (int)rank, world, status_ptr(dev), tp::to_ptrs(sig_flags),
      reinterpret_cast<const unsigned*>(epoch.data_ptr()), (unsigned)sig_idx, tp::done_ctr(dev));
  SCIRS_CHECK_LAUNCH();
}

// Expert-parallel combine (see ep_combine_kernel): `srcs[w]` is rank w's
// output buffer [L, W, C, D]; waits for signal `wait_idx` when `flags` given.
void ep_combine(std::vector<int64_t> srcs, torch::Tensor expert, torch::Tensor slot, c10::optional<torch::Tensor> wt,
                torch::Tensor out, int64_t L, int64_t C, int64_t rank, c10::optional<torch::Tensor> flags,
                torch::Tensor epoch, int64_t wait_idx, double timeout_s) {
  CHECK_DTYPE(expert, at::kInt);
  CHECK_DTYPE(slot, at::kInt);
  CHECK_CONTIG(expert);
  CHECK_CONTIG(slot);
  CHECK_DTYPE(out, at::kBFloat16);
  CHECK_CONTIG(out);
  TORCH_CHECK(expert.dim() == 2 && expert.sizes() == slot.sizes() && expert.size(1) <= tp::kEpMaxK,
              "expert / slot [T, k], k <= 8");
  TORCH_CHECK(out.dim() == 2 && out.size(0) == expert.size(0) && out.size(1) % 8 == 0, "out [T, D]");
  const float* wp = nullptr;
  if (wt.has_value() && wt->defined()) {
    CHECK_DTYPE((*wt), at::kFloat);
    CHECK_CONTIG((*wt));
    TORCH_CHECK(wt->sizes() == expert.sizes(), "wt [T, k]");
    wp = wt->data_ptr<float>();
  }
  const int world = (int)srcs.size();
  const int dev = out.get_device();
  c10::cuda::CUDAGuard guard(dev);
  const unsigned* fp = (flags.has_value() && flags->defined()) ? reinterpret_cast<const unsigned*>(flags->data_ptr())
                                                               : nullptr;
  tp::ep_combine_kernel<<<warp_grid(out.size(0), dev), 256, 0, cur_stream()>>>(
      to_base(srcs), expert.data_ptr<int>(), slot.data_ptr<int>(), wp, (int)expert.size(1), out.size(0), (int)L,
      (int)C, (int)out.size(1), (int)rank, world, fp, reinterpret_cast<const unsigned*>(epoch.data_ptr()),
      (unsigned)wait_idx, (long long)(timeout_s * 1e9), status_ptr(dev),
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  SCIRS_CHECK_LAUNCH();
}

// gw[t, j] = <dout[t], expert output j of token t> (0 for dropped assignments).
void ep_grad_w(std::vector<int64_t> srcs, torch::Tensor expert, torch::Tensor slot, torch::Tensor dout,
               torch::Tensor gw, int64_t L, int64_t C, int64_t rank) {
  CHECK_DTYPE(expert, at::kInt);
  CHECK_DTYPE(slot, at::kInt);
  CHECK_CONTIG(expert);
  CHECK_CONTIG(slot);
  CHECK_DTYPE(dout, at::kBFloat16);
  CHECK_CONTIG(dout);
  CHECK_DTYPE(gw, at::kFloat);
  CHECK_CONTIG(gw);
  TORCH_CHECK(expert.dim() == 2 && expert.sizes() == slot.sizes() && gw.sizes() == expert.sizes(),
              "expert / slot / gw [T, k]");
  TORCH_CHECK(dout.dim() == 2 && dout.size(0) == expert.size(0) && dout.size(1) % 8 == 0, "dout [T, D]");
  const int dev = dout.get_device();
  c10::cuda::CUDAGuard guard(dev);
  tp::ep_grad_w_kernel<<<warp_grid(expert.numel(), dev), 256, 0, cur_stream()>>>(
      to_base(srcs), expert.data_ptr<int>(), slot.data_ptr<int>(),
      reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), gw.data_ptr<float>(), (int)expert.size(1),
      expert.size(0), (int)L, (int)C, (int)dout.size(1), (int)rank, (int)srcs.size(), status_ptr(dev));
  SCIRS_CHECK_LAUNCH();
}

// Vocabulary-gradient routing (see vocab_route_kernel): rows[w] / ids[w] are
// rank w's receive buffers [W, M, D] bf16 and [W, M] int32.
void vocab_route(torch::Tensor tok, torch::Tensor dout, int64_t R, int64_t V, std::vector<int64_t> rows,
                 std::vector<int64_t> ids, int64_t rank, std::vector<int64_t> sig_flags, torch::Tensor epoch,
                 int64_t sig_idx) {
  CHECK_DTYPE(tok, at::kLong);
  CHECK_CONTIG(tok);
  CHECK_DTYPE(dout, at::kBFloat16);
  CHECK_CONTIG(dout);
  TORCH_CHECK(dout.dim() == 2 && dout.size(0) == tok.numel() && dout.size(1) % 8 == 0, "dout [M, D], D % 8 == 0");
  const int world = (int)rows.size();
  TORCH_CHECK(world >= 1 && world <= tp::kMaxPeers && (int)ids.size() == world && (int)sig_flags.size() == world,
              "one receive buffer, id buffer and signal word per rank");
  TORCH_CHECK(R > 0 && R * world >= V, "rows per rank must cover the vocabulary");
  const int dev = tok.get_device();
  c10::cuda::CUDAGuard guard(dev);
  tp::vocab_route_kernel<<<warp_grid(tok.numel(), dev), 256, 0, cur_stream()>>>(
      tok.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), tok.numel(),
      (int)dout.size(1), R, V, to_base(rows), to_base(ids), (int)rank, world, status_ptr(dev), tp::to_ptrs(sig_flags),
      reinterpret_cast<const unsigned*>(epoch.data_ptr()), (unsigned)sig_idx, tp::done_ctr(dev));
  SCIRS_CHECK_LAUNCH();
}

// shard [R, D] fp32 += scale * (received rows routed to this rank).
void vocab_accum(torch::Tensor rows, torch::Tensor ids, torch::Tensor shard, double scale, int64_t rank,
                 torch::Tensor flags, torch::Tensor epoch, int64_t wait_idx, double timeout_s) {
  CHECK_DTYPE(rows, at::kBFloat16);
  CHECK_CONTIG(rows);
  CHECK_DTYPE(ids, at::kInt);
  CHECK_CONTIG(ids);
  CHECK_DTYPE(shard, at::kFloat);
  CHECK_CONTIG(shard);
  TORCH_CHECK(rows.dim() == 3 && ids.dim() == 2 && rows.size(0) == ids.size(0) && rows.size(1) == ids.size(1),
              "rows [W, M, D], ids [W, M]");
  TORCH_CHECK(shard.dim() == 2 && shard.size(1) == rows.size(2) && rows.size(2) % 8 == 0, "shard [R, D]");
  const int world = (int)rows.size(0);
  TORCH_CHECK(world <= tp::kMaxPeers && flags.numel() >= world && flags.element_size() == 4, "flags per rank");
  const int dev = rows.get_device();
  c10::cuda::CUDAGuard guard(dev);
  tp::vocab_accum_kernel<<<warp_grid(ids.numel(), dev), 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(rows.data_ptr()), ids.data_ptr<int>(), shard.data_ptr<float>(),
      (float)scale, rows.size(1), (int)rows.size(2), shard.size(0), (int)rank, world,
      reinterpret_cast<const unsigned*>(flags.data_ptr()), reinterpret_cast<const unsigned*>(epoch.data_ptr()),
      (unsigned)wait_idx, (long long)(timeout_s * 1e9), status_ptr(dev));
  SCIRS_CHECK_LAUNCH();
}

void tp_wait(torch::Tensor flags, torch::Tensor epoch, int64_t idx, int64_t rank, int64_t world, double timeout_s) {
  TORCH_CHECK(world >= 1 && world <= tp::kMaxPeers && flags.numel() >= world && flags.element_size() == 4,
              "flags: one 32-bit word per rank");
  const int dev = flags.get_device();
  c10::cuda::CUDAGuard guard(dev);
  tp::wait_kernel<<<1, 32, 0, cur_stream()>>>(reinterpret_cast<const unsigned*>(flags.data_ptr()),
                                              reinterpret_cast<const unsigned*>(epoch.data_ptr()), (unsigned)idx,
                                              (int)rank, (int)world, (long long)(timeout_s * 1e9), status_ptr(dev));
  SCIRS_CHECK_LAUNCH();
}

}  // namespace scirs
