// Paged KV cache kernels for decoding: append new tokens' K/V into pages,
// and single-query attention over each sequence's page chain (split over
// the key axis, then combined), with grouped-query heads.
//
// Pool layout: k_pool / v_pool [num_pages, block_size, Hkv, HD] bf16; a
// sequence's page chain is a row of block_tables [B, max_pages] (int32 page
// ids); seq_lens [B] (int32) counts its tokens.
//
// Decode attention (one new query per sequence, H query heads sharing Hkv
// key/value heads, G = H / Hkv): grid (splits, Hkv, B), 128 threads. A CTA
// walks its split's tokens in chunks of 128 (one token per thread for the
// scores of all G heads, K row read with 16-byte loads), keeps a running
// max / sum per head in shared memory, and accumulates P V with threads
// laid out over (head, 8-dim slice). Decoding is bandwidth-bound: every K/V
// byte of the chain is read once per (sequence, KV head). Each split writes
// (max, sum, unnormalised O); the combine kernel merges the splits.
//
// Reference parity: scirs2-neural/src/inference/paged_attention.rs:113-283
// (PagedAttentionForward::forward over a KvPagePool page chain),
// kv_page.rs:96-140 (write_kv), block_manager.rs:161-196 (write_token_kv).
#include "host_common.h"

#include <type_traits>

namespace scirs {
namespace paged {

constexpr int kT = 128;  // tokens per chunk = threads per CTA
constexpr int kMaxG = 8;
constexpr int kMaxHD = 128;

// k_new/v_new [n, Hkv, HD] for tokens at positions pos[i] of sequences
// seq[i]; slot = block_tables[seq][pos / bs], pos % bs.
__global__ void append_kernel(const __nv_bfloat16* __restrict__ k_new, const __nv_bfloat16* __restrict__ v_new,
                              __nv_bfloat16* __restrict__ k_pool, __nv_bfloat16* __restrict__ v_pool,
                              const int* __restrict__ block_tables, const int* __restrict__ seq,
                              const int* __restrict__ pos, int n, int max_pages, int bs, int row_vecs,
                              int num_seqs, int num_pages, DevStatus* st) {
  const long total = (long)n * row_vecs;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int tok = (int)(i / row_vecs), c = (int)(i % row_vecs);
    const int s = seq[tok], p = pos[tok];
    if (!input_in_range(s, num_seqs, st, 90) || !input_in_range(p / bs, max_pages, st, 91) || p < 0) continue;
    const int page = block_tables[(long)s * max_pages + p / bs];
    if (!input_in_range(page, num_pages, st, 92)) continue;
    const long dst = ((long)page * bs + p % bs) * row_vecs + c;
    reinterpret_cast<uint4*>(k_pool)[dst] = reinterpret_cast<const uint4*>(k_new)[i];
    reinterpret_cast<uint4*>(v_pool)[dst] = reinterpret_cast<const uint4*>(v_new)[i];
  }
}

template <int HD>
__global__ void __launch_bounds__(kT) decode_kernel(const __nv_bfloat16* __restrict__ q,
                                                    const __nv_bfloat16* __restrict__ k_pool,
                                                    const __nv_bfloat16* __restrict__ v_pool,
                                                    const int* __restrict__ block_tables,
                                                    const int* __restrict__ seq_lens, float* __restrict__ part_o,
                                                    float* __restrict__ part_ml, int H, int Hkv, int bs,
                                                    int max_pages, int tokens_per_split, float scale_log2,
                                                    int num_pages, DevStatus* st) {
  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int G = H / Hkv;
  const int tid = threadIdx.x;
  __shared__ float qs[kMaxG][HD];
  __shared__ float ps[kMaxG][kT];
  __shared__ float red[kMaxG][kT / 32];
  __shared__ float m_run[kMaxG], l_run[kMaxG], alpha_s[kMaxG];
  for (int i = tid; i < G * HD; i += kT) {
    const int g = i / HD, d = i % HD;
    qs[g][d] = __bfloat162float(q[((long)b * H + hk * G + g) * HD + d]);
  }
  if (tid < G) {
    m_run[tid] = -INFINITY;
    l_run[tid] = 0.f;
  }
  // output slice owned by this thread: head og, dims [od, od + ODIM)
  constexpr int ODIM = (HD * kMaxG) / kT;  // 4 (HD 64) or 8 (HD 128) when G = 8
  const int og = tid / (HD / ODIM), od = (tid % (HD / ODIM)) * ODIM;
  float acc[ODIM];
#pragma unroll
  for (int e = 0; e < ODIM; ++e) acc[e] = 0.f;
  __syncthreads();
  const int len = min(seq_lens[b], max_pages * bs);  // tokens past the page table are not addressable
  if (tid == 0 && seq_lens[b] > max_pages * bs) report_status(st, kStBounds, 93, (unsigned)seq_lens[b]);
  const int t_begin = split * tokens_per_split;
  const int t_end = min(len, t_begin + tokens_per_split);
  const long row = (long)Hkv * HD;  // elements per token slot
  const int* bt = block_tables + (long)b * max_pages;
  for (int c0 = t_begin; c0 < t_end; c0 += kT) {
    // ---- scores: thread = token
    const int t = c0 + tid;
    float sc[kMaxG];
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) sc[g] = -INFINITY;
    const int kpage = (t < t_end) ? bt[t / bs] : 0;
    if (t < t_end && input_in_range(kpage, num_pages, st, 94)) {
      const int page = kpage;
      const __nv_bfloat16* kr = k_pool + ((long)page * bs + t % bs) * row + (long)hk * HD;
#pragma unroll
      for (int g = 0; g < kMaxG; ++g) sc[g] = 0.f;
#pragma unroll
      for (int d = 0; d < HD; d += 8) {
        const uint4 u = *reinterpret_cast<const uint4*>(kr + d);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float k0 = bf16_lo(w[e]), k1 = bf16_hi(w[e]);
#pragma unroll
          for (int g = 0; g < kMaxG; ++g)
            if (g < G) sc[g] = fmaf(qs[g][d + 2 * e], k0, fmaf(qs[g][d + 2 * e + 1], k1, sc[g]));
        }
      }
#pragma unroll
      for (int g = 0; g < kMaxG; ++g) sc[g] *= scale_log2;
    }
    // ---- chunk max per head
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
      if (g >= G) break;
      const float m = warp_max(sc[g]);
      if ((tid & 31) == 0) red[g][tid >> 5] = m;
    }
    __syncthreads();
    if (tid < G) {
      float m = red[tid][0];
      for (int w = 1; w < kT / 32; ++w) m = fmaxf(m, red[tid][w]);
      const float m_new = fmaxf(m_run[tid], m);
      alpha_s[tid] = (m_run[tid] == -INFINITY) ? 0.f : ex2_fast(m_run[tid] - m_new);
      m_run[tid] = m_new;
    }
    __syncthreads();
    // ---- probabilities and chunk sums
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
      if (g >= G) break;
      const float mr = m_run[g];
      const float pv = (sc[g] == -INFINITY || mr == -INFINITY) ? 0.f : ex2_fast(sc[g] - mr);
      ps[g][tid] = pv;
      const float s = warp_sum(pv);
      if ((tid & 31) == 0) red[g][tid >> 5] = s;
    }
    __syncthreads();
    if (tid < G) {
      float s = 0.f;
      for (int w = 0; w < kT / 32; ++w) s += red[tid][w];
      l_run[tid] = l_run[tid] * alpha_s[tid] + s;
    }
    // ---- O += P V (thread = head og, dims od..od+ODIM)
    if (og < G) {
      const float al = alpha_s[og];
#pragma unroll
      for (int e = 0; e < ODIM; ++e) acc[e] *= al;
      const int n = min(kT, t_end - c0);
      int i = 0;
      // eight tokens per step: their page ids and V slices are all loaded before the FMAs,
      // so each thread has eight independent loads in flight instead of one
      constexpr int kU = 8;
      using VT = typename std::conditional<ODIM == 8, uint4, uint2>::type;
      for (; i + kU <= n; i += kU) {
        VT vv[kU];
        float pw[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int tt = c0 + i + u;
          const int page = bt[tt / bs];
          const bool okp = page >= 0 && page < num_pages;  // a bad page was reported in the score pass
          const __nv_bfloat16* vr = v_pool + ((long)(okp ? page : 0) * bs + tt % bs) * row + (long)hk * HD + od;
          vv[u] = *reinterpret_cast<const VT*>(vr);
          pw[u] = okp ? ps[og][i + u] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const uint32_t* w = reinterpret_cast<const uint32_t*>(&vv[u]);
#pragma unroll
          for (int e = 0; e < ODIM / 2; ++e) {
            acc[2 * e] = fmaf(pw[u], bf16_lo(w[e]), acc[2 * e]);
            acc[2 * e + 1] = fmaf(pw[u], bf16_hi(w[e]), acc[2 * e + 1]);
          }
        }
      }
      for (; i < n; ++i) {
        const int tt = c0 + i;
        const int page = bt[tt / bs];
        if (page < 0 || page >= num_pages) continue;  // reported in the score pass; its score is -inf
        const __nv_bfloat16* vr = v_pool + ((long)page * bs + tt % bs) * row + (long)hk * HD + od;
        const float pv = ps[og][i];
        if (ODIM == 8) {
          const uint4 u = *reinterpret_cast<const uint4*>(vr);
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            acc[2 * e] = fmaf(pv, bf16_lo(w[e]), acc[2 * e]);
            acc[2 * e + 1] = fmaf(pv, bf16_hi(w[e]), acc[2 * e + 1]);
          }
        } else {
          const uint2 u = *reinterpret_cast<const uint2*>(vr);
          acc[0] = fmaf(pv, bf16_lo(u.x), acc[0]);
          acc[1] = fmaf(pv, bf16_hi(u.x), acc[1]);
          acc[2] = fmaf(pv, bf16_lo(u.y), acc[2]);
          acc[3] = fmaf(pv, bf16_hi(u.y), acc[3]);
        }
      }
    }
    __syncthreads();
  }
  // ---- partial results of this split, laid out [b, head, split]
  if (og < G) {
    float* o = part_o + ((((long)b * H + hk * G + og) * gridDim.x + split) * HD) + od;
#pragma unroll
    for (int e = 0; e < ODIM; ++e) o[e] = acc[e];
  }
  if (tid < G) {
    float* ml = part_ml + ((((long)b * H + hk * G + tid) * gridDim.x + split) * 2);
    ml[0] = m_run[tid];
    ml[1] = l_run[tid];
  }
}

// out[b, h, :] = sum_s exp2(m_s - M) O_s / sum_s exp2(m_s - M) l_s
__global__ void combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml,
                               __nv_bfloat16* __restrict__ out, int splits, int HD) {
  const long bh = blockIdx.x;
  const float* ml = part_ml + bh * splits * 2;
  float M = -INFINITY;
  for (int s = 0; s < splits; ++s) M = fmaxf(M, ml[2 * s]);
  for (int d = threadIdx.x; d < HD; d += blockDim.x) {
    float num = 0.f, den = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float m = ml[2 * s];
      if (m == -INFINITY) continue;
      const float w = ex2_fast(m - M);
      num += w * part_o[(bh * splits + s) * HD + d];
      den += w * ml[2 * s + 1];
    }
    out[bh * HD + d] = __float2bfloat16(den > 0.f ? num / den : 0.f);
  }
}

}  // namespace paged

void paged_kv_append(torch::Tensor k_new, torch::Tensor v_new, torch::Tensor k_pool, torch::Tensor v_pool,
                     torch::Tensor block_tables, torch::Tensor seq, torch::Tensor pos) {
  for (auto* t : {&k_new, &v_new, &k_pool, &v_pool}) {
    CHECK_DTYPE((*t), at::kBFloat16);
    CHECK_CONTIG((*t));
  }
  for (auto* t : {&block_tables, &seq, &pos}) {
    TORCH_CHECK(t->scalar_type() == at::kInt && t->is_contiguous(), "index tensors must be contiguous int32");
  }
  TORCH_CHECK(k_pool.dim() == 4 && k_pool.sizes() == v_pool.sizes(), "pools [num_pages, block_size, Hkv, HD]");
  const int bs = k_pool.size(1);
  const long row = k_pool.size(2) * k_pool.size(3);
  TORCH_CHECK(row % 8 == 0 && k_new.numel() == seq.numel() * row && v_new.numel() == k_new.numel(),
              "k_new/v_new must be [n, Hkv, HD] matching the pool");
  TORCH_CHECK(pos.numel() == seq.numel(), "seq/pos size mismatch");
  const int n = seq.numel();
  if (n == 0) return;
  c10::cuda::CUDAGuard guard(k_pool.get_device());
  const long work = (long)n * (row / 8);
  const int grid = (int)std::max<long>(1, std::min<long>((work + 255) / 256, 4L * num_sms(k_pool.get_device())));
  paged::append_kernel<<<grid, 256, 0, cur_stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(k_new.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(v_new.data_ptr()),
      reinterpret_cast<__nv_bfloat16*>(k_pool.data_ptr()), reinterpret_cast<__nv_bfloat16*>(v_pool.data_ptr()),
      block_tables.data_ptr<int>(), seq.data_ptr<int>(), pos.data_ptr<int>(), n, (int)block_tables.size(1), bs,
      (int)(row / 8), (int)block_tables.size(0), (int)k_pool.size(0), status_ptr(k_pool.get_device()));
  SCIRS_CHECK_LAUNCH();
}

// q [B, H, HD] bf16 -> out [B, H, HD] bf16. part_o fp32 [B, H, splits, HD] and
// part_ml fp32 [B, H, splits, 2] are scratch (caller-provided).
void paged_attention_decode(torch::Tensor q, torch::Tensor k_pool, torch::Tensor v_pool, torch::Tensor block_tables,
                            torch::Tensor seq_lens, torch::Tensor out, torch::Tensor part_o, torch::Tensor part_ml,
                            int64_t tokens_per_split, double scale) {
  CHECK_DTYPE(q, at::kBFloat16);
  CHECK_DTYPE(out, at::kBFloat16);
  CHECK_CONTIG(q);
  CHECK_CONTIG(out);
  CHECK_DTYPE(part_o, at::kFloat);
  CHECK_DTYPE(part_ml, at::kFloat);
  TORCH_CHECK(q.dim() == 3, "q must be [B, H, HD]");
  const int B = q.size(0), H = q.size(1), HD = q.size(2);
  TORCH_CHECK(k_pool.dim() == 4 && k_pool.size(3) == HD, "pool head_dim mismatch");
  const int Hkv = k_pool.size(2), bs = k_pool.size(1);
  TORCH_CHECK(H % Hkv == 0 && H / Hkv <= paged::kMaxG, "query heads per KV head must be <= 8");
  TORCH_CHECK(HD == 64 || HD == 128, "head_dim must be 64 or 128");
  TORCH_CHECK(tokens_per_split > 0 && tokens_per_split % paged::kT == 0, "tokens_per_split must be a multiple of 128");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt && seq_lens.scalar_type() == at::kInt, "int32 tables");
  const int splits = part_ml.size(2);
  TORCH_CHECK(part_ml.numel() == (long)B * H * splits * 2 && part_o.numel() == (long)B * H * splits * HD,
              "scratch sizes must be [B, H, splits, HD] and [B, H, splits, 2]");
  TORCH_CHECK((long)splits * tokens_per_split >= (long)block_tables.size(1) * bs, "splits do not cover the chain");
  c10::cuda::CUDAGuard guard(q.get_device());
  dim3 grid(splits, Hkv, B);
  const float sl2 = (float)(scale * 1.4426950408889634);
  auto st = cur_stream();
  if (HD == 64)
    paged::decode_kernel<64><<<grid, paged::kT, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(k_pool.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(v_pool.data_ptr()), block_tables.data_ptr<int>(),
        seq_lens.data_ptr<int>(), part_o.data_ptr<float>(), part_ml.data_ptr<float>(), H, Hkv, bs,
        (int)block_tables.size(1), (int)tokens_per_split, sl2, (int)k_pool.size(0), status_ptr(q.get_device()));
  else
    paged::decode_kernel<128><<<grid, paged::kT, 0, st>>>(
        reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(k_pool.data_ptr()),
        reinterpret_cast<const __nv_bfloat16*>(v_pool.data_ptr()), block_tables.data_ptr<int>(),
        seq_lens.data_ptr<int>(), part_o.data_ptr<float>(), part_ml.data_ptr<float>(), H, Hkv, bs,
        (int)block_tables.size(1), (int)tokens_per_split, sl2, (int)k_pool.size(0), status_ptr(q.get_device()));
  SCIRS_CHECK_LAUNCH();
  paged::combine_kernel<<<B * H, 64, 0, st>>>(part_o.data_ptr<float>(), part_ml.data_ptr<float>(),
                                              reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), splits, HD);
  SCIRS_CHECK_LAUNCH();
}

}  // namespace scirs
