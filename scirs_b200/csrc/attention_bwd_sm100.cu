// FlashAttention backward on tcgen05 for head_dim 128.
//
// One CTA = one 128-key tile of one (batch, head); it walks the 64-query
// blocks that can see those keys (all, or q >= k for causal). Per block:
//
//   S^T  = K Q^T     [128 keys x 64 q]   TMEM cols [  0,  64)
//   dP^T = V dO^T    [128 keys x 64 q]   TMEM cols [ 64, 128)
//   P^T  = exp2(S^T * scale * log2e - lse2_q),  dS^T = P^T (dP^T - delta_q)
//          (8 warps, thread = key row x 32 query columns) -> bf16 smem
//   dV  += P^T dO    [128 keys x 128]    TMEM cols [128, 256)
//   dK  += dS^T Q    [128 keys x 128]    TMEM cols [256, 384)
//   dQ^T = K^T dS^T  [128 hd x 64 q]     TMEM cols [384, 448)
//          -> the same 8 warps add it into the fp32 dQ accumulator with TMA
//             reduce-add (staged through shared memory, transposed)
//
// Computing dQ transposed keeps every MMA at M = 128 with 64-query blocks,
// which fits dV, dK (2 x 128 columns) and both score tiles in TMEM.
//   warp 0      TMA producer: K, V once; Q_i / dO_i into a 2-stage ring
//   warp 1      TMEM owner; one thread issues the MMAs
//   warps 2-9   softmax-gradient / dQ drain: warp w owns TMEM lane quarter
//               w % 4 and query columns [32 (w-2)/4, +32)
// dK is scaled by the softmax scale at the end; dQ in the conversion kernel.
// Every mbarrier wait is bounded.
//
// Reference parity: the reference's FlashAttention layers have no backward
// (scirs2-neural/src/layers/flash_attention_v2.rs:484-491 NotImplemented);
// the math is the standard FlashAttention-2 backward, checked against
// PyTorch autograd of the fp32 attention.
#include "host_common.h"

namespace scirs {
namespace fabw128 {

using bf16 = __nv_bfloat16;
constexpr int HD = 128, BK = 128, BQ = 64;
constexpr int kThreads = 320;
constexpr int KV_BYTES = BK * HD * 2;     // 32 KB: two 64-column atoms of 16 KB
constexpr int QT_BYTES = BQ * HD * 2;     // 16 KB: two 64-column atoms of 8 KB
constexpr int PT_BYTES = BK * BQ * 2;     // 16 KB: one atom [128 keys][64 q]
constexpr int OFF_K = 0;
constexpr int OFF_V = OFF_K + KV_BYTES;
constexpr int OFF_Q = OFF_V + KV_BYTES;         // 2 stages
constexpr int OFF_DO = OFF_Q + 2 * QT_BYTES;    // 2 stages
constexpr int OFF_PT = OFF_DO + 2 * QT_BYTES;
constexpr int OFF_DST = OFF_PT + PT_BYTES;
constexpr int OFF_DQS = OFF_DST + PT_BYTES;     // 8 warps x 4 KB staging (32 q x 32 hd fp32)
constexpr int OFF_LD = OFF_DQS + 8 * 4096;      // lse2 / delta [2 buffers][2][64] fp32
constexpr int OFF_BAR = OFF_LD + 2 * 2 * BQ * 4;
constexpr int SMEM = OFF_BAR + 256 + 1024;
constexpr uint32_t IDESC_S = umma_idesc_bf16(128, BQ, 0, 0);   // S^T, dP^T
constexpr uint32_t IDESC_KV = umma_idesc_bf16(128, HD, 0, 1);  // dV, dK: A K-major, B MN-major
constexpr uint32_t IDESC_Q = umma_idesc_bf16(128, BQ, 1, 1);   // dQ^T: A = K^T MN-major, B = dS^T MN-major
constexpr uint32_t T_S = 0, T_DP = 64, T_DV = 128, T_DK = 256, T_DQ = 384;

struct Params {
  const float* lse;    // [B, H, S] natural log
  const float* delta;  // [B, H, S]
  bf16* dk;
  bf16* dv;
  long dk_rs, dv_rs;
  int B, H, S;  // S: query length
  int Sk;       // key / value length
  float scale, scale_log2;
  DevStatus* st;
  AttnSparse sp;  // SPARSE: per key tile, the list of 64-query blocks to visit
};

template <bool CAUSAL, bool SPARSE = false>
__global__ void __launch_bounds__(kThreads, 1)
    fa_bwd_h128_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                       const __grid_constant__ CUtensorMap tmDQ, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;   // [2]
  uint64_t* qdo_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* p_full = bars + 6;     // 8 warps
  uint64_t* pt_free = bars + 7;
  uint64_t* dq_full = bars + 8;
  uint64_t* dq_free = bars + 9;    // 8 warps
  uint64_t* dkv_full = bars + 10;
  uint64_t* drain = bars + 11;
  uint64_t* ld_bar = bars + 12;    // [2]: lse / delta of a query block staged (8 warps)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* sLD = reinterpret_cast<float*>(smem + OFF_LD);  // [buf][0: lse2, 1: delta][64]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.S, Sk = p.Sk, H = p.H;
  const int kb = blockIdx.x;
  const int b = blockIdx.y / H, h = blockIdx.y % H;
  const int k0 = kb * BK;
  const int row_base = b * S;   // query rows (Q, dO, dQ)
  const int kv_base = b * Sk;   // key rows (K, V, dK, dV)
  const int nq = (S + BQ - 1) / BQ;
  const int i0 = CAUSAL ? k0 / BQ : 0;
  const int lb = SPARSE ? __ldg(p.sp.ptr + kb) : 0;
  const int niter = SPARSE ? __ldg(p.sp.ptr + kb + 1) - lb : max(nq - i0, 0);
  auto qblk = [&](int n) -> int { return SPARSE ? __ldg(p.sp.idx + lb + n) : i0 + n; };
  const int col = h * HD;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qdo_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
      mbar_init(&ld_bar[i], 8);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 8);
    mbar_init(pt_free, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 8);
    mbar_init(dkv_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    prefetch_tmap(&tmDO);
    prefetch_tmap(&tmDQ);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * KV_BYTES);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tma_load_2d(smem + OFF_K + c * (BK * 128), &tmK, kv_full, col + c * 64, kv_base + k0);
        tma_load_2d(smem + OFF_V + c * (BK * 128), &tmV, kv_full, col + c * 64, kv_base + k0);
      }
      for (int n = 0; n < niter; ++n) {
        const int i = qblk(n);
        const int st = n & 1;
        if (!mbar_wait(&qdo_empty[st], ((n >> 1) & 1) ^ 1, p.st, 80, abort_flag)) break;
        mbar_arrive_expect_tx(&qdo_full[st], 2 * QT_BYTES);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tma_load_2d(smem + OFF_Q + st * QT_BYTES + c * (BQ * 128), &tmQ, &qdo_full[st], col + c * 64,
                      row_base + i * BQ);
          tma_load_2d(smem + OFF_DO + st * QT_BYTES + c * (BQ * 128), &tmDO, &qdo_full[st], col + c * 64,
                      row_base + i * BQ);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA
    if (lane == 0) {
      bool ok = mbar_wait(kv_full, 0, p.st, 81, abort_flag);
      tc_fence_after();
      const uint32_t k_addr = smem_u32(smem + OFF_K), v_addr = smem_u32(smem + OFF_V);
      const uint32_t pt_addr = smem_u32(smem + OFF_PT), ds_addr = smem_u32(smem + OFF_DST);
      for (int n = 0; n < niter && ok; ++n) {
        const int st = n & 1;
        // the score tiles are free once the warps published P^T / dS^T of the
        // previous block (p_full, waited for below in iteration n - 1)
        if (!mbar_wait(&qdo_full[st], (n >> 1) & 1, p.st, 82, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t q_addr = smem_u32(smem + OFF_Q + st * QT_BYTES);
        const uint32_t do_addr = smem_u32(smem + OFF_DO + st * QT_BYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t ak = (kk >> 2) * (BK * 128) + (kk & 3) * 32;  // K / V atoms of 16 KB
          const uint32_t bq = (kk >> 2) * (BQ * 128) + (kk & 3) * 32;  // Q / dO atoms of 8 KB
          tc_mma_f16_ss(tmem + T_S, umma_desc_sw128(k_addr + ak, 16, 1024), umma_desc_sw128(q_addr + bq, 16, 1024),
                        IDESC_S, kk > 0 ? 1u : 0u);
          tc_mma_f16_ss(tmem + T_DP, umma_desc_sw128(v_addr + ak, 16, 1024),
                        umma_desc_sw128(do_addr + bq, 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
        }
        tc_commit(s_full);
        if (!mbar_wait(p_full, n & 1, p.st, 83, abort_flag)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {
          // A = P^T / dS^T [keys][q] K-major (one atom); B = dO / Q [q][hd] MN-major
          // (two 64-column atoms 8 KB apart; k-step = 16 query rows = 2 KB)
          const uint64_t bdo = umma_desc_sw128(do_addr + kk * 2048, BQ * 128, 1024);
          const uint64_t bq = umma_desc_sw128(q_addr + kk * 2048, BQ * 128, 1024);
          tc_mma_f16_ss(tmem + T_DV, umma_desc_sw128(pt_addr + kk * 32, 16, 1024), bdo, IDESC_KV,
                        (n > 0 || kk > 0) ? 1u : 0u);
          tc_mma_f16_ss(tmem + T_DK, umma_desc_sw128(ds_addr + kk * 32, 16, 1024), bq, IDESC_KV,
                        (n > 0 || kk > 0) ? 1u : 0u);
        }
        if (!mbar_wait(dq_free, (n & 1) ^ 1, p.st, 84, abort_flag)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          // A = K^T [hd][keys]: K read MN-major (hd atoms 16 KB apart, k-step 16 key rows);
          // B = dS^T [keys][q] MN-major (one 64-query atom)
          tc_mma_f16_ss(tmem + T_DQ, umma_desc_sw128(k_addr + kk * 2048, BK * 128, 1024),
                        umma_desc_sw128(ds_addr + kk * 2048, BK * 128, 1024), IDESC_Q, kk > 0 ? 1u : 0u);
        }
        tc_commit(pt_free);
        tc_commit(dq_full);
        tc_commit(&qdo_empty[st]);
      }
      tc_commit(dkv_full);
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr, 0, nullptr);
    }
  } else {
    // ------------------------------------------------------------ gradient warps
    const int w8 = warp - 2;
    const int q4 = warp & 3;      // TMEM lane quarter
    const int ch = w8 >> 2;       // query column half (32 columns)
    const int r = q4 * 32 + lane; // key row (S^T / dP^T / dV / dK) or hd index (dQ^T)
    const int key = k0 + r;
    const uint32_t lane_base = tmem + (uint32_t(q4 * 32) << 16);
    const float* lse_g = p.lse + ((long)b * H + h) * S;
    const float* del_g = p.delta + ((long)b * H + h) * S;
    uint8_t* pt_row = smem + OFF_PT + r * 128;
    uint8_t* ds_row = smem + OFF_DST + r * 128;
    float* stage = reinterpret_cast<float*>(smem + OFF_DQS + w8 * 4096);  // [32 q][32 hd]
    const float LOG2E = 1.4426950408889634f;
    bool ok = true;
    for (int n = 0; n < niter && ok; ++n) {
      const int q0 = qblk(n) * BQ;
      float* sL = sLD + (n & 1) * 2 * BQ;
      if (w8 < 4) {  // 128 threads stage the 64 lse and 64 delta values
        const int t = w8 * 32 + lane;
        const int q = q0 + (t & 63);
        if (t < 64) sL[t] = q < S ? lse_g[q] * LOG2E : 0.f;
        else sL[t] = q < S ? del_g[q] : 0.f;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ld_bar[n & 1]);
      if (!mbar_wait(&ld_bar[n & 1], (n >> 1) & 1, p.st, 85, abort_flag)) { ok = false; break; }
      if (!mbar_wait(s_full, n & 1, p.st, 86, abort_flag)) { ok = false; break; }
      if (!mbar_wait(pt_free, (n & 1) ^ 1, p.st, 87, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const int c0 = ch * 32;
      uint32_t sv[32], dv[32];
      tmem_ld_32x32b_x32(lane_base + T_S + c0, sv);
      tmem_ld_32x32b_x32(lane_base + T_DP + c0, dv);
      tc_wait_ld();
      const bool need_mask = (q0 + BQ > S) || (k0 + BK > Sk) || (CAUSAL && q0 < k0 + BK) ||
                             (SPARSE && !attn_block_full(p.sp, q0, q0 + BQ - 1, k0, k0 + BK - 1));
      const AttnSpan span = attn_queries_of_key<SPARSE>(p.sp, key, q0, S, Sk, CAUSAL);
      uint32_t pp[16], dd[16];
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        float pr[2], ds[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int ql = c0 + e + u;
          float pv = ex2_fast(fmaf(__uint_as_float(sv[e + u]), p.scale_log2, -sL[ql]));
          if (need_mask && !attn_span_has(span, ql)) pv = 0.f;
          pr[u] = pv;
          ds[u] = pv * (__uint_as_float(dv[e + u]) - sL[BQ + ql]);
        }
        pp[e >> 1] = pack_bf16x2(pr[0], pr[1]);
        dd[e >> 1] = pack_bf16x2(ds[0], ds[1]);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int so = ((ch * 4 + u) ^ (r & 7)) << 4;  // 128-byte swizzle within the row
        *reinterpret_cast<uint4*>(pt_row + so) = make_uint4(pp[4 * u], pp[4 * u + 1], pp[4 * u + 2], pp[4 * u + 3]);
        *reinterpret_cast<uint4*>(ds_row + so) = make_uint4(dd[4 * u], dd[4 * u + 1], dd[4 * u + 2], dd[4 * u + 3]);
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      // ---- dQ^T drain: lane r = hd index, columns = this warp's 32 queries
      if (!mbar_wait(dq_full, n & 1, p.st, 88, abort_flag)) { ok = false; break; }
      tc_fence_after();
      uint32_t a[32];
      tmem_ld_32x32b_x32(lane_base + T_DQ + c0, a);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_free);
      if (lane == 0) tma_store_wait_read0();  // the previous block's reduce-add has read the stage
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 32; ++j) stage[j * 32 + lane] = __uint_as_float(a[j]);  // [q][hd], conflict-free
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int row = row_base + q0 + c0;
        asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                         &tmDQ), "r"(smem_u32(stage)), "r"(col + q4 * 32), "r"(row) : "memory");
        tma_store_commit();
      }
    }
    if (lane == 0) tma_store_wait0();
    __syncwarp();
    // ---- dK, dV: lane = key row, this warp's half of the 128 columns
    if (ok && mbar_wait(dkv_full, 0, p.st, 89, abort_flag)) {
      tc_fence_after();
      uint32_t kv[32];
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        bf16* dst = which ? (p.dv + (long)(kv_base + key) * p.dv_rs + col)
                          : (p.dk + (long)(kv_base + key) * p.dk_rs + col);
        const float sc = which ? 1.f : p.scale;
        const bool empty = SPARSE && niter == 0;  // no query sees these keys: zero gradients
#pragma unroll 1
        for (int c = ch * 64; c < ch * 64 + 64; c += 32) {
          tmem_ld_32x32b_x32(lane_base + (which ? T_DV : T_DK) + c, kv);
          tc_wait_ld();
          if (empty) {
#pragma unroll
            for (int e = 0; e < 32; ++e) kv[e] = 0u;
          }
          if (key < Sk) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float* f = reinterpret_cast<const float*>(kv) + 8 * u;
              uint4 o;
              o.x = pack_bf16x2(f[0] * sc, f[1] * sc);
              o.y = pack_bf16x2(f[2] * sc, f[3] * sc);
              o.z = pack_bf16x2(f[4] * sc, f[5] * sc);
              o.w = pack_bf16x2(f[6] * sc, f[7] * sc);
              *reinterpret_cast<uint4*>(dst + c + 8 * u) = o;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}


// ---------------------------------------------------------------------------
// Pipelined variant (same CTA shape, roles and outputs as fa_bwd_h128_kernel).
// The tensor core no longer waits for the gradient warps between blocks:
//   * the warps copy S^T out of TMEM first and release it, so S^T of the next
//     block is computed while they work on this one;
//   * P^T (bf16) goes to TMEM columns [448, 480) and dV += P^T dO reads it
//     from there, issued as soon as P^T is written;
//   * dS^T (bf16) goes to TMEM over the dP^T columns each warp has read (dK
//     reads it from there) and to shared memory (B operand of dQ^T);
//   * dQ^T of block n - 1 is drained between P and dS of block n, so the dQ
//     MMA of block n never waits for it;
//   * dP^T of the next block is issued right after dQ^T of this one.
// dS is formed from the bf16 P that dV uses.
// MMA issue order per block n: S_{n+1} | dV_n | dK_n | dQ^T_n | dP_{n+1}.
// ---------------------------------------------------------------------------
template <bool CAUSAL, bool SPARSE = false>
__global__ void __launch_bounds__(kThreads, 1)
    fa_bwd_h128_pipe_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                            const __grid_constant__ CUtensorMap tmDQ, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;   // [2]
  uint64_t* qdo_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;     // MMA commit
  uint64_t* s_free = bars + 6;     // 8 warps copied S^T out
  uint64_t* dp_full = bars + 7;    // MMA commit
  uint64_t* pt_full = bars + 8;    // 8 warps wrote P^T
  uint64_t* pt_free = bars + 9;    // MMA commit after dV
  uint64_t* ds_full = bars + 10;   // 8 warps wrote dS^T
  uint64_t* dq_full = bars + 11;
  uint64_t* dq_free = bars + 12;   // 8 warps
  uint64_t* dkv_full = bars + 13;
  uint64_t* drain = bars + 14;
  uint64_t* ld_bar = bars + 15;    // [2]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* sLD = reinterpret_cast<float*>(smem + OFF_LD);  // [buf][0: lse2, 1: delta][64]
  constexpr uint32_t T_PT = 448;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.S, Sk = p.Sk, H = p.H;
  const int kb = blockIdx.x;
  const int b = blockIdx.y / H, h = blockIdx.y % H;
  const int k0 = kb * BK;
  const int row_base = b * S;
  const int kv_base = b * Sk;
  const int nq = (S + BQ - 1) / BQ;
  const int i0 = CAUSAL ? k0 / BQ : 0;
  const int lb = SPARSE ? __ldg(p.sp.ptr + kb) : 0;
  const int niter = SPARSE ? __ldg(p.sp.ptr + kb + 1) - lb : max(nq - i0, 0);
  auto qblk = [&](int n) -> int { return SPARSE ? __ldg(p.sp.idx + lb + n) : i0 + n; };
  const int col = h * HD;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qdo_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
      mbar_init(&ld_bar[i], 8);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 8);
    mbar_init(dp_full, 1);
    mbar_init(pt_full, 8);
    mbar_init(pt_free, 1);
    mbar_init(ds_full, 8);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 8);
    mbar_init(dkv_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
    prefetch_tmap(&tmDO);
    prefetch_tmap(&tmDQ);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * KV_BYTES);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tma_load_2d(smem + OFF_K + c * (BK * 128), &tmK, kv_full, col + c * 64, kv_base + k0);
        tma_load_2d(smem + OFF_V + c * (BK * 128), &tmV, kv_full, col + c * 64, kv_base + k0);
      }
      for (int n = 0; n < niter; ++n) {
        const int i = qblk(n);
        const int st = n & 1;
        if (!mbar_wait(&qdo_empty[st], ((n >> 1) & 1) ^ 1, p.st, 80, abort_flag)) break;
        mbar_arrive_expect_tx(&qdo_full[st], 2 * QT_BYTES);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tma_load_2d(smem + OFF_Q + st * QT_BYTES + c * (BQ * 128), &tmQ, &qdo_full[st], col + c * 64,
                      row_base + i * BQ);
          tma_load_2d(smem + OFF_DO + st * QT_BYTES + c * (BQ * 128), &tmDO, &qdo_full[st], col + c * 64,
                      row_base + i * BQ);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA
    if (lane == 0) {
      const uint32_t k_addr = smem_u32(smem + OFF_K), v_addr = smem_u32(smem + OFF_V);
      const uint32_t ds_addr = smem_u32(smem + OFF_DST);
      auto q_at = [&](int n) { return smem_u32(smem + OFF_Q + (n & 1) * QT_BYTES); };
      auto do_at = [&](int n) { return smem_u32(smem + OFF_DO + (n & 1) * QT_BYTES); };
      auto issue_s = [&](int n) {  // S^T = K Q_n^T
        const uint32_t q_addr = q_at(n);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t ak = (kk >> 2) * (BK * 128) + (kk & 3) * 32;
          const uint32_t bq = (kk >> 2) * (BQ * 128) + (kk & 3) * 32;
          tc_mma_f16_ss(tmem + T_S, umma_desc_sw128(k_addr + ak, 16, 1024), umma_desc_sw128(q_addr + bq, 16, 1024),
                        IDESC_S, kk > 0 ? 1u : 0u);
        }
        tc_commit(s_full);
      };
      auto issue_dp = [&](int n) {  // dP^T = V dO_n^T
        const uint32_t do_addr = do_at(n);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t ak = (kk >> 2) * (BK * 128) + (kk & 3) * 32;
          const uint32_t bq = (kk >> 2) * (BQ * 128) + (kk & 3) * 32;
          tc_mma_f16_ss(tmem + T_DP, umma_desc_sw128(v_addr + ak, 16, 1024),
                        umma_desc_sw128(do_addr + bq, 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
        }
        tc_commit(dp_full);
      };
      bool ok = mbar_wait(kv_full, 0, p.st, 81, abort_flag);
      if (ok && niter > 0) {
        ok = mbar_wait(&qdo_full[0], 0, p.st, 82, abort_flag);
        if (ok) {
          tc_fence_after();
          issue_s(0);
          issue_dp(0);
        }
      }
      for (int n = 0; n < niter && ok; ++n) {
        const int st = n & 1;
        if (n + 1 < niter) {
          ok = mbar_wait(&qdo_full[(n + 1) & 1], ((n + 1) >> 1) & 1, p.st, 82, abort_flag) &&
               mbar_wait(s_free, n & 1, p.st, 90, abort_flag);
          if (!ok) break;
          tc_fence_after();
          issue_s(n + 1);
        }
        const uint32_t q_addr = q_at(n), do_addr = do_at(n);
        if (!mbar_wait(pt_full, n & 1, p.st, 83, abort_flag)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)  // dV += P^T dO, A = P^T in TMEM (8 packed columns per k-step)
          tc_mma_f16_ts(tmem + T_DV, tmem + T_PT + kk * 8, umma_desc_sw128(do_addr + kk * 2048, BQ * 128, 1024),
                        IDESC_KV, (n > 0 || kk > 0) ? 1u : 0u);
        tc_commit(pt_free);
        if (!mbar_wait(ds_full, n & 1, p.st, 91, abort_flag)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)  // dK += dS^T Q, A = dS^T in TMEM over the dP^T columns
          tc_mma_f16_ts(tmem + T_DK, tmem + T_DP + (kk >> 1) * 32 + (kk & 1) * 8,
                        umma_desc_sw128(q_addr + kk * 2048, BQ * 128, 1024), IDESC_KV, (n > 0 || kk > 0) ? 1u : 0u);
        if (!mbar_wait(dq_free, (n & 1) ^ 1, p.st, 84, abort_flag)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          tc_mma_f16_ss(tmem + T_DQ, umma_desc_sw128(k_addr + kk * 2048, BK * 128, 1024),
                        umma_desc_sw128(ds_addr + kk * 2048, BK * 128, 1024), IDESC_Q, kk > 0 ? 1u : 0u);
        tc_commit(dq_full);
        tc_commit(&qdo_empty[st]);
        if (n + 1 < niter) issue_dp(n + 1);
      }
      tc_commit(dkv_full);
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr, 0, nullptr);
    }
  } else {
    // ------------------------------------------------------------ gradient warps
    const int w8 = warp - 2;
    const int q4 = warp & 3;
    const int ch = w8 >> 2;        // query half (32 of the block's 64)
    const int r = q4 * 32 + lane;  // key row, or hd index for dQ^T
    const int key = k0 + r;
    const uint32_t lane_base = tmem + (uint32_t(q4 * 32) << 16);
    const float* lse_g = p.lse + ((long)b * H + h) * S;
    const float* del_g = p.delta + ((long)b * H + h) * S;
    uint8_t* ds_row = smem + OFF_DST + r * 128;
    float* stage = reinterpret_cast<float*>(smem + OFF_DQS + w8 * 4096);  // [32 q][32 hd]
    const float LOG2E = 1.4426950408889634f;
    const int c0 = ch * 32;
    const int t = w8 * 32 + lane;  // t < 128 stage the block's 64 lse and 64 delta values
    float nv = 0.f;
    if (t < 128 && niter > 0) {
      const int q = qblk(0) * BQ + (t & 63);
      nv = q < S ? (t < 64 ? lse_g[q] * LOG2E : del_g[q]) : 0.f;
    }
    // dQ^T of block m: lane = hd index, columns = this warp's 32 queries
    auto drain_dq = [&](int m) -> bool {
      if (!mbar_wait(dq_full, m & 1, p.st, 88, abort_flag)) return false;
      tc_fence_after();
      uint32_t a[32];
      tmem_ld_32x32b_x32(lane_base + T_DQ + c0, a);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_free);
      if (lane == 0) tma_store_wait_read0();
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 32; ++j) stage[j * 32 + lane] = __uint_as_float(a[j]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int row = row_base + qblk(m) * BQ + c0;
        asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                         &tmDQ), "r"(smem_u32(stage)), "r"(col + q4 * 32), "r"(row) : "memory");
        tma_store_commit();
      }
      return true;
    };
    bool ok = true;
    for (int n = 0; n < niter && ok; ++n) {
      const int q0 = qblk(n) * BQ;
      float* sL = sLD + (n & 1) * 2 * BQ;
      if (t < 128) {
        sL[t] = nv;
        if (n + 1 < niter) {
          const int q = qblk(n + 1) * BQ + (t & 63);
          nv = q < S ? (t < 64 ? lse_g[q] * LOG2E : del_g[q]) : 0.f;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ld_bar[n & 1]);
      if (!mbar_wait(&ld_bar[n & 1], (n >> 1) & 1, p.st, 85, abort_flag)) { ok = false; break; }
      if (!mbar_wait(s_full, n & 1, p.st, 86, abort_flag)) { ok = false; break; }
      tc_fence_after();
      uint32_t sv[32];
      tmem_ld_32x32b_x32(lane_base + T_S + c0, sv);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);
      const bool need_mask = (q0 + BQ > S) || (k0 + BK > Sk) || (CAUSAL && q0 < k0 + BK) ||
                             (SPARSE && !attn_block_full(p.sp, q0, q0 + BQ - 1, k0, k0 + BK - 1));
      const AttnSpan span = attn_queries_of_key<SPARSE>(p.sp, key, q0, S, Sk, CAUSAL);
      uint32_t pp[16];
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        float pr[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int ql = c0 + e + u;
          float pv = ex2_fast(fmaf(__uint_as_float(sv[e + u]), p.scale_log2, -sL[ql]));
          if (need_mask && !attn_span_has(span, ql)) pv = 0.f;
          pr[u] = pv;
        }
        pp[e >> 1] = pack_bf16x2(pr[0], pr[1]);
      }
      if (!mbar_wait(pt_free, (n & 1) ^ 1, p.st, 87, abort_flag)) { ok = false; break; }
      tc_fence_after();
      tmem_st_32x32b_x16(lane_base + T_PT + (c0 >> 1), pp);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pt_full);
      if (n > 0 && !drain_dq(n - 1)) { ok = false; break; }
      if (!mbar_wait(dp_full, n & 1, p.st, 92, abort_flag)) { ok = false; break; }
      tc_fence_after();
      uint32_t dv[32];
      tmem_ld_32x32b_x32(lane_base + T_DP + c0, dv);
      tc_wait_ld();
      uint32_t dd[16];
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        const uint32_t pq = pp[e >> 1];
        const float d0 = bf16_lo(pq) * (__uint_as_float(dv[e]) - sL[BQ + c0 + e]);
        const float d1 = bf16_hi(pq) * (__uint_as_float(dv[e + 1]) - sL[BQ + c0 + e + 1]);
        dd[e >> 1] = pack_bf16x2(d0, d1);
      }
      tmem_st_32x32b_x16(lane_base + T_DP + c0, dd);  // over dP^T columns this warp has read
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int so = ((ch * 4 + u) ^ (r & 7)) << 4;
        *reinterpret_cast<uint4*>(ds_row + so) = make_uint4(dd[4 * u], dd[4 * u + 1], dd[4 * u + 2], dd[4 * u + 3]);
      }
      tc_wait_st();
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_full);
    }
    if (ok && niter > 0) ok = drain_dq(niter - 1);
    if (lane == 0) tma_store_wait0();
    __syncwarp();
    if (ok && mbar_wait(dkv_full, 0, p.st, 89, abort_flag)) {
      tc_fence_after();
      uint32_t kv[32];
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        bf16* dst = which ? (p.dv + (long)(kv_base + key) * p.dv_rs + col)
                          : (p.dk + (long)(kv_base + key) * p.dk_rs + col);
        const float sc = which ? 1.f : p.scale;
        const bool empty = SPARSE && niter == 0;
#pragma unroll 1
        for (int c = ch * 64; c < ch * 64 + 64; c += 32) {
          tmem_ld_32x32b_x32(lane_base + (which ? T_DV : T_DK) + c, kv);
          tc_wait_ld();
          if (empty) {
#pragma unroll
            for (int e = 0; e < 32; ++e) kv[e] = 0u;
          }
          if (key < Sk) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float* f = reinterpret_cast<const float*>(kv) + 8 * u;
              uint4 o;
              o.x = pack_bf16x2(f[0] * sc, f[1] * sc);
              o.y = pack_bf16x2(f[2] * sc, f[3] * sc);
              o.z = pack_bf16x2(f[4] * sc, f[5] * sc);
              o.w = pack_bf16x2(f[6] * sc, f[7] * sc);
              *reinterpret_cast<uint4*>(dst + c + 8 * u) = o;
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace fabw128

void flash_attn_bwd_h128(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor lse,
                         torch::Tensor delta, torch::Tensor dk, torch::Tensor dv, torch::Tensor dq_acc, bool causal,
                         double scale, const AttnSparse& sp, bool pipelined) {
  const int64_t B = q.size(0), S = q.size(1), H = q.size(2), HD = q.size(3);
  const int64_t Sk = k.size(1);
  TORCH_CHECK(HD == 128, "this backward kernel is for head_dim 128");
  for (auto* t : {&q, &k, &v, &dout, &dk, &dv}) {
    const int64_t St = (t == &k || t == &v || t == &dk || t == &dv) ? Sk : S;
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->dim() == 4 && t->size(0) == B && t->size(1) == St &&
                    t->size(2) == H && t->size(3) == HD,
                "q/dout must be bf16 [B, S, H, HD] and k/v/dk/dv bf16 [B, Sk, H, HD]");
    TORCH_CHECK(t->stride(3) == 1 && t->stride(2) == HD && t->stride(0) == St * t->stride(1),
                "tensors must be token-major with contiguous heads");
  }
  TORCH_CHECK(dq_acc.scalar_type() == at::kFloat && dq_acc.numel() >= B * S * H * HD, "dq_acc fp32 [B*S*H*HD]");
  c10::cuda::CUDAGuard guard(q.get_device());
  auto mk = [&](const torch::Tensor& t, int64_t len, uint32_t rows) {
    return make_tmap_2d(t.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)(H * HD), (uint64_t)(B * len),
                        (uint64_t)t.stride(1) * 2, 64, rows, CU_TENSOR_MAP_SWIZZLE_128B);
  };
  CUtensorMap tq = mk(q, S, 64), tk = mk(k, Sk, 128), tv = mk(v, Sk, 128), tdo = mk(dout, S, 64);
  // dQ staging tiles are plain row-major [32 q][32 hd] fp32
  CUtensorMap tdq = make_tmap_2d(dq_acc.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (uint64_t)(H * HD),
                                 (uint64_t)(B * S), (uint64_t)(H * HD) * 4, 32, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
  fabw128::Params p{};
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.dk = reinterpret_cast<fabw128::bf16*>(dk.data_ptr());
  p.dv = reinterpret_cast<fabw128::bf16*>(dv.data_ptr());
  p.dk_rs = dk.stride(1);
  p.dv_rs = dv.stride(1);
  p.B = (int)B;
  p.H = (int)H;
  p.S = (int)S;
  p.Sk = (int)Sk;
  p.scale = (float)scale;
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  p.st = status_ptr(q.get_device());
  p.sp = sp;
  const bool sparse = sp.ptr != nullptr;
  dim3 grid((unsigned)((Sk + 127) / 128), (unsigned)(B * H));
  auto st = cur_stream();
#define FABW128(C_, SP_)                                                   \
  {                                                                        \
    auto kern = pipelined ? fabw128::fa_bwd_h128_pipe_kernel<C_, SP_> : fabw128::fa_bwd_h128_kernel<C_, SP_>; \
    set_max_smem((const void*)kern, fabw128::SMEM);                        \
    kern<<<grid, fabw128::kThreads, fabw128::SMEM, st>>>(tq, tk, tv, tdo, tdq, p); \
  }
  if (sparse) {
    if (causal) FABW128(true, true) else FABW128(false, true)
  } else {
    if (causal) FABW128(true, false) else FABW128(false, false)
  }
#undef FABW128
  SCIRS_CHECK_LAUNCH();
}

}  // namespace scirs
