// FlashAttention forward on the 5th-generation tensor cores (tcgen05/TMEM).
//
// One CTA = one 128-query tile of one (batch, head). Q, K, V are read with
// TMA straight out of token-major buffers (e.g. the fused QKV projection
// [B*S, 3*H*HD]); no transposes.
//
//   warp 0     TMA producer: Q once, then K_j / V_j into a 2-stage ring
//   warp 1     owns TMEM; one thread issues  S_j = Q K_j^T  (M=128,N=128,K=HD)
//              into S[j%2] and  O_j = P_j V_j  (M=128,N=HD,K=128) into O[j%2]
//   warps 2-5  softmax: thread t owns query row t (TMEM lane t), so row max /
//              row sum need no cross-thread reduction. Reads S_j from TMEM,
//              writes P_j = exp2(S_j*scale*log2e - m_j) as bf16 into a
//              128B-swizzled smem tile (the K-major A operand of the PV MMA),
//              and folds O_{j-1} into a register accumulator (one block
//              behind, rescaled by exp2(m_{j-2} - m_{j-1})).
//
// TMEM columns: NSB S buffers of 128, then NSB O buffers of HD (NSB = 1 for
// head_dim 64 -> 256 columns, two CTAs per SM; NSB = 2 for head_dim 128).
// Causal masking applies only to the diagonal block (BM == BN == 128); keys
// >= S are masked, rows >= S are not stored. Every mbarrier wait is bounded.
//
// Reference parity: same math as the reference's CPU FlashAttention-2
// forward (scirs2-neural/src/layers/flash_attention_v2.rs:220,369-482,
// scirs2-neural/src/attention/flash_v2.rs:96-300); LSE is natural-log.
#include "host_common.h"

namespace scirs {
namespace fatc {

using bf16 = __nv_bfloat16;
constexpr int BM = 128, BN = 128;
constexpr int kThreads = 192;

struct Params {
  bf16* out;
  float* lse;
  long o_rs;
  int B, H, S;
  float scale_log2;
  DevStatus* st;
};

template <int HD>
struct Cfg {
  static constexpr int Q_BYTES = BM * HD * 2;
  static constexpr int KV_BYTES = BN * HD * 2;
  static constexpr int P_BYTES = BM * BN * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;          // 2 stages
  static constexpr int OFF_V = OFF_K + 2 * KV_BYTES;     // 2 stages
  static constexpr int OFF_P = OFF_V + 2 * KV_BYTES;
  static constexpr int OFF_BAR = OFF_P + P_BYTES;
  // 512 bytes of alignment slack (the kernel checks the base alignment at
  // run time); with 1024 two 112 KB CTAs would not fit one SM.
  static constexpr int SLACK = 512;
  static constexpr int SMEM = OFF_BAR + 256 + SLACK;
  // TMEM: NSB buffers of S (128 fp32 columns) then NSB buffers of O (HD
  // columns). head_dim 64 uses one buffer each (256 columns), so two CTAs
  // share an SM and their softmax / MMA phases interleave.
  static constexpr int NSB = (HD == 64) ? 1 : 2;
  static constexpr int TMEM_COLS = (NSB * (128 + HD) <= 256) ? 256 : 512;
  static constexpr int MIN_BLOCKS = (HD == 64) ? 2 : 1;
  static constexpr uint32_t IDESC_S = umma_idesc_bf16(BM, BN, 0, 0);
  static constexpr uint32_t IDESC_O = umma_idesc_bf16(BM, HD, 0, 1);
};

template <int HD, bool CAUSAL>
__global__ void __launch_bounds__(kThreads, Cfg<HD>::MIN_BLOCKS)
    fa_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const Params p) {
  using C = Cfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  if (smem - smem_raw > C::SLACK) {  // dynamic smem less aligned than assumed: refuse, do not overrun
    if (threadIdx.x == 0) report_status(p.st, kStBadArg, 40, (unsigned)(smem - smem_raw));
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* v_full = bars + 3;   // [2]
  uint64_t* kv_empty = bars + 5; // [2]
  uint64_t* s_full = bars + 7;   // [2]
  uint64_t* s_free = bars + 9;   // [2]
  uint64_t* o_full = bars + 11;  // [2]
  uint64_t* o_free = bars + 13;  // [2]
  uint64_t* p_full = bars + 15;
  uint64_t* p_free = bars + 16;
  uint64_t* drain = bars + 17;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.S, H = p.H;
  const int qb = gridDim.x - 1 - blockIdx.x;  // longest causal tiles first
  const int b = blockIdx.y / H, h = blockIdx.y % H;
  const int q0 = qb * BM;
  const int row_base = b * S;  // token row of position 0 of this sequence
  const int nkv_all = (S + BN - 1) / BN;
  const int nkv = CAUSAL ? min(nkv_all, qb + 1) : nkv_all;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(p_free, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      const int col = h * HD;
      mbar_arrive_expect_tx(q_full, C::Q_BYTES);
#pragma unroll
      for (int c = 0; c < HD / 64; ++c)
        tma_load_2d(smem + C::OFF_Q + c * (BM * 128), &tmQ, q_full, col + c * 64, row_base + q0);
      for (int j = 0; j < nkv; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&kv_empty[s], ((j >> 1) & 1) ^ 1, p.st, 20, abort_flag)) break;
        mbar_arrive_expect_tx(&k_full[s], C::KV_BYTES);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_2d(smem + C::OFF_K + s * C::KV_BYTES + c * (BN * 128), &tmK, &k_full[s], col + c * 64,
                      row_base + j * BN);
        mbar_arrive_expect_tx(&v_full[s], C::KV_BYTES);
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_2d(smem + C::OFF_V + s * C::KV_BYTES + c * (BN * 128), &tmV, &v_full[s], col + c * 64,
                      row_base + j * BN);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, p.st, 21, abort_flag);
      tc_fence_after();
      const uint32_t q_addr = smem_u32(smem + C::OFF_Q);
      const uint32_t p_addr = smem_u32(smem + C::OFF_P);
      auto issue_pv = [&](int i) -> bool {
        const int s = i & 1;                  // K/V smem stage
        const int ob = i % C::NSB;            // O TMEM buffer
        if (!mbar_wait(p_full, i & 1, p.st, 22, abort_flag)) return false;
        if (!mbar_wait(&v_full[s], (i >> 1) & 1, p.st, 23, abort_flag)) return false;
        if (!mbar_wait(&o_free[ob], ((i / C::NSB) & 1) ^ 1, p.st, 24, abort_flag)) return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(smem + C::OFF_V + s * C::KV_BYTES);
        const uint32_t d_tmem = tmem + C::NSB * BN + ob * HD;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          // A = P [128 q][128 keys] K-major in two 64-key column blocks
          const uint64_t adesc = umma_desc_sw128(p_addr + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 16, 1024);
          // B = V [keys][HD] MN-major: k-step = 16 key rows = 2048 bytes
          const uint64_t bdesc = umma_desc_sw128(v_addr + kk * 2048, BN * 128, 1024);
          tc_mma_f16_ss(d_tmem, adesc, bdesc, C::IDESC_O, kk > 0 ? 1u : 0u);
        }
        tc_commit(p_free);
        tc_commit(&o_full[ob]);
        tc_commit(&kv_empty[s]);
        return true;
      };
      for (int j = 0; j < nkv && ok; ++j) {
        const int s = j & 1;        // K/V smem stage
        const int sb = j % C::NSB;  // S TMEM buffer
        ok = mbar_wait(&k_full[s], (j >> 1) & 1, p.st, 25, abort_flag) &&
             mbar_wait(&s_free[sb], ((j / C::NSB) & 1) ^ 1, p.st, 26, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + C::OFF_K + s * C::KV_BYTES);
        const uint32_t d_tmem = tmem + sb * BN;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint32_t offk = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          tc_mma_f16_ss(d_tmem, umma_desc_sw128(q_addr + off, 16, 1024), umma_desc_sw128(k_addr + offk, 16, 1024),
                        C::IDESC_S, kk > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[sb]);
        if (j >= 1) ok = issue_pv(j - 1);
      }
      if (ok && nkv >= 1) issue_pv(nkv - 1);
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr, 0, nullptr);
    }
  } else {
    // ---------------------------------------------------------------- softmax
    const int q = warp & 3;          // TMEM lane quarter
    const int r = q * 32 + lane;     // query row within the tile
    const int qrow = q0 + r;         // position within the sequence
    const uint32_t lane_base = tmem + (uint32_t(q * 32) << 16);
    uint8_t* prow = smem + C::OFF_P + r * 128;
    float oacc[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) oacc[i] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_pend = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv && ok; ++j) {
      const int s = j % C::NSB;  // S TMEM buffer
      if (!mbar_wait(&s_full[s], (j / C::NSB) & 1, p.st, 30, abort_flag)) { ok = false; break; }
      tc_fence_after();
      const int kv0 = j * BN;
      const bool mask = (kv0 + BN > S) || (CAUSAL && j == qb);
      // pass 1: row max
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(lane_base + s * BN + c, v);
        tc_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          float x = __uint_as_float(v[e]);
          const int key = kv0 + c + e;
          if (mask && (key >= S || (CAUSAL && key > qrow))) x = -INFINITY;
          mx = fmaxf(mx, x);
        }
      }
      const float m_new = fmaxf(m, mx * p.scale_log2);
      const float ref = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = ex2_fast(m - ref);
      // P may be overwritten once the previous PV MMA has consumed it
      if (j >= 1 && !mbar_wait(p_free, (j - 1) & 1, p.st, 31, abort_flag)) { ok = false; break; }
      // pass 2: P = exp2(S*scale_log2 - m_new) -> bf16 swizzled smem tile
      float rs = 0.f;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(lane_base + s * BN + c, v);
        tc_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float x0 = __uint_as_float(v[e]), x1 = __uint_as_float(v[e + 1]);
          const int key = kv0 + c + e;
          if (mask && (key >= S || (CAUSAL && key > qrow))) x0 = -INFINITY;
          if (mask && (key + 1 >= S || (CAUSAL && key + 1 > qrow))) x1 = -INFINITY;
          const float p0 = ex2_fast(fmaf(x0, p.scale_log2, -ref));
          const float p1 = ex2_fast(fmaf(x1, p.scale_log2, -ref));
          rs += p0 + p1;
          pk[e >> 1] = pack_bf16x2(p0, p1);
        }
        // 32 keys = four 16-byte units of the row; key block c/64, unit (c%64)/8 + u
        uint8_t* blk = prow + (c >> 6) * (BM * 128);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int unit = ((c & 63) >> 3) + u;
          *reinterpret_cast<uint4*>(blk + ((unit ^ (r & 7)) << 4)) =
              make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s_free[s]);
        mbar_arrive(p_full);
      }
      l = l * alpha + rs;
      m = m_new;
      // fold O_{j-1} (relative to m_{j-1}) into the accumulator
      if (j >= 1) {
        const int so = (j - 1) % C::NSB;
        if (!mbar_wait(&o_full[so], ((j - 1) / C::NSB) & 1, p.st, 32, abort_flag)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < HD; c += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(lane_base + C::NSB * BN + so * HD + c, v);
          tc_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) oacc[c + e] = fmaf(oacc[c + e], alpha_pend, __uint_as_float(v[e]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_free[so]);
      }
      alpha_pend = alpha;
    }
    if (ok && nkv >= 1) {
      const int so = (nkv - 1) % C::NSB;
      if (mbar_wait(&o_full[so], ((nkv - 1) / C::NSB) & 1, p.st, 33, abort_flag)) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < HD; c += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(lane_base + C::NSB * BN + so * HD + c, v);
          tc_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) oacc[c + e] = fmaf(oacc[c + e], alpha_pend, __uint_as_float(v[e]));
        }
        if (qrow < S) {
          const float inv = l > 0.f ? 1.f / l : 0.f;
          bf16* orow = p.out + (long)(row_base + qrow) * p.o_rs + h * HD;
#pragma unroll
          for (int c = 0; c < HD; c += 8) {
            uint4 o;
            o.x = pack_bf16x2(oacc[c] * inv, oacc[c + 1] * inv);
            o.y = pack_bf16x2(oacc[c + 2] * inv, oacc[c + 3] * inv);
            o.z = pack_bf16x2(oacc[c + 4] * inv, oacc[c + 5] * inv);
            o.w = pack_bf16x2(oacc[c + 6] * inv, oacc[c + 7] * inv);
            *reinterpret_cast<uint4*>(orow + c) = o;
          }
          p.lse[((long)b * H + h) * S + qrow] = (m + log2f(l)) * 0.6931471805599453f;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace fatc

// q/k/v/out: [B, S, H, HD] token-major views with contiguous heads; lse [B,H,S].
void flash_attn_fwd_tc(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                       bool causal, double scale) {
  const int64_t B = q.size(0), S = q.size(1), H = q.size(2), HD = q.size(3);
  TORCH_CHECK(HD == 64 || HD == 128, "head_dim must be 64 or 128");
  for (auto* t : {&q, &k, &v, &out}) {
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->dim() == 4 && t->size(0) == B && t->size(1) == S &&
                    t->size(2) == H && t->size(3) == HD,
                "q/k/v/out must be bf16 [B, S, H, HD]");
    TORCH_CHECK(t->stride(3) == 1 && t->stride(2) == HD && t->stride(0) == S * t->stride(1),
                "q/k/v/out must be token-major with contiguous heads");
  }
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.numel() == B * H * S && lse.is_contiguous(), "lse fp32 [B,H,S]");
  c10::cuda::CUDAGuard guard(q.get_device());
  auto mk = [&](const torch::Tensor& t) {
    return make_tmap_2d(t.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)(H * HD), (uint64_t)(B * S),
                        (uint64_t)t.stride(1) * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  };
  CUtensorMap tq = mk(q), tk = mk(k), tv = mk(v);
  fatc::Params p{};
  p.out = reinterpret_cast<fatc::bf16*>(out.data_ptr());
  p.lse = lse.data_ptr<float>();
  p.o_rs = out.stride(1);
  p.B = (int)B;
  p.H = (int)H;
  p.S = (int)S;
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  p.st = status_ptr(q.get_device());
  dim3 grid((unsigned)((S + 127) / 128), (unsigned)(B * H));
  auto st = cur_stream();
#define FATC(HD_, C_)                                                                                      \
  {                                                                                                        \
    auto kern = fatc::fa_fwd_tc_kernel<HD_, C_>;                                                           \
    set_max_smem((const void*)kern, fatc::Cfg<HD_>::SMEM);                                          \
    kern<<<grid, fatc::kThreads, fatc::Cfg<HD_>::SMEM, st>>>(tq, tk, tv, p);                               \
  }
  if (HD == 64) {
    if (causal) FATC(64, true) else FATC(64, false)
  } else {
    if (causal) FATC(128, true) else FATC(128, false)
  }
#undef FATC
  SCIRS_CHECK_LAUNCH();
}



// ===========================================================================
// FlashAttention backward on tcgen05 (head_dim 64).
//
// One CTA = one 128-key tile of one (batch, head); it walks the 128-query
// blocks that can see those keys (all of them, or q >= k for causal).
//
//   warp 0     TMA: K, V once; Q_i, dO_i into a 2-stage ring
//   warp 1     MMA thread, per query block i:
//                S^T  = K Q_i^T        (TMEM [0,128))
//                dP^T = V dO_i^T       (TMEM [128,256))
//                -- dS warps turn them into P^T, dS^T (bf16 smem) --
//                dV  += P^T dO_i       (TMEM [256,320), accumulated over i)
//                dK  += dS^T Q_i       (TMEM [320,384), accumulated over i)
//                dQ_i = dS K           (TMEM [384,448); A = dS^T read MN-major)
//   warps 2-9  dS: thread = key row, warps 2-5 take queries [0, 64) of the
//              block and warps 6-9 queries [64, 128) (two warps per scheduler
//              share the exponentials). P = exp2(S*scale*log2e - LSE*log2e)
//              (masked to 0), dS = P (dP - delta); both stored as
//              128B-swizzled K-major bf16 tiles [key][q].
//   warps 6-9  also move dQ_i: TMEM -> 128B-swizzled fp32 smem slots -> TMA
//              reduce-add into the fp32 dQ accumulator [B*S, H*HD] (while the
//              tensor core starts the next block); at the end they write
//              dK * scale and dV (bf16).
// dQ is scaled by the softmax scale in the follow-up conversion kernel.
// ===========================================================================
namespace fabw {

using bf16 = __nv_bfloat16;
constexpr int HD = 64, BK = 128, BQ = 128;
// 16 warps = 4 warpgroups: 0 = TMA warp, MMA warp, two idle warps; 1 and 2 =
// the eight dS warps; 3 = the dQ-drain / dK-dV epilogue warps. Launched with
// 128 registers per thread (65536 / 512); the control and drain warpgroups
// give registers to the dS warpgroups: 128 x 64 + 256 x 176 + 128 x 96 = 512 x 128.
constexpr int kThreads = 512;
constexpr int kRegsLaunch = 128, kRegsCtl = 64, kRegsDs = 176, kRegsDrain = 96;
static_assert(128 * kRegsCtl + 256 * kRegsDs + 128 * kRegsDrain <= kThreads * kRegsLaunch,
              "register split exceeds the launch");
constexpr int T_BYTES = 128 * HD * 2;    // one 128-row x 64-col bf16 tile (16 KB)
constexpr int P_BYTES = BK * BQ * 2;     // 128 x 128 bf16 (32 KB)
constexpr int OFF_K = 0;
constexpr int OFF_V = OFF_K + T_BYTES;
constexpr int OFF_Q = OFF_V + T_BYTES;      // 2 stages
constexpr int OFF_DO = OFF_Q + 2 * T_BYTES; // 2 stages
constexpr int OFF_PT = OFF_DO + 2 * T_BYTES;
constexpr int OFF_DST = OFF_PT + P_BYTES;
constexpr int OFF_DQS = OFF_DST + P_BYTES;  // 4 warps x 2 slots x 4 KB
constexpr int OFF_LD = OFF_DQS + 4 * 2 * 4096;  // lse / delta [2][2][128] fp32
constexpr int OFF_BAR = OFF_LD + 4 * 128 * 4;
constexpr int SMEM = OFF_BAR + 256 + 1024;
constexpr uint32_t IDESC_S = umma_idesc_bf16(128, 128, 0, 0);
constexpr uint32_t IDESC_KV = umma_idesc_bf16(128, HD, 0, 1);   // dV, dK: A K-major, B MN-major
constexpr uint32_t IDESC_Q = umma_idesc_bf16(128, HD, 1, 1);    // dQ: A (dS^T) MN-major, B MN-major

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
  AttnSparse sp;  // SPARSE: per key tile, the list of 128-query blocks to visit
  // optional phase timing of the pipelined kernel (clock64 cycles summed over a CTA's blocks):
  // [CTA][16] = dS warp 4 lane 0: ld_bar, s_full, S copy, exponentials, pt_free, P store,
  // dp_full, dS; MMA thread: next-S waits, S issue, pt_full, ds_full, dq_free, other issue;
  // [14] = blocks; nullptr = off
  unsigned long long* trace;
};

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

template <bool CAUSAL, bool SPARSE = false>
__global__ void __launch_bounds__(kThreads, 1)
    fa_bwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                     const __grid_constant__ CUtensorMap tmDQ, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;   // [2]
  uint64_t* qdo_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* s_free = bars + 6;
  uint64_t* p_full = bars + 7;
  uint64_t* pt_free = bars + 8;
  uint64_t* dq_full = bars + 9;
  uint64_t* dq_free = bars + 10;
  uint64_t* dkv_full = bars + 11;
  uint64_t* drain = bars + 12;
  uint64_t* ld_bar = bars + 13;  // [2]: the 4 dS warps have staged LSE / delta of a query block
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 15);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* sLD = reinterpret_cast<float*>(smem + OFF_LD);  // [buf][0: lse2, 1: delta][128]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.S, Sk = p.Sk, H = p.H;
  const int kb = blockIdx.x;
  const int b = blockIdx.y / H, h = blockIdx.y % H;
  const int k0 = kb * BK;
  const int row_base = b * S;   // query rows (Q, dO, dQ)
  const int kv_base = b * Sk;   // key rows (K, V, dK, dV)
  const int nq = (S + BQ - 1) / BQ;
  const int i0 = CAUSAL ? kb : 0;
  const int lb = SPARSE ? __ldg(p.sp.ptr + kb) : 0;
  const int niter = SPARSE ? __ldg(p.sp.ptr + kb + 1) - lb : max(nq - i0, 0);
  auto qblk = [&](int n) -> int { return SPARSE ? __ldg(p.sp.idx + lb + n) : i0 + n; };
  const int col = h * HD;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qdo_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 8);
    mbar_init(p_full, 8);
    mbar_init(pt_free, 1);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 4);
    mbar_init(dkv_full, 1);
    mbar_init(drain, 1);
    mbar_init(&ld_bar[0], 4);
    mbar_init(&ld_bar[1], 4);
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
  constexpr uint32_t T_S = 0, T_DP = 128, T_DV = 256, T_DK = 256 + HD, T_DQ = 256 + 2 * HD;

  if (warp < 4) {
  setmaxnreg_dec<kRegsCtl>();
  if (warp == 0) {
    // ------------------------------------------------------------ TMA
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * T_BYTES);
      tma_load_2d(smem + OFF_K, &tmK, kv_full, col, kv_base + k0);
      tma_load_2d(smem + OFF_V, &tmV, kv_full, col, kv_base + k0);
      for (int n = 0; n < niter; ++n) {
        const int i = qblk(n);
        const int st = n & 1;
        if (!mbar_wait(&qdo_empty[st], ((n >> 1) & 1) ^ 1, p.st, 50, abort_flag)) break;
        mbar_arrive_expect_tx(&qdo_full[st], 2 * T_BYTES);
        tma_load_2d(smem + OFF_Q + st * T_BYTES, &tmQ, &qdo_full[st], col, row_base + i * BQ);
        tma_load_2d(smem + OFF_DO + st * T_BYTES, &tmDO, &qdo_full[st], col, row_base + i * BQ);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA
    if (lane == 0) {
      bool ok = mbar_wait(kv_full, 0, p.st, 51, abort_flag);
      tc_fence_after();
      const uint32_t k_addr = smem_u32(smem + OFF_K), v_addr = smem_u32(smem + OFF_V);
      const uint32_t pt_addr = smem_u32(smem + OFF_PT), ds_addr = smem_u32(smem + OFF_DST);
      for (int n = 0; n < niter && ok; ++n) {
        const int st = n & 1;
        ok = mbar_wait(&qdo_full[st], (n >> 1) & 1, p.st, 52, abort_flag) &&
             mbar_wait(s_free, (n & 1) ^ 1, p.st, 53, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(smem + OFF_Q + st * T_BYTES);
        const uint32_t do_addr = smem_u32(smem + OFF_DO + st * T_BYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          tc_mma_f16_ss(tmem + T_S, umma_desc_sw128(k_addr + kk * 32, 16, 1024),
                        umma_desc_sw128(q_addr + kk * 32, 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          tc_mma_f16_ss(tmem + T_DP, umma_desc_sw128(v_addr + kk * 32, 16, 1024),
                        umma_desc_sw128(do_addr + kk * 32, 16, 1024), IDESC_S, kk > 0 ? 1u : 0u);
        }
        tc_commit(s_full);
        if (!mbar_wait(p_full, n & 1, p.st, 54, abort_flag)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {
          const uint32_t aoff = (kk >> 2) * (BK * 128) + (kk & 3) * 32;  // K-major [key][q] tiles
          tc_mma_f16_ss(tmem + T_DV, umma_desc_sw128(pt_addr + aoff, 16, 1024),
                        umma_desc_sw128(do_addr + kk * 2048, 128 * 128, 1024), IDESC_KV,
                        (n > 0 || kk > 0) ? 1u : 0u);
          tc_mma_f16_ss(tmem + T_DK, umma_desc_sw128(ds_addr + aoff, 16, 1024),
                        umma_desc_sw128(q_addr + kk * 2048, 128 * 128, 1024), IDESC_KV,
                        (n > 0 || kk > 0) ? 1u : 0u);
        }
        if (!mbar_wait(dq_free, (n & 1) ^ 1, p.st, 55, abort_flag)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          // A = dS [q][key] = dS^T read MN-major: q atoms of 64 (16 KB apart), key rows 8 per 1 KB
          tc_mma_f16_ss(tmem + T_DQ, umma_desc_sw128(ds_addr + kk * 2048, BK * 128, 1024),
                        umma_desc_sw128(k_addr + kk * 2048, 128 * 128, 1024), IDESC_Q, kk > 0 ? 1u : 0u);
        }
        tc_commit(pt_free);
        tc_commit(dq_full);
        tc_commit(&qdo_empty[st]);
      }
      tc_commit(dkv_full);
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr, 0, nullptr);
    }
  }
  } else if (warp < 12) {
    setmaxnreg_inc<kRegsDs>();
    // ------------------------------------------------------------ dS warps
    // Eight warps compute P / dS for each query block: warps 4-7 the first
    // 64 queries of every key row, warps 8-11 the other 64 (two warps per
    // scheduler share the MUFU / issue work).
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;   // key row in the tile
    const int key = k0 + r;
    const bool stager = warp < 8;   // warps 4-7 stage the block's LSE / delta
    const int t128 = (warp - 4) * 32 + lane;
    const uint32_t lane_base = tmem + (uint32_t(q4 * 32) << 16);
    const float* lse_g = p.lse + ((long)b * H + h) * S;
    const float* del_g = p.delta + ((long)b * H + h) * S;
    uint8_t* pt_row = smem + OFF_PT + r * 128;
    uint8_t* ds_row = smem + OFF_DST + r * 128;
    const float LOG2E = 1.4426950408889634f;
    const int c_begin = stager ? 0 : BQ / 2;
    for (int n = 0; n < niter; ++n) {
      const int i = qblk(n);
      const int q0 = i * BQ;
      float* sL = sLD + (n & 1) * 256;
      if (stager) {
        const int q = q0 + t128;
        sL[t128] = q < S ? lse_g[q] * LOG2E : 0.f;
        sL[128 + t128] = q < S ? del_g[q] : 0.f;
        __syncwarp();
        if (lane == 0) mbar_arrive(&ld_bar[n & 1]);
      }
      if (!mbar_wait(&ld_bar[n & 1], (n >> 1) & 1, p.st, 60, abort_flag)) break;
      if (!mbar_wait(s_full, n & 1, p.st, 56, abort_flag)) break;
      if (!mbar_wait(pt_free, (n & 1) ^ 1, p.st, 57, abort_flag)) break;
      tc_fence_after();
      const bool need_mask = (q0 + BQ > S) || (k0 + BK > Sk) || (CAUSAL && q0 < k0 + BK) ||
                             (SPARSE && !attn_block_full(p.sp, q0, q0 + BQ - 1, k0, k0 + BK - 1));
      const AttnSpan span = attn_queries_of_key<SPARSE>(p.sp, key, q0, S, Sk, CAUSAL);
#pragma unroll 1
      for (int c = c_begin; c < c_begin + BQ / 2; c += 32) {
        uint32_t sv[32], dv[32];
        tmem_ld_32x32b_x32(lane_base + T_S + c, sv);
        tmem_ld_32x32b_x32(lane_base + T_DP + c, dv);
        tc_wait_ld();
        uint32_t pp[16], dd[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float pr[2], ds[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int ql = c + e + u;
            float pv = ex2_fast(fmaf(__uint_as_float(sv[e + u]), p.scale_log2, -sL[ql]));
            if (need_mask && !attn_span_has(span, ql)) pv = 0.f;
            pr[u] = pv;
            ds[u] = pv * (__uint_as_float(dv[e + u]) - sL[128 + ql]);
          }
          pp[e >> 1] = pack_bf16x2(pr[0], pr[1]);
          dd[e >> 1] = pack_bf16x2(ds[0], ds[1]);
        }
        const int blk = (c >> 6) * (BK * 128);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int unit = ((c & 63) >> 3) + u;
          const int so = blk + ((unit ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(pt_row + so) = make_uint4(pp[4 * u], pp[4 * u + 1], pp[4 * u + 2], pp[4 * u + 3]);
          *reinterpret_cast<uint4*>(ds_row + so) = make_uint4(dd[4 * u], dd[4 * u + 1], dd[4 * u + 2], dd[4 * u + 3]);
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(s_free);
        mbar_arrive(p_full);
      }
    }
  } else {
    setmaxnreg_dec<kRegsDrain>();
    // ------------------------------------------------------------ dQ drain, then dK / dV
    // Warps 12-15 move each block's dQ out of TMEM (lane quarter warp % 4):
    // TMEM -> 128B-swizzled fp32 smem slots -> TMA reduce-add into the fp32
    // dQ accumulator [B*S, H*HD], while the dS warps work on the next block.
    const int q4 = warp & 3;
    const uint32_t lane_base = tmem + (uint32_t(q4 * 32) << 16);
    uint8_t* slot0 = smem + OFF_DQS + (warp - 12) * 8192;
    uint8_t* slot1 = slot0 + 4096;
    bool ok = true;
    for (int n = 0; n < niter; ++n) {
      const int i = qblk(n);
      if (!mbar_wait(dq_full, n & 1, p.st, 58, abort_flag)) { ok = false; break; }
      tc_fence_after();
      uint32_t a0[32], a1[32];
      tmem_ld_32x32b_x32(lane_base + T_DQ, a0);
      tmem_ld_32x32b_x32(lane_base + T_DQ + 32, a1);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_free);
      if (lane == 0) tma_store_wait_read0();
      __syncwarp();
      // 32 rows x 32 fp32 per slot, 128-byte swizzle: unit u of row r at (u ^ (r & 7)) * 16
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        *reinterpret_cast<uint4*>(slot0 + lane * 128 + ((u ^ (lane & 7)) << 4)) =
            make_uint4(a0[4 * u], a0[4 * u + 1], a0[4 * u + 2], a0[4 * u + 3]);
        *reinterpret_cast<uint4*>(slot1 + lane * 128 + ((u ^ (lane & 7)) << 4)) =
            make_uint4(a1[4 * u], a1[4 * u + 1], a1[4 * u + 2], a1[4 * u + 3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int row = row_base + i * BQ + q4 * 32;
        asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                         &tmDQ), "r"(smem_u32(slot0)), "r"(col), "r"(row) : "memory");
        asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                         &tmDQ), "r"(smem_u32(slot1)), "r"(col + 32), "r"(row) : "memory");
        tma_store_commit();
      }
    }
    if (lane == 0) tma_store_wait0();
    __syncwarp();
    // dK, dV (TMEM lane = key row)
    if (ok && mbar_wait(dkv_full, 0, p.st, 59, abort_flag)) {
      tc_fence_after();
      const int r = q4 * 32 + lane;
      const int key = k0 + r;
      uint32_t kv[32];
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        bf16* dst = which ? (p.dv + (long)(kv_base + key) * p.dv_rs + col)
                          : (p.dk + (long)(kv_base + key) * p.dk_rs + col);
        const float sc = which ? 1.f : p.scale;
        const bool empty = SPARSE && niter == 0;  // no query sees these keys: zero gradients
#pragma unroll
        for (int c = 0; c < HD; c += 32) {
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
// Pipelined variant of the head_dim-64 backward. Same CTA shape, warp roles
// and outputs as fa_bwd_tc_kernel; the schedule differs so that the tensor
// core and the dS warps overlap instead of taking turns, and fewer operand
// bytes go through shared memory:
//
//   * the dS warps copy S^T of a query block out of TMEM first and release it
//     at once, so the MMA warp computes S^T of the NEXT block while the dS
//     warps are still on the exponentials of this one;
//   * P^T (bf16) goes to TMEM columns [448, 512) and dV += P^T dO reads it
//     from there (A operand in TMEM), issued as soon as P^T is written;
//   * dS^T (bf16) goes both to TMEM, over the dP^T columns this warp has
//     already read (dK += dS^T Q reads it from there), and to shared memory
//     (dQ = dS K needs it as an MN-major A operand);
//   * dP^T of the next block is issued right after dQ of this one;
//   * the staging warps load LSE / delta of the next block while this block
//     is in flight.
// dS is formed from the bf16 P that dV uses (32 live registers instead of 64).
//
// MMA issue order per block n: S_{n+1} | dV_n | dK_n | dQ_n | dP_{n+1}.
// TMEM columns: S^T [0,128), dP^T / dS^T [128,256), dV [256,320),
// dK [320,384), dQ [384,448), P^T [448,512).
// ---------------------------------------------------------------------------
template <bool CAUSAL, bool SPARSE = false, bool TRACE = false>
__global__ void __launch_bounds__(kThreads, 1)
    fa_bwd_pipe_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                       const __grid_constant__ CUtensorMap tmDQ, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;   // [2]
  uint64_t* qdo_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;     // S^T of a block is in TMEM (MMA commit)
  uint64_t* s_free = bars + 6;     // the 8 dS warps have copied S^T out
  uint64_t* dp_full = bars + 7;    // dP^T of a block is in TMEM (MMA commit)
  uint64_t* pt_full = bars + 8;    // P^T written to TMEM (8 warps)
  uint64_t* pt_free = bars + 9;    // dV MMA done with P^T (MMA commit)
  uint64_t* ds_full = bars + 10;   // dS^T written to TMEM and smem (8 warps)
  uint64_t* dq_full = bars + 11;
  uint64_t* dq_free = bars + 12;
  uint64_t* dkv_full = bars + 13;
  uint64_t* drain = bars + 14;
  uint64_t* ld_bar = bars + 15;    // [2]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 17);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* sLD = reinterpret_cast<float*>(smem + OFF_LD);  // [buf][0: lse2, 1: delta][128]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.S, Sk = p.Sk, H = p.H;
  const int kb = blockIdx.x;
  const int b = blockIdx.y / H, h = blockIdx.y % H;
  const int k0 = kb * BK;
  const int row_base = b * S;
  const int kv_base = b * Sk;
  const int nq = (S + BQ - 1) / BQ;
  const int i0 = CAUSAL ? kb : 0;
  const int lb = SPARSE ? __ldg(p.sp.ptr + kb) : 0;
  const int niter = SPARSE ? __ldg(p.sp.ptr + kb + 1) - lb : max(nq - i0, 0);
  auto qblk = [&](int n) -> int { return SPARSE ? __ldg(p.sp.idx + lb + n) : i0 + n; };
  const int col = h * HD;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qdo_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
      mbar_init(&ld_bar[i], 4);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 8);
    mbar_init(dp_full, 1);
    mbar_init(pt_full, 8);
    mbar_init(pt_free, 1);
    mbar_init(ds_full, 8);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 4);
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
  constexpr uint32_t T_S = 0, T_DP = 128, T_DV = 256, T_DK = 256 + HD, T_DQ = 256 + 2 * HD, T_PT = 448;

  if (warp < 4) {
  setmaxnreg_dec<kRegsCtl>();
  if (warp == 0) {
    // ------------------------------------------------------------ TMA
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * T_BYTES);
      tma_load_2d(smem + OFF_K, &tmK, kv_full, col, kv_base + k0);
      tma_load_2d(smem + OFF_V, &tmV, kv_full, col, kv_base + k0);
      for (int n = 0; n < niter; ++n) {
        const int i = qblk(n);
        const int st = n & 1;
        if (!mbar_wait(&qdo_empty[st], ((n >> 1) & 1) ^ 1, p.st, 50, abort_flag)) break;
        mbar_arrive_expect_tx(&qdo_full[st], 2 * T_BYTES);
        tma_load_2d(smem + OFF_Q + st * T_BYTES, &tmQ, &qdo_full[st], col, row_base + i * BQ);
        tma_load_2d(smem + OFF_DO + st * T_BYTES, &tmDO, &qdo_full[st], col, row_base + i * BQ);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA
    if (lane == 0) {
      const uint32_t k_addr = smem_u32(smem + OFF_K), v_addr = smem_u32(smem + OFF_V);
      const uint32_t ds_addr = smem_u32(smem + OFF_DST);
      auto q_at = [&](int n) { return smem_u32(smem + OFF_Q + (n & 1) * T_BYTES); };
      auto do_at = [&](int n) { return smem_u32(smem + OFF_DO + (n & 1) * T_BYTES); };
      // loop-invariant descriptors (K, V, dS^T); the Q / dO ones are built once per block and
      // stepped through k with desc_off
      const uint64_t dk_km = umma_desc_sw128(k_addr, 16, 1024), dv_km = umma_desc_sw128(v_addr, 16, 1024);
      const uint64_t dk_mn = umma_desc_sw128(k_addr, 128 * 128, 1024);
      const uint64_t dds_mn = umma_desc_sw128(ds_addr, BK * 128, 1024);
      auto issue_s = [&](int n) {  // S^T = K Q_n^T -> T_S
        const uint64_t dq = umma_desc_sw128(q_at(n), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          tc_mma_f16_ss(tmem + T_S, desc_off(dk_km, kk * 32), desc_off(dq, kk * 32), IDESC_S, kk > 0 ? 1u : 0u);
        tc_commit(s_full);
      };
      auto issue_dp = [&](int n) {  // dP^T = V dO_n^T -> T_DP
        const uint64_t ddo = umma_desc_sw128(do_at(n), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          tc_mma_f16_ss(tmem + T_DP, desc_off(dv_km, kk * 32), desc_off(ddo, kk * 32), IDESC_S, kk > 0 ? 1u : 0u);
        tc_commit(dp_full);
      };
      unsigned long long tm[6] = {0, 0, 0, 0, 0, 0};
      long long tkm = TRACE ? clock64() : 0;
      auto lapm = [&](int q) {
        if (TRACE) {
          const long long now = clock64();
          tm[q] += (unsigned long long)(now - tkm);
          tkm = now;
        }
      };
      bool ok = mbar_wait(kv_full, 0, p.st, 51, abort_flag);
      if (ok && niter > 0) {
        ok = mbar_wait(&qdo_full[0], 0, p.st, 52, abort_flag);
        if (ok) {
          tc_fence_after();
          issue_s(0);
          issue_dp(0);
        }
      }
      for (int n = 0; n < niter && ok; ++n) {
        const int st = n & 1;
        if (n + 1 < niter) {
          // next block's scores as soon as this block's S^T has been copied out
          lapm(5);
          ok = mbar_wait(&qdo_full[(n + 1) & 1], ((n + 1) >> 1) & 1, p.st, 52, abort_flag) &&
               mbar_wait(s_free, n & 1, p.st, 53, abort_flag);
          if (!ok) break;
          lapm(0);
          tc_fence_after();
          issue_s(n + 1);
          lapm(1);
        }
        if (!mbar_wait(pt_full, n & 1, p.st, 54, abort_flag)) { ok = false; break; }
        lapm(2);
        tc_fence_after();
        const uint64_t ddo_mn = umma_desc_sw128(do_at(n), 128 * 128, 1024);
        const uint64_t dq_mn = umma_desc_sw128(q_at(n), 128 * 128, 1024);
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)  // dV += P^T dO: A = P^T from TMEM (8 packed columns per k-step)
          tc_mma_f16_ts(tmem + T_DV, tmem + T_PT + kk * 8, desc_off(ddo_mn, kk * 2048), IDESC_KV,
                        (n > 0 || kk > 0) ? 1u : 0u);
        tc_commit(pt_free);
        lapm(5);
        if (!mbar_wait(ds_full, n & 1, p.st, 56, abort_flag)) { ok = false; break; }
        lapm(3);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)  // dK += dS^T Q: A = dS^T from TMEM (over the dP^T columns)
          tc_mma_f16_ts(tmem + T_DK, tmem + T_DP + (kk >> 2) * 64 + (kk & 3) * 8, desc_off(dq_mn, kk * 2048),
                        IDESC_KV, (n > 0 || kk > 0) ? 1u : 0u);
        lapm(5);
        if (!mbar_wait(dq_free, (n & 1) ^ 1, p.st, 55, abort_flag)) { ok = false; break; }
        lapm(4);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          tc_mma_f16_ss(tmem + T_DQ, desc_off(dds_mn, kk * 2048), desc_off(dk_mn, kk * 2048), IDESC_Q,
                        kk > 0 ? 1u : 0u);
        tc_commit(dq_full);
        tc_commit(&qdo_empty[st]);
        if (n + 1 < niter) issue_dp(n + 1);
        lapm(5);
      }
      if (TRACE) {
        unsigned long long* dst = p.trace + (long)(blockIdx.y * gridDim.x + blockIdx.x) * 16;
#pragma unroll
        for (int q = 0; q < 6; ++q) dst[8 + q] = tm[q];
        dst[14] = (unsigned long long)niter;
      }
      tc_commit(dkv_full);
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr, 0, nullptr);
    }
  }
  } else if (warp < 12) {
    setmaxnreg_inc<kRegsDs>();
    // ------------------------------------------------------------ dS warps
    // warps 4-7: queries [0, 64) of the block, warps 8-11: [64, 128);
    // thread = key row r (TMEM lane).
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const int key = k0 + r;
    const bool stager = warp < 8;
    const int t128 = (warp - 4) * 32 + lane;
    const uint32_t lane_base = tmem + (uint32_t(q4 * 32) << 16);
    const float* lse_g = p.lse + ((long)b * H + h) * S;
    const float* del_g = p.delta + ((long)b * H + h) * S;
    uint8_t* ds_row = smem + OFF_DST + r * 128;
    const float LOG2E = 1.4426950408889634f;
    const int hq = stager ? 0 : 1;         // query half of the block
    const int c_begin = hq * (BQ / 2);
    const bool tr = TRACE && warp == 4 && lane == 0;
    unsigned long long td[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    long long tkd = tr ? clock64() : 0;
    auto lapd = [&](int q) {
      if (TRACE && tr) {
        const long long now = clock64();
        td[q] += (unsigned long long)(now - tkd);
        tkd = now;
      }
    };
    float nl = 0.f, nd = 0.f;              // staged LSE / delta of the next block (stagers)
    if (stager && niter > 0) {
      const int q = qblk(0) * BQ + t128;
      nl = q < S ? lse_g[q] * LOG2E : 0.f;
      nd = q < S ? del_g[q] : 0.f;
    }
    for (int n = 0; n < niter; ++n) {
      const int i = qblk(n);
      const int q0 = i * BQ;
      float* sL = sLD + (n & 1) * 256;
      if (stager) {
        sL[t128] = nl;
        sL[128 + t128] = nd;
        __syncwarp();
        if (lane == 0) mbar_arrive(&ld_bar[n & 1]);
        if (n + 1 < niter) {  // prefetch the next block's rows while this one runs
          const int q = qblk(n + 1) * BQ + t128;
          nl = q < S ? lse_g[q] * LOG2E : 0.f;
          nd = q < S ? del_g[q] : 0.f;
        }
      }
      if (!mbar_wait(&ld_bar[n & 1], (n >> 1) & 1, p.st, 60, abort_flag)) break;
      lapd(0);
      if (!mbar_wait(s_full, n & 1, p.st, 57, abort_flag)) break;
      lapd(1);
      tc_fence_after();
      uint32_t sv[64];
      tmem_ld_32x32b_x32(lane_base + T_S + c_begin, sv);
      tmem_ld_32x32b_x32(lane_base + T_S + c_begin + 32, sv + 32);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);  // the tensor core may overwrite S^T now
      lapd(2);
      const bool need_mask = (q0 + BQ > S) || (k0 + BK > Sk) || (CAUSAL && q0 < k0 + BK) ||
                             (SPARSE && !attn_block_full(p.sp, q0, q0 + BQ - 1, k0, k0 + BK - 1));
      const AttnSpan span = attn_queries_of_key<SPARSE>(p.sp, key, q0, S, Sk, CAUSAL);
      uint32_t pk[32];
#pragma unroll
      for (int e = 0; e < 64; e += 4) {
        const float4 l4 = *reinterpret_cast<const float4*>(sL + c_begin + e);  // one broadcast load for 4 queries
        const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
        float pr[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int ql = c_begin + e + u;
          float pv = ex2_fast(fmaf(__uint_as_float(sv[e + u]), p.scale_log2, -lv[u]));
          if (need_mask && !attn_span_has(span, ql)) pv = 0.f;
          pr[u] = pv;
        }
        pk[e >> 1] = pack_bf16x2(pr[0], pr[1]);
        pk[(e >> 1) + 1] = pack_bf16x2(pr[2], pr[3]);
      }
      lapd(3);
      if (!mbar_wait(pt_free, (n & 1) ^ 1, p.st, 58, abort_flag)) break;
      lapd(4);
      tc_fence_after();
      tmem_st_32x32b_x16(lane_base + T_PT + (c_begin >> 1), pk);
      tmem_st_32x32b_x16(lane_base + T_PT + (c_begin >> 1) + 16, pk + 16);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pt_full);
      lapd(5);
      if (!mbar_wait(dp_full, n & 1, p.st, 59, abort_flag)) break;
      lapd(6);
      tc_fence_after();
      uint32_t dva[64];  // both halves of this thread's dP^T columns, one TMEM round trip
      tmem_ld_32x32b_x32(lane_base + T_DP + c_begin, dva);
      tmem_ld_32x32b_x32(lane_base + T_DP + c_begin + 32, dva + 32);
      tc_wait_ld();
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int c = c_begin + half * 32;
        const uint32_t* dv = dva + half * 32;
        uint32_t dd[16];
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          const float4 d4 = *reinterpret_cast<const float4*>(sL + 128 + c + e);
          const uint32_t pa = pk[(half * 32 + e) >> 1], pb = pk[((half * 32 + e) >> 1) + 1];
          dd[e >> 1] = pack_bf16x2(bf16_lo(pa) * (__uint_as_float(dv[e]) - d4.x),
                                   bf16_hi(pa) * (__uint_as_float(dv[e + 1]) - d4.y));
          dd[(e >> 1) + 1] = pack_bf16x2(bf16_lo(pb) * (__uint_as_float(dv[e + 2]) - d4.z),
                                         bf16_hi(pb) * (__uint_as_float(dv[e + 3]) - d4.w));
        }
        // TMEM copy for dK (over dP^T columns this thread has read), smem copy for dQ
        tmem_st_32x32b_x16(lane_base + T_DP + hq * 64 + half * 16, dd);
        const int blk = (c >> 6) * (BK * 128);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int unit = ((c & 63) >> 3) + u;
          const int so = blk + ((unit ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(ds_row + so) = make_uint4(dd[4 * u], dd[4 * u + 1], dd[4 * u + 2], dd[4 * u + 3]);
        }
      }
      tc_wait_st();
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_full);
      lapd(7);
    }
    if (TRACE && tr) {
      unsigned long long* dst = p.trace + (long)(blockIdx.y * gridDim.x + blockIdx.x) * 16;
#pragma unroll
      for (int q = 0; q < 8; ++q) dst[q] = td[q];
    }
  } else {
    setmaxnreg_dec<kRegsDrain>();
    // ------------------------------------------------------------ dQ drain, then dK / dV
    const int q4 = warp & 3;
    const uint32_t lane_base = tmem + (uint32_t(q4 * 32) << 16);
    uint8_t* slot0 = smem + OFF_DQS + (warp - 12) * 8192;
    uint8_t* slot1 = slot0 + 4096;
    bool ok = true;
    for (int n = 0; n < niter; ++n) {
      const int i = qblk(n);
      if (!mbar_wait(dq_full, n & 1, p.st, 61, abort_flag)) { ok = false; break; }
      tc_fence_after();
      uint32_t a0[32], a1[32];
      tmem_ld_32x32b_x32(lane_base + T_DQ, a0);
      tmem_ld_32x32b_x32(lane_base + T_DQ + 32, a1);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_free);
      if (lane == 0) tma_store_wait_read0();
      __syncwarp();
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        *reinterpret_cast<uint4*>(slot0 + lane * 128 + ((u ^ (lane & 7)) << 4)) =
            make_uint4(a0[4 * u], a0[4 * u + 1], a0[4 * u + 2], a0[4 * u + 3]);
        *reinterpret_cast<uint4*>(slot1 + lane * 128 + ((u ^ (lane & 7)) << 4)) =
            make_uint4(a1[4 * u], a1[4 * u + 1], a1[4 * u + 2], a1[4 * u + 3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int row = row_base + i * BQ + q4 * 32;
        asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                         &tmDQ), "r"(smem_u32(slot0)), "r"(col), "r"(row) : "memory");
        asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                         &tmDQ), "r"(smem_u32(slot1)), "r"(col + 32), "r"(row) : "memory");
        tma_store_commit();
      }
    }
    if (lane == 0) tma_store_wait0();
    __syncwarp();
    if (ok && mbar_wait(dkv_full, 0, p.st, 62, abort_flag)) {
      tc_fence_after();
      const int r = q4 * 32 + lane;
      const int key = k0 + r;
      uint32_t kv[32];
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        bf16* dst = which ? (p.dv + (long)(kv_base + key) * p.dv_rs + col)
                          : (p.dk + (long)(kv_base + key) * p.dk_rs + col);
        const float sc = which ? 1.f : p.scale;
        const bool empty = SPARSE && niter == 0;
#pragma unroll
        for (int c = 0; c < HD; c += 32) {
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
// Persistent head_dim-64 backward (non-sparse): one CTA per SM walks pairs
// of key tiles (see Sched: balanced under a causal mask, heads in order so
// that concurrent CTAs share L2-resident Q / dO / dQ). The per-block
// schedule is the pipelined one above, run as ONE stream of query blocks
// across all of a CTA's tiles, so the fixed cost of a tile (TMEM allocation,
// barrier set-up, K / V load latency, pipeline fill and drain, dK / dV
// write-out) overlaps the neighbouring tiles' work:
//   * K / V are double-buffered; the TMA warp loads the next tile's pair
//     while the current tile's last query blocks are in flight;
//   * S^T of the next tile's first block is issued before this tile ends;
//   * the drain warps copy dK / dV out of TMEM right after the tile's last
//     MMA, release the columns (dkv_free) and write them to global memory
//     while the next tile's first block runs.
// Barrier phases follow a per-CTA block counter g (blocks) and tile counter lt.
// ---------------------------------------------------------------------------
namespace ps {
constexpr int OFF_K = 0;                       // 2 stages x 16 KB
constexpr int OFF_V = OFF_K + 2 * T_BYTES;     // 2 stages
constexpr int OFF_Q = OFF_V + 2 * T_BYTES;     // 2 stages
constexpr int OFF_DO = OFF_Q + 2 * T_BYTES;    // 2 stages
constexpr int OFF_DST = OFF_DO + 2 * T_BYTES;  // dS^T [key][q] bf16, 32 KB
constexpr int OFF_DQS = OFF_DST + P_BYTES;     // 4 warps x 2 slots x 4 KB
constexpr int OFF_LD = OFF_DQS + 4 * 2 * 4096; // lse / delta [2][2][128] fp32
constexpr int OFF_BAR = OFF_LD + 4 * 128 * 4;
constexpr int SMEM = OFF_BAR + 256 + 1024;

struct Tile {
  int b, h, k0, i0, niter;
};
// The CTA's tiles. Work is handed out in PAIRS p = blockIdx.x + m * gridDim.x: pair p of
// (batch x head) bh = p / half covers the key tiles kp = p % half and nkb - 1 - kp (one tile
// when they coincide), so under a causal mask every pair holds nkb + 1 query blocks and a static
// assignment is balanced. Pairs are bh-major: the CTAs running at the same time share a few
// heads, whose Q, dO and dQ accumulator then stay in L2. A tile is named by code = 2 m + second.
struct Sched {
  int P, half, nkb, G, BH, H, nq;
  bool causal;
  __device__ __forceinline__ int pair(int code) const { return (int)blockIdx.x + (code >> 1) * G; }
  __device__ __forceinline__ bool valid(int code) const { return pair(code) < P; }
  __device__ __forceinline__ int next(int code) const {
    const int kp = pair(code) % half;
    return ((code & 1) == 0 && nkb - 1 - kp != kp) ? code + 1 : (code | 1) + 1;
  }
  __device__ __forceinline__ Tile tile(int code) const {
    const int p = pair(code);
    const int bh = p / half, kp = p - bh * half;
    const int kb = (code & 1) ? nkb - 1 - kp : kp;
    Tile t;
    t.b = bh / H;
    t.h = bh - t.b * H;
    t.k0 = kb * BK;
    t.i0 = causal ? kb : 0;
    t.niter = causal ? nq - kb : nq;
    return t;
  }
};
}  // namespace ps

template <bool CAUSAL>
__global__ void __launch_bounds__(kThreads, 1)
    fa_bwd_persist_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                          const __grid_constant__ CUtensorMap tmDQ, const Params p) {
  using namespace ps;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + ps::OFF_BAR);
  uint64_t* kv_full = bars + 0;    // [2]
  uint64_t* kv_empty = bars + 2;   // [2]
  uint64_t* qdo_full = bars + 4;   // [2]
  uint64_t* qdo_empty = bars + 6;  // [2]
  uint64_t* s_full = bars + 8;
  uint64_t* s_free = bars + 9;
  uint64_t* dp_full = bars + 10;
  uint64_t* pt_full = bars + 11;
  uint64_t* pt_free = bars + 12;
  uint64_t* ds_full = bars + 13;
  uint64_t* dq_full = bars + 14;
  uint64_t* dq_free = bars + 15;
  uint64_t* dkv_full = bars + 16;
  uint64_t* dkv_free = bars + 17;
  uint64_t* drain = bars + 18;
  uint64_t* ld_bar = bars + 19;    // [2]
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 21);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* sLD = reinterpret_cast<float*>(smem + ps::OFF_LD);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.S, Sk = p.Sk, H = p.H;
  const int BH = p.B * H;
  const int nq = (S + BQ - 1) / BQ;
  ps::Sched sc;
  sc.nkb = (Sk + BK - 1) / BK;
  sc.half = (sc.nkb + 1) / 2;
  sc.BH = BH;
  sc.P = BH * sc.half;
  sc.G = gridDim.x;
  sc.H = H;
  sc.nq = nq;
  sc.causal = CAUSAL;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&qdo_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
      mbar_init(&ld_bar[i], 4);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 8);
    mbar_init(dp_full, 1);
    mbar_init(pt_full, 8);
    mbar_init(pt_free, 1);
    mbar_init(ds_full, 8);
    mbar_init(dq_full, 1);
    mbar_init(dq_free, 4);
    mbar_init(dkv_full, 1);
    mbar_init(dkv_free, 4);
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
  constexpr uint32_t T_S = 0, T_DP = 128, T_DV = 256, T_DK = 256 + HD, T_DQ = 256 + 2 * HD, T_PT = 448;

  if (warp < 4) {
  setmaxnreg_dec<kRegsCtl>();
  if (warp == 0) {
    // ------------------------------------------------------------ TMA
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int j = 0, lt = 0; sc.valid(j) && ok; j = sc.next(j), ++lt) {
        const Tile tl = sc.tile(j);
        const int col = tl.h * HD;
        const int ks = lt & 1;
        if (!mbar_wait(&kv_empty[ks], ((lt >> 1) & 1) ^ 1, p.st, 63, abort_flag)) break;
        mbar_arrive_expect_tx(&kv_full[ks], 2 * T_BYTES);
        tma_load_2d(smem + ps::OFF_K + ks * T_BYTES, &tmK, &kv_full[ks], col, tl.b * Sk + tl.k0);
        tma_load_2d(smem + ps::OFF_V + ks * T_BYTES, &tmV, &kv_full[ks], col, tl.b * Sk + tl.k0);
        for (int n = 0; n < tl.niter; ++n, ++g) {
          const int st = g & 1;
          if (!mbar_wait(&qdo_empty[st], ((g >> 1) & 1) ^ 1, p.st, 50, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&qdo_full[st], 2 * T_BYTES);
          const int row = tl.b * S + (tl.i0 + n) * BQ;
          tma_load_2d(smem + ps::OFF_Q + st * T_BYTES, &tmQ, &qdo_full[st], col, row);
          tma_load_2d(smem + ps::OFF_DO + st * T_BYTES, &tmDO, &qdo_full[st], col, row);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA
    if (lane == 0) {
      const uint32_t ds_addr = smem_u32(smem + ps::OFF_DST);
      auto k_at = [&](int lt) { return smem_u32(smem + ps::OFF_K + (lt & 1) * T_BYTES); };
      auto v_at = [&](int lt) { return smem_u32(smem + ps::OFF_V + (lt & 1) * T_BYTES); };
      auto q_at = [&](int g) { return smem_u32(smem + ps::OFF_Q + (g & 1) * T_BYTES); };
      auto do_at = [&](int g) { return smem_u32(smem + ps::OFF_DO + (g & 1) * T_BYTES); };
      const uint64_t dds_mn = umma_desc_sw128(ds_addr, BK * 128, 1024);
      auto issue_s = [&](int lt, int g) {
        const uint64_t dk = umma_desc_sw128(k_at(lt), 16, 1024), dq = umma_desc_sw128(q_at(g), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          tc_mma_f16_ss(tmem + T_S, desc_off(dk, kk * 32), desc_off(dq, kk * 32), IDESC_S, kk > 0 ? 1u : 0u);
        tc_commit(s_full);
      };
      auto issue_dp = [&](int lt, int g) {
        const uint64_t dv = umma_desc_sw128(v_at(lt), 16, 1024), ddo = umma_desc_sw128(do_at(g), 16, 1024);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          tc_mma_f16_ss(tmem + T_DP, desc_off(dv, kk * 32), desc_off(ddo, kk * 32), IDESC_S, kk > 0 ? 1u : 0u);
        tc_commit(dp_full);
      };
      // cursor over the CTA's stream of query blocks: (tile counter, item, block in tile)
      int lt = 0, j = 0, n = 0;
      int niter = sc.valid(j) ? sc.tile(j).niter : 0;
      bool ok = true;
      if (sc.valid(j)) {
        ok = mbar_wait(&kv_full[0], 0, p.st, 64, abort_flag) && mbar_wait(&qdo_full[0], 0, p.st, 52, abort_flag);
        if (ok) {
          tc_fence_after();
          issue_s(0, 0);
          issue_dp(0, 0);
        }
      }
      for (int g = 0; sc.valid(j) && ok; ++g) {
        // the block after this one
        int lt2 = lt, j2 = j, n2 = n + 1, niter2 = niter;
        if (n2 == niter) {
          ++lt2;
          j2 = sc.next(j);
          n2 = 0;
          niter2 = sc.valid(j2) ? sc.tile(j2).niter : 0;
        }
        const bool has_next = sc.valid(j2);
        if (has_next) {
          ok = (n2 != 0 || mbar_wait(&kv_full[lt2 & 1], (lt2 >> 1) & 1, p.st, 64, abort_flag)) &&
               mbar_wait(&qdo_full[(g + 1) & 1], ((g + 1) >> 1) & 1, p.st, 52, abort_flag) &&
               mbar_wait(s_free, g & 1, p.st, 53, abort_flag);
          if (!ok) break;
          tc_fence_after();
          issue_s(lt2, g + 1);
        }
        if (!mbar_wait(pt_full, g & 1, p.st, 54, abort_flag)) { ok = false; break; }
        // a tile's first dV / dK overwrite the accumulators: the drain warps must
        // have copied the previous tile's dK / dV out
        if (n == 0 && lt > 0 && !mbar_wait(dkv_free, (lt - 1) & 1, p.st, 65, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint64_t ddo_mn = umma_desc_sw128(do_at(g), 128 * 128, 1024);
        const uint64_t dq_mn = umma_desc_sw128(q_at(g), 128 * 128, 1024);
        const uint64_t dk_mn = umma_desc_sw128(k_at(lt), 128 * 128, 1024);
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)
          tc_mma_f16_ts(tmem + T_DV, tmem + T_PT + kk * 8, desc_off(ddo_mn, kk * 2048), IDESC_KV,
                        (n > 0 || kk > 0) ? 1u : 0u);
        tc_commit(pt_free);
        if (!mbar_wait(ds_full, g & 1, p.st, 56, abort_flag)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)
          tc_mma_f16_ts(tmem + T_DK, tmem + T_DP + (kk >> 2) * 64 + (kk & 3) * 8, desc_off(dq_mn, kk * 2048),
                        IDESC_KV, (n > 0 || kk > 0) ? 1u : 0u);
        if (!mbar_wait(dq_free, (g & 1) ^ 1, p.st, 55, abort_flag)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          tc_mma_f16_ss(tmem + T_DQ, desc_off(dds_mn, kk * 2048), desc_off(dk_mn, kk * 2048), IDESC_Q,
                        kk > 0 ? 1u : 0u);
        tc_commit(dq_full);
        tc_commit(&qdo_empty[g & 1]);
        if (n + 1 == niter) {
          tc_commit(dkv_full);
          tc_commit(&kv_empty[lt & 1]);
        }
        if (has_next) issue_dp(lt2, g + 1);
        lt = lt2;
        j = j2;
        n = n2;
        niter = niter2;
      }
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr, 0, nullptr);
    }
  }
  } else if (warp < 12) {
    setmaxnreg_inc<kRegsDs>();
    // ------------------------------------------------------------ dS warps
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const bool stager = warp < 8;
    const int t128 = (warp - 4) * 32 + lane;
    const uint32_t lane_base = tmem + (uint32_t(q4 * 32) << 16);
    uint8_t* ds_row = smem + ps::OFF_DST + r * 128;
    const float LOG2E = 1.4426950408889634f;
    const int hq = stager ? 0 : 1;
    const int c_begin = hq * (BQ / 2);
    // staged LSE / delta of the next block (stagers), across tile boundaries
    auto load_ld = [&](int jj, int nn, float& l_, float& d_) {
      const Tile tl = sc.tile(jj);
      const long base = ((long)tl.b * H + tl.h) * S;
      const int q = (tl.i0 + nn) * BQ + t128;
      l_ = q < S ? p.lse[base + q] * LOG2E : 0.f;
      d_ = q < S ? p.delta[base + q] : 0.f;
    };
    float nl = 0.f, nd = 0.f;
    if (stager && sc.valid(0)) load_ld(0, 0, nl, nd);
    bool ok = true;
    int g = 0;
    for (int j = 0; sc.valid(j) && ok; j = sc.next(j)) {
      const Tile tl = sc.tile(j);
      const int key = tl.k0 + r;
      for (int n = 0; n < tl.niter; ++n, ++g) {
        const int q0 = (tl.i0 + n) * BQ;
        float* sL = sLD + (g & 1) * 256;
        if (stager) {
          sL[t128] = nl;
          sL[128 + t128] = nd;
          __syncwarp();
          if (lane == 0) mbar_arrive(&ld_bar[g & 1]);
          if (n + 1 < tl.niter) load_ld(j, n + 1, nl, nd);
          else if (sc.valid(sc.next(j))) load_ld(sc.next(j), 0, nl, nd);
        }
        if (!mbar_wait(&ld_bar[g & 1], (g >> 1) & 1, p.st, 60, abort_flag)) { ok = false; break; }
        if (!mbar_wait(s_full, g & 1, p.st, 57, abort_flag)) { ok = false; break; }
        tc_fence_after();
        uint32_t sv[64];
        tmem_ld_32x32b_x32(lane_base + T_S + c_begin, sv);
        tmem_ld_32x32b_x32(lane_base + T_S + c_begin + 32, sv + 32);
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_free);
        const bool need_mask = (q0 + BQ > S) || (tl.k0 + BK > Sk) || (CAUSAL && q0 < tl.k0 + BK);
        const AttnSpan span = attn_queries_of_key<false>(p.sp, key, q0, S, Sk, CAUSAL);
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 64; e += 4) {
          const float4 l4 = *reinterpret_cast<const float4*>(sL + c_begin + e);  // one broadcast load for 4 queries
          const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
          float pr[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int ql = c_begin + e + u;
            float pv = ex2_fast(fmaf(__uint_as_float(sv[e + u]), p.scale_log2, -lv[u]));
            if (need_mask && !attn_span_has(span, ql)) pv = 0.f;
            pr[u] = pv;
          }
          pk[e >> 1] = pack_bf16x2(pr[0], pr[1]);
          pk[(e >> 1) + 1] = pack_bf16x2(pr[2], pr[3]);
        }
        if (!mbar_wait(pt_free, (g & 1) ^ 1, p.st, 58, abort_flag)) { ok = false; break; }
        tc_fence_after();
        tmem_st_32x32b_x16(lane_base + T_PT + (c_begin >> 1), pk);
        tmem_st_32x32b_x16(lane_base + T_PT + (c_begin >> 1) + 16, pk + 16);
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(pt_full);
        if (!mbar_wait(dp_full, g & 1, p.st, 59, abort_flag)) { ok = false; break; }
        tc_fence_after();
        uint32_t dva[64];
        tmem_ld_32x32b_x32(lane_base + T_DP + c_begin, dva);
        tmem_ld_32x32b_x32(lane_base + T_DP + c_begin + 32, dva + 32);
        tc_wait_ld();
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int c = c_begin + half * 32;
          const uint32_t* dv = dva + half * 32;
          uint32_t dd[16];
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const float4 d4 = *reinterpret_cast<const float4*>(sL + 128 + c + e);
            const uint32_t pa = pk[(half * 32 + e) >> 1], pb = pk[((half * 32 + e) >> 1) + 1];
            dd[e >> 1] = pack_bf16x2(bf16_lo(pa) * (__uint_as_float(dv[e]) - d4.x),
                                     bf16_hi(pa) * (__uint_as_float(dv[e + 1]) - d4.y));
            dd[(e >> 1) + 1] = pack_bf16x2(bf16_lo(pb) * (__uint_as_float(dv[e + 2]) - d4.z),
                                           bf16_hi(pb) * (__uint_as_float(dv[e + 3]) - d4.w));
          }
          tmem_st_32x32b_x16(lane_base + T_DP + hq * 64 + half * 16, dd);
          const int blk = (c >> 6) * (BK * 128);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int unit = ((c & 63) >> 3) + u;
            const int so = blk + ((unit ^ (r & 7)) << 4);
            *reinterpret_cast<uint4*>(ds_row + so) = make_uint4(dd[4 * u], dd[4 * u + 1], dd[4 * u + 2], dd[4 * u + 3]);
          }
        }
        tc_wait_st();
        tc_fence_before();
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(ds_full);
      }
    }
  } else {
    setmaxnreg_dec<kRegsDrain>();
    // ------------------------------------------------------------ dQ drain and dK / dV write-out
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;
    const uint32_t lane_base = tmem + (uint32_t(q4 * 32) << 16);
    uint8_t* slot0 = smem + ps::OFF_DQS + (warp - 12) * 8192;
    uint8_t* slot1 = slot0 + 4096;
    bool ok = true;
    int g = 0;
    for (int j = 0, lt = 0; sc.valid(j) && ok; j = sc.next(j), ++lt) {
      const Tile tl = sc.tile(j);
      const int col = tl.h * HD;
      for (int n = 0; n < tl.niter; ++n, ++g) {
        if (!mbar_wait(dq_full, g & 1, p.st, 61, abort_flag)) { ok = false; break; }
        tc_fence_after();
        uint32_t a0[32], a1[32];
        tmem_ld_32x32b_x32(lane_base + T_DQ, a0);
        tmem_ld_32x32b_x32(lane_base + T_DQ + 32, a1);
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dq_free);
        if (lane == 0) tma_store_wait_read0();
        __syncwarp();
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          *reinterpret_cast<uint4*>(slot0 + lane * 128 + ((u ^ (lane & 7)) << 4)) =
              make_uint4(a0[4 * u], a0[4 * u + 1], a0[4 * u + 2], a0[4 * u + 3]);
          *reinterpret_cast<uint4*>(slot1 + lane * 128 + ((u ^ (lane & 7)) << 4)) =
              make_uint4(a1[4 * u], a1[4 * u + 1], a1[4 * u + 2], a1[4 * u + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const int row = tl.b * S + (tl.i0 + n) * BQ + q4 * 32;
          asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                           &tmDQ), "r"(smem_u32(slot0)), "r"(col), "r"(row) : "memory");
          asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                           &tmDQ), "r"(smem_u32(slot1)), "r"(col + 32), "r"(row) : "memory");
          tma_store_commit();
        }
      }
      if (!ok || !mbar_wait(dkv_full, lt & 1, p.st, 62, abort_flag)) { ok = false; break; }
      tc_fence_after();
      // copy dK / dV out chunk by chunk (TMEM lane = key row); the columns are
      // released after the last TMEM load, the global stores follow
      const int key = tl.k0 + r;
      const long kvrow = (long)tl.b * Sk + key;
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        const int which = ch >> 1, c = (ch & 1) * 32;
        uint32_t kv[32];
        tmem_ld_32x32b_x32(lane_base + (which ? T_DV : T_DK) + c, kv);
        tc_wait_ld();
        if (ch == 3) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(dkv_free);
        }
        if (key < Sk) {
          bf16* dst = which ? (p.dv + kvrow * p.dv_rs + col) : (p.dk + kvrow * p.dk_rs + col);
          const float sc = which ? 1.f : p.scale;
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
    if (lane == 0) tma_store_wait0();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace fabw

// Phase trace of the last traced backward launch: [CTAs, 16] int64 (see fabw::Params::trace).
static torch::Tensor g_bwd_trace;
torch::Tensor attn_bwd_trace() { return g_bwd_trace; }

// Attention backward core on tcgen05 (head_dim 64): writes dK, dV and
// reduce-adds the unscaled dQ into dq_acc (fp32 [B*S, H*HD], pre-zeroed by
// the caller). lse / delta fp32 [B, H, S]. q/dout [B, S, H, 64], k/v/dk/dv
// [B, Sk, H, 64]; `sp` (block lists of 128-query blocks per 128-key tile,
// and the element predicate) selects the sparse instantiation.
void flash_attn_bwd_tc(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor lse,
                       torch::Tensor delta, torch::Tensor dk, torch::Tensor dv, torch::Tensor dq_acc, bool causal,
                       double scale, const AttnSparse& sp, int schedule) {
  const int64_t B = q.size(0), S = q.size(1), H = q.size(2), HD = q.size(3);
  const int64_t Sk = k.size(1);
  TORCH_CHECK(HD == 64, "tcgen05 attention backward supports head_dim 64");
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
  auto mk = [&](const torch::Tensor& t, int64_t len) {
    return make_tmap_2d(t.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)(H * HD), (uint64_t)(B * len),
                        (uint64_t)t.stride(1) * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  };
  CUtensorMap tq = mk(q, S), tk = mk(k, Sk), tv = mk(v, Sk), tdo = mk(dout, S);
  CUtensorMap tdq = make_tmap_2d(dq_acc.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (uint64_t)(H * HD),
                                 (uint64_t)(B * S), (uint64_t)(H * HD) * 4, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  fabw::Params p{};
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.dk = reinterpret_cast<fabw::bf16*>(dk.data_ptr());
  p.dv = reinterpret_cast<fabw::bf16*>(dv.data_ptr());
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
  const bool pipelined = schedule >= 1;
  dim3 grid((unsigned)((Sk + 127) / 128), (unsigned)(B * H));
  auto st = cur_stream();
  {
    // phase trace of the pipelined kernel (profiling aid): SCIRS_ATTN_BWD_TRACE=1
    const char* e = getenv("SCIRS_ATTN_BWD_TRACE");
    if (e != nullptr && e[0] == '1' && pipelined && !sparse) {
      g_bwd_trace = torch::zeros({(long)grid.x * grid.y, 16}, q.options().dtype(at::kLong));
      p.trace = reinterpret_cast<unsigned long long*>(g_bwd_trace.data_ptr());
      auto kern = causal ? fabw::fa_bwd_pipe_kernel<true, false, true> : fabw::fa_bwd_pipe_kernel<false, false, true>;
      set_max_smem((const void*)kern, fabw::SMEM);
      kern<<<grid, fabw::kThreads, fabw::SMEM, st>>>(tq, tk, tv, tdo, tdq, p);
      SCIRS_CHECK_LAUNCH();
      return;
    }
  }
  if (schedule == 2 && !sparse) {
    // persistent: one CTA per SM over the (key tile, batch x head) items
    const long pairs = (long)((grid.x + 1) / 2) * grid.y;
    const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
    const unsigned g = (unsigned)std::min<long>(pairs, sms);
    auto kern = causal ? fabw::fa_bwd_persist_kernel<true> : fabw::fa_bwd_persist_kernel<false>;
    set_max_smem((const void*)kern, fabw::ps::SMEM);
    kern<<<g, fabw::kThreads, fabw::ps::SMEM, st>>>(tq, tk, tv, tdo, tdq, p);
    SCIRS_CHECK_LAUNCH();
    return;
  }
#define FABW(C_, SP_)                                                  \
  {                                                                    \
    auto kern = pipelined ? fabw::fa_bwd_pipe_kernel<C_, SP_> : fabw::fa_bwd_tc_kernel<C_, SP_>; \
    set_max_smem((const void*)kern, fabw::SMEM);                       \
    kern<<<grid, fabw::kThreads, fabw::SMEM, st>>>(tq, tk, tv, tdo, tdq, p); \
  }
  if (sparse) {
    if (causal) FABW(true, true) else FABW(false, true)
  } else {
    if (causal) FABW(true, false) else FABW(false, false)
  }
#undef FABW
  SCIRS_CHECK_LAUNCH();
}

}  // namespace scirs
