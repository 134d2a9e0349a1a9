// FlashAttention forward, second design: two query tiles per CTA in
// ping-pong, O accumulated in TMEM by the tensor cores, P handed to the PV
// MMA through TMEM, lazy rescaling.
//
// One CTA = 256 queries (two 128-row tiles t = 0, 1) of one (batch, head);
// both tiles share the K/V stream.
//
//   warp 0     TMA producer: Q0, Q1 once, then K_j / V_j into a 3-stage (head_dim
//              64) or 2-stage (128) ring
//   warp 1     owns TMEM (512 columns); one thread issues, per key block j,
//              PV_t(j) = P_t(j) V_j (A = P from TMEM, accumulated into O_t)
//              followed by S_t(j+1) = Q_t K_{j+1}^T, alternating t, so the
//              tensor core works on one tile while the other tile's softmax
//              warps run
//   warps 2-3  idle (their registers go to the softmax warpgroups)
//   warps 4-7  softmax of tile 0, warps 8-11 softmax of tile 1: thread owns
//              one query row (TMEM lane); reads the 128 scores of its row in
//              one go, takes the row max, and keeps a running reference max
//              that is raised only when a score exceeds it by more than
//              2^8 (then the O row in TMEM and the row sum are rescaled;
//              otherwise P = exp2(s - ref) <= 256 is exact enough in bf16 and
//              fp32). P is written back into the S columns as packed bf16
//              (tcgen05.st) and consumed there by the PV MMA.
//
// TMEM columns: S_t at [128 t, 128 t + 128) (P_t aliases its first 64),
// O_t at [256 + HD t, 256 + HD (t + 1)).
// MMAs issued by one thread complete in issue order, so S_t(j+1) may reuse
// the columns PV_t(j) reads, and the completion of S_t(j+1) (s_full) implies
// PV_t(j) has finished accumulating into O_t (which the softmax warps may
// then rescale). Causal masking touches only the diagonal block; keys >= S
// are masked; rows >= S are not stored. Every mbarrier wait is bounded.
//
// Reference parity: same math as the reference's CPU FlashAttention-2
// forward (scirs2-neural/src/layers/flash_attention_v2.rs:220,369-482,
// scirs2-neural/src/attention/flash_v2.rs:96-300); LSE is natural-log.
#include "host_common.h"

namespace scirs {
namespace fa2t {

using bf16 = __nv_bfloat16;
constexpr int BM = 128, BN = 128;
// 12 warps = 3 warpgroups: warpgroup 0 = TMA warp, MMA warp and two idle
// warps (registers given away), warpgroups 1 and 2 = the softmax warps of
// tile 0 and tile 1 (registers taken). The block launches with 168 registers
// per thread (65536 / 384 rounded down to 8), split as below.
constexpr int kThreads = 384;
// The control warps walk the persistent item list and keep 72 registers, the softmax warps
// 216: 128 x 72 + 256 x 216 = 384 x 168 (ptxas: no spills at head_dim 64).
constexpr int kRegsLaunch = 168;
template <int HD>
struct Regs {
  static constexpr int kCtl = 72;
  static constexpr int kSoftmax = 216;
  static_assert(128 * kCtl + 256 * kSoftmax <= kThreads * kRegsLaunch, "register split exceeds the launch");
};
constexpr float kRescaleLog2 = 8.f;  // raise the reference max only past 2^8

struct Params {
  bf16* out;
  float* lse;
  long o_rs;
  int B, H, S;  // S: query length
  int Sk;       // key / value length (cross-attention; = S for self-attention)
  float scale_log2;
  DevStatus* st;
  AttnSparse sp;  // used by the SPARSE instantiations
  // optional phase timing (clock64 cycles summed over the loop) of one
  // softmax thread per tile: [CTA][tile][wait S, TMEM load, max/rescale,
  // exp + P store, signal]; nullptr = off
  unsigned long long* trace;
};

template <int HD>
struct Cfg {
  static constexpr int Q_BYTES = BM * HD * 2;
  static constexpr int KV_BYTES = BN * HD * 2;
  // K/V ring depth: 3 stages for head_dim 64 (which also keeps the CTA at
  // one per SM, matching its 512-column TMEM allocation), 2 for 128
  static constexpr int NST = (HD == 64) ? 3 : 2;
  static constexpr int OFF_Q = 0;                         // 2 tiles
  static constexpr int OFF_K = OFF_Q + 2 * Q_BYTES;       // NST stages
  static constexpr int OFF_V = OFF_K + NST * KV_BYTES;    // NST stages
  static constexpr int OFF_BAR = OFF_V + NST * KV_BYTES;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;
  static constexpr int TMEM_COLS = 512;
  static constexpr uint32_t IDESC_S = umma_idesc_bf16(BM, BN, 0, 0);
  static constexpr uint32_t IDESC_O = umma_idesc_bf16(BM, HD, 0, 1);
};

// 2^x on the FMA pipe (for x <= 0, softmax arguments): x = n + f with n the
// nearest integer (added into the low mantissa bits of 1.5 * 2^23) and f in
// [-0.5, 0.5]; 2^f by a degree-3 polynomial whose coefficients come from a
// Remez fit of the relative error on [-0.5, 0.5] (max 7.5e-5, far below the
// bf16 rounding of P); 2^n is applied by adding n to the exponent field.
// Arguments below -125 return 0, as ex2 of a masked (-inf) score does.
__device__ __forceinline__ float exp2_poly3(float x) {
  const float xc = fmaxf(x, -125.f);
  const float j = xc + 12582912.f;
  const float f = xc - (j - 12582912.f);
  float q = fmaf(5.517166906e-02f, f, 2.426111222e-01f);
  q = fmaf(q, f, 6.932609855e-01f);
  q = fmaf(q, f, 9.999280735e-01f);
  const float r = __int_as_float(__float_as_int(q) + (__float_as_int(j) << 23));
  return x < -125.f ? 0.f : r;
}

// exp2_poly3 for a pair, the floating-point steps as packed f32x2
// instructions (one FADD2 / FFMA2 per step for both values): the same
// rounding split and Remez cubic as exp2_poly3, 2^n added to the exponent
// field per value.
__device__ __forceinline__ void exp2_poly3_x2(float x0, float x1, float& r0, float& r1) {
  const uint64_t xc = f2_pack(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
  const uint64_t j = f2_add(xc, f2_pack(12582912.f, 12582912.f));
  const uint64_t jr = f2_add(j, f2_pack(-12582912.f, -12582912.f));
  const uint64_t f = f2_fma(jr, f2_pack(-1.f, -1.f), xc);
  uint64_t q = f2_fma(f2_pack(5.517166906e-02f, 5.517166906e-02f), f, f2_pack(2.426111222e-01f, 2.426111222e-01f));
  q = f2_fma(q, f, f2_pack(6.932609855e-01f, 6.932609855e-01f));
  q = f2_fma(q, f, f2_pack(9.999280735e-01f, 9.999280735e-01f));
  float q0, q1, j0, j1;
  f2_unpack(q, q0, q1);
  f2_unpack(j, j0, j1);
  r0 = x0 < -125.f ? 0.f : __int_as_float(__float_as_int(q0) + (__float_as_int(j0) << 23));
  r1 = x1 < -125.f ? 0.f : __int_as_float(__float_as_int(q1) + (__float_as_int(j1) << 23));
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

template <int HD, bool CAUSAL, bool POLY = false, bool TRACE = false, bool X2 = false, bool SPARSE = false,
          bool BF2 = false>
__global__ void __launch_bounds__(kThreads, 1)
    fa_fwd_pp_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const Params p) {
  using C = Cfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  constexpr int NST = C::NST;
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;              // [NST] stages
  uint64_t* v_full = k_full + NST;          // [NST]
  uint64_t* kv_empty = v_full + NST;        // [NST]
  uint64_t* s_full = kv_empty + NST;        // [2] tiles
  uint64_t* p_full = s_full + 2;            // [2] tiles (4 warps each)
  uint64_t* o_final = p_full + 2;           // [2] tiles
  uint64_t* drain = o_final + 2;
  uint64_t* q_empty = drain + 1;            // the MMAs of an item are done with Q
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(q_empty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.S, Sk = p.Sk, H = p.H;
  // Work items: (query pair qp, batch x head bh); item i has qp = nqp - 1 - i / BH (the longest causal
  // work first) and bh = i % BH. A CTA takes items item0, item0 + istride, ...: with a grid of
  // (nqp, B*H) that is exactly one item per CTA, with a grid of one CTA per SM the kernel is persistent.
  const int BH = p.B * H;
  const int nqp = (S + 2 * BM - 1) / (2 * BM);
  const int nitems = nqp * BH;
  const int item0 = blockIdx.x * gridDim.y + blockIdx.y;
  const int istride = gridDim.x * gridDim.y;
  const int nkv_all = (Sk + BN - 1) / BN;
  struct Item {
    int b, h, q0, lb, nkv0, nkv1, nkv;
  };
  auto item_of = [&](int i) -> Item {
    Item I;
    const int qp = nqp - 1 - i / BH, bh = i % BH;
    I.b = bh / H;
    I.h = bh % H;
    I.q0 = qp * 2 * BM;
    // SPARSE: the item visits the key blocks of its list (both tiles)
    I.lb = SPARSE ? __ldg(p.sp.ptr + qp) : 0;
    const int cnt = SPARSE ? __ldg(p.sp.ptr + qp + 1) - I.lb : 0;
    // key blocks each tile needs (tile t covers queries [q0 + 128 t, +128))
    I.nkv0 = (I.q0 >= S) ? 0 : (SPARSE ? cnt : (CAUSAL ? min(nkv_all, I.q0 / BM + 1) : nkv_all));
    I.nkv1 = (I.q0 + BM >= S) ? 0 : (SPARSE ? cnt : (CAUSAL ? min(nkv_all, I.q0 / BM + 2) : nkv_all));
    I.nkv = max(I.nkv0, I.nkv1);
    return I;
  };
  auto kblk = [&](const Item& I, int j) -> int { return SPARSE ? __ldg(p.sp.idx + I.lb + j) : j; };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_final[i], 1);
    }
    mbar_init(drain, 1);
    mbar_init(q_empty, 1);
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
  if (warp < 4) {
  setmaxnreg_dec<Regs<HD>::kCtl>();
  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      int jg = 0;  // K / V ring position over all of this CTA's key blocks
      bool ok = true;
      for (int it = item0, ii = 0; it < nitems && ok; it += istride, ++ii) {
        const Item I = item_of(it);
        const int col = I.h * HD;
        // the previous item's score MMAs have read Q
        if (!mbar_wait(q_empty, (ii & 1) ^ 1, p.st, 49, abort_flag)) break;
        mbar_arrive_expect_tx(q_full, 2 * C::Q_BYTES);
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int c = 0; c < HD / 64; ++c)
            tma_load_2d(smem + C::OFF_Q + t * C::Q_BYTES + c * (BM * 128), &tmQ, q_full, col + c * 64,
                        I.b * S + I.q0 + t * BM);
        for (int j = 0; j < I.nkv; ++j, ++jg) {
          const int s = jg % NST;
          if (!mbar_wait(&kv_empty[s], ((jg / NST) & 1) ^ 1, p.st, 50, abort_flag)) { ok = false; break; }
          const int krow = I.b * Sk + kblk(I, j) * BN;
          mbar_arrive_expect_tx(&k_full[s], C::KV_BYTES);
#pragma unroll
          for (int c = 0; c < HD / 64; ++c)
            tma_load_2d(smem + C::OFF_K + s * C::KV_BYTES + c * (BN * 128), &tmK, &k_full[s], col + c * 64, krow);
          mbar_arrive_expect_tx(&v_full[s], C::KV_BYTES);
#pragma unroll
          for (int c = 0; c < HD / 64; ++c)
            tma_load_2d(smem + C::OFF_V + s * C::KV_BYTES + c * (BN * 128), &tmV, &v_full[s], col + c * 64, krow);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      const uint32_t q_addr = smem_u32(smem + C::OFF_Q);
      // jg: K / V ring position of the item's first key block; c0 / c1: blocks of
      // tile 0 / 1 in earlier items (phases of s_full / p_full)
      int jg = 0, c0 = 0, c1 = 0;
      bool ok = true;
      auto issue_s = [&](int t, int j) -> bool {
        const int s = (jg + j) % NST;
        if (!mbar_wait(&k_full[s], ((jg + j) / NST) & 1, p.st, 52, abort_flag)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(smem + C::OFF_K + s * C::KV_BYTES);
        const uint32_t qa = q_addr + t * C::Q_BYTES;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint32_t offk = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          tc_mma_f16_ss(tmem + t * BN, umma_desc_sw128(qa + off, 16, 1024), umma_desc_sw128(k_addr + offk, 16, 1024),
                        C::IDESC_S, kk > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[t]);
        return true;
      };
      for (int it = item0, ii = 0; it < nitems && ok; it += istride, ++ii) {
      const Item I = item_of(it);
      if (!mbar_wait(q_full, ii & 1, p.st, 51, abort_flag)) { ok = false; break; }
      tc_fence_after();
      if (I.nkv0 > 0) ok = issue_s(0, 0);
      if (ok && I.nkv1 > 0) ok = issue_s(1, 0);
      if (ok && I.nkv <= 1) tc_commit(q_empty);  // every score MMA of the item is issued
      for (int j = 0; j < I.nkv && ok; ++j) {
        const int s = (jg + j) % NST;
        bool v_ready = false;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int nt = t ? I.nkv1 : I.nkv0;
          if (!ok || j >= nt) continue;
          if (!mbar_wait(&p_full[t], ((t ? c1 : c0) + j) & 1, p.st, 53, abort_flag)) { ok = false; break; }
          if (!v_ready) {
            if (!mbar_wait(&v_full[s], ((jg + j) / NST) & 1, p.st, 54, abort_flag)) { ok = false; break; }
            v_ready = true;
          }
          tc_fence_after();
          const uint32_t v_addr = smem_u32(smem + C::OFF_V + s * C::KV_BYTES);
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            // A = P_t from TMEM (16 keys = 8 packed columns per step);
            // B = V [keys][HD] MN-major: k-step = 16 key rows = 2048 bytes
            const uint64_t bdesc = umma_desc_sw128(v_addr + kk * 2048, BN * 128, 1024);
            tc_mma_f16_ts(tmem + 2 * BN + t * HD, tmem + t * BN + kk * 8, bdesc, C::IDESC_O,
                          (j > 0 || kk > 0) ? 1u : 0u);
          }
          if (j + 1 < nt) {
            ok = issue_s(t, j + 1);
          } else {
            tc_commit(&o_final[t]);
          }
        }
        if (ok && j == I.nkv - 2) tc_commit(q_empty);  // the item's last score MMAs are issued
        if (ok) tc_commit(&kv_empty[s]);
      }
      jg += I.nkv;
      c0 += I.nkv0;
      c1 += I.nkv1;
      }
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr, 0, nullptr);
    }
  }
  } else {
    setmaxnreg_inc<Regs<HD>::kSoftmax>();
    // ---------------------------------------------------------------- softmax
    const int t = (warp - 4) >> 2;   // tile of this warpgroup
    const int q = warp & 3;          // TMEM lane quarter
    const int r = q * 32 + lane;     // query row within the tile
    const uint32_t lane_off = uint32_t(q * 32) << 16;
    const uint32_t s_base = tmem + lane_off + t * BN;
    const uint32_t o_base = tmem + lane_off + 2 * BN + t * HD;
    bool ok = true;
    const bool tr = TRACE && q == 0 && lane == 0;
    unsigned long long ph[5] = {0, 0, 0, 0, 0};
    long long tk = (TRACE && tr) ? clock64() : 0;
    auto lap = [&](int k) {
      if (TRACE && tr) {
        const long long now = clock64();
        ph[k] += (unsigned long long)(now - tk);
        tk = now;
      }
    };
    int cb = 0, ni = 0;  // this tile's blocks in earlier items; earlier items with blocks
    for (int it = item0; it < nitems && ok; it += istride) {
    // only the query offset, the tile's block count and the block list start stay live across the
    // block loop (the softmax warps are at their register limit); the rest is recomputed below
    const Item I = item_of(it);
    const int q0 = I.q0;
    const int my_nkv = t ? I.nkv1 : I.nkv0;
    float m_ref = -INFINITY, l = 0.f;
    for (int j = 0; j < my_nkv && ok; ++j) {
      if (!mbar_wait(&s_full[t], (cb + j) & 1, p.st, 55, abort_flag)) { ok = false; break; }
      tc_fence_after();
      lap(0);
      float sv[BN];
      {
        uint32_t* u = reinterpret_cast<uint32_t*>(sv);
#pragma unroll
        for (int c = 0; c < BN; c += 32) tmem_ld_32x32b_x32(s_base + c, u + c);
        tc_wait_ld();
      }
      lap(1);
      const int kv0 = kblk(I, j) * BN;
      const bool mask = (kv0 + BN > Sk) || (CAUSAL && kv0 + BN > q0 + t * BM) ||
                        (SPARSE && !attn_block_full(p.sp, q0 + t * BM, q0 + t * BM + BM - 1, kv0, kv0 + BN - 1));
      if (mask) {
        const AttnSpan span = attn_keys_of_query<SPARSE>(p.sp, q0 + t * BM + r, kv0, Sk, CAUSAL);
#pragma unroll
        for (int e = 0; e < BN; ++e) sv[e] = attn_span_has(span, e) ? sv[e] : -INFINITY;
      }
      // row max: four independent chains of 3-input max instructions
      float m4[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
      for (int e = 4; e < BN; e += 8) {
        m4[0] = fmax3(m4[0], sv[e], sv[e + 4]);
        m4[1] = fmax3(m4[1], sv[e + 1], sv[e + 5]);
        m4[2] = fmax3(m4[2], sv[e + 2], sv[e + 6]);
        m4[3] = fmax3(m4[3], sv[e + 3], sv[e + 7]);
      }
      const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * p.scale_log2;
      // raise the reference max (and rescale O and l) only when needed
      const bool raise = mx > m_ref + kRescaleLog2;
      float alpha = 1.f;
      if (raise) {
        alpha = (m_ref == -INFINITY) ? 0.f : ex2_fast(m_ref - mx);
        m_ref = mx;
        l *= alpha;
      }
      if (j > 0 && __any_sync(0xffffffffu, raise)) {
        // O_t holds PV_t(0..j-1), complete (implied by s_full above)
#pragma unroll 1
        for (int c = 0; c < HD; c += 32) {
          uint32_t ov[32];
          tmem_ld_32x32b_x32(o_base + c, ov);
          tc_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
          tmem_st_32x32b_x16(o_base + c, ov);
          tmem_st_32x32b_x16(o_base + c + 16, ov + 16);
        }
        tc_wait_st();
      }
      lap(2);
      const float ref = (m_ref == -INFINITY) ? 0.f : m_ref;
      float rs[4] = {0.f, 0.f, 0.f, 0.f};
      uint64_t rs2[2] = {0ull, 0ull};  // X2: packed row-sum accumulators
      const uint64_t sc2 = f2_pack(p.scale_log2, p.scale_log2), nref2 = f2_pack(-ref, -ref);
#pragma unroll
      for (int c = 0; c < BN; c += 32) {
        // 32 scores -> 16 packed bf16 pairs -> TMEM columns [c/2, c/2 + 16);
        // with POLY every second exponential runs on the FMA pipe, halving
        // the MUFU work; with X2 the scale / subtract and the row sums run
        // as packed pair instructions
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float p0, p1;
          if (BF2) {
            // two exponentials per MUFU instruction; P comes out packed
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(sv[c + e], sv[c + e + 1]), sc2, nref2), x0, x1);
            const uint32_t pp = ex2_bf16x2(x0, x1);
            pk[e >> 1] = pp;
            rs2[(e >> 1) & 1] = f2_add(rs2[(e >> 1) & 1], f2_pack(bf16_lo(pp), bf16_hi(pp)));
            continue;
          }
          if (X2) {
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(sv[c + e], sv[c + e + 1]), sc2, nref2), x0, x1);
            if (POLY && ((e >> 1) & 1)) {
              // every second pair on the FMA pipe: the MUFU unit is the
              // busiest pipe of this loop
              exp2_poly3_x2(x0, x1, p0, p1);
            } else {
              p0 = ex2_fast(x0);
              p1 = ex2_fast(x1);
            }
            rs2[(e >> 1) & 1] = f2_add(rs2[(e >> 1) & 1], f2_pack(p0, p1));
          } else {
            p0 = ex2_fast(fmaf(sv[c + e], p.scale_log2, -ref));
            const float x1 = fmaf(sv[c + e + 1], p.scale_log2, -ref);
            p1 = POLY ? exp2_poly3(x1) : ex2_fast(x1);
            rs[(e >> 1) & 3] += p0 + p1;
          }
          pk[e >> 1] = pack_bf16x2(p0, p1);
        }
        tmem_st_32x32b_x16(s_base + (c >> 1), pk);
      }
      if (X2 || BF2) {
        f2_unpack(f2_add(rs2[0], rs2[1]), rs[0], rs[1]);
        l += rs[0] + rs[1];
      } else {
        l += (rs[0] + rs[1]) + (rs[2] + rs[3]);
      }
      tc_wait_st();
      lap(3);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
      lap(4);
    }
    int it2 = it;
    asm volatile("" : "+r"(it2));  // an opaque copy: recompute the item's fields instead of keeping them
    const Item I2 = item_of(it2);
    const int b = I2.b, h = I2.h;
    const int row_base = b * S;
    const int qrow = I2.q0 + t * BM + r;
    const bool fin = ok && my_nkv > 0;
    if (fin && !mbar_wait(&o_final[t], ni & 1, p.st, 56, abort_flag)) ok = false;
    if (fin && ok) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      bf16* orow = p.out + (long)(row_base + qrow) * p.o_rs + h * HD;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        uint32_t ov[32];
        tmem_ld_32x32b_x32(o_base + c, ov);
        tc_wait_ld();
        if (qrow < S) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 o;
            const float* f = reinterpret_cast<const float*>(ov) + g * 8;
            o.x = pack_bf16x2(f[0] * inv, f[1] * inv);
            o.y = pack_bf16x2(f[2] * inv, f[3] * inv);
            o.z = pack_bf16x2(f[4] * inv, f[5] * inv);
            o.w = pack_bf16x2(f[6] * inv, f[7] * inv);
            *reinterpret_cast<uint4*>(orow + c + g * 8) = o;
          }
        }
      }
      if (qrow < S) p.lse[((long)b * H + h) * S + qrow] = (m_ref + log2f(l)) * 0.6931471805599453f;
    } else if (SPARSE && ok && my_nkv == 0 && qrow < S) {
      // an empty key list: zero output, -inf log-sum-exp
      bf16* orow = p.out + (long)(row_base + qrow) * p.o_rs + h * HD;
      for (int c = 0; c < HD; c += 8) *reinterpret_cast<uint4*>(orow + c) = make_uint4(0u, 0u, 0u, 0u);
      p.lse[((long)b * H + h) * S + qrow] = -INFINITY;
    }
    cb += my_nkv;
    ni += my_nkv > 0 ? 1 : 0;
    }
    if (TRACE && tr) {
      unsigned long long* dst = p.trace + ((long)(blockIdx.y * gridDim.x + blockIdx.x) * 2 + t) * 5;
#pragma unroll
      for (int k = 0; k < 5; ++k) dst[k] = ph[k];
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace fa2t

// Fill an AttnSparse from optional tensors (block lists int32, bitmap uint8).
AttnSparse attn_sparse_args(const c10::optional<torch::Tensor>& ptr, const c10::optional<torch::Tensor>& idx,
                            const c10::optional<torch::Tensor>& bmap, int64_t wl, int64_t wr, int64_t ng,
                            int64_t rows) {
  AttnSparse a{};
  a.wl = (int)wl;
  a.wr = (int)wr;
  a.ng = (int)ng;
  const bool has = ptr.has_value() && ptr->defined();
  TORCH_CHECK(has == (idx.has_value() && idx->defined()), "block lists need both ptr and idx");
  if (has) {
    TORCH_CHECK(ptr->scalar_type() == at::kInt && idx->scalar_type() == at::kInt && ptr->is_contiguous() &&
                    idx->is_contiguous() && ptr->is_cuda() && idx->is_cuda(),
                "block lists: contiguous int32 CUDA tensors");
    TORCH_CHECK(ptr->numel() == rows + 1, "block list ptr must have one entry per CTA plus one");
    a.ptr = ptr->data_ptr<int>();
    a.idx = idx->data_ptr<int>();
  }
  if (bmap.has_value() && bmap->defined()) {
    TORCH_CHECK(bmap->scalar_type() == at::kByte && bmap->dim() == 2 && bmap->is_contiguous() && bmap->is_cuda(),
                "block bitmap: contiguous uint8 CUDA [q blocks, k blocks]");
    a.bmap = bmap->data_ptr<uint8_t>();
    a.bmap_ld = (int)bmap->size(1);
  }
  return a;
}

// q/out: [B, S, H, HD], k/v: [B, Sk, H, HD] token-major views with contiguous
// heads; lse [B, H, S]. With block lists (blk_ptr / blk_idx: for CTA c, which
// covers queries [256 c, 256 c + 256), the key blocks blk_idx[blk_ptr[c] ..
// blk_ptr[c + 1]) of 128 keys) the kernel visits only those blocks and masks
// with the element predicate (window wl / wr with ng global tokens, and the
// optional 128 x 128 block bitmap).
void flash_attn_fwd_pp(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                       bool causal, double scale, bool poly, c10::optional<torch::Tensor> trace, bool x2,
                       c10::optional<torch::Tensor> blk_ptr, c10::optional<torch::Tensor> blk_idx,
                       c10::optional<torch::Tensor> bmap, int64_t wl, int64_t wr, int64_t ng, bool bf2,
                       int64_t persist_req) {
  const int64_t B = q.size(0), S = q.size(1), H = q.size(2), HD = q.size(3);
  const int64_t Sk = k.size(1);
  TORCH_CHECK(HD == 64 || HD == 128, "head_dim must be 64 or 128");
  TORCH_CHECK(!causal || Sk == S, "causal attention needs equal query and key lengths");
  for (auto* t : {&q, &k, &v, &out}) {
    const int64_t St = (t == &k || t == &v) ? Sk : S;
    TORCH_CHECK(t->scalar_type() == at::kBFloat16 && t->dim() == 4 && t->size(0) == B && t->size(1) == St &&
                    t->size(2) == H && t->size(3) == HD,
                "q/out must be bf16 [B, S, H, HD] and k/v bf16 [B, Sk, H, HD]");
    TORCH_CHECK(t->stride(3) == 1 && t->stride(2) == HD && t->stride(0) == St * t->stride(1),
                "q/k/v/out must be token-major with contiguous heads");
  }
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.numel() == B * H * S && lse.is_contiguous(), "lse fp32 [B,H,S]");
  c10::cuda::CUDAGuard guard(q.get_device());
  auto mk = [&](const torch::Tensor& t, int64_t rows) {
    return make_tmap_2d(t.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (uint64_t)(H * HD), (uint64_t)(B * rows),
                        (uint64_t)t.stride(1) * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B);
  };
  CUtensorMap tq = mk(q, S), tk = mk(k, Sk), tv = mk(v, Sk);
  fa2t::Params p{};
  p.out = reinterpret_cast<fa2t::bf16*>(out.data_ptr());
  p.lse = lse.data_ptr<float>();
  p.o_rs = out.stride(1);
  p.B = (int)B;
  p.H = (int)H;
  p.S = (int)S;
  p.Sk = (int)Sk;
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  p.st = status_ptr(q.get_device());
  // one CTA per (query pair, batch x head) item, or one CTA per SM walking the
  // items
  dim3 grid((unsigned)((S + 255) / 256), (unsigned)(B * H));
  const int64_t nqp = grid.x;
  p.sp = attn_sparse_args(blk_ptr, blk_idx, bmap, wl, wr, ng, nqp);
  const bool sparse = p.sp.ptr != nullptr || p.sp.bmap != nullptr || p.sp.wl >= 0 || p.sp.ng > 0;
  TORCH_CHECK(!sparse || p.sp.ptr != nullptr, "a sparsity predicate needs block lists");
  if (trace.has_value() && trace->defined()) {
    TORCH_CHECK(trace->scalar_type() == at::kLong && trace->is_contiguous() &&
                    trace->numel() >= (long)grid.x * grid.y * 2 * 5,
                "trace: int64 [grid, 2, 5]");
    p.trace = reinterpret_cast<unsigned long long*>(trace->data_ptr());
  }
  {
    const char* e = getenv("SCIRS_ATTN_FWD_PERSIST");
    // persist_req: 1 / 0 = the caller's choice, -1 = by size: persistent for head_dim 64, and for
    // 128 up to 1,024 queries (measured faster there). SCIRS_ATTN_FWD_PERSIST=0 / 1 overrides.
    const bool dflt = persist_req >= 0 ? persist_req == 1 : (HD == 64 || S <= 1024);
    const bool persist = (e != nullptr ? e[0] == '1' : dflt) && p.trace == nullptr;
    const long items = (long)grid.x * grid.y;
    const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
    if (persist && items > sms) grid = dim3((unsigned)sms, 1u);
  }
  auto st = cur_stream();
#define FA2T(HD_, C_, P_, R_, X_, SP_, ...)                                    \
  {                                                                            \
    auto kern = fa2t::fa_fwd_pp_kernel<HD_, C_, P_, R_, X_, SP_, ##__VA_ARGS__>; \
    set_max_smem((const void*)kern, fa2t::Cfg<HD_>::SMEM);                     \
    kern<<<grid, fa2t::kThreads, fa2t::Cfg<HD_>::SMEM, st>>>(tq, tk, tv, p);   \
  }
#define FA2T_HD(P_, R_, X_, SP_)                                                       \
  if (HD == 64) {                                                                      \
    if (causal) FA2T(64, true, P_, R_, X_, SP_) else FA2T(64, false, P_, R_, X_, SP_)  \
  } else {                                                                             \
    if (causal) FA2T(128, true, P_, R_, X_, SP_) else FA2T(128, false, P_, R_, X_, SP_) \
  }
  const bool traced = p.trace != nullptr;
  TORCH_CHECK(!(traced && poly), "the trace is available for the plain variant");
  TORCH_CHECK(!(sparse && (traced || poly || bf2)), "sparse attention uses the packed-pair variant");
  TORCH_CHECK(!(bf2 && (traced || poly || x2)), "the bf16x2-exponential variant is exclusive");
  if (bf2) {
    if (HD == 64) {
      if (causal) FA2T(64, true, false, false, false, false, true) else FA2T(64, false, false, false, false, false, true)
    } else {
      if (causal) FA2T(128, true, false, false, false, false, true) else FA2T(128, false, false, false, false, false, true)
    }
  } else if (sparse) {
    FA2T_HD(false, false, true, true)
  } else if (traced) {
    if (x2) {
      FA2T_HD(false, true, true, false)
    } else {
      FA2T_HD(false, true, false, false)
    }
  } else if (poly) {
    // packed-pair variant with every second pair's exponentials on the FMA pipe
    FA2T_HD(true, false, true, false)
  } else if (x2) {
    FA2T_HD(false, false, true, false)
  } else {
    FA2T_HD(false, false, false, false)
  }
#undef FA2T_HD
#undef FA2T
  SCIRS_CHECK_LAUNCH();
}

}  // namespace scirs
