// FlashAttention-2 style fused attention, forward and backward, bf16 in /
// fp32 accumulation, head_dim 64 or 128, optional causal mask, any sequence
// length (out-of-range keys are masked, out-of-range queries not stored).
//
// Q, K, V and dO are read straight out of strided token-major buffers (for a
// GPT block: the fused QKV projection output [B*S, 3*H*HD]), so no
// transposes or head splits are materialised. Forward writes O [B*S, H*HD]
// and the natural-log row logsumexp LSE [B, H, S]; backward recomputes the
// probabilities from LSE.
//
// Tensor-core path: warp-level mma.sync m16n8k16 with ldmatrix from
// XOR-swizzled shared memory and a cp.async double-buffered K/V (forward) or
// Q/dO (backward) pipeline. dQ is accumulated across key blocks with fp32
// atomics and converted to bf16 by a small follow-up kernel.
//
// Reference parity: the reference computes this forward-only on the CPU
// (scirs2-neural/src/layers/flash_attention_v2.rs:220,369-482 and
// scirs2-neural/src/attention/flash_v2.rs:96-300, online softmax with
// Br=Bc=128 blocks); its backward is NotImplemented
// (flash_attention_v2.rs:484-491). The backward here is the standard one and
// is tested against a torch fp32 restatement.
#include "host_common.h"

namespace scirs {
namespace attn {

using bf16 = __nv_bfloat16;

struct Params {
  const bf16* q;
  const bf16* k;
  const bf16* v;
  const bf16* o;
  const bf16* dout;
  bf16* out;
  float* lse;  // [B, H, S], natural log
  float* delta;
  float* dq_acc;  // [B*S, H*HD] fp32
  bf16* dq;
  bf16* dk;
  bf16* dv;
  long q_rs, k_rs, v_rs, o_rs, do_rs, dq_rs, dk_rs, dv_rs;  // token row strides (elements)
  int B, H, S;
  float scale;       // softmax scale
  float scale_log2;  // scale * log2(e)
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(pred ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Byte offset of 16-byte chunk `c` of row `r` in a [rows x HD] bf16 tile with
// the chunk index XOR-swizzled by the row (conflict-free ldmatrix).
template <int HD>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)(r * HD * 2 + ((c ^ (r & 7)) << 4));
}

// Asynchronously copy rows [row0, row0+R) of a token-major matrix (HD
// columns, row stride rs) into a swizzled tile; rows >= S are zero-filled.
template <int R, int HD, int NT>
__device__ __forceinline__ void load_tile(uint32_t sdst, const bf16* g, long rs, int row0, int S) {
  constexpr int CPR = HD / 8;  // chunks per row
#pragma unroll
  for (int idx = threadIdx.x; idx < R * CPR; idx += NT) {
    const int r = idx / CPR, c = idx % CPR;
    const int row = row0 + r;
    const bool ok = row < S;
    const bf16* src = g + (long)(ok ? row : 0) * rs + c * 8;
    cp_async16(sdst + swz<HD>(r, c), src, ok);
  }
}

// ===========================================================================
// forward: CTA = 8 warps x 16 query rows (BM = 128), key blocks of BN = 64.
// ===========================================================================
template <int HD>
struct FwdCfg {
  static constexpr int BM = 128, BN = 64, NT = 256;
  static constexpr int Q_BYTES = BM * HD * 2, KV_BYTES = BN * HD * 2;
  static constexpr int SMEM = Q_BYTES + 4 * KV_BYTES;
};

template <int HD, bool CAUSAL>
__global__ void __launch_bounds__(256) fa_fwd_kernel(const Params p) {
  using C = FwdCfg<HD>;
  constexpr int BM = C::BM, BN = C::BN, KSTEPS = HD / 16, NTS = BN / 8, NTO = HD / 8;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + C::Q_BYTES;
  const uint32_t sV0 = sK0 + C::KV_BYTES;
  const uint32_t sK1 = sV0 + C::KV_BYTES;
  const uint32_t sV1 = sK1 + C::KV_BYTES;

  const int S = p.S, H = p.H;
  const int qb = gridDim.x - 1 - blockIdx.x;  // longest (causal) blocks first
  const int b = blockIdx.y / H, h = blockIdx.y % H;
  const int q0 = qb * BM;
  const bf16* qg = p.q + (long)b * S * p.q_rs + h * HD;
  const bf16* kg = p.k + (long)b * S * p.k_rs + h * HD;
  const bf16* vg = p.v + (long)b * S * p.v_rs + h * HD;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3, mat = lane >> 3, r8 = lane & 7;

  const int nkv_all = (S + BN - 1) / BN;
  const int nkv = CAUSAL ? min(nkv_all, (q0 + BM + BN - 1) / BN) : nkv_all;

  load_tile<BM, HD, 256>(sQ, qg, p.q_rs, q0, S);
  load_tile<BN, HD, 256>(sK0, kg, p.k_rs, 0, S);
  load_tile<BN, HD, 256>(sV0, vg, p.v_rs, 0, S);
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();

  uint32_t qf[KSTEPS][4];
#pragma unroll
  for (int kk = 0; kk < KSTEPS; ++kk) {
    const int row = warp * 16 + (mat & 1) * 8 + r8;
    ldsm_x4(sQ + swz<HD>(row, 2 * kk + (mat >> 1)), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
  }

  float o[NTO][4];
#pragma unroll
  for (int i = 0; i < NTO; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  const int row_a = q0 + warp * 16 + g, row_b = row_a + 8;

  for (int j = 0; j < nkv; ++j) {
    if (j + 1 < nkv) {
      const uint32_t nk = ((j + 1) & 1) ? sK1 : sK0, nv = ((j + 1) & 1) ? sV1 : sV0;
      load_tile<BN, HD, 256>(nk, kg, p.k_rs, (j + 1) * BN, S);
      load_tile<BN, HD, 256>(nv, vg, p.v_rs, (j + 1) * BN, S);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t sK = (j & 1) ? sK1 : sK0, sV = (j & 1) ? sV1 : sV0;
    const int kv0 = j * BN;

    float s[NTS][4];
#pragma unroll
    for (int i = 0; i < NTS; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
#pragma unroll
      for (int pp = 0; pp < BN / 16; ++pp) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sK + swz<HD>(pp * 16 + (mat >> 1) * 8 + r8, 2 * kk + (mat & 1)), b0, b1, b2, b3);
        mma16816(s[2 * pp], qf[kk], b0, b1);
        mma16816(s[2 * pp + 1], qf[kk], b2, b3);
      }
    }
    // scale, mask, online softmax
    const bool need_mask = (kv0 + BN > S) || (CAUSAL && kv0 + BN - 1 > q0 + warp * 16);
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < NTS; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float va = s[nt][e] * p.scale_log2, vb = s[nt][2 + e] * p.scale_log2;
        if (need_mask) {
          const int key = kv0 + nt * 8 + 2 * t + e;
          if (key >= S || (CAUSAL && key > row_a)) va = -INFINITY;
          if (key >= S || (CAUSAL && key > row_b)) vb = -INFINITY;
        }
        s[nt][e] = va;
        s[nt][2 + e] = vb;
        mx_a = fmaxf(mx_a, va);
        mx_b = fmaxf(mx_b, vb);
      }
    }
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    const float ref_a = (mn_a == -INFINITY) ? 0.f : mn_a, ref_b = (mn_b == -INFINITY) ? 0.f : mn_b;
    const float al_a = exp2f(m_a - ref_a), al_b = exp2f(m_b - ref_b);
    m_a = mn_a;
    m_b = mn_b;
    float rs_a = 0.f, rs_b = 0.f;
    uint32_t pa[BN / 16][4];
#pragma unroll
    for (int nt = 0; nt < NTS; ++nt) {
      const float p0 = exp2f(s[nt][0] - ref_a), p1 = exp2f(s[nt][1] - ref_a);
      const float p2 = exp2f(s[nt][2] - ref_b), p3 = exp2f(s[nt][3] - ref_b);
      rs_a += p0 + p1;
      rs_b += p2 + p3;
      pa[nt >> 1][(nt & 1) * 2 + 0] = pack_bf16x2(p0, p1);
      pa[nt >> 1][(nt & 1) * 2 + 1] = pack_bf16x2(p2, p3);
    }
    l_a = l_a * al_a + rs_a;
    l_b = l_b * al_b + rs_b;
#pragma unroll
    for (int i = 0; i < NTO; ++i) {
      o[i][0] *= al_a;
      o[i][1] *= al_a;
      o[i][2] *= al_b;
      o[i][3] *= al_b;
    }
    // O += P V
#pragma unroll
    for (int js = 0; js < BN / 16; ++js) {
#pragma unroll
      for (int qq = 0; qq < HD / 16; ++qq) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(sV + swz<HD>(js * 16 + (mat & 1) * 8 + r8, 2 * qq + (mat >> 1)), b0, b1, b2, b3);
        mma16816(o[2 * qq], pa[js], b0, b1);
        mma16816(o[2 * qq + 1], pa[js], b2, b3);
      }
    }
    __syncthreads();
  }

  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  const float inv_a = l_a > 0.f ? 1.f / l_a : 0.f, inv_b = l_b > 0.f ? 1.f / l_b : 0.f;
  bf16* og = p.out + (long)b * S * p.o_rs + h * HD;
#pragma unroll
  for (int nt = 0; nt < NTO; ++nt) {
    const int col = nt * 8 + 2 * t;
    if (row_a < S)
      *reinterpret_cast<uint32_t*>(og + (long)row_a * p.o_rs + col) = pack_bf16x2(o[nt][0] * inv_a, o[nt][1] * inv_a);
    if (row_b < S)
      *reinterpret_cast<uint32_t*>(og + (long)row_b * p.o_rs + col) = pack_bf16x2(o[nt][2] * inv_b, o[nt][3] * inv_b);
  }
  if (t == 0) {
    const float ln2 = 0.6931471805599453f;
    float* lse = p.lse + ((long)b * H + h) * S;
    if (row_a < S) lse[row_a] = (m_a + log2f(l_a)) * ln2;
    if (row_b < S) lse[row_b] = (m_b + log2f(l_b)) * ln2;
  }
}

// delta[b, h, s] = sum_d dO[s, h, d] * O[s, h, d]; HD/8 lanes per (token,
// head), 16-byte loads, shuffle reduction within the lane group.
template <int HD>
__global__ void fa_bwd_delta_kernel(const Params p) {
  constexpr int G = HD / 8;  // lanes per (token, head): 8 or 16
  const long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const long idx = gid / G;  // (b*S + s)*H + h
  const int sub = (int)(gid % G);
  const long total = (long)p.B * p.S * p.H;
  const bool ok = idx < total;
  float acc = 0.f;
  long tok = 0;
  int h = 0;
  if (ok) {
    h = (int)(idx % p.H);
    tok = idx / p.H;
    const uint4 ov = *reinterpret_cast<const uint4*>(p.o + tok * p.o_rs + h * HD + sub * 8);
    const uint4 dv = *reinterpret_cast<const uint4*>(p.dout + tok * p.do_rs + h * HD + sub * 8);
    const uint32_t oa[4] = {ov.x, ov.y, ov.z, ov.w}, da[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) acc += bf16_lo(oa[e]) * bf16_lo(da[e]) + bf16_hi(oa[e]) * bf16_hi(da[e]);
    // zero this (token, head)'s slice of the fp32 dQ accumulator [B*S, H*HD]
    // that the backward kernels reduce-add into
    float4* z = reinterpret_cast<float4*>(p.dq_acc + tok * ((long)p.H * HD) + h * HD + sub * 8);
    z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (ok && sub == 0) {
    const int b = (int)(tok / p.S), s = (int)(tok % p.S);
    p.delta[((long)b * p.H + h) * p.S + s] = acc;
  }
}

// ===========================================================================
// backward: CTA = 4 warps x 16 keys (BN = 64), query blocks of BM = 64.
// ===========================================================================
template <int HD>
struct BwdCfg {
  static constexpr int BN = 64, BM = 64, NT = 128;
  static constexpr int T_BYTES = 64 * HD * 2;  // one 64-row tile
  static constexpr int DS_BYTES = 64 * 64 * 2;
  static constexpr int SMEM = 6 * T_BYTES + DS_BYTES + 4 * 64 * 4;
};

template <int HD, bool CAUSAL>
__global__ void __launch_bounds__(128) fa_bwd_kernel(const Params p) {
  using C = BwdCfg<HD>;
  constexpr int BN = C::BN, BM = C::BM, KSTEPS = HD / 16, NTO = HD / 8;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + C::T_BYTES;
  const uint32_t sQb[2] = {sV + C::T_BYTES, sV + 2 * C::T_BYTES};
  const uint32_t sdOb[2] = {sV + 3 * C::T_BYTES, sV + 4 * C::T_BYTES};
  const uint32_t sdS = sV + 5 * C::T_BYTES;
  float* sLse = reinterpret_cast<float*>(smem + 6 * C::T_BYTES + C::DS_BYTES);  // [2][64]
  float* sDel = sLse + 128;                                                     // [2][64]

  const int S = p.S, H = p.H;
  const int kb = blockIdx.x;
  const int b = blockIdx.y / H, h = blockIdx.y % H;
  const int kv0 = kb * BN;
  const long tok0 = (long)b * S;
  const bf16* qg = p.q + tok0 * p.q_rs + h * HD;
  const bf16* kg = p.k + tok0 * p.k_rs + h * HD;
  const bf16* vg = p.v + tok0 * p.v_rs + h * HD;
  const bf16* dog = p.dout + tok0 * p.do_rs + h * HD;
  const float* lse_g = p.lse + ((long)b * H + h) * S;
  const float* del_g = p.delta + ((long)b * H + h) * S;
  float* dqa = p.dq_acc + tok0 * (long)H * HD + h * HD;
  const long dqa_rs = (long)H * HD;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3, mat = lane >> 3, r8 = lane & 7;
  const float LOG2E = 1.4426950408889634f;

  const int nq = (S + BM - 1) / BM;
  const int i0 = CAUSAL ? (kv0 / BM) : 0;

  auto load_q_block = [&](int i, int buf) {
    load_tile<BM, HD, 128>(sQb[buf], qg, p.q_rs, i * BM, S);
    load_tile<BM, HD, 128>(sdOb[buf], dog, p.do_rs, i * BM, S);
    if (threadIdx.x < 64) {
      const int q = i * BM + threadIdx.x;
      sLse[buf * 64 + threadIdx.x] = q < S ? lse_g[q] * LOG2E : 0.f;
      sDel[buf * 64 + threadIdx.x] = q < S ? del_g[q] : 0.f;
    }
  };

  load_tile<BN, HD, 128>(sK, kg, p.k_rs, kv0, S);
  load_tile<BN, HD, 128>(sV, vg, p.v_rs, kv0, S);
  if (i0 < nq) load_q_block(i0, 0);
  cp_async_commit();

  float dk[NTO][4], dv[NTO][4];
#pragma unroll
  for (int i = 0; i < NTO; ++i) {
    dk[i][0] = dk[i][1] = dk[i][2] = dk[i][3] = 0.f;
    dv[i][0] = dv[i][1] = dv[i][2] = dv[i][3] = 0.f;
  }
  const int key_a = kv0 + warp * 16 + g, key_b = key_a + 8;

  for (int i = i0; i < nq; ++i) {
    const int buf = (i - i0) & 1;
    if (i + 1 < nq) {
      load_q_block(i + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const uint32_t sQ = sQb[buf], sdO = sdOb[buf];
    const float* lse = sLse + buf * 64;
    const float* del = sDel + buf * 64;
    const int q0 = i * BM;

    // S^T = K Q^T and dP^T = V dO^T  (16 keys x 64 queries per warp)
    float st[8][4], dpt[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      st[n][0] = st[n][1] = st[n][2] = st[n][3] = 0.f;
      dpt[n][0] = dpt[n][1] = dpt[n][2] = dpt[n][3] = 0.f;
    }
#pragma unroll
    for (int kk = 0; kk < KSTEPS; ++kk) {
      uint32_t ka[4], va[4];
      const int row = warp * 16 + (mat & 1) * 8 + r8;
      ldsm_x4(sK + swz<HD>(row, 2 * kk + (mat >> 1)), ka[0], ka[1], ka[2], ka[3]);
      ldsm_x4(sV + swz<HD>(row, 2 * kk + (mat >> 1)), va[0], va[1], va[2], va[3]);
#pragma unroll
      for (int pp = 0; pp < BM / 16; ++pp) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sQ + swz<HD>(pp * 16 + (mat >> 1) * 8 + r8, 2 * kk + (mat & 1)), b0, b1, b2, b3);
        mma16816(st[2 * pp], ka, b0, b1);
        mma16816(st[2 * pp + 1], ka, b2, b3);
        ldsm_x4(sdO + swz<HD>(pp * 16 + (mat >> 1) * 8 + r8, 2 * kk + (mat & 1)), b0, b1, b2, b3);
        mma16816(dpt[2 * pp], va, b0, b1);
        mma16816(dpt[2 * pp + 1], va, b2, b3);
      }
    }
    // P^T and dS^T
    uint32_t pT[4][4], dsT[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float pv[4], dsv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ql = nt * 8 + 2 * t + (e & 1);
        const int q = q0 + ql;
        const int key = (e < 2) ? key_a : key_b;
        const bool masked = (q >= S) || (key >= S) || (CAUSAL && key > q);
        const float pr = masked ? 0.f : exp2f(st[nt][e] * p.scale_log2 - lse[ql]);
        pv[e] = pr;
        dsv[e] = pr * (dpt[nt][e] - del[ql]);
      }
      pT[nt >> 1][(nt & 1) * 2 + 0] = pack_bf16x2(pv[0], pv[1]);
      pT[nt >> 1][(nt & 1) * 2 + 1] = pack_bf16x2(pv[2], pv[3]);
      dsT[nt >> 1][(nt & 1) * 2 + 0] = pack_bf16x2(dsv[0], dsv[1]);
      dsT[nt >> 1][(nt & 1) * 2 + 1] = pack_bf16x2(dsv[2], dsv[3]);
      // dS^T tile to shared memory ([key][q], swizzled 64-wide rows)
      const int kr = warp * 16 + g;
      const int qc = nt * 8 + 2 * t;
      const uint32_t off_a = (uint32_t)(kr * 128 + ((((qc >> 3) ^ (kr & 7))) << 4) + (qc & 7) * 2);
      const uint32_t off_b = (uint32_t)((kr + 8) * 128 + ((((qc >> 3) ^ ((kr + 8) & 7))) << 4) + (qc & 7) * 2);
      asm volatile("st.shared.b32 [%0], %1;" ::"r"(sdS + off_a), "r"(dsT[nt >> 1][(nt & 1) * 2 + 0]));
      asm volatile("st.shared.b32 [%0], %1;" ::"r"(sdS + off_b), "r"(dsT[nt >> 1][(nt & 1) * 2 + 1]));
    }
    // dV += P^T dO ; dK += dS^T Q   (B operands: trans ldmatrix of dO / Q)
#pragma unroll
    for (int js = 0; js < BM / 16; ++js) {
#pragma unroll
      for (int qq = 0; qq < HD / 16; ++qq) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(sdO + swz<HD>(js * 16 + (mat & 1) * 8 + r8, 2 * qq + (mat >> 1)), b0, b1, b2, b3);
        mma16816(dv[2 * qq], pT[js], b0, b1);
        mma16816(dv[2 * qq + 1], pT[js], b2, b3);
        ldsm_x4_t(sQ + swz<HD>(js * 16 + (mat & 1) * 8 + r8, 2 * qq + (mat >> 1)), b0, b1, b2, b3);
        mma16816(dk[2 * qq], dsT[js], b0, b1);
        mma16816(dk[2 * qq + 1], dsT[js], b2, b3);
      }
    }
    __syncthreads();
    // dQ[q rows of this warp] += dS K, accumulated with fp32 atomics.
    {
      float dq[NTO][4];
#pragma unroll
      for (int n = 0; n < NTO; ++n) dq[n][0] = dq[n][1] = dq[n][2] = dq[n][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < BN / 16; ++ks) {
        uint32_t a[4];
        {
          const int kr = ks * 16 + (mat >> 1) * 8 + r8;
          const int ch = 2 * warp + (mat & 1);
          ldsm_x4_t(sdS + (uint32_t)(kr * 128 + ((ch ^ (kr & 7)) << 4)), a[0], a[1], a[2], a[3]);
        }
#pragma unroll
        for (int qq = 0; qq < HD / 16; ++qq) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(sK + swz<HD>(ks * 16 + (mat & 1) * 8 + r8, 2 * qq + (mat >> 1)), b0, b1, b2, b3);
          mma16816(dq[2 * qq], a, b0, b1);
          mma16816(dq[2 * qq + 1], a, b2, b3);
        }
      }
      const int qa = q0 + warp * 16 + g, qb2 = qa + 8;
#pragma unroll
      for (int nt = 0; nt < NTO; ++nt) {
        const int col = nt * 8 + 2 * t;
        if (qa < S) atomicAdd(reinterpret_cast<float2*>(dqa + (long)qa * dqa_rs + col), make_float2(dq[nt][0], dq[nt][1]));
        if (qb2 < S)
          atomicAdd(reinterpret_cast<float2*>(dqa + (long)qb2 * dqa_rs + col), make_float2(dq[nt][2], dq[nt][3]));
      }
    }
    __syncthreads();
  }
  // write dK (scaled) and dV
  bf16* dkg = p.dk + tok0 * p.dk_rs + h * HD;
  bf16* dvg = p.dv + tok0 * p.dv_rs + h * HD;
#pragma unroll
  for (int nt = 0; nt < NTO; ++nt) {
    const int col = nt * 8 + 2 * t;
    if (key_a < S) {
      *reinterpret_cast<uint32_t*>(dkg + (long)key_a * p.dk_rs + col) = pack_bf16x2(dk[nt][0] * p.scale, dk[nt][1] * p.scale);
      *reinterpret_cast<uint32_t*>(dvg + (long)key_a * p.dv_rs + col) = pack_bf16x2(dv[nt][0], dv[nt][1]);
    }
    if (key_b < S) {
      *reinterpret_cast<uint32_t*>(dkg + (long)key_b * p.dk_rs + col) = pack_bf16x2(dk[nt][2] * p.scale, dk[nt][3] * p.scale);
      *reinterpret_cast<uint32_t*>(dvg + (long)key_b * p.dv_rs + col) = pack_bf16x2(dv[nt][2], dv[nt][3]);
    }
  }
}

// dq[tok, h*HD + d] = dq_acc[tok, h*HD + d] * scale  (bf16, strided output)
__global__ void fa_dq_convert_kernel(const float* __restrict__ acc, bf16* __restrict__ dq, long dq_rs, long ntok,
                                     int width, float scale) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;  // index of a 4-element group
  const long n4 = ntok * width / 4;
  if (i >= n4) return;
  const long e = i * 4;
  const long tok = e / width;
  const int c = (int)(e % width);
  const float4 v = reinterpret_cast<const float4*>(acc)[i];
  uint2 o;
  o.x = pack_bf16x2(v.x * scale, v.y * scale);
  o.y = pack_bf16x2(v.z * scale, v.w * scale);
  *reinterpret_cast<uint2*>(dq + tok * dq_rs + c) = o;
}

}  // namespace attn

static void check_qkv_view(const torch::Tensor& t, const char* name, int64_t B, int64_t S, int64_t H, int64_t HD) {
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, " must be bf16");
  TORCH_CHECK(t.dim() == 4 && t.size(0) == B && t.size(1) == S && t.size(2) == H && t.size(3) == HD, name,
              " must be [B, S, H, HD]");
  TORCH_CHECK(t.stride(3) == 1 && t.stride(2) == HD, name, " must have contiguous heads");
  TORCH_CHECK(t.stride(0) == S * t.stride(1), name, " must be token-major");
  TORCH_CHECK(t.stride(1) % 8 == 0, name, " token stride must be a multiple of 8");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, name, " must be 16-byte aligned");
}

// q/k/v/out: [B, S, H, HD] views (token-major, heads contiguous); lse fp32 [B, H, S].
void flash_attn_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out, torch::Tensor lse,
                    bool causal, double scale) {
  const int64_t B = q.size(0), S = q.size(1), H = q.size(2), HD = q.size(3);
  check_qkv_view(q, "q", B, S, H, HD);
  check_qkv_view(k, "k", B, S, H, HD);
  check_qkv_view(v, "v", B, S, H, HD);
  check_qkv_view(out, "out", B, S, H, HD);
  TORCH_CHECK(HD == 64 || HD == 128, "head_dim must be 64 or 128");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.numel() == B * H * S && lse.is_contiguous(), "lse [B,H,S] fp32");
  c10::cuda::CUDAGuard guard(q.get_device());
  attn::Params p{};
  p.q = (const attn::bf16*)q.data_ptr();
  p.k = (const attn::bf16*)k.data_ptr();
  p.v = (const attn::bf16*)v.data_ptr();
  p.out = (attn::bf16*)out.data_ptr();
  p.lse = lse.data_ptr<float>();
  p.q_rs = q.stride(1);
  p.k_rs = k.stride(1);
  p.v_rs = v.stride(1);
  p.o_rs = out.stride(1);
  p.B = (int)B;
  p.H = (int)H;
  p.S = (int)S;
  p.scale = (float)scale;
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  dim3 grid((unsigned)((S + 127) / 128), (unsigned)(B * H));
  auto st = cur_stream();
#define FA_FWD(HD_, CAUSAL_)                                                                             \
  {                                                                                                      \
    auto kern = attn::fa_fwd_kernel<HD_, CAUSAL_>;                                                       \
    set_max_smem((const void*)kern, attn::FwdCfg<HD_>::SMEM);                                     \
    kern<<<grid, 256, attn::FwdCfg<HD_>::SMEM, st>>>(p);                                                 \
  }
  if (HD == 64) {
    if (causal) FA_FWD(64, true) else FA_FWD(64, false)
  } else {
    if (causal) FA_FWD(128, true) else FA_FWD(128, false)
  }
#undef FA_FWD
  SCIRS_CHECK_LAUNCH();
}

// dq/dk/dv: [B, S, H, HD] bf16 views; dq_acc fp32 scratch [B*S*H*HD] (zeroed
// here); delta fp32 scratch [B*H*S].
void flash_attn_bwd_tc(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor lse,
                       torch::Tensor delta, torch::Tensor dk, torch::Tensor dv, torch::Tensor dq_acc, bool causal,
                       double scale, const AttnSparse& sp, int schedule);

// impl: 0 = warp-level mma.sync kernel, 1 = tcgen05 kernels (serial schedule),
// 2 = tcgen05 kernels with the pipelined schedule, 3 = pipelined and, for head_dim 64
// without a sparsity pattern, persistent (one CTA per SM), 4 = 3 up to 1,024 keys, else 2.
void flash_attn_bwd_h128(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor lse,
                         torch::Tensor delta, torch::Tensor dk, torch::Tensor dv, torch::Tensor dq_acc, bool causal,
                         double scale, const AttnSparse& sp, bool pipelined);

// Sk = k.size(1) may differ from S (cross-attention; tcgen05 kernels only).
// Optional block lists (per 128-key tile: the query blocks that see it, in
// units of 128 queries for head_dim 64 and 64 for head_dim 128) and the
// element predicate select the sparse kernels.
void flash_attn_bwd(torch::Tensor dout, torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor out,
                    torch::Tensor lse, torch::Tensor dq, torch::Tensor dk, torch::Tensor dv, torch::Tensor dq_acc,
                    torch::Tensor delta, bool causal, double scale, int64_t impl,
                    c10::optional<torch::Tensor> blk_ptr, c10::optional<torch::Tensor> blk_idx,
                    c10::optional<torch::Tensor> bmap, int64_t wl, int64_t wr, int64_t ng) {
  const int64_t B = q.size(0), S = q.size(1), H = q.size(2), HD = q.size(3);
  const int64_t Sk = k.size(1);
  check_qkv_view(q, "q", B, S, H, HD);
  check_qkv_view(k, "k", B, Sk, H, HD);
  check_qkv_view(v, "v", B, Sk, H, HD);
  check_qkv_view(out, "out", B, S, H, HD);
  check_qkv_view(dout, "dout", B, S, H, HD);
  check_qkv_view(dq, "dq", B, S, H, HD);
  check_qkv_view(dk, "dk", B, Sk, H, HD);
  check_qkv_view(dv, "dv", B, Sk, H, HD);
  TORCH_CHECK(!causal || Sk == S, "causal attention needs equal query and key lengths");
  const AttnSparse sp = attn_sparse_args(blk_ptr, blk_idx, bmap, wl, wr, ng, (Sk + 127) / 128);
  const bool sparse = sp.ptr != nullptr || sp.bmap != nullptr || sp.wl >= 0 || sp.ng > 0;
  TORCH_CHECK(!sparse || sp.ptr != nullptr, "a sparsity predicate needs block lists");
  TORCH_CHECK(impl >= 1 || (!sparse && Sk == S), "sparse and cross attention need the tcgen05 kernels");
  TORCH_CHECK(HD == 64 || HD == 128, "head_dim must be 64 or 128");
  TORCH_CHECK(dq_acc.scalar_type() == at::kFloat && dq_acc.numel() >= B * S * H * HD, "dq_acc too small");
  TORCH_CHECK(delta.scalar_type() == at::kFloat && delta.numel() >= B * H * S, "delta too small");
  c10::cuda::CUDAGuard guard(q.get_device());
  auto st = cur_stream();
  attn::Params p{};
  p.q = (const attn::bf16*)q.data_ptr();
  p.k = (const attn::bf16*)k.data_ptr();
  p.v = (const attn::bf16*)v.data_ptr();
  p.o = (const attn::bf16*)out.data_ptr();
  p.dout = (const attn::bf16*)dout.data_ptr();
  p.lse = lse.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.dq_acc = dq_acc.data_ptr<float>();
  p.dq = (attn::bf16*)dq.data_ptr();
  p.dk = (attn::bf16*)dk.data_ptr();
  p.dv = (attn::bf16*)dv.data_ptr();
  p.q_rs = q.stride(1);
  p.k_rs = k.stride(1);
  p.v_rs = v.stride(1);
  p.o_rs = out.stride(1);
  p.do_rs = dout.stride(1);
  p.dq_rs = dq.stride(1);
  p.dk_rs = dk.stride(1);
  p.dv_rs = dv.stride(1);
  p.B = (int)B;
  p.H = (int)H;
  p.S = (int)S;
  p.scale = (float)scale;
  p.scale_log2 = (float)(scale * 1.4426950408889634);
  {
    // delta = rowsum(O * dO), and the dQ accumulator zeroed in the same pass
    const long rows = B * S * H;  // one 8-lane group per (token, head), 16-byte loads
    if (HD == 64) attn::fa_bwd_delta_kernel<64><<<(unsigned)((rows * 8 + 255) / 256), 256, 0, st>>>(p);
    else attn::fa_bwd_delta_kernel<128><<<(unsigned)((rows * 16 + 255) / 256), 256, 0, st>>>(p);
    SCIRS_CHECK_LAUNCH();
  }
  if (impl >= 1 && HD == 64) {
    // auto (4): persistent up to 1,024 keys (measured faster there), pipelined above
    const int sched = impl == 4 ? (Sk <= 1024 ? 2 : 1) : (int)impl - 1;
    flash_attn_bwd_tc(dout, q, k, v, lse, delta, dk, dv, dq_acc, causal, scale, sp, sched);
  } else if (impl >= 1 && HD == 128) {
    flash_attn_bwd_h128(dout, q, k, v, lse, delta, dk, dv, dq_acc, causal, scale, sp, impl >= 2);
  } else {
  dim3 grid((unsigned)((S + 63) / 64), (unsigned)(B * H));
#define FA_BWD(HD_, CAUSAL_)                                                                             \
  {                                                                                                      \
    auto kern = attn::fa_bwd_kernel<HD_, CAUSAL_>;                                                       \
    set_max_smem((const void*)kern, attn::BwdCfg<HD_>::SMEM);                                     \
    kern<<<grid, 128, attn::BwdCfg<HD_>::SMEM, st>>>(p);                                                 \
  }
  if (HD == 64) {
    if (causal) FA_BWD(64, true) else FA_BWD(64, false)
  } else {
    if (causal) FA_BWD(128, true) else FA_BWD(128, false)
  }
#undef FA_BWD
  SCIRS_CHECK_LAUNCH();
  }
  {
    const long n4 = B * S * H * HD / 4;
    attn::fa_dq_convert_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(p.dq_acc, p.dq, p.dq_rs, B * S,
                                                                              (int)(H * HD), 1.0f * (float)scale);
    SCIRS_CHECK_LAUNCH();
  }
}

}  // namespace scirs
