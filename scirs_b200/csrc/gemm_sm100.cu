// Persistent bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
//   C[M,N] = op(A) * op(B)  with fp32 accumulation in TMEM and a fused epilogue.
//
// Operand forms (row-major storage, "major" = which dimension is contiguous):
//   A K-major : a is [M, K]           A MN-major : a is [K, M]
//   B K-major : b is [N, K] (C=A b^T) B MN-major : b is [K, N] (C=A b)
// so one kernel family serves a Linear layer's forward (x W^T), data
// gradient (dY W) and weight gradient (dY^T X) without transposes.
//
// CTA layout (320 threads, one CTA per SM, persistent over output tiles):
//   warp 0      : TMA producer (one thread), fills a STAGES-deep smem ring
//   warp 1      : owns TMEM; one elected thread issues tcgen05.mma
//   warps 2..9  : epilogue; tcgen05.ld from TMEM -> fused math -> global
//                 (warp w reads TMEM lane quarter w%4; warps 2-5 take the
//                 left half of the tile's columns, warps 6-9 the right half)
// The accumulator is double-buffered in TMEM (2 x BN fp32 columns), so the
// epilogue of tile i overlaps the MMAs of tile i+1.
//
// Pair mode (PAIR = true, BN = 256): two CTAs of a cluster compute one
// 256 x 256 tile with tcgen05.mma.cta_group::2. Each CTA loads its own 128
// rows of A and its own 128 of the 256 columns of B (so each SM moves 32 KB
// per 64-deep k-block instead of 48 KB: the single-CTA kernel is bound by
// L2->SM bandwidth), both CTAs' TMA loads complete on the leader CTA's
// full barrier (cp.async.bulk.tensor .cta_group::2, no multicast), the leader
// alone issues the MMAs, and its commits arrive on both CTAs' empty / tfull
// barriers (tcgen05.commit .multicast::cluster). Each CTA's TMEM holds its
// 128 rows x 256 columns; the epilogue is unchanged, and both CTAs'
// epilogue warps release the accumulator on the leader's tempty barrier.
//
// Reference parity: replaces the SIMT / WMMA GEMMs of the reference
// (scirs2-core/src/gpu/kernels/gemm_f32.cu:4, scirs2-core/src/gpu/tensor_cores.rs:636,
// scirs2-linalg/kernels/matmul_f32.cu:159) and the Dense layer's forward and
// backward products (scirs2-neural/src/layers/dense.rs:174-212, :302-400).
#include "host_common.h"

namespace scirs {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2..9 epilogue
constexpr int kEpiWarps = 8;
constexpr int kMaxPeers = 8;
constexpr unsigned kSigStride = 4096;  // signals per step (flag values are epoch * kSigStride + idx)

enum Epi : int {
  EPI_BF16 = 0,       // C = acc (+ bias)
  EPI_BIAS_GELU = 1,  // C2 = acc + bias (pre-activation), C = gelu(C2)
  EPI_RESID = 2,      // C = acc (+ bias) + aux
  EPI_DGELU = 3,      // C = acc * gelu'(aux)
  EPI_F32 = 4,        // C(fp32) = acc, or += acc (atomic) when accumulating / split-K
  EPI_ROPE = 5,       // C = rope(acc + bias) on the first rope_cols columns, acc + bias after
};

struct Args {
  int M, N, K;
  int num_kb;
  int splits;
  int kb_per_split;
  int m_blocks, n_blocks;
  int num_units;
  int group_m;
  void* C;
  long ldc;
  void* C2;
  long ldc2;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* aux;
  long ldaux;
  float* bias_grad;  // EPI_DGELU: += column sums of the output (fp32 [N])
  int atomic_out;
  int gelu_x2;  // EPI_BIAS_GELU / EPI_DGELU: GELU and its derivative in packed f32x2 instructions
  // EPI_ROPE: rotary embedding of the q and k parts of a fused [rows, 3, H, hd]
  // output (columns [0, rope_cols) = q and k heads), half-rotation form
  //   x[d]        -> x[d] cos(pos w_d) - x[d + hd/2] sin(pos w_d)
  //   x[d + hd/2] -> x[d + hd/2] cos(pos w_d) + x[d] sin(pos w_d),  d < hd/2,
  // pos = row % rope_S; tables fp32 [rope_S, hd/2]
  const float* rope_cos;
  const float* rope_sin;
  int rope_S, rope_hd, rope_cols;
  DevStatus* st;
  int m_rot;   // rotation of the m-block order (tensor parallel: start with local rows)
  int kb_rot;  // rotation of the k-block order (tensor parallel: start with local K rows)
  // ---- tensor-parallel extensions (gemm_tp_kernel only) ----
  int rank, world;
  int a_seg, b_seg;            // >0: the operand's split dimension (A: M rows if K-major, K rows if
                               // MN-major; B: K rows, MN-major) is split over the ranks in segments of
                               // this many elements, rank r's segment read through peer map r
  const unsigned* wait_flags;  // [world] local flag words written by the peers
  const unsigned* epoch_ptr;   // device step counter; flag value = epoch * kSigStride + idx
  unsigned wait_idx;
  long long timeout_ns;
  __nv_bfloat16* rs_dst[kMaxPeers];  // GEMM->RS: owner r's receive slot for this rank's partial
  int rs_seg;                        // output rows per owner (0: plain output)
  long rs_ld;
  unsigned* sig_flags[kMaxPeers];    // flag words [peer r][this rank] set when the kernel is done
  unsigned sig_idx;
  unsigned* done_ctr;                // local counter for the last-CTA signal
};

struct PeerMaps {
  CUtensorMap a[kMaxPeers];
  CUtensorMap b[kMaxPeers];
};

template <int BN, bool PAIR = false>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = (PAIR ? BN / 2 : BN) * BK * 2;  // pair: this CTA's half of B
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = PAIR ? 6 : ((BN == 256) ? 4 : 6);
  static constexpr int TMEM_COLS = 2 * BN;
  // Epilogue staging: per epilogue warp two 2 KB slots (32 rows x 64 bytes,
  // 64-byte swizzle) that feed TMA stores / reduce-adds.
  static constexpr int SLOT_BYTES = 2048;
  static constexpr int STAGING_OFF = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = STAGING_OFF + kEpiWarps * 2 * SLOT_BYTES;
  static constexpr int SMEM = BAR_OFF + 256 /*barriers*/ + 1024 /*align*/;
};

// Write 16 bytes `v` as 16-byte unit `u` (0..3) of row `r` of a 32x64B slot
// with the TMA 64-byte swizzle (unit index XOR (row/2)%4; slot 512B-aligned).
__device__ __forceinline__ void slot_st16(uint8_t* slot, int r, int u, uint4 v) {
  *reinterpret_cast<uint4*>(slot + r * 64 + ((u ^ ((r >> 1) & 3)) << 4)) = v;
}

__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* smem_src, int c0, int c1) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   map),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}

__device__ __forceinline__ void decode_unit(const Args& a, int u, int& m_blk, int& n_blk, int& split) {
  split = u % a.splits;
  int t = u / a.splits;
  // grouped rasterisation: G m-blocks x all n-blocks per group, m fastest
  int per_group = a.group_m * a.n_blocks;
  int g = t / per_group;
  int first_m = g * a.group_m;
  int gsize = min(a.group_m, a.m_blocks - first_m);
  int r = t % per_group;
  m_blk = first_m + r % gsize;
  n_blk = r / gsize;
  if (a.m_rot) m_blk = (m_blk + a.m_rot) % a.m_blocks;
}

__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys_u32(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// ---- cluster-pair helpers (PAIR mode) ----
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of `p` (a local shared variable) in CTA `rank`
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA load into this CTA's smem whose completion is counted on the leader's
// barrier (`bar_cluster`, a shared::cluster address). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster, int c0,
                                                 int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(map), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tc_mma_f16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                   uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// commit the leader's MMAs to the barrier at the same offset in both CTAs
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::
                   "r"(smem_u32(bar)),
               "h"((uint16_t)3)
               : "memory");
}
__device__ __forceinline__ void tc_commit_pair_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Wait (bounded) until peer r's flag reaches this kernel's expected value;
// afterwards the peer's data may be read, also by TMA (async proxy).
__device__ __forceinline__ bool wait_peer(const Args& a, int r, volatile int* abort_flag) {
  const unsigned want = *a.epoch_ptr * kSigStride + a.wait_idx;
  const unsigned* f = a.wait_flags + r;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while ((int)(ld_acquire_sys_u32(f) - want) < 0) {
    if ((++spins & 255u) == 0) {
      if (*abort_flag) return false;
      if ((long long)(globaltimer_ns() - t0) > a.timeout_ns) {
        report_status(a.st, kStPeerTimeout, 60, (unsigned)r);
        *abort_flag = 1;
        return false;
      }
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

// Tensor map and coordinate for a tile of an operand whose split dimension
// may live on the peers (coordinate `c` along that dimension is rewritten to
// the owner's local coordinate).
template <bool PEER>
__device__ __forceinline__ const CUtensorMap* pick_map(const CUtensorMap* local, const CUtensorMap* peers, int seg,
                                                        int& c, const Args& a, uint32_t& ready, bool& ok,
                                                        volatile int* abort_flag) {
  if (!PEER || seg == 0) return local;
  const int r = c / seg;
  c -= r * seg;
  if (r != a.rank && a.wait_flags != nullptr && !(ready & (1u << r))) {
    if (!wait_peer(a, r, abort_flag)) ok = false;
    ready |= 1u << r;
  }
  return peers + r;
}

template <int BN, int A_MN, int B_MN, int EPI, bool PEER, bool PAIR = false>
__device__ __forceinline__ void gemm_body(const CUtensorMap* pA, const CUtensorMap* pB, const CUtensorMap* pC,
                                          const CUtensorMap* pC2, const PeerMaps* pm, const Args& args) {
  static_assert(!PAIR || (BN == 256 && !PEER), "pair mode: BN 256, local operands");
  using C = Cfg<BN, PAIR>;
  const CUtensorMap& tmA = *pA;
  const CUtensorMap& tmB = *pB;
  const CUtensorMap& tmC = *pC;
  const CUtensorMap& tmC2 = *pC2;
  constexpr int STAGES = C::STAGES;
  constexpr uint32_t IDESC = umma_idesc_bf16(PAIR ? 2 * BM : BM, BN, A_MN, B_MN);
  // pair mode: CTA rank in the pair, the units are walked per cluster
  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = crank == 0;
  const int unit0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int ustep = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int row_sub = PAIR ? (int)crank * BM : 0;  // this CTA's rows within the unit's 256
  constexpr int MT = PAIR ? 2 * BM : BM;            // rows per unit

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* aux_bar = drain + 1;  // [kEpiWarps]: TMA loads of the epilogue's aux operand
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(aux_bar + kEpiWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], PAIR ? 2 * kEpiWarps : kEpiWarps);
    }
    mbar_init(drain, 1);
    for (int w = 0; w < kEpiWarps; ++w) mbar_init(&aux_bar[w], 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmC);
    if (EPI == EPI_BIAS_GELU || EPI == EPI_RESID || EPI == EPI_DGELU) prefetch_tmap(&tmC2);
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(tmem_holder, C::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_holder, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if (PAIR)
    cluster_sync_all();  // both CTAs' barriers exist before any remote arrive / TMA completion
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      uint32_t ready = 0;  // peers whose data is known to be ready
      const uint32_t full_leader0 = PAIR ? mapa_shared(&full[0], 0) : 0u;
      for (int u = unit0; u < args.num_units && ok; u += ustep) {
        int m_blk, n_blk, split;
        decode_unit(args, u, m_blk, n_blk, split);
        const int kb0 = split * args.kb_per_split;
        const int kb1 = min(args.num_kb, kb0 + args.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, args.st, 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sA = smem + s * C::STAGE_BYTES;
          uint8_t* sB = sA + C::A_BYTES;
          const int kbp = args.kb_rot ? (kb + args.kb_rot) % args.num_kb : kb;
          // split coordinates (rewritten to the owner's local coordinate for peer operands)
          if (PAIR) {
            // this CTA's 128 rows of A and 128 columns of B; completion on the leader's barrier
            const uint32_t fb = full_leader0 + s * 8;
            const int arow = m_blk * MT + row_sub;
            const int bcol = n_blk * BN + (int)crank * (BN / 2);
            if (leader) mbar_arrive_expect_tx(&full[s], 2 * C::STAGE_BYTES);
            if (A_MN) {
              tma_load_2d_pair(sA, &tmA, fb, arow, kbp * BK);
              tma_load_2d_pair(sA + 8192, &tmA, fb, arow + 64, kbp * BK);
            } else {
              tma_load_2d_pair(sA, &tmA, fb, kbp * BK, arow);
            }
            if (B_MN) {
              tma_load_2d_pair(sB, &tmB, fb, bcol, kbp * BK);
              tma_load_2d_pair(sB + 8192, &tmB, fb, bcol + 64, kbp * BK);
            } else {
              tma_load_2d_pair(sB, &tmB, fb, kbp * BK, bcol);
            }
            continue;
          }
          int ca = A_MN ? kbp * BK : m_blk * BM;
          int cb = kbp * BK;
          const CUtensorMap* mA =
              pick_map<PEER>(&tmA, PEER ? pm->a : nullptr, args.a_seg, ca, args, ready, ok, abort_flag);
          const CUtensorMap* mB =
              pick_map<PEER>(&tmB, PEER ? pm->b : nullptr, B_MN ? args.b_seg : 0, cb, args, ready, ok, abort_flag);
          if (!ok) break;
          mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
          if (A_MN) {
            tma_load_2d(sA, mA, &full[s], m_blk * BM, ca);
            tma_load_2d(sA + 8192, mA, &full[s], m_blk * BM + 64, ca);
          } else {
            tma_load_2d(sA, mA, &full[s], kbp * BK, ca);
          }
          if (B_MN) {
#pragma unroll
            for (int h = 0; h < BN / 64; ++h) tma_load_2d(sB + h * 8192, mB, &full[s], n_blk * BN + h * 64, cb);
          } else {
            tma_load_2d(sB, mB, &full[s], kbp * BK, n_blk * BN);
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        // Let copies already in flight land before the CTA exits (pair mode:
        // they complete on the leader's barriers; the final cluster barrier
        // keeps both CTAs alive until then).
        for (int j = 1; j <= STAGES && it - j >= 0 && (!PAIR || leader); ++j) {
          const int i2 = it - j;
          mbar_wait(&full[i2 % STAGES], (i2 / STAGES) & 1, nullptr, 0, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && (!PAIR || leader)) {
      int it = 0, local = 0;
      bool ok = true;
      for (int u = unit0; u < args.num_units && ok; u += ustep, ++local) {
        int m_blk, n_blk, split;
        decode_unit(args, u, m_blk, n_blk, split);
        const int kb0 = split * args.kb_per_split;
        const int kb1 = min(args.num_kb, kb0 + args.kb_per_split);
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], aph ^ 1, args.st, 2, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full[s], ph, args.st, 3, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + s * C::STAGE_BYTES);
          const uint32_t b_base = a_base + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t adesc = A_MN ? umma_desc_sw128(a_base + kk * 2048, 8192, 1024)
                                        : umma_desc_sw128(a_base + kk * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? umma_desc_sw128(b_base + kk * 2048, 8192, 1024)
                                        : umma_desc_sw128(b_base + kk * 32, 16, 1024);
            if (PAIR)
              tc_mma_f16_ss_pair(d_tmem, adesc, bdesc, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
            else
              tc_mma_f16_ss(d_tmem, adesc, bdesc, IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          if (PAIR)
            tc_commit_pair(&empty[s]);
          else
            tc_commit(&empty[s]);
        }
        if (!ok) break;
        if (PAIR)
          tc_commit_pair(&tfull[acc]);
        else
          tc_commit(&tfull[acc]);
      }
      // Drain: make sure every MMA this thread issued has completed before
      // TMEM is released at the end of the kernel.
      if (PAIR)
        tc_commit_pair_local(drain);
      else
        tc_commit(drain);
      mbar_wait(drain, 0, nullptr, 0, nullptr);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // TMEM -> registers -> fused math -> swizzled smem slot -> TMA store
    // (bf16 outputs) or TMA reduce-add / store (fp32 outputs, 16-col halves).
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    // two warps per lane quarter; each takes one half of the tile's columns
    const int c_begin = (warp < 6) ? 0 : BN / 2;
    uint8_t* slot0 = smem + C::STAGING_OFF + (warp - 2) * 2 * C::SLOT_BYTES;
    uint8_t* slot1 = slot0 + C::SLOT_BYTES;
    // Epilogues with an aux operand (residual / GELU pre-activation) TMA-load
    // each 32x32 aux chunk into slot1 one chunk ahead; outputs go via slot0.
    constexpr bool HAS_AUX = (EPI == EPI_RESID || EPI == EPI_DGELU);
    uint64_t* my_aux_bar = &aux_bar[warp - 2];
    uint32_t aux_phase = 0;
    int local = 0;
    // the accumulator is released on the leader's tempty barrier (pair mode)
    const uint32_t tempty_leader0 = PAIR ? mapa_shared(&tempty[0], 0) : 0u;
    auto release_acc = [&](int acc) {
      if (PAIR)
        mbar_arrive_cluster(tempty_leader0 + acc * 8);
      else
        mbar_arrive(&tempty[acc]);
    };
    for (int u = unit0; u < args.num_units; u += ustep, ++local) {
      int m_blk, n_blk, split;
      decode_unit(args, u, m_blk, n_blk, split);
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      const int row0 = m_blk * MT + row_sub + q * 32;
      const int row = row0 + lane;
      const bool row_ok = row < args.M;
      // number of 32-column chunks of this warp's half that lie inside N
      const int nch = max(0, min(BN / 64, (args.N - (n_blk * BN + c_begin) + 31) / 32));
      if (HAS_AUX && nch > 0 && lane == 0) {
        mbar_arrive_expect_tx(my_aux_bar, C::SLOT_BYTES);
        tma_load_2d(slot1, &tmC2, my_aux_bar, n_blk * BN + c_begin, row0);
      }
      if (!mbar_wait(&tfull[acc], aph, args.st, 4, abort_flag)) break;
      tc_fence_after();
      const uint32_t trow = tmem_base + (uint32_t(q * 32) << 16) + acc * BN;
      if (nch == 0) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release_acc(acc);
      }
      // TMEM reads are software-pipelined: chunk ci+1 is loaded while chunk
      // ci is processed (two register buffers; the dGELU epilogue, which
      // needs its registers for the column-sum butterfly, loads one at a time)
      constexpr bool PREFETCH = (EPI != EPI_DGELU && EPI != EPI_ROPE);
      uint32_t rb0[32], rb1[32];
      if (PREFETCH && nch > 0) tmem_ld_32x32b_x32(trow + c_begin, rb0);
#pragma unroll
      for (int ci = 0; ci < BN / 64; ++ci) {
        if (ci >= nch) break;
        const int c = c_begin + ci * 32;
        const int col0 = n_blk * BN + c;
        uint32_t* r = (ci & 1) ? rb1 : rb0;
        // RoPE: the partner half of this chunk's head (same TMEM lane = same
        // row, columns hd/2 away; heads never straddle a tile since BN % hd == 0)
        uint32_t* pr = (ci & 1) ? rb0 : rb1;
        const bool rot = (EPI == EPI_ROPE) && col0 < args.rope_cols;
        const int rhalf = (EPI == EPI_ROPE) ? (args.rope_hd >> 1) : 0;
        const int rd0 = rot ? col0 % args.rope_hd : 0;
        const int rpoff = rd0 < rhalf ? rhalf : -rhalf;  // partner column offset
        if (PREFETCH) {
          tc_wait_ld_regs(r);
          if (ci + 1 < nch) tmem_ld_32x32b_x32(trow + c + 32, (ci & 1) ? rb0 : rb1);
        } else {
          tmem_ld_32x32b_x32(trow + c, r);
          if (EPI == EPI_ROPE && rot) tmem_ld_32x32b_x32(trow + c + rpoff, pr);
          tc_wait_ld_regs(r);
          if (EPI == EPI_ROPE && rot) tc_wait_ld_regs(pr);
        }
        if (ci == nch - 1) {
          // last TMEM read of this tile by this warp: release the accumulator
          // so the MMA warp can start the next tile while we finish the math
          tc_fence_before();
          __syncwarp();
          if (lane == 0) release_acc(acc);
        }
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = row_ok ? __uint_as_float(r[j]) : 0.f;
        if (EPI != EPI_F32 && EPI != EPI_DGELU && args.bias != nullptr) {
          const uint4* bp = reinterpret_cast<const uint4*>(args.bias + col0);
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            if (col0 + g * 8 >= args.N) break;
            uint4 b4 = __ldg(bp + g);
            uint32_t bw[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              v[g * 8 + 2 * e] += bf16_lo(bw[e]);
              v[g * 8 + 2 * e + 1] += bf16_hi(bw[e]);
            }
          }
        }
        if (EPI == EPI_ROPE && rot) {
          float pv[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) pv[j] = __uint_as_float(pr[j]);
          if (args.bias != nullptr) {
            const uint4* bp = reinterpret_cast<const uint4*>(args.bias + col0 + rpoff);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              uint4 b4 = __ldg(bp + g);
              uint32_t bw[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                pv[g * 8 + 2 * e] += bf16_lo(bw[e]);
                pv[g * 8 + 2 * e + 1] += bf16_hi(bw[e]);
              }
            }
          }
          // first half: x cos - partner sin; second half: x cos + partner sin
          const float sgn = rd0 < rhalf ? -1.f : 1.f;
          const long toff = (long)(row % args.rope_S) * rhalf + (rd0 < rhalf ? rd0 : rd0 - rhalf);
          const float4* cp = reinterpret_cast<const float4*>(args.rope_cos + toff);
          const float4* sp4 = reinterpret_cast<const float4*>(args.rope_sin + toff);
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            const float4 c4 = __ldg(cp + g), s4 = __ldg(sp4 + g);
            v[4 * g + 0] = fmaf(v[4 * g + 0], c4.x, sgn * pv[4 * g + 0] * s4.x);
            v[4 * g + 1] = fmaf(v[4 * g + 1], c4.y, sgn * pv[4 * g + 1] * s4.y);
            v[4 * g + 2] = fmaf(v[4 * g + 2], c4.z, sgn * pv[4 * g + 2] * s4.z);
            v[4 * g + 3] = fmaf(v[4 * g + 3], c4.w, sgn * pv[4 * g + 3] * s4.w);
          }
        }
        if (HAS_AUX) {
          // aux chunk (rows beyond M / cols beyond N arrive zero-filled)
          mbar_wait(my_aux_bar, aux_phase, args.st, 5, abort_flag);
          aux_phase ^= 1;
          uint4 ax[4];
#pragma unroll
          for (int g = 0; g < 4; ++g)
            ax[g] = *reinterpret_cast<const uint4*>(slot1 + lane * 64 + ((g ^ ((lane >> 1) & 3)) << 4));
          fence_proxy_async_smem();
          __syncwarp();
          if (ci + 1 < nch && lane == 0) {
            mbar_arrive_expect_tx(my_aux_bar, C::SLOT_BYTES);
            tma_load_2d(slot1, &tmC2, my_aux_bar, col0 + 32, row0);
          }
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 x4 = ax[g];
            uint32_t xw[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float x0 = bf16_lo(xw[e]), x1 = bf16_hi(xw[e]);
              if (EPI == EPI_RESID) {
                v[g * 8 + 2 * e] += x0;
                v[g * 8 + 2 * e + 1] += x1;
              } else if (args.gelu_x2) {
                const uint64_t d = f2_mul(f2_pack(v[g * 8 + 2 * e], v[g * 8 + 2 * e + 1]),
                                          gelu_tanh_grad2(f2_pack(x0, x1)));
                f2_unpack(d, v[g * 8 + 2 * e], v[g * 8 + 2 * e + 1]);
              } else {
                v[g * 8 + 2 * e] *= gelu_tanh_grad(x0);
                v[g * 8 + 2 * e + 1] *= gelu_tanh_grad(x1);
              }
            }
          }
        }
        if (PEER && args.rs_seg > 0) {
          // GEMM -> reduce-scatter: push the chunk's bf16 partial sums
          // straight into the owners' receive slots over NVLink. The chunk
          // (32 rows x 64 bytes, one row per lane) is transposed through this
          // warp's staging slot so that each store instruction writes eight
          // whole 64-byte row segments (four lanes per row) instead of 32
          // scattered 16-byte pieces.
#pragma unroll
          for (int uu = 0; uu < 4; ++uu) {
            const int j = uu * 8;
            slot_st16(slot0, lane, uu,
                      make_uint4(pack_bf16x2(v[j], v[j + 1]), pack_bf16x2(v[j + 2], v[j + 3]),
                                 pack_bf16x2(v[j + 4], v[j + 5]), pack_bf16x2(v[j + 6], v[j + 7])));
          }
          __syncwarp();
          const int u = lane & 3;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int r = k * 8 + (lane >> 2);
            const int grow = row0 + r;
            const uint4 val = *reinterpret_cast<const uint4*>(slot0 + r * 64 + ((u ^ ((r >> 1) & 3)) << 4));
            if (grow < args.M && col0 + u * 8 < args.N) {
              const int owner = grow / args.rs_seg;
              *reinterpret_cast<uint4*>(args.rs_dst[owner] + (long)(grow - owner * args.rs_seg) * args.rs_ld + col0 +
                                        u * 8) = val;
            }
          }
          __syncwarp();  // the slot is rewritten by the next chunk
          continue;
        }
        // slots are free once the previous chunk's stores have read them
        if (lane == 0) tma_store_wait_read0();
        __syncwarp();
        if (EPI == EPI_F32) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint8_t* sl = hh ? slot1 : slot0;
#pragma unroll
            for (int uu = 0; uu < 4; ++uu) {
              const int j = hh * 16 + uu * 4;
              slot_st16(sl, lane, uu,
                        make_uint4(__float_as_uint(v[j]), __float_as_uint(v[j + 1]), __float_as_uint(v[j + 2]),
                                   __float_as_uint(v[j + 3])));
            }
          }
        } else {
          if (EPI == EPI_BIAS_GELU) {
#pragma unroll
            for (int uu = 0; uu < 4; ++uu) {
              const int j = uu * 8;
              slot_st16(slot1, lane, uu,
                        make_uint4(pack_bf16x2(v[j], v[j + 1]), pack_bf16x2(v[j + 2], v[j + 3]),
                                   pack_bf16x2(v[j + 4], v[j + 5]), pack_bf16x2(v[j + 6], v[j + 7])));
            }
#pragma unroll
            if (args.gelu_x2) {
#pragma unroll
              for (int j = 0; j < 32; j += 2) f2_unpack(gelu_tanh2(f2_pack(v[j], v[j + 1])), v[j], v[j + 1]);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
            }
          }
#pragma unroll
          for (int uu = 0; uu < 4; ++uu) {
            const int j = uu * 8;
            slot_st16(slot0, lane, uu,
                      make_uint4(pack_bf16x2(v[j], v[j + 1]), pack_bf16x2(v[j + 2], v[j + 3]),
                                 pack_bf16x2(v[j + 4], v[j + 5]), pack_bf16x2(v[j + 6], v[j + 7])));
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (EPI == EPI_F32) {
            if (args.atomic_out) {
              tma_reduce_add_2d(&tmC, slot0, col0, row0);
              if (col0 + 16 < args.N) tma_reduce_add_2d(&tmC, slot1, col0 + 16, row0);
            } else {
              tma_store_2d(&tmC, slot0, col0, row0);
              if (col0 + 16 < args.N) tma_store_2d(&tmC, slot1, col0 + 16, row0);
            }
          } else {
            tma_store_2d(&tmC, slot0, col0, row0);
            if (EPI == EPI_BIAS_GELU) tma_store_2d(&tmC2, slot1, col0, row0);
          }
          tma_store_commit();
        }
        if (EPI == EPI_DGELU && args.bias_grad != nullptr) {
          // Column sums over this warp's 32 rows: butterfly reduce-scatter,
          // after which lane l holds the sum of column col0 + l.
#pragma unroll
          for (int s = 16; s >= 1; s >>= 1) {
            const bool upper = (lane & s) != 0;
#pragma unroll
            for (int i = 0; i < s; ++i) {
              const float send = upper ? v[i] : v[i + s];
              const float recv = __shfl_xor_sync(0xffffffffu, send, s);
              v[i] = (upper ? v[i + s] : v[i]) + recv;
            }
          }
          if (col0 + lane < args.N) atomicAdd(args.bias_grad + col0 + lane, v[0]);
        }
      }
    }
    if (lane == 0) tma_store_wait0();
    __syncwarp();
  }

  tc_fence_before();
  if (PAIR)
    cluster_sync_all();  // no CTA leaves while its pair still signals its barriers / reads its smem
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    else
      tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if (PEER && args.sig_flags[0] != nullptr && threadIdx.x == 0) {
    // last CTA to finish tells every peer that this rank's output is complete
    __threadfence_system();
    if (atomicAdd(args.done_ctr, 1u) == gridDim.x - 1) {
      *args.done_ctr = 0u;
      const unsigned v = *args.epoch_ptr * kSigStride + args.sig_idx;
      __threadfence_system();
      for (int r = 0; r < args.world; ++r) st_release_sys_u32(args.sig_flags[r], v);
    }
  }
}

template <int BN, int A_MN, int B_MN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmC2, const Args args) {
  gemm_body<BN, A_MN, B_MN, EPI, false>(&tmA, &tmB, &tmC, &tmC2, nullptr, args);
}

// Pair variant: clusters of two CTAs share each 256 x 256 tile (cta_group::2).
template <int A_MN, int B_MN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmC2,
                     const Args args) {
  gemm_body<256, A_MN, B_MN, EPI, false, true>(&tmA, &tmB, &tmC, &tmC2, nullptr, args);
}

// Tensor-parallel variant: operands may be split over the ranks' symmetric
// buffers (one TMA map per rank, plain TMA loads, no multicast), the output
// may be pushed to the owners of its rows, and the kernel can signal peers.
template <int BN, int A_MN, int B_MN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tp_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmC2,
                   const __grid_constant__ PeerMaps pm, const Args args) {
  gemm_body<BN, A_MN, B_MN, EPI, true>(&tmA, &tmB, &tmC, &tmC2, &pm, args);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct TmapKey {
  const void* p;
  uint64_t inner, outer, stride;
  uint32_t bi, bo, dtype, swz;
  bool operator==(const TmapKey& o) const {
    return p == o.p && inner == o.inner && outer == o.outer && stride == o.stride && bi == o.bi && bo == o.bo &&
           dtype == o.dtype && swz == o.swz;
  }
};
struct TmapHash {
  size_t operator()(const TmapKey& k) const {
    size_t h = std::hash<const void*>()(k.p);
    h ^= std::hash<uint64_t>()(k.inner * 1315423911ull + k.outer * 2654435761ull + k.stride * 97 + k.bi * 31 +
                               k.bo * 7 + k.dtype * 3 + k.swz);
    return h;
  }
};

static std::mutex g_tm_mu;
static std::unordered_map<TmapKey, CUtensorMap, TmapHash> g_tmaps;

// Cached tensor map. Operand maps use bf16 + 128B swizzle; output maps use a
// 64B swizzle that matches the epilogue staging slots.
static CUtensorMap get_tmap(const void* p, uint64_t inner, uint64_t outer, uint64_t stride_bytes, uint32_t bi,
                            uint32_t bo, CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                            CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  TmapKey k{p, inner, outer, stride_bytes, bi, bo, (uint32_t)dt, (uint32_t)swz};
  std::lock_guard<std::mutex> lk(g_tm_mu);
  auto it = g_tmaps.find(k);
  if (it != g_tmaps.end()) return it->second;
  if (g_tmaps.size() > 4096) g_tmaps.clear();
  CUtensorMap m = make_tmap_2d(p, dt, inner, outer, stride_bytes, bi, bo, swz);
  g_tmaps.emplace(k, m);
  return m;
}

struct Maps {
  CUtensorMap a, b, c, c2;
};

template <int BN, int A_MN, int B_MN, int EPI>
static void launch_t(const Maps& m, const Args& args, int grid, cudaStream_t stream) {
  auto kern = gemm_tc_kernel<BN, A_MN, B_MN, EPI>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    SCIRS_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<BN>::SMEM));
    attr_set[dev] = true;
  }
  kern<<<grid, kThreads, Cfg<BN>::SMEM, stream>>>(m.a, m.b, m.c, m.c2, args);
  SCIRS_CHECK_LAUNCH();
}

template <int BN, int A_MN, int B_MN>
static void launch_epi(int epi, const Maps& m, const Args& args, int grid, cudaStream_t s) {
  switch (epi) {
    case EPI_BF16: launch_t<BN, A_MN, B_MN, EPI_BF16>(m, args, grid, s); break;
    case EPI_BIAS_GELU: launch_t<BN, A_MN, B_MN, EPI_BIAS_GELU>(m, args, grid, s); break;
    case EPI_RESID: launch_t<BN, A_MN, B_MN, EPI_RESID>(m, args, grid, s); break;
    case EPI_DGELU: launch_t<BN, A_MN, B_MN, EPI_DGELU>(m, args, grid, s); break;
    case EPI_F32: launch_t<BN, A_MN, B_MN, EPI_F32>(m, args, grid, s); break;
    case EPI_ROPE:
      if (!A_MN && !B_MN) launch_t<BN, 0, 0, EPI_ROPE>(m, args, grid, s);
      else TORCH_CHECK(false, "the RoPE epilogue takes K-major operands");
      break;
    default: TORCH_CHECK(false, "bad epilogue ", epi);
  }
}

template <int BN>
static void launch_bn(int a_mn, int b_mn, int epi, const Maps& m, const Args& args, int grid, cudaStream_t s) {
  if (!a_mn && !b_mn) launch_epi<BN, 0, 0>(epi, m, args, grid, s);
  else if (!a_mn && b_mn) launch_epi<BN, 0, 1>(epi, m, args, grid, s);
  else if (a_mn && !b_mn) launch_epi<BN, 1, 0>(epi, m, args, grid, s);
  else launch_epi<BN, 1, 1>(epi, m, args, grid, s);
}

// Clusters of two that can be resident at once (SMs of a GPC pair up; an odd
// SM count leaves one out). A persistent grid larger than this would run its
// last clusters after the others finished.
static int pair_slots(int dev) {
  static int slots[64] = {0};
  if (slots[dev] == 0) {
    auto kern = gemm_pair_kernel<0, 0, EPI_BF16>;
    set_max_smem(reinterpret_cast<const void*>(kern), Cfg<256, true>::SMEM);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * num_sms(dev), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = Cfg<256, true>::SMEM;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, reinterpret_cast<const void*>(kern), &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms(dev) / 2;
    }
    slots[dev] = std::min(n, num_sms(dev) / 2);
  }
  return slots[dev];
}

template <int A_MN, int B_MN, int EPI>
static void launch_pair_t(const Maps& m, const Args& args, int grid, cudaStream_t stream) {
  auto kern = gemm_pair_kernel<A_MN, B_MN, EPI>;
  set_max_smem(reinterpret_cast<const void*>(kern), Cfg<256, true>::SMEM);
  kern<<<grid, kThreads, Cfg<256, true>::SMEM, stream>>>(m.a, m.b, m.c, m.c2, args);
  SCIRS_CHECK_LAUNCH();
}

template <int A_MN, int B_MN>
static void launch_pair_epi(int epi, const Maps& m, const Args& args, int grid, cudaStream_t s) {
  switch (epi) {
    case EPI_BF16: launch_pair_t<A_MN, B_MN, EPI_BF16>(m, args, grid, s); break;
    case EPI_BIAS_GELU: launch_pair_t<A_MN, B_MN, EPI_BIAS_GELU>(m, args, grid, s); break;
    case EPI_RESID: launch_pair_t<A_MN, B_MN, EPI_RESID>(m, args, grid, s); break;
    case EPI_DGELU: launch_pair_t<A_MN, B_MN, EPI_DGELU>(m, args, grid, s); break;
    case EPI_F32: launch_pair_t<A_MN, B_MN, EPI_F32>(m, args, grid, s); break;
    case EPI_ROPE:
      if (!A_MN && !B_MN) launch_pair_t<0, 0, EPI_ROPE>(m, args, grid, s);
      else TORCH_CHECK(false, "the RoPE epilogue takes K-major operands");
      break;
    default: TORCH_CHECK(false, "bad epilogue ", epi);
  }
}

static void launch_pair(int a_mn, int b_mn, int epi, const Maps& m, const Args& args, int grid, cudaStream_t s) {
  if (!a_mn && !b_mn) launch_pair_epi<0, 0>(epi, m, args, grid, s);
  else if (!a_mn && b_mn) launch_pair_epi<0, 1>(epi, m, args, grid, s);
  else if (a_mn && !b_mn) launch_pair_epi<1, 0>(epi, m, args, grid, s);
  else launch_pair_epi<1, 1>(epi, m, args, grid, s);
}

// Packed f32x2 GELU / GELU' in the bias + GELU and dGELU epilogues:
// SCIRS_GEMM_GELU_X2=0 selects the scalar forms, read once per process.
static bool gelu_x2_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("SCIRS_GEMM_GELU_X2");
    v = (e == nullptr) ? 1 : atoi(e);
  }
  return v != 0;
}

// 2-CTA (cta_group::2) tiles for large GEMMs: SCIRS_GEMM_PAIR=0 disables,
// =1 enables (default), read once per process.
static bool pair_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("SCIRS_GEMM_PAIR");
    v = (e == nullptr) ? 1 : atoi(e);
  }
  return v != 0;
}

template <int A_MN, int B_MN, int EPI>
static void launch_tp_t(const Maps& m, const PeerMaps& pm, const Args& args, int grid, cudaStream_t stream) {
  constexpr int BN = 256;
  auto kern = gemm_tp_kernel<BN, A_MN, B_MN, EPI>;
  set_max_smem(reinterpret_cast<const void*>(kern), Cfg<BN>::SMEM);
  kern<<<grid, kThreads, Cfg<BN>::SMEM, stream>>>(m.a, m.b, m.c, m.c2, pm, args);
  SCIRS_CHECK_LAUNCH();
}

// Operand forms used by the tensor-parallel layers (BN = 256):
//   (K, K, BF16/BIAS_GELU) forward column-parallel (A rows gathered from the
//   peers) and row-parallel (output rows pushed to their owners);
//   (K, MN, BF16/DGELU) data gradients; (MN, MN, F32) weight gradients with
//   the K (token) dimension of one operand gathered from the peers.
static void launch_tp(int a_mn, int b_mn, int epi, const Maps& m, const PeerMaps& pm, const Args& args, int grid,
                      cudaStream_t s) {
  if (!a_mn && !b_mn && epi == EPI_BF16) launch_tp_t<0, 0, EPI_BF16>(m, pm, args, grid, s);
  else if (!a_mn && !b_mn && epi == EPI_BIAS_GELU) launch_tp_t<0, 0, EPI_BIAS_GELU>(m, pm, args, grid, s);
  else if (!a_mn && !b_mn && epi == EPI_ROPE) launch_tp_t<0, 0, EPI_ROPE>(m, pm, args, grid, s);
  else if (!a_mn && b_mn && epi == EPI_BF16) launch_tp_t<0, 1, EPI_BF16>(m, pm, args, grid, s);
  else if (!a_mn && b_mn && epi == EPI_DGELU) launch_tp_t<0, 1, EPI_DGELU>(m, pm, args, grid, s);
  else if (a_mn && b_mn && epi == EPI_F32) launch_tp_t<1, 1, EPI_F32>(m, pm, args, grid, s);
  else TORCH_CHECK(false, "tensor-parallel GEMM form not supported: a_mn=", a_mn, " b_mn=", b_mn, " epi=", epi);
}

// EPI_ROPE arguments: fp32 [S, hd/2] cos / sin tables, hd a multiple of 64
// (so that a 32-column chunk and its partner lie in one half each), the
// rotated columns a whole number of heads, N a whole number of heads.
static void set_rope(Args& args, int64_t epi, const c10::optional<torch::Tensor>& cos_t,
                     const c10::optional<torch::Tensor>& sin_t, int64_t S, int64_t hd, int64_t cols, int64_t N) {
  if (epi != EPI_ROPE) return;
  TORCH_CHECK(cos_t.has_value() && cos_t->defined() && sin_t.has_value() && sin_t->defined(),
              "the RoPE epilogue needs cos / sin tables");
  CHECK_DTYPE((*cos_t), at::kFloat);
  CHECK_DTYPE((*sin_t), at::kFloat);
  TORCH_CHECK(cos_t->is_contiguous() && sin_t->is_contiguous(), "rope tables must be contiguous");
  TORCH_CHECK(hd > 0 && hd % 64 == 0, "RoPE epilogue: head_dim must be a multiple of 64");
  TORCH_CHECK(S > 0 && cos_t->numel() >= S * hd / 2 && sin_t->numel() >= S * hd / 2, "rope tables too small");
  TORCH_CHECK(cols >= 0 && cols % hd == 0 && cols <= N && N % hd == 0, "RoPE columns must be whole heads");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(cos_t->data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(sin_t->data_ptr()) & 15) == 0, "rope tables must be 16-byte aligned");
  args.rope_cos = cos_t->data_ptr<float>();
  args.rope_sin = sin_t->data_ptr<float>();
  args.rope_S = (int)S;
  args.rope_hd = (int)hd;
  args.rope_cols = (int)cols;
}

// ---------------------------------------------------------------------------
// Split-K for bf16 outputs (small M, long K): the product is reduce-added in
// fp32 into a zeroed workspace (stream-ordered allocation, so it also works
// under CUDA-graph capture) by the split-K weight-gradient path (2-SM pair
// tiles), then one pass converts it to bf16 with the bias and the residual.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) splitk_finalize_kernel(const float* __restrict__ ws,
                                                              __nv_bfloat16* __restrict__ out,
                                                              long ldo, const __nv_bfloat16* __restrict__ bias,
                                                              const __nv_bfloat16* __restrict__ aux, long ldaux, int M,
                                                              int N) {
  const long nvec = (long)M * (N / 8);
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < nvec; i += (long)gridDim.x * blockDim.x) {
    const long row = i / (N / 8);
    const int col = (int)(i % (N / 8)) * 8;
    const float4* w = reinterpret_cast<const float4*>(ws + row * N + col);
    const float4 w0 = __ldcs(w), w1 = __ldcs(w + 1);
    float f[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    if (bias != nullptr) {
      const uint4 b4 = __ldg(reinterpret_cast<const uint4*>(bias + col));
      const uint32_t bw[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        f[2 * e] += bf16_lo(bw[e]);
        f[2 * e + 1] += bf16_hi(bw[e]);
      }
    }
    if (aux != nullptr) {
      const uint4 a4 = *reinterpret_cast<const uint4*>(aux + row * ldaux + col);
      const uint32_t aw[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        f[2 * e] += bf16_lo(aw[e]);
        f[2 * e + 1] += bf16_hi(aw[e]);
      }
    }
    *reinterpret_cast<uint4*>(out + row * ldo + col) =
        make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
  }
}

// SCIRS_GEMM_SPLITK_BF16=0 disables the split-K path for bf16 outputs.
static bool splitk_bf16_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("SCIRS_GEMM_SPLITK_BF16");
    v = (e == nullptr) ? 1 : atoi(e);
  }
  return v != 0;
}

static unsigned* done_counter(int dev) {
  static unsigned* ctr[64] = {nullptr};
  if (ctr[dev] == nullptr) {
    SCIRS_CHECK_CUDA(cudaMalloc(&ctr[dev], sizeof(unsigned)));
    SCIRS_CHECK_CUDA(cudaMemset(ctr[dev], 0, sizeof(unsigned)));
  }
  return ctr[dev];
}

}  // namespace gemm

// Tensor-parallel GEMM (fused all-gather -> GEMM and GEMM -> reduce-scatter).
//   a_peers (optional): base address of A's segment on every rank (symmetric
//     buffers; `a` is this rank's segment): A K-major [Mr, K] -> rows
//     gathered, M = world * Mr; A MN-major [Kr, M] -> K gathered, K = world*Kr.
//   b_peers (optional, B MN-major [Kr, N]): K gathered, K = world * Kr.
//   rs_dst (optional): owner r's receive-slot address for this rank's rows;
//     `out` is then this rank's receive buffer [world, Mr, N] (shape check
//     only) and output rows [r*Mr, (r+1)*Mr) are pushed to owner r.
//   flags / epoch / wait_idx: before reading a peer's segment the producer
//     waits (bounded) until flags[peer] >= epoch * 4096 + wait_idx.
//   sig_flags / sig_idx (optional): when every CTA is done, each peer's flag
//     word for this rank is set to epoch * 4096 + sig_idx.
void gemm_tp(torch::Tensor a, torch::Tensor b, torch::Tensor out, int64_t a_mn, int64_t b_mn, int64_t epi,
             c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> aux, c10::optional<torch::Tensor> out2,
             bool accumulate, int64_t splits, int64_t rank, int64_t world, std::vector<int64_t> a_peers,
             std::vector<int64_t> b_peers, std::vector<int64_t> rs_dst, c10::optional<torch::Tensor> flags,
             c10::optional<torch::Tensor> epoch, int64_t wait_idx, std::vector<int64_t> sig_flags, int64_t sig_idx,
             double timeout_s, c10::optional<torch::Tensor> rope_cos, c10::optional<torch::Tensor> rope_sin,
             int64_t rope_S, int64_t rope_hd, int64_t rope_cols) {
  using namespace gemm;
  CHECK_DTYPE(a, at::kBFloat16);
  CHECK_DTYPE(b, at::kBFloat16);
  TORCH_CHECK(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world, "bad rank/world");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2, "gemm operands must be 2-D");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1, "gemm operands need unit inner stride");
  const bool ap = !a_peers.empty(), bp = !b_peers.empty(), rs = !rs_dst.empty();
  TORCH_CHECK(!ap || (int64_t)a_peers.size() == world, "a_peers needs one address per rank");
  TORCH_CHECK(!bp || ((int64_t)b_peers.size() == world && b_mn), "b_peers: one address per rank, B MN-major");
  TORCH_CHECK(!rs || ((int64_t)rs_dst.size() == world && epi == EPI_BF16 && !a_mn), "rs_dst: one per rank, bf16");
  const int64_t Ml = a_mn ? a.size(1) : a.size(0);
  const int64_t Kl = a_mn ? a.size(0) : a.size(1);
  const int64_t M = (ap && !a_mn) ? Ml * world : Ml;
  const int64_t K = (ap && a_mn) ? Kl * world : Kl;
  const int64_t Kb = b_mn ? b.size(0) * (bp ? world : 1) : b.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK(K == Kb, "gemm K mismatch: ", K, " vs ", Kb);
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0, "tensor-parallel gemm needs K and N multiples of 8");
  TORCH_CHECK(!((ap && !a_mn) || rs) || M % (BM * world) == 0, "row-split operands need M % (128*world) == 0");
  if (ap) TORCH_CHECK(a_mn ? (a.size(0) % BK == 0) : (a.size(0) % BM == 0), "segment not tile aligned");
  if (bp) TORCH_CHECK(b.size(0) % BK == 0, "B segment not tile aligned");
  const int dev = a.get_device();
  c10::cuda::CUDAGuard guard(dev);
  const int sms = num_sms(dev);
  Args args{};
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.num_kb = (int)((K + BK - 1) / BK);
  args.m_blocks = (int)((M + BM - 1) / BM);
  args.st = status_ptr(dev);
  args.group_m = 16;
  args.rank = (int)rank;
  args.world = (int)world;
  args.timeout_ns = (long long)(timeout_s * 1e9);
  if (epoch.has_value() && epoch->defined()) {
    TORCH_CHECK(epoch->element_size() == 4 && epoch->is_cuda(), "epoch: 32-bit device scalar");
    args.epoch_ptr = reinterpret_cast<const unsigned*>(epoch->data_ptr());
  }
  if (flags.has_value() && flags->defined()) {
    TORCH_CHECK(flags->numel() >= world && flags->element_size() == 4, "flags: 32-bit [world]");
    TORCH_CHECK(args.epoch_ptr != nullptr, "waiting on flags needs the epoch counter");
    args.wait_flags = reinterpret_cast<const unsigned*>(flags->data_ptr());
    args.wait_idx = (unsigned)wait_idx;
  }
  if (!sig_flags.empty()) {
    TORCH_CHECK((int64_t)sig_flags.size() == world && args.epoch_ptr != nullptr, "sig_flags: one per rank + epoch");
    for (int r = 0; r < world; ++r) args.sig_flags[r] = reinterpret_cast<unsigned*>(sig_flags[r]);
    args.sig_idx = (unsigned)sig_idx;
    args.done_ctr = done_counter(dev);
  }
  if (bias.has_value() && bias->defined()) {
    CHECK_DTYPE((*bias), at::kBFloat16);
    TORCH_CHECK(bias->numel() >= N && bias->is_contiguous(), "bias must hold N contiguous values");
    args.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  }
  if (epi == EPI_DGELU) {
    TORCH_CHECK(aux.has_value() && aux->defined() && aux->size(0) == M && aux->size(1) == N, "dgelu needs aux [M,N]");
    args.aux = reinterpret_cast<const __nv_bfloat16*>(aux->data_ptr());
    args.ldaux = aux->stride(0);
  }
  Maps maps;
  if (rs) {
    TORCH_CHECK(out.dim() == 3 && out.size(0) == world && out.size(1) * world == M && out.size(2) == N &&
                    out.is_contiguous(), "out must be this rank's receive buffer [world, M/world, N]");
    CHECK_DTYPE(out, at::kBFloat16);
    args.rs_seg = (int)(M / world);
    args.rs_ld = N;
    for (int r = 0; r < world; ++r) args.rs_dst[r] = reinterpret_cast<__nv_bfloat16*>(rs_dst[r]);
    // start with the next rank's rows so that every rank pushes to a different owner
    args.m_rot = (int)(((rank + 1) % world) * (args.rs_seg / BM));
    maps.c = get_tmap(out.data_ptr(), (uint64_t)N, (uint64_t)M, (uint64_t)N * 2, 32, 32,
                      CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, CU_TENSOR_MAP_SWIZZLE_64B);
  } else {
    TORCH_CHECK(out.dim() == 2 && out.size(0) == M && out.size(1) == N && out.stride(1) == 1, "out must be [M, N]");
    if (epi == EPI_F32) {
      CHECK_DTYPE(out, at::kFloat);
    } else {
      CHECK_DTYPE(out, at::kBFloat16);
    }
    args.C = out.data_ptr();
    args.ldc = out.stride(0);
    TORCH_CHECK((reinterpret_cast<uintptr_t>(args.C) & 15) == 0 && args.ldc % 8 == 0,
                "out must be 16-byte aligned with rows a multiple of 8 elements");
    if (epi == EPI_F32)
      maps.c = get_tmap(out.data_ptr(), (uint64_t)N, (uint64_t)M, (uint64_t)out.stride(0) * 4, 16, 32,
                        CU_TENSOR_MAP_DATA_TYPE_FLOAT32, CU_TENSOR_MAP_SWIZZLE_64B);
    else
      maps.c = get_tmap(out.data_ptr(), (uint64_t)N, (uint64_t)M, (uint64_t)out.stride(0) * 2, 32, 32,
                        CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, CU_TENSOR_MAP_SWIZZLE_64B);
    if (ap && !a_mn) args.m_rot = (int)(rank * (Ml / BM));  // local rows first
  }
  maps.c2 = maps.c;
  if (epi == EPI_DGELU)
    maps.c2 = get_tmap(args.aux, (uint64_t)N, (uint64_t)M, (uint64_t)args.ldaux * 2, 32, 32,
                       CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, CU_TENSOR_MAP_SWIZZLE_64B);
  if (epi == EPI_BIAS_GELU) {
    TORCH_CHECK(out2.has_value() && out2->defined() && out2->size(0) == M && out2->size(1) == N, "gelu needs out2");
    args.C2 = out2->data_ptr();
    args.ldc2 = out2->stride(0);
    TORCH_CHECK((reinterpret_cast<uintptr_t>(args.C2) & 15) == 0 && args.ldc2 % 8 == 0, "out2 must be 16-byte aligned");
    maps.c2 = get_tmap(args.C2, (uint64_t)N, (uint64_t)M, (uint64_t)args.ldc2 * 2, 32, 32,
                       CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, CU_TENSOR_MAP_SWIZZLE_64B);
  }
  const uint64_t lda_b = (uint64_t)a.stride(0) * 2, ldb_b = (uint64_t)b.stride(0) * 2;
  PeerMaps pm;
  memset(&pm, 0, sizeof(pm));
  // local maps (own segment) and one map per rank for peer operands
  maps.a = a_mn ? get_tmap(a.data_ptr(), (uint64_t)Ml, (uint64_t)a.size(0), lda_b, 64, 64)
                : get_tmap(a.data_ptr(), (uint64_t)Kl, (uint64_t)a.size(0), lda_b, 64, BM);
  maps.b = b_mn ? get_tmap(b.data_ptr(), (uint64_t)N, (uint64_t)b.size(0), ldb_b, 64, 64)
                : get_tmap(b.data_ptr(), (uint64_t)b.size(1), (uint64_t)N, ldb_b, 64, 256);
  if (ap) {
    args.a_seg = (int)a.size(0);
    for (int r = 0; r < world; ++r) {
      const void* p = reinterpret_cast<const void*>(a_peers[r]);
      TORCH_CHECK((a_peers[r] & 15) == 0, "peer operand must be 16-byte aligned");
      pm.a[r] = a_mn ? get_tmap(p, (uint64_t)Ml, (uint64_t)a.size(0), lda_b, 64, 64)
                     : get_tmap(p, (uint64_t)Kl, (uint64_t)a.size(0), lda_b, 64, BM);
    }
    if (a_mn) args.kb_rot = (int)(rank * (a.size(0) / BK));
  }
  if (bp) {
    args.b_seg = (int)b.size(0);
    for (int r = 0; r < world; ++r) {
      TORCH_CHECK((b_peers[r] & 15) == 0, "peer operand must be 16-byte aligned");
      pm.b[r] = get_tmap(reinterpret_cast<const void*>(b_peers[r]), (uint64_t)N, (uint64_t)b.size(0), ldb_b, 64, 64);
    }
    args.kb_rot = (int)(rank * (b.size(0) / BK));
  }
  set_rope(args, epi, rope_cos, rope_sin, rope_S, rope_hd, rope_cols, N);
  args.n_blocks = (int)((N + 255) / 256);
  const long tiles = (long)args.m_blocks * args.n_blocks;
  int sp = 1;
  if (epi == EPI_F32) {
    if (splits > 0) sp = (int)splits;
    else if (tiles < 2L * sms) sp = (int)std::max<long>(1, std::min<long>(16, (2L * sms + tiles - 1) / tiles));
    sp = std::max(1, std::min(sp, args.num_kb));
  }
  args.kb_per_split = (args.num_kb + sp - 1) / sp;
  sp = (args.num_kb + args.kb_per_split - 1) / args.kb_per_split;
  args.splits = sp;
  args.atomic_out = (epi == EPI_F32 && (accumulate || sp > 1)) ? 1 : 0;
  args.gelu_x2 = gelu_x2_enabled() ? 1 : 0;
  if (epi == EPI_F32 && sp > 1 && !accumulate) out.zero_();
  args.num_units = (int)(tiles * sp);
  const int grid = (int)std::min<long>(args.num_units, sms);
  launch_tp((int)a_mn, (int)b_mn, (int)epi, maps, pm, args, grid, cur_stream());
}

// Python entry: see scirs_b200/ops/gemm.py for the calling convention.
//   a        : bf16 2-D, [M,K] (a_mn=0) or [K,M] (a_mn=1)
//   b        : bf16 2-D, [N,K] (b_mn=0) or [K,N] (b_mn=1)
//   out      : bf16 [M,N] (epi 0-3) or fp32 [M,N] (epi 4)
//   out2     : bf16 [M,N] pre-activation (epi 1)
//   aux      : bf16 [M,N] residual (epi 2) / pre-activation (epi 3)
//   accumulate (epi 4): add into out instead of overwriting
//   bias_grad (epi 3)  : fp32 [N], accumulates the column sums of out
//   splits   : split-K factor (0 = automatic; epi 4 only)
static void gemm_tc_impl(torch::Tensor a, torch::Tensor b, torch::Tensor out, int64_t a_mn, int64_t b_mn,
                         int64_t epi, c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> aux,
                         c10::optional<torch::Tensor> out2, bool accumulate, int64_t splits, int64_t bn_force,
                         c10::optional<torch::Tensor> bias_grad, c10::optional<torch::Tensor> rope_cos,
                         c10::optional<torch::Tensor> rope_sin, int64_t rope_S, int64_t rope_hd, int64_t rope_cols,
                         bool allow_split_bf16);

void gemm_tc(torch::Tensor a, torch::Tensor b, torch::Tensor out, int64_t a_mn, int64_t b_mn, int64_t epi,
             c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> aux, c10::optional<torch::Tensor> out2,
             bool accumulate, int64_t splits, int64_t bn_force, c10::optional<torch::Tensor> bias_grad,
             c10::optional<torch::Tensor> rope_cos, c10::optional<torch::Tensor> rope_sin, int64_t rope_S,
             int64_t rope_hd, int64_t rope_cols) {
  gemm_tc_impl(a, b, out, a_mn, b_mn, epi, bias, aux, out2, accumulate, splits, bn_force, bias_grad, rope_cos,
               rope_sin, rope_S, rope_hd, rope_cols, true);
}

static void gemm_tc_impl(torch::Tensor a, torch::Tensor b, torch::Tensor out, int64_t a_mn, int64_t b_mn,
                         int64_t epi, c10::optional<torch::Tensor> bias, c10::optional<torch::Tensor> aux,
                         c10::optional<torch::Tensor> out2, bool accumulate, int64_t splits, int64_t bn_force,
                         c10::optional<torch::Tensor> bias_grad, c10::optional<torch::Tensor> rope_cos,
                         c10::optional<torch::Tensor> rope_sin, int64_t rope_S, int64_t rope_hd, int64_t rope_cols,
                         bool allow_split_bf16) {
  using namespace gemm;
  CHECK_CUDA_TENSOR(a);
  CHECK_CUDA_TENSOR(b);
  CHECK_CUDA_TENSOR(out);
  CHECK_DTYPE(a, at::kBFloat16);
  CHECK_DTYPE(b, at::kBFloat16);
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 2, "gemm operands must be 2-D");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && out.stride(1) == 1, "gemm operands need unit inner stride");
  const int64_t M = a_mn ? a.size(1) : a.size(0);
  const int64_t K = a_mn ? a.size(0) : a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  const int64_t Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "gemm K mismatch: ", K, " vs ", Kb);
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "gemm out shape mismatch");
  // TMA: the contiguous dimension of every operand must span a multiple of
  // 16 bytes (N is the output's contiguous dimension)
  TORCH_CHECK(N % 8 == 0, "gemm N must be a multiple of 8");
  TORCH_CHECK((a_mn ? M : K) % 8 == 0, "gemm: A's contiguous dimension must be a multiple of 8");
  TORCH_CHECK((b_mn || K % 8 == 0), "gemm: B's contiguous dimension (K) must be a multiple of 8");
  if (epi == EPI_F32) {
    CHECK_DTYPE(out, at::kFloat);
  } else {
    CHECK_DTYPE(out, at::kBFloat16);
  }
  TORCH_CHECK(out.stride(0) % 8 == 0, "out row stride must be a multiple of 8 elements");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0, "out must be 16-byte aligned");

  const int dev = a.get_device();
  c10::cuda::CUDAGuard guard(dev);
  const int sms = num_sms(dev);

  Args args{};
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.num_kb = (int)((K + BK - 1) / BK);
  args.m_blocks = (int)((M + BM - 1) / BM);
  args.C = out.data_ptr();
  args.ldc = out.stride(0);
  args.st = status_ptr(dev);
  args.group_m = 16;

  if (bias.has_value() && bias->defined()) {
    CHECK_DTYPE((*bias), at::kBFloat16);
    TORCH_CHECK(bias->numel() >= N && bias->is_contiguous(), "bias must hold N contiguous values");
    TORCH_CHECK((reinterpret_cast<uintptr_t>(bias->data_ptr()) & 15) == 0, "bias must be 16-byte aligned");
    args.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  }
  if (epi == EPI_RESID || epi == EPI_DGELU) {
    TORCH_CHECK(aux.has_value() && aux->defined(), "epilogue needs aux");
    CHECK_DTYPE((*aux), at::kBFloat16);
    TORCH_CHECK(aux->size(0) == M && aux->size(1) == N && aux->stride(1) == 1 && aux->stride(0) % 8 == 0,
                "aux must be [M,N] with 16-byte aligned rows");
    args.aux = reinterpret_cast<const __nv_bfloat16*>(aux->data_ptr());
    args.ldaux = aux->stride(0);
  }
  if (bias_grad.has_value() && bias_grad->defined()) {
    TORCH_CHECK(epi == EPI_DGELU, "fused bias gradient is only available with the dGELU epilogue");
    CHECK_DTYPE((*bias_grad), at::kFloat);
    TORCH_CHECK(bias_grad->numel() == N && bias_grad->is_contiguous(), "bias_grad must be fp32 [N]");
    args.bias_grad = bias_grad->data_ptr<float>();
  }
  if (epi == EPI_BIAS_GELU) {
    TORCH_CHECK(out2.has_value() && out2->defined(), "gelu epilogue needs out2");
    CHECK_DTYPE((*out2), at::kBFloat16);
    TORCH_CHECK(out2->size(0) == M && out2->size(1) == N && out2->stride(1) == 1 && out2->stride(0) % 8 == 0,
                "out2 must be [M,N]");
    args.C2 = out2->data_ptr();
    args.ldc2 = out2->stride(0);
    TORCH_CHECK((reinterpret_cast<uintptr_t>(args.C2) & 15) == 0, "out2 must be 16-byte aligned");
  }

  // Small M with a long K and few output tiles (e.g. a data gradient into
  // d_model at a few thousand tokens): split K over 2-SM pair tiles into the
  // fp32 workspace, then convert with the bias / residual.
  if (allow_split_bf16 && (epi == EPI_BF16 || epi == EPI_RESID) && bn_force == 0 && !accumulate && splits == 0 &&
      splitk_bf16_enabled() && pair_enabled() && M >= 2 * BM && N % 8 == 0 && args.num_kb >= 32) {
    const long pair_tiles = (long)((M + 2 * BM - 1) / (2 * BM)) * ((N + 255) / 256);
    const int usms = pair_slots(dev);
    // 2-4 splits of at least 16 k-blocks each, scored by how well the units
    // fill whole waves of SM pairs, with a penalty per split for the fp32
    // reduce-add traffic
    int best_s = 0;
    double best = -1e9;
    for (int sp = 2; sp <= 4; ++sp) {
      if (args.num_kb / sp < 16) break;
      const double units = (double)pair_tiles * sp;
      const double eff = units / (std::ceil(units / usms) * usms);
      if (eff - 0.05 * sp > best) {
        best = eff - 0.05 * sp;
        best_s = sp;
      }
    }
    // Worth it (measured on the GPT-2 / ViT per-rank shapes) when the
    // unsplit 128 x 128 tiles fill their last wave poorly, or when K is so
    // long (>= 8192) that the workspace passes are noise next to the product;
    // otherwise the zeroing, reduce-add and conversion passes cost more than
    // the better wave fill gains.
    const long t128 = (long)args.m_blocks * ((N + 127) / 128);
    const double e128 = (double)t128 / (std::ceil((double)t128 / sms) * sms);
    if (pair_tiles < usms * 2L && best_s > 0 && (e128 < 0.75 || args.num_kb >= 128)) {
      cudaStream_t st0 = cur_stream();
      auto wst = torch::zeros({M, N}, torch::TensorOptions().dtype(torch::kFloat).device(out.device()));
      const float* ws = wst.data_ptr<float>();
      gemm_tc_impl(a, b, wst, a_mn, b_mn, EPI_F32, c10::nullopt, c10::nullopt, c10::nullopt, /*accumulate=*/true,
                   best_s, 0, c10::nullopt, c10::nullopt, c10::nullopt, 0, 0, 0, false);
      const long nvec = (long)M * (N / 8);
      const int grid = (int)std::min<long>((nvec + 255) / 256, (long)sms * 8);
      splitk_finalize_kernel<<<grid, 256, 0, st0>>>(ws, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                                    out.stride(0), args.bias, epi == EPI_RESID ? args.aux : nullptr,
                                                    args.ldaux, (int)M, (int)N);
      SCIRS_CHECK_LAUNCH();
      return;
    }
  }

  // Tile width: BN=256 unless BN=128 gives fewer waves for this shape.
  // Split-K (fp32 outputs only) turns a few large-K tiles into enough work
  // units to fill every SM.
  const bool can_split = (epi == EPI_F32);
  int BN = 256;
  {
    auto cost = [&](int bn) {
      long tiles = (long)args.m_blocks * ((N + bn - 1) / bn);
      long waves = (tiles + sms - 1) / sms;
      return waves * (bn + 48);
    };
    if (N <= 128 || (!can_split && cost(128) < cost(256))) BN = 128;
  }
  if (bn_force == 128 || bn_force == 256) BN = (int)bn_force;
  set_rope(args, epi, rope_cos, rope_sin, rope_S, rope_hd, rope_cols, N);
  TORCH_CHECK(epi != EPI_ROPE || (!a_mn && !b_mn && BN % rope_hd == 0), "RoPE epilogue: K-major operands, BN % hd == 0");
  // Pair mode (two SMs per 256 x 256 tile) when the tiles are wide and there
  // are enough of them to fill the GPU with pairs.
  // (fp32 weight gradients count their split-K work units: a long K splits
  // into enough units even when the output has few tiles)
  const long pair_tiles = (long)((M + 2 * BM - 1) / (2 * BM)) * ((N + 255) / 256);
  const long pair_units = can_split ? pair_tiles * std::max(1, std::min(16, args.num_kb / 4)) : pair_tiles;
  const bool pair = pair_enabled() && BN == 256 && bn_force != 128 && M >= 2 * BM && pair_units >= sms / 2;
  if (pair) args.m_blocks = (int)((M + 2 * BM - 1) / (2 * BM));
  const int usms = pair ? pair_slots(dev) : sms;  // scheduling slots: resident SM pairs in pair mode
  args.n_blocks = (int)((N + BN - 1) / BN);
  const long tiles = (long)args.m_blocks * args.n_blocks;

  int sp = 1;
  if (can_split) {
    if (splits > 0) {
      sp = (int)splits;
    } else if (tiles < 2L * usms) {
      // choose the split that fills whole waves best (mild penalty per split)
      const int max_sp = std::max(1, std::min(16, args.num_kb / 4));
      double best = -1e9;
      for (int s = 1; s <= max_sp; ++s) {
        const double units = (double)tiles * s;
        const double waves = std::ceil(units / usms);
        const double eff = units / (waves * usms);
        const double score = eff - 0.01 * s - (units < usms ? 0.5 : 0.0);
        if (score > best) {
          best = score;
          sp = s;
        }
      }
    }
    sp = std::max(1, std::min(sp, args.num_kb));
  }
  args.kb_per_split = (args.num_kb + sp - 1) / sp;
  sp = (args.num_kb + args.kb_per_split - 1) / args.kb_per_split;  // every split non-empty
  args.splits = sp;
  args.atomic_out = (epi == EPI_F32 && (accumulate || sp > 1)) ? 1 : 0;
  args.gelu_x2 = gelu_x2_enabled() ? 1 : 0;
  if (epi == EPI_F32 && sp > 1 && !accumulate) out.zero_();
  args.num_units = (int)(tiles * sp);
  const int grid = pair ? 2 * (int)std::min<long>(args.num_units, usms) : (int)std::min<long>(args.num_units, sms);

  // Operand maps (SWIZZLE_128B, 64-element inner boxes) and output maps
  // (32x32 bf16 or 32x16 fp32 boxes, SWIZZLE_64B, matching the staging slots).
  const uint64_t lda_b = (uint64_t)a.stride(0) * 2, ldb_b = (uint64_t)b.stride(0) * 2;
  Maps maps;
  maps.a = a_mn ? get_tmap(a.data_ptr(), (uint64_t)M, (uint64_t)K, lda_b, 64, 64)
                : get_tmap(a.data_ptr(), (uint64_t)K, (uint64_t)M, lda_b, 64, BM);
  maps.b = b_mn ? get_tmap(b.data_ptr(), (uint64_t)N, (uint64_t)K, ldb_b, 64, 64)
                : get_tmap(b.data_ptr(), (uint64_t)K, (uint64_t)N, ldb_b, 64, (uint32_t)(pair ? BN / 2 : BN));
  if (epi == EPI_F32) {
    maps.c = get_tmap(out.data_ptr(), (uint64_t)N, (uint64_t)M, (uint64_t)out.stride(0) * 4, 16, 32,
                      CU_TENSOR_MAP_DATA_TYPE_FLOAT32, CU_TENSOR_MAP_SWIZZLE_64B);
  } else {
    maps.c = get_tmap(out.data_ptr(), (uint64_t)N, (uint64_t)M, (uint64_t)out.stride(0) * 2, 32, 32,
                      CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, CU_TENSOR_MAP_SWIZZLE_64B);
  }
  maps.c2 = maps.c;
  if (epi == EPI_RESID || epi == EPI_DGELU) {  // aux operand, loaded by the epilogue via TMA
    maps.c2 = get_tmap(args.aux, (uint64_t)N, (uint64_t)M, (uint64_t)args.ldaux * 2, 32, 32,
                       CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, CU_TENSOR_MAP_SWIZZLE_64B);
  }
  if (epi == EPI_BIAS_GELU) {
    maps.c2 = get_tmap(args.C2, (uint64_t)N, (uint64_t)M, (uint64_t)args.ldc2 * 2, 32, 32,
                       CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, CU_TENSOR_MAP_SWIZZLE_64B);
  }

  cudaStream_t s = cur_stream();
  if (pair) launch_pair((int)a_mn, (int)b_mn, (int)epi, maps, args, grid, s);
  else if (BN == 256) launch_bn<256>((int)a_mn, (int)b_mn, (int)epi, maps, args, grid, s);
  else launch_bn<128>((int)a_mn, (int)b_mn, (int)epi, maps, args, grid, s);
}

}  // namespace scirs
