// Shared device-side helpers for the sm_100a kernels of scirs_b200.
//
// Everything here is inline PTX for Blackwell (sm_100a): mbarriers, TMA tile
// copies (never with cluster multicast), tcgen05 MMA / TMEM management and the
// bounded-wait primitives that every spin loop in this library goes through.
// A wait that runs out of budget records an error in the caller's status word
// and returns false; no kernel here traps or spins forever.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace scirs {

// Sparsity of an attention call. Block lists (CSR, one row per CTA: the
// forward's 256-query CTAs list 128-key blocks, the backward's 128-key CTAs
// list query blocks) choose the tiles a CTA visits; the element predicate
// masks inside them. A pair (q, k) is allowed when it is in the union of the
// components given: the window [q - wl, q + wr], the global tokens (q < ng
// or k < ng) and the 128 x 128 block bitmap (causal masking comes on top).
struct AttnSparse {
  const int* ptr;
  const int* idx;
  const uint8_t* bmap;
  int bmap_ld;
  int wl, wr, ng;  // wl < 0: no window
};


// ---------------------------------------------------------------------------
// Device status word. Kernels record the FIRST error they meet here; the host
// reads it after a synchronize (see status_check in host_common.h).
// ---------------------------------------------------------------------------
struct DevStatus {
  unsigned int code;   // 0 = ok
  unsigned int where;  // site id (kernel-specific)
  unsigned int block;  // blockIdx.x of the reporter
  unsigned int info;   // extra detail (stage, peer rank, ...)
};

enum StatusCode : unsigned int {
  kStOk = 0,
  kStMbarTimeout = 1,   // an mbarrier wait ran out of budget
  kStPeerTimeout = 2,   // a wait on another GPU's flag ran out of budget
  kStBounds = 3,        // a bounds check failed (debug builds)
  kStBadArg = 4,
};

#ifdef __CUDACC__
__device__ __forceinline__ void report_status(DevStatus* st, unsigned code, unsigned where, unsigned info) {
  if (st != nullptr && atomicCAS(&st->code, 0u, code) == 0u) {
    st->where = where;
    st->block = blockIdx.x;
    st->info = info;
  }
}

// Bounds checks. Indices that come from user data (token ids, page tables)
// are always checked: an out-of-range value is recorded as kStBounds in the
// status word and the access is skipped (the host raises on the next
// check_status). Checks of internal index arithmetic compile in only with
// -DSCIRS_KCHECK (setup.py: SCIRS_KCHECK=1), for debug builds.
__device__ __forceinline__ bool input_in_range(long v, long n, DevStatus* st, unsigned where) {
  if (v >= 0 && v < n) return true;
  report_status(st, kStBounds, where, (unsigned)v);
  return false;
}
#ifdef SCIRS_KCHECK
#define SCIRS_KCHECK_IDX(v, n, st, where) ::scirs::input_in_range((long)(v), (long)(n), (st), (where))
#else
#define SCIRS_KCHECK_IDX(v, n, st, where) true
#endif

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Budget for intra-CTA pipeline waits. A healthy pipeline never waits more
// than a few microseconds; two seconds means the pipeline is broken.
constexpr uint64_t kMbarTimeoutNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t lane_id() {
  uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

__device__ __forceinline__ bool elect_one_sync() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, %1;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(pred)
      : "r"(0xffffffffu));
  return pred != 0;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase. `abort_flag` (shared memory, may be
// null) lets the other roles of a CTA stop waiting as soon as one role has
// given up. Returns false on timeout / abort.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, DevStatus* st, unsigned where,
                                          volatile int* abort_flag) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    #pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(addr, parity)) return true;
    if (abort_flag != nullptr && *abort_flag) return false;
    if (globaltimer_ns() - t0 > kMbarTimeoutNs) {
      report_status(st, kStMbarTimeout, where, parity);
      if (abort_flag != nullptr) *abort_flag = 1;
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor). Loads land in this CTA's shared memory and
// signal an mbarrier with complete_tx. No multicast variants exist in this
// library on purpose.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}

__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

__device__ __forceinline__ void tma_store_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

__device__ __forceinline__ void tma_store_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 / TMEM
// ---------------------------------------------------------------------------
// Allocate `ncols` TMEM columns (power of two >= 32). Warp-collective; the
// allocated base address is written to *smem_dst.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D(tmem) (+)= A(smem desc) * B(smem desc), kind::f16 (bf16 in, fp32 accum).
__device__ __forceinline__ void tc_mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D(tmem) (+)= A(tmem) * B(smem desc): A operand read from TMEM.
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread
// have completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Wait for this thread's TMEM loads, naming the 32 destination registers of
// the load being waited on as read-write operands: the compiler then cannot
// move any use (or copy) of them above the wait, which matters when another
// load is in flight while they are processed.
__device__ __forceinline__ void tc_wait_ld_regs(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Load 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Load 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Store 16 consecutive 32-bit columns into this thread's TMEM lane.
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// ---------------------------------------------------------------------------
// UMMA shared-memory matrix descriptor (64-bit), SWIZZLE_128B layouts.
//   bits [0,14)  start address >> 4
//   bits [16,30) leading-dimension byte offset >> 4
//   bits [32,46) stride-dimension byte offset >> 4
//   bits [46,48) descriptor version (1 on sm_100)
//   bits [49,52) base offset (0: atoms are 1024-byte aligned)
//   bits [61,64) layout: 2 = SWIZZLE_128B
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// The descriptor of an operand `bytes` further into the same swizzled tile: only
// the start-address field (low 14 bits, in 16-byte units) changes, and it cannot
// carry into the next field while the address stays inside shared memory, so a
// 32-bit add on the low word is enough (one instruction per MMA in the k loops).
__device__ __forceinline__ uint64_t desc_off(uint64_t d, uint32_t bytes) {
  return (d & 0xFFFFFFFF00000000ull) | (uint64_t)((uint32_t)d + (bytes >> 4));
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 accumulator.
//   [4,6) c_format=1 (F32); [7,10) a_format=1 (BF16); [10,13) b_format=1;
//   [15] a_major (1 = MN-major); [16] b_major; [17,23) N>>3; [24,29) M>>4.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn_major << 15) | ((uint32_t)b_mn_major << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------------------
// small numeric helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float warp_sum(float v) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Hardware tanh approximation (PTX tanh.approx.f32, sm_75+); max relative
// error ~2^-11, below bf16 resolution, so used for activations whose outputs
// are stored in bf16.
__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x via the PTX ex2.approx instruction (flush-to-zero; 2^-inf = 0).
__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x of two values in one MUFU instruction: the arguments are rounded to
// bf16 (round to nearest) and the results come back as packed bf16x2
// {lo: 2^lo, hi: 2^hi}; -inf gives 0.
__device__ __forceinline__ uint32_t ex2_bf16x2(float lo, float hi) {
  uint32_t in, out;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(in) : "f"(hi), "f"(lo));
  asm("ex2.approx.ftz.bf16x2 %0, %1;" : "=r"(out) : "r"(in));
  return out;
}

// GELU, tanh form: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))).
// The two constants are the definition of the approximation (Hendrycks &
// Gimpel 2016), not taken from any library.
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  float u = k0 * fmaf(k1 * x, x * x, x);
  return 0.5f * x * (1.f + tanh_fast(u));
}

// Packed fp32 pairs (Blackwell f32x2 instructions): one FFMA2 / FADD2 does
// the work of two scalar instructions.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// gelu_tanh of two packed fp32 values: the polynomial and the final
// 0.5 x (1 + t) in f32x2 instructions, the two tanh evaluations scalar.
__device__ __forceinline__ uint64_t gelu_tanh2(uint64_t x) {
  const uint64_t k0 = f2_pack(0.7978845608028654f, 0.7978845608028654f);
  const uint64_t k1 = f2_pack(0.044715f, 0.044715f);
  const uint64_t one = f2_pack(1.f, 1.f), half = f2_pack(0.5f, 0.5f);
  const uint64_t a = f2_fma(f2_mul(x, x), k1, one);  // 1 + k1 x^2
  float u0, u1;
  f2_unpack(f2_mul(f2_mul(x, a), k0), u0, u1);      // k0 (x + k1 x^3)
  const uint64_t t = f2_pack(tanh_fast(u0), tanh_fast(u1));
  const uint64_t hx = f2_mul(x, half);
  return f2_fma(hx, t, hx);
}

// d/dx of gelu_tanh.
__device__ __forceinline__ float gelu_tanh_grad(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  float x2 = x * x;
  float u = k0 * fmaf(k1 * x, x2, x);
  float t = tanh_fast(u);
  return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * k0 * fmaf(3.f * k1, x2, 1.f);
}

// gelu_tanh_grad of two packed fp32 values (f32x2 instructions except the
// two tanh evaluations):
// 0.5 (1 + t) + 0.5 x k0 (1 + 3 k1 x^2) (1 - t^2), t = tanh(k0 (x + k1 x^3)).
__device__ __forceinline__ uint64_t gelu_tanh_grad2(uint64_t x) {
  const uint64_t k0 = f2_pack(0.7978845608028654f, 0.7978845608028654f);
  const uint64_t k1 = f2_pack(0.044715f, 0.044715f), k13 = f2_pack(3.f * 0.044715f, 3.f * 0.044715f);
  const uint64_t one = f2_pack(1.f, 1.f), half = f2_pack(0.5f, 0.5f);
  const uint64_t xx = f2_mul(x, x);
  float u0, u1;
  f2_unpack(f2_mul(f2_mul(x, f2_fma(xx, k1, one)), k0), u0, u1);
  const float t0 = tanh_fast(u0), t1 = tanh_fast(u1);
  const uint64_t t = f2_pack(t0, t1), nt = f2_pack(-t0, -t1);
  const uint64_t c = f2_mul(f2_mul(x, half), f2_mul(k0, f2_fma(xx, k13, one)));  // 0.5 x k0 (1 + 3 k1 x^2)
  return f2_fma(c, f2_fma(nt, t, one), f2_fma(half, t, half));
}

// Warpgroup register reallocation (all 128 threads of a warpgroup execute
// the same instruction). The shares of all warpgroups must not exceed the
// registers the block was launched with (threads x registers per thread).
template <int N>
__device__ __forceinline__ void setmaxnreg_inc() {
  static_assert(N % 8 == 0 && N >= 24 && N <= 256, "setmaxnreg: multiple of 8 in [24, 256]");
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_dec() {
  static_assert(N % 8 == 0 && N >= 24 && N <= 256, "setmaxnreg: multiple of 8 in [24, 256]");
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// True when every pair of queries [q0, q1] x keys [k0, k1] is allowed, so a
// tile needs no element mask (block bitmap entries cover whole 128 x 128
// blocks; q0 / k0 are multiples of 64 / 128 and the ranges lie in one block).
__device__ __forceinline__ bool attn_block_full(const AttnSparse& a, int q0, int q1, int k0, int k1) {
  if (a.bmap == nullptr && a.wl < 0 && a.ng <= 0) return true;
  if (a.bmap != nullptr && a.bmap[(long)(q0 >> 7) * a.bmap_ld + (k0 >> 7)] != 0) return true;
  if (a.wl >= 0 && k0 >= q1 - a.wl && k1 <= q0 + a.wr) return true;
  return q1 < a.ng || k1 < a.ng;
}

__device__ __forceinline__ bool attn_allowed(const AttnSparse& a, int q, int k) {
  // union of the components that are present (none present: everything)
  if (a.bmap == nullptr && a.wl < 0 && a.ng <= 0) return true;
  if (a.wl >= 0 && k >= q - a.wl && k <= q + a.wr) return true;
  if (q < a.ng || k < a.ng) return true;
  return a.bmap != nullptr && a.bmap[(long)(q >> 7) * a.bmap_ld + (k >> 7)] != 0;
}

// The allowed positions of one row of a score block, as the union of at
// most two inclusive intervals [a0, b0] and [a1, b1] of block-relative
// indices. Built once per row and block, so that the element loop masks with
// two compares and a select per score, without branches or memory loads.
struct AttnSpan {
  int a0, b0, a1, b1;
};

__device__ __forceinline__ bool attn_span_has(const AttnSpan& m, int e) {
  return (e >= m.a0 && e <= m.b0) || (e >= m.a1 && e <= m.b1);
}

// Forward: keys k0 + e allowed for query q (k0 a multiple of 128): the key
// length and causal bound, then the pattern (all keys when the row is a
// global token or its 128 x 128 bitmap block is set; else the window and the
// global keys).
template <bool SPARSE>
__device__ __forceinline__ AttnSpan attn_keys_of_query(const AttnSparse& a, int q, int k0, int Sk, bool causal) {
  int hi = Sk - 1 - k0;
  if (causal) hi = min(hi, q - k0);
  AttnSpan m{0, hi, 1, 0};
  if (!SPARSE) return m;
  const bool none = a.bmap == nullptr && a.wl < 0 && a.ng <= 0;
  if (none || q < a.ng || (a.bmap != nullptr && a.bmap[(long)(q >> 7) * a.bmap_ld + (k0 >> 7)] != 0)) return m;
  m.a0 = a.wl >= 0 ? q - a.wl - k0 : 1;
  m.b0 = a.wl >= 0 ? min(q + a.wr - k0, hi) : 0;
  m.a1 = 0;
  m.b1 = min(a.ng - 1 - k0, hi);
  return m;
}

// Backward: queries q0 + e that see key k (q0 a multiple of the query block,
// which divides 128): q < S, q >= k when causal, nothing for k >= Sk; then
// the pattern (every query for a global key or a set bitmap block; else the
// window q in [k - wr, k + wl] and the global queries q < ng).
template <bool SPARSE>
__device__ __forceinline__ AttnSpan attn_queries_of_key(const AttnSparse& a, int k, int q0, int S, int Sk,
                                                        bool causal) {
  const int lo = causal ? k - q0 : 0;
  const int hi = k < Sk ? S - 1 - q0 : -1;
  AttnSpan m{lo, hi, 1, 0};
  if (!SPARSE) return m;
  const bool none = a.bmap == nullptr && a.wl < 0 && a.ng <= 0;
  if (none || k < a.ng || (a.bmap != nullptr && a.bmap[(long)(q0 >> 7) * a.bmap_ld + (k >> 7)] != 0)) return m;
  m.a0 = a.wl >= 0 ? max(k - a.wr - q0, lo) : 1;
  m.b0 = a.wl >= 0 ? min(k + a.wl - q0, hi) : 0;
  m.a1 = lo;
  m.b1 = min(a.ng - 1 - q0, hi);
  return m;
}

#endif  // __CUDACC__

}  // namespace scirs
