// In-kernel NVLink collectives over symmetric peer memory.
//
// Every rank owns one "symmetric" device buffer of the same size, mapped into
// every other rank's address space with CUDA IPC (handles exchanged over the
// process group by the Python side). Kernels here read and write peers'
// buffers directly (P2P loads/stores over NVLink 5 / NVSwitch) and
// synchronise with per-block epoch flags:
//
//   signal: __syncthreads; thread i < world stores `epoch` into peer i's flag
//           slot [barrier][block][my_rank] with st.release.sys
//   wait  : thread i < world spins (bounded by a globaltimer budget) with
//           ld.acquire.sys on my flag slot [barrier][block][i]; __syncthreads
//
// Block b of every rank works on the same slice of the payload, so the
// barriers are per block and no grid-wide synchronisation is needed. A wait
// that runs out of budget records kStPeerTimeout in the status word and the
// kernel finishes without hanging (its output is then invalid; the host
// raises when it reads the status word).
//
// Buffer layout (bytes): [ area0 | area1 | flags ]   area = data_cap / 2.
//   all-reduce : area0 holds the scaled bf16 inputs, area1 the reduced pieces
//   reduce-scat: area0 holds the scaled bf16 inputs
//   all-gather : area0 holds the gathered bf16 payload
//   Every kernel ends with an exit barrier and all kinds share one epoch
//   sequence per block, so consecutive collectives of any kind may reuse the
//   buffer safely.
//
// Reference parity: replaces the single-process simulations of the
// reference's distributed gradient primitives
// (scirs2-autograd/src/distributed/mod.rs:47-84 local averaging,
// scirs2-core/src/gpu/multi_gpu_sync.cu:18 "ring" inside one buffer,
// scirs2-core/src/gpu/multi_gpu_sync.cu:381,410 ZeRO partition/gather index
// math, scirs2-autograd/src/distributed_grad.rs:100-330 simulated ring and
// bucketing) with real cross-GPU collectives.
#include "host_common.h"

namespace scirs {
namespace comm {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 256;
constexpr int kBarriers = 3;  // phase barriers 0, 1 and the exit barrier 2
constexpr long kFlagBytes = (long)kBarriers * kMaxBlocks * kMaxRanks * 4;

struct Peers {
  char* base[kMaxRanks];
};

struct Args {
  Peers peers;
  int rank, world;
  long area_bytes;   // bytes of one data area
  long n;            // payload elements
  const float* in32;  // fp32 input (all-reduce / reduce-scatter)
  float* out32;       // fp32 output
  const __nv_bfloat16* in16;  // bf16 input (all-gather shard)
  __nv_bfloat16* out16;       // bf16 output (all-gather full)
  float scale;
  unsigned* epochs;  // local per-block counters [kMaxBlocks]
  DevStatus* st;
  long long timeout_ns;
};

__device__ __forceinline__ unsigned* flag_ptr(char* base, long area_bytes, int barrier, int block, int src) {
  return reinterpret_cast<unsigned*>(base + 2 * area_bytes) + ((barrier * kMaxBlocks + block) * kMaxRanks + src);
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Cross-rank barrier among the blocks with this blockIdx.x. Returns false
// (and records the status) if a peer did not arrive within the budget.
__device__ bool block_barrier(const Args& a, int barrier, unsigned epoch, volatile int* sfail) {
  __syncthreads();
  const int i = threadIdx.x;
  if (i < a.world) {
    __threadfence_system();
    st_release_sys(flag_ptr(a.peers.base[i], a.area_bytes, barrier, blockIdx.x, a.rank), epoch);
  }
  if (i < a.world) {
    const unsigned* f = flag_ptr(a.peers.base[a.rank], a.area_bytes, barrier, blockIdx.x, i);
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while ((int)(ld_acquire_sys(f) - epoch) < 0) {
      if ((++spins & 255u) == 0 && (long long)(globaltimer_ns() - t0) > a.timeout_ns) {
        report_status(a.st, kStPeerTimeout, 100 + barrier, (unsigned)i);
        *sfail = 1;
        break;
      }
    }
  }
  __syncthreads();
  return *sfail == 0;
}

__device__ __forceinline__ void load8f(const float* p, float* f) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
__device__ __forceinline__ void store8f(float* p, const float* f) {
  reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
}
__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 q;
  q.x = pack_bf16x2(f[0], f[1]);
  q.y = pack_bf16x2(f[2], f[3]);
  q.z = pack_bf16x2(f[4], f[5]);
  q.w = pack_bf16x2(f[6], f[7]);
  return q;
}
__device__ __forceinline__ void acc8(const uint4& q, float* f) {
  f[0] += bf16_lo(q.x); f[1] += bf16_hi(q.x);
  f[2] += bf16_lo(q.y); f[3] += bf16_hi(q.y);
  f[4] += bf16_lo(q.z); f[5] += bf16_hi(q.z);
  f[6] += bf16_lo(q.w); f[7] += bf16_hi(q.w);
}
__device__ __forceinline__ void unpack8(const uint4& q, float* f) {
  f[0] = bf16_lo(q.x); f[1] = bf16_hi(q.x);
  f[2] = bf16_lo(q.y); f[3] = bf16_hi(q.y);
  f[4] = bf16_lo(q.z); f[5] = bf16_hi(q.z);
  f[6] = bf16_lo(q.w); f[7] = bf16_hi(q.w);
}

// Slice of the payload (in 8-element vectors) owned by this block, and the
// piece of that slice owned by rank r.
__device__ __forceinline__ void block_slice(long nvec, int world, long& v0, long& v1) {
  const long per = ((nvec + gridDim.x - 1) / gridDim.x + world - 1) / world * world;
  v0 = min(nvec, (long)blockIdx.x * per);
  v1 = min(nvec, v0 + per);
}
__device__ __forceinline__ void piece(long v0, long v1, int world, int r, long& p0, long& p1) {
  const long per = (v1 - v0 + world - 1) / world;
  p0 = min(v1, v0 + r * per);
  p1 = min(v1, p0 + per);
}

// Memory-level parallelism: every thread keeps kU independent 16-byte vectors
// in flight per step (phase 2 keeps one vector per peer in flight instead),
// and blocks are kept small in registers (<= 64) so they can co-reside with
// a persistent GEMM CTA while overlapping the backward pass.
constexpr int kU = 4;
constexpr int kCommThreads = 256;

// ---------------------------------------------------------------------------
// All-reduce (sum * scale), fp32 in -> fp32 out, bf16 on the wire.
// Two-shot: publish scaled bf16 copy; reduce own piece from all peers into
// area1; gather every reduced piece. Every rank ends with bit-identical output.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kCommThreads, 4) allreduce_kernel(const Args a) {
  __shared__ volatile int sfail;
  if (threadIdx.x == 0) sfail = 0;
  const unsigned epoch = a.epochs[blockIdx.x] + 1;
  const long nvec = a.n / 8;
  const long bd = blockDim.x;
  long v0, v1;
  block_slice(nvec, a.world, v0, v1);
  uint4* my_in = reinterpret_cast<uint4*>(a.peers.base[a.rank]);
  // phase 1: scale + cast + publish
  for (long base = v0 + threadIdx.x; base < v1; base += bd * kU) {
    float f[kU][8];
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (base + u * bd < v1) load8f(a.in32 + (base + u * bd) * 8, f[u]);
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      if (base + u * bd < v1) {
#pragma unroll
        for (int e = 0; e < 8; ++e) f[u][e] *= a.scale;
        my_in[base + u * bd] = pack8(f[u]);
      }
    }
  }
  bool ok = block_barrier(a, 0, epoch, &sfail);
  // phase 2: reduce my piece (one load per peer in flight per vector)
  long p0, p1;
  piece(v0, v1, a.world, a.rank, p0, p1);
  if (ok) {
    uint4* my_out = reinterpret_cast<uint4*>(a.peers.base[a.rank] + a.area_bytes);
    for (long v = p0 + threadIdx.x; v < p1; v += bd) {
      uint4 x[kMaxRanks];
#pragma unroll
      for (int k = 0; k < kMaxRanks; ++k)
        if (k < a.world) x[k] = __ldcg(reinterpret_cast<const uint4*>(a.peers.base[(a.rank + k) % a.world]) + v);
      float f[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
      for (int k = 0; k < kMaxRanks; ++k)
        if (k < a.world) acc8(x[k], f);
      my_out[v] = pack8(f);
    }
    ok = block_barrier(a, 1, epoch, &sfail);
  }
  // phase 3: gather every reduced piece (own included, for bit-identical results)
  if (ok) {
    const long per = (v1 - v0 + a.world - 1) / a.world;
    for (long base = v0 + threadIdx.x; base < v1; base += bd * kU) {
      uint4 x[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const long v = base + u * bd;
        if (v < v1) {
          const int src = (int)((v - v0) / per);
          x[u] = __ldcg(reinterpret_cast<const uint4*>(a.peers.base[src] + a.area_bytes) + v);
        }
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const long v = base + u * bd;
        if (v < v1) {
          float f[8];
          unpack8(x[u], f);
          store8f(a.out32 + v * 8, f);
        }
      }
    }
  }
  __syncthreads();
  // exit barrier: every peer is done reading this call's buffers, so the next
  // collective (of any kind) may overwrite them
  if (sfail == 0) block_barrier(a, 2, epoch, &sfail);
  if (threadIdx.x == 0) a.epochs[blockIdx.x] = epoch;
}

// ---------------------------------------------------------------------------
// Reduce-scatter (sum * scale): fp32 full input -> fp32 shard output.
// Rank r's shard is elements [r*n/world, (r+1)*n/world).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kCommThreads, 4) reduce_scatter_kernel(const Args a) {
  __shared__ volatile int sfail;
  if (threadIdx.x == 0) sfail = 0;
  const unsigned epoch = a.epochs[blockIdx.x] + 1;
  const long area = 0;
  const long bd = blockDim.x;
  const long shard_vec = a.n / 8 / a.world;
  // Block b handles vectors [b*per, ...) of every shard.
  const long per = (shard_vec + gridDim.x - 1) / gridDim.x;
  const long s0 = min(shard_vec, (long)blockIdx.x * per), s1 = min(shard_vec, s0 + per);
  uint4* my_in = reinterpret_cast<uint4*>(a.peers.base[a.rank] + area);
  const long span = s1 - s0;
  // phase 1: publish the block's slice of every shard (scaled, bf16)
  for (long base = threadIdx.x; base < span * a.world; base += bd * kU) {
    float f[kU][8];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const long t = base + u * bd;
      if (t < span * a.world) load8f(a.in32 + ((t / span) * shard_vec + s0 + t % span) * 8, f[u]);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const long t = base + u * bd;
      if (t < span * a.world) {
#pragma unroll
        for (int e = 0; e < 8; ++e) f[u][e] *= a.scale;
        my_in[(t / span) * shard_vec + s0 + t % span] = pack8(f[u]);
      }
    }
  }
  const bool ok = block_barrier(a, 0, epoch, &sfail);
  if (ok) {
    const long off = (long)a.rank * shard_vec;
    for (long v = s0 + threadIdx.x; v < s1; v += bd) {
      uint4 x[kMaxRanks];
#pragma unroll
      for (int k = 0; k < kMaxRanks; ++k)
        if (k < a.world)
          x[k] = __ldcg(reinterpret_cast<const uint4*>(a.peers.base[(a.rank + k) % a.world] + area) + off + v);
      float f[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
      for (int k = 0; k < kMaxRanks; ++k)
        if (k < a.world) acc8(x[k], f);
      store8f(a.out32 + v * 8, f);
    }
  }
  __syncthreads();
  if (sfail == 0) block_barrier(a, 2, epoch, &sfail);
  if (threadIdx.x == 0) a.epochs[blockIdx.x] = epoch;
}

// ---------------------------------------------------------------------------
// All-gather: bf16 shard in -> bf16 full output. Push model: every rank
// stores its shard straight into every peer's buffer, then one barrier.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kCommThreads, 4) allgather_kernel(const Args a) {
  __shared__ volatile int sfail;
  if (threadIdx.x == 0) sfail = 0;
  const unsigned epoch = a.epochs[blockIdx.x] + 1;
  const long area = 0;
  const long bd = blockDim.x;
  const long shard_vec = a.n / 8 / a.world;
  const long per = (shard_vec + gridDim.x - 1) / gridDim.x;
  const long s0 = min(shard_vec, (long)blockIdx.x * per), s1 = min(shard_vec, s0 + per);
  const long off = (long)a.rank * shard_vec;
  const uint4* src = reinterpret_cast<const uint4*>(a.in16);
  for (long base = s0 + threadIdx.x; base < s1; base += bd * kU) {
    uint4 q[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u)
      if (base + u * bd < s1) q[u] = src[base + u * bd];
    for (int k = 0; k < a.world; ++k) {
      uint4* dst = reinterpret_cast<uint4*>(a.peers.base[(a.rank + k) % a.world] + area) + off;
#pragma unroll
      for (int u = 0; u < kU; ++u)
        if (base + u * bd < s1) dst[base + u * bd] = q[u];
    }
  }
  const bool ok = block_barrier(a, 0, epoch, &sfail);
  if (ok && a.out16 != nullptr) {
    const uint4* full = reinterpret_cast<const uint4*>(a.peers.base[a.rank] + area);
    uint4* out = reinterpret_cast<uint4*>(a.out16);
    const long span = s1 - s0;
    for (long base = threadIdx.x; base < span * a.world; base += bd * kU) {
      uint4 x[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const long t = base + u * bd;
        if (t < span * a.world) x[u] = __ldcg(full + (t / span) * shard_vec + s0 + t % span);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const long t = base + u * bd;
        if (t < span * a.world) out[(t / span) * shard_vec + s0 + t % span] = x[u];
      }
    }
  }
  __syncthreads();
  if (sfail == 0) block_barrier(a, 2, epoch, &sfail);
  if (threadIdx.x == 0) a.epochs[blockIdx.x] = epoch;
}

// Fault-injection helper for tests: waits on a flag nothing ever sets, with
// the same bounded wait as the collectives, so the timeout path and the
// status word can be exercised on a single GPU without any hang.
__global__ void timeout_probe_kernel(const unsigned* flag, DevStatus* st, long long timeout_ns, int* out) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  int result = 0;
  while (ld_acquire_sys(flag) == 0u) {
    if ((++spins & 255u) == 0 && (long long)(globaltimer_ns() - t0) > timeout_ns) {
      report_status(st, kStPeerTimeout, 999, 0);
      result = 1;
      break;
    }
  }
  *out = result;
}

}  // namespace comm

// ===========================================================================
// host side
// ===========================================================================
namespace {
struct CommState {
  int rank = 0, world = 1, device = 0;
  long area_bytes = 0;
  char* local = nullptr;
  comm::Peers peers{};
  unsigned* epochs_ar = nullptr;
  unsigned* epochs_rs = nullptr;
  unsigned* epochs_ag = nullptr;
  std::vector<char*> opened;
};
std::unordered_map<int64_t, CommState> g_comms;
int64_t g_next_id = 1;
std::mutex g_mu;
}  // namespace

// Allocate this rank's symmetric buffer (2 data areas of area_bytes + flags)
// and return (comm id, IPC handle bytes).
std::tuple<int64_t, py::bytes> comm_create(int64_t device, int64_t rank, int64_t world, int64_t area_bytes) {
  TORCH_CHECK(world >= 1 && world <= comm::kMaxRanks, "world size must be 1..8");
  TORCH_CHECK(area_bytes % 256 == 0, "area_bytes must be a multiple of 256");
  c10::cuda::CUDAGuard guard((int)device);
  CommState cs;
  cs.rank = (int)rank;
  cs.world = (int)world;
  cs.device = (int)device;
  cs.area_bytes = area_bytes;
  const size_t total = 2 * area_bytes + comm::kFlagBytes;
  SCIRS_CHECK_CUDA(cudaMalloc(&cs.local, total));
  SCIRS_CHECK_CUDA(cudaMemset(cs.local, 0, total));
  SCIRS_CHECK_CUDA(cudaMalloc(&cs.epochs_ar, 3 * comm::kMaxBlocks * sizeof(unsigned)));
  SCIRS_CHECK_CUDA(cudaMemset(cs.epochs_ar, 0, 3 * comm::kMaxBlocks * sizeof(unsigned)));
  cs.epochs_rs = cs.epochs_ar + comm::kMaxBlocks;
  cs.epochs_ag = cs.epochs_rs + comm::kMaxBlocks;
  SCIRS_CHECK_CUDA(cudaDeviceSynchronize());
  cudaIpcMemHandle_t h;
  SCIRS_CHECK_CUDA(cudaIpcGetMemHandle(&h, cs.local));
  std::lock_guard<std::mutex> lk(g_mu);
  const int64_t id = g_next_id++;
  cs.peers.base[cs.rank] = cs.local;
  g_comms[id] = cs;
  return {id, py::bytes(reinterpret_cast<const char*>(&h), sizeof(h))};
}

// Open the peers' handles (index = rank; own entry ignored).
void comm_open_peers(int64_t id, std::vector<py::bytes> handles) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_comms.find(id);
  TORCH_CHECK(it != g_comms.end(), "unknown comm id");
  CommState& cs = it->second;
  TORCH_CHECK((int)handles.size() == cs.world, "need one handle per rank");
  c10::cuda::CUDAGuard guard(cs.device);
  for (int r = 0; r < cs.world; ++r) {
    if (r == cs.rank) continue;
    std::string s = handles[r];
    TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "bad handle size");
    cudaIpcMemHandle_t h;
    memcpy(&h, s.data(), sizeof(h));
    void* p = nullptr;
    SCIRS_CHECK_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    cs.peers.base[r] = reinterpret_cast<char*>(p);
    cs.opened.push_back(reinterpret_cast<char*>(p));
  }
}

void comm_destroy(int64_t id) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_comms.find(id);
  if (it == g_comms.end()) return;
  CommState& cs = it->second;
  c10::cuda::CUDAGuard guard(cs.device);
  cudaDeviceSynchronize();
  for (char* p : cs.opened) cudaIpcCloseMemHandle(p);
  cudaFree(cs.local);
  cudaFree(cs.epochs_ar);
  g_comms.erase(it);
}

static comm::Args make_args(const CommState& cs, long n, double timeout_s) {
  comm::Args a{};
  a.peers = cs.peers;
  a.rank = cs.rank;
  a.world = cs.world;
  a.area_bytes = cs.area_bytes;
  a.n = n;
  a.st = status_ptr(cs.device);
  a.timeout_ns = (long long)(timeout_s * 1e9);
  return a;
}

static CommState& get_cs(int64_t id) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_comms.find(id);
  TORCH_CHECK(it != g_comms.end(), "unknown comm id");
  return it->second;
}

static int pick_blocks(long nvec_total, int world, int64_t blocks) {
  if (blocks > 0) return (int)std::min<int64_t>(blocks, comm::kMaxBlocks);
  // at least kU vectors per thread per block; up to two blocks per SM for
  // large payloads (the blocks are small enough to co-reside with a GEMM CTA)
  long b = (nvec_total + (long)comm::kCommThreads * comm::kU - 1) / ((long)comm::kCommThreads * comm::kU);
  return (int)std::max<long>(1, std::min<long>(b, comm::kMaxBlocks));
}

// out32 = scale * sum_over_ranks(in32); in/out fp32 contiguous, may alias.
void comm_allreduce(int64_t id, torch::Tensor in32, torch::Tensor out32, double scale, int64_t blocks,
                    double timeout_s) {
  CommState& cs = get_cs(id);
  CHECK_DTYPE(in32, at::kFloat);
  CHECK_DTYPE(out32, at::kFloat);
  CHECK_CONTIG(in32);
  CHECK_CONTIG(out32);
  const long n = in32.numel();
  TORCH_CHECK(out32.numel() == n, "size mismatch");
  TORCH_CHECK(n % 8 == 0, "all-reduce payload must be a multiple of 8 elements");
  TORCH_CHECK(n * 2 <= cs.area_bytes, "payload larger than the symmetric buffer area");
  comm::Args a = make_args(cs, n, timeout_s);
  a.in32 = in32.data_ptr<float>();
  a.out32 = out32.data_ptr<float>();
  a.scale = (float)scale;
  a.epochs = cs.epochs_ar;
  c10::cuda::CUDAGuard guard(cs.device);
  const int nb = pick_blocks(n / 8, cs.world, blocks);
  comm::allreduce_kernel<<<nb, comm::kCommThreads, 0, cur_stream()>>>(a);
  SCIRS_CHECK_LAUNCH();
}

// out32 (shard, n/world) = scale * sum_over_ranks(in32[rank shard]).
void comm_reduce_scatter(int64_t id, torch::Tensor in32, torch::Tensor out32, double scale, int64_t blocks,
                         double timeout_s) {
  CommState& cs = get_cs(id);
  CHECK_DTYPE(in32, at::kFloat);
  CHECK_DTYPE(out32, at::kFloat);
  CHECK_CONTIG(in32);
  CHECK_CONTIG(out32);
  const long n = in32.numel();
  TORCH_CHECK(n % (8L * cs.world) == 0, "reduce-scatter payload must be a multiple of 8*world");
  TORCH_CHECK(out32.numel() == n / cs.world, "out must hold one shard");
  TORCH_CHECK(n * 2 <= cs.area_bytes, "payload larger than the symmetric buffer area");
  comm::Args a = make_args(cs, n, timeout_s);
  a.in32 = in32.data_ptr<float>();
  a.out32 = out32.data_ptr<float>();
  a.scale = (float)scale;
  a.epochs = cs.epochs_ar;  // one epoch sequence per block shared by every collective kind
  c10::cuda::CUDAGuard guard(cs.device);
  const int nb = pick_blocks(n / 8 / cs.world, cs.world, blocks);
  comm::reduce_scatter_kernel<<<nb, comm::kCommThreads, 0, cur_stream()>>>(a);
  SCIRS_CHECK_LAUNCH();
}

// out16 (full, n) = concat over ranks of in16 (shard, n/world).
void comm_allgather(int64_t id, torch::Tensor in16, torch::Tensor out16, int64_t blocks, double timeout_s) {
  CommState& cs = get_cs(id);
  CHECK_DTYPE(in16, at::kBFloat16);
  CHECK_DTYPE(out16, at::kBFloat16);
  CHECK_CONTIG(in16);
  CHECK_CONTIG(out16);
  const long n = out16.numel();
  TORCH_CHECK(n % (8L * cs.world) == 0, "all-gather payload must be a multiple of 8*world");
  TORCH_CHECK(in16.numel() == n / cs.world, "in must hold one shard");
  TORCH_CHECK(n * 2 <= cs.area_bytes, "payload larger than the symmetric buffer area");
  comm::Args a = make_args(cs, n, timeout_s);
  a.in16 = reinterpret_cast<const __nv_bfloat16*>(in16.data_ptr());
  a.out16 = reinterpret_cast<__nv_bfloat16*>(out16.data_ptr());
  a.epochs = cs.epochs_ar;
  c10::cuda::CUDAGuard guard(cs.device);
  const int nb = pick_blocks(n / 8 / cs.world, cs.world, blocks);
  comm::allgather_kernel<<<nb, comm::kCommThreads, 0, cur_stream()>>>(a);
  SCIRS_CHECK_LAUNCH();
}

// Runs a bounded wait on a flag that is never set; returns the status word
// the kernel left behind. Used by the failure-detection tests.
std::vector<int64_t> comm_timeout_probe(int64_t device, double timeout_s) {
  c10::cuda::CUDAGuard guard((int)device);
  auto opts = torch::TensorOptions().device(torch::kCUDA, device);
  auto flag = torch::zeros({1}, opts.dtype(torch::kInt32));
  auto out = torch::full({1}, -1, opts.dtype(torch::kInt32));
  status_read_and_clear((int)device);
  comm::timeout_probe_kernel<<<1, 1, 0, cur_stream()>>>(reinterpret_cast<const unsigned*>(flag.data_ptr()),
                                                        status_ptr((int)device), (long long)(timeout_s * 1e9),
                                                        out.data_ptr<int>());
  SCIRS_CHECK_LAUNCH();
  auto st = status_read_and_clear((int)device);
  st.push_back(out.item<int>());
  return st;
}

}  // namespace scirs
