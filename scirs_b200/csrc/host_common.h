// Host-side helpers shared by the extension's launchers: argument checks,
// TMA tensor-map encoding (through the driver entry point, so the extension
// does not need to link libcuda) and the per-device status word.
#pragma once

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>
#include <string>
#include <unordered_map>

#include "common.cuh"

#define SCIRS_CHECK_CUDA(expr)                                                                       \
  do {                                                                                               \
    cudaError_t _e = (expr);                                                                         \
    TORCH_CHECK(_e == cudaSuccess, "CUDA error ", cudaGetErrorString(_e), " at ", __FILE__, ":", __LINE__); \
  } while (0)

#define SCIRS_CHECK_LAUNCH() SCIRS_CHECK_CUDA(cudaGetLastError())

#define CHECK_CUDA_TENSOR(t) TORCH_CHECK((t).is_cuda(), #t " must be a CUDA tensor")
#define CHECK_DTYPE(t, dt) TORCH_CHECK((t).scalar_type() == (dt), #t " has wrong dtype ", (t).scalar_type())
#define CHECK_CONTIG(t) TORCH_CHECK((t).is_contiguous(), #t " must be contiguous")

namespace scirs {

// Per-device status word (4 x u32, see DevStatus). Allocated on first use.
DevStatus* status_ptr(int device);
// Reads and clears the status word of `device` (synchronizes the device).
std::vector<int64_t> status_read_and_clear(int device);

int num_sms(int device);

// Encode a 2-D tiled tensor map. `inner` is the contiguous extent, `outer`
// the row count, `row_stride_bytes` the distance between rows.
CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, uint64_t inner, uint64_t outer,
                         uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle);

inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

}  // namespace scirs

#include <set>

namespace scirs {
// Set a kernel's max dynamic shared memory once per device (keeps the call
// out of later launches, e.g. while a CUDA graph is being captured).
inline void set_max_smem(const void* kern, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  SCIRS_CHECK_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  if (done.count({kern, dev})) return;
  SCIRS_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.insert({kern, dev});
}
// Attention sparsity arguments from optional tensors (attention_fwd_sm100.cu).
AttnSparse attn_sparse_args(const c10::optional<torch::Tensor>& ptr, const c10::optional<torch::Tensor>& idx,
                            const c10::optional<torch::Tensor>& bmap, int64_t wl, int64_t wr, int64_t ng,
                            int64_t rows);

}  // namespace scirs
