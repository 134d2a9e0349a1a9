#include "host_common.h"

#include <cudaTypedefs.h>

namespace scirs {

namespace {
std::mutex g_mu;
DevStatus* g_status[64] = {nullptr};
int g_sms[64] = {0};
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    SCIRS_CHECK_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && fn != nullptr, "cuTensorMapEncodeTiled not available");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  return g_encode;
}
}  // namespace

DevStatus* status_ptr(int device) {
  TORCH_CHECK(device >= 0 && device < 64, "bad device");
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_status[device] == nullptr) {
    c10::cuda::CUDAGuard guard(device);
    void* p = nullptr;
    SCIRS_CHECK_CUDA(cudaMalloc(&p, sizeof(DevStatus)));
    SCIRS_CHECK_CUDA(cudaMemset(p, 0, sizeof(DevStatus)));
    SCIRS_CHECK_CUDA(cudaDeviceSynchronize());
    g_status[device] = reinterpret_cast<DevStatus*>(p);
  }
  return g_status[device];
}

std::vector<int64_t> status_read_and_clear(int device) {
  DevStatus* p = status_ptr(device);
  c10::cuda::CUDAGuard guard(device);
  DevStatus h;
  SCIRS_CHECK_CUDA(cudaDeviceSynchronize());
  SCIRS_CHECK_CUDA(cudaMemcpy(&h, p, sizeof(h), cudaMemcpyDeviceToHost));
  SCIRS_CHECK_CUDA(cudaMemset(p, 0, sizeof(DevStatus)));
  SCIRS_CHECK_CUDA(cudaDeviceSynchronize());
  return {(int64_t)h.code, (int64_t)h.where, (int64_t)h.block, (int64_t)h.info};
}

int num_sms(int device) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_sms[device] == 0) {
    int v = 0;
    SCIRS_CHECK_CUDA(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device));
    g_sms[device] = v;
  }
  return g_sms[device];
}

CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dtype, uint64_t inner, uint64_t outer,
                         uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                         CUtensorMapSwizzle swizzle) {
  TORCH_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base address must be 16-byte aligned");
  TORCH_CHECK(row_stride_bytes % 16 == 0, "TMA row stride must be a multiple of 16 bytes, got ", row_stride_bytes);
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(&m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with code ", (int)r, " (inner=", inner,
              " outer=", outer, " stride=", row_stride_bytes, " box=", box_inner, "x", box_outer, ")");
  return m;
}

}  // namespace scirs
