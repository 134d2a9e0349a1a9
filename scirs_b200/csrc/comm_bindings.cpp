// Python bindings of the NVLink collective kernels (module scirs_b200._comm).
#include "host_common.h"

namespace scirs {
std::tuple<int64_t, py::bytes> comm_create(int64_t device, int64_t rank, int64_t world, int64_t area_bytes);
void comm_open_peers(int64_t id, std::vector<py::bytes> handles);
void comm_destroy(int64_t id);
void comm_allreduce(int64_t id, torch::Tensor in32, torch::Tensor out32, double scale, int64_t blocks,
                    double timeout_s, int64_t algo);
void comm_allreduce_nvls(int64_t id, torch::Tensor buf, int64_t mc_addr, double scale, int64_t blocks,
                         double timeout_s);
void comm_reduce_scatter_nvls(int64_t id, torch::Tensor full, int64_t mc_addr, torch::Tensor shard, double scale,
                              int64_t blocks, double timeout_s);
void comm_allgather_nvls(int64_t id, torch::Tensor shard, torch::Tensor full, int64_t mc_addr, int64_t blocks,
                         double timeout_s);
void comm_reduce_scatter(int64_t id, torch::Tensor in32, torch::Tensor out32, double scale, int64_t blocks,
                         double timeout_s);
void comm_allgather(int64_t id, torch::Tensor in16, torch::Tensor out16, int64_t blocks, double timeout_s);
std::vector<int64_t> comm_timeout_probe(int64_t device, double timeout_s);
std::tuple<int64_t, py::bytes> sym_create(int64_t device, int64_t rank, int64_t world, int64_t bytes);
void sym_open(int64_t id, std::vector<py::bytes> handles);
torch::Tensor sym_tensor(int64_t id);
std::vector<int64_t> sym_ptrs(int64_t id);
void sym_destroy(int64_t id);
void peer_copy(std::vector<int64_t> dsts, int64_t src, int64_t nbytes);
}  // namespace scirs

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "scirs_b200 in-kernel NVLink collectives";
  m.def("create", &scirs::comm_create);
  m.def("open_peers", &scirs::comm_open_peers);
  m.def("destroy", &scirs::comm_destroy);
  m.def("allreduce", &scirs::comm_allreduce, py::arg("id"), py::arg("in32"), py::arg("out32"), py::arg("scale"),
        py::arg("blocks"), py::arg("timeout_s"), py::arg("algo") = 0);
  m.def("allreduce_nvls", &scirs::comm_allreduce_nvls);
  m.def("reduce_scatter", &scirs::comm_reduce_scatter);
  m.def("reduce_scatter_nvls", &scirs::comm_reduce_scatter_nvls);
  m.def("allgather_nvls", &scirs::comm_allgather_nvls);
  m.def("allgather", &scirs::comm_allgather);
  m.def("timeout_probe", &scirs::comm_timeout_probe);
  m.def("sym_create", &scirs::sym_create);
  m.def("sym_open", &scirs::sym_open);
  m.def("sym_tensor", &scirs::sym_tensor);
  m.def("sym_ptrs", &scirs::sym_ptrs);
  m.def("sym_destroy", &scirs::sym_destroy);
  m.def("peer_copy", &scirs::peer_copy);
  m.def("status_read_and_clear", &scirs::status_read_and_clear);
}
