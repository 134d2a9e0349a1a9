// Native batch prefetcher for in-memory datasets (module scirs_b200._data).
//
// Worker threads gather the rows of each batch (in a seeded shuffled or
// sequential order) from the dataset's host arrays into a ring of pinned
// staging slots, so that the host->device copy of batch i+1 (issued
// asynchronously by the Python side from pinned memory) and the gather of
// batch i+2 both overlap the GPU step on batch i. Batches come out in order;
// a slot is reused only after the consumer releases it.
//
// Reference parity: scirs2-neural/src/data/dataloader.rs:18-168 (DataLoader
// over a Dataset with batch size, shuffle, drop_last, prefetch) and
// data/memory_pool.rs (reusable batch buffers); there in Rust on the host.
#include <torch/extension.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstring>
#include <mutex>
#include <random>
#include <thread>
#include <vector>

namespace scirs {

class BatchPrefetcher {
 public:
  BatchPrefetcher(std::vector<torch::Tensor> arrays, int64_t batch_size, int64_t num_slots, int64_t num_threads,
                  bool shuffle, int64_t seed, bool drop_last, bool pin)
      : arrays_(std::move(arrays)), bs_(batch_size), nslots_(num_slots), shuffle_(shuffle), seed_(seed),
        drop_last_(drop_last) {
    TORCH_CHECK(!arrays_.empty(), "need at least one array");
    TORCH_CHECK(batch_size > 0 && num_slots >= 2 && num_threads >= 1, "bad prefetcher sizes");
    n_ = arrays_[0].size(0);
    for (auto& a : arrays_) {
      TORCH_CHECK(a.device().is_cpu() && a.is_contiguous(), "arrays must be contiguous host tensors");
      TORCH_CHECK(a.size(0) == n_, "arrays must share their first dimension");
      row_bytes_.push_back(a.numel() == 0 ? 0 : a.nbytes() / n_);
    }
    for (int64_t s = 0; s < nslots_; ++s) {
      std::vector<torch::Tensor> bufs;
      for (auto& a : arrays_) {
        auto shape = a.sizes().vec();
        shape[0] = bs_;
        auto opts = torch::TensorOptions().dtype(a.scalar_type()).pinned_memory(pin);
        bufs.push_back(torch::empty(shape, opts));
      }
      slots_.push_back(std::move(bufs));
    }
    slot_state_.assign(nslots_, kFree);
    slot_batch_.assign(nslots_, -1);
    slot_rows_.assign(nslots_, 0);
    for (int64_t t = 0; t < num_threads; ++t) workers_.emplace_back([this] { work(); });
  }

  ~BatchPrefetcher() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& w : workers_) w.join();
  }

  int64_t num_batches() const { return drop_last_ ? n_ / bs_ : (n_ + bs_ - 1) / bs_; }

  // Start an epoch: new order (seed + epoch when shuffling), clear the ring.
  void start_epoch(int64_t epoch) {
    std::unique_lock<std::mutex> lk(mu_);
    cv_.wait(lk, [&] { return busy_ == 0; });
    order_.resize(n_);
    for (int64_t i = 0; i < n_; ++i) order_[i] = i;
    if (shuffle_) {
      std::mt19937_64 rng((uint64_t)seed_ * 1000003ull + (uint64_t)epoch);
      std::shuffle(order_.begin(), order_.end(), rng);
    }
    std::fill(slot_state_.begin(), slot_state_.end(), kFree);
    next_produce_ = 0;
    next_consume_ = 0;
    epoch_active_ = true;
    lk.unlock();
    cv_.notify_all();
  }

  // Wait for the next batch in order; returns (slot, rows, tensors) or
  // slot -1 at the end of the epoch. The tensors stay valid until release(slot).
  std::tuple<int64_t, int64_t, std::vector<torch::Tensor>> next() {
    std::unique_lock<std::mutex> lk(mu_);
    if (!epoch_active_ || next_consume_ >= num_batches()) return {-1, 0, {}};
    const int64_t b = next_consume_;
    int64_t slot = -1;
    cv_.wait(lk, [&] {
      for (int64_t s = 0; s < nslots_; ++s)
        if (slot_state_[s] == kReady && slot_batch_[s] == b) {
          slot = s;
          return true;
        }
      return stop_;
    });
    if (slot < 0) return {-1, 0, {}};
    slot_state_[slot] = kHeld;
    ++next_consume_;
    const int64_t rows = slot_rows_[slot];
    std::vector<torch::Tensor> out;
    for (auto& t : slots_[slot]) out.push_back(t.narrow(0, 0, rows));
    return {slot, rows, out};
  }

  void release(int64_t slot) {
    {
      std::lock_guard<std::mutex> lk(mu_);
      TORCH_CHECK(slot >= 0 && slot < nslots_ && slot_state_[slot] == kHeld, "slot is not held");
      slot_state_[slot] = kFree;
    }
    cv_.notify_all();
  }

 private:
  enum State { kFree = 0, kFilling = 1, kReady = 2, kHeld = 3 };

  void work() {
    while (true) {
      int64_t slot = -1, b = -1;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] {
          if (stop_) return true;
          if (!epoch_active_ || next_produce_ >= num_batches()) return false;
          // never run more than nslots batches ahead of the consumer
          if (next_produce_ >= next_consume_ + nslots_) return false;
          for (int64_t s = 0; s < nslots_; ++s)
            if (slot_state_[s] == kFree) return true;
          return false;
        });
        if (stop_) return;
        for (int64_t s = 0; s < nslots_; ++s)
          if (slot_state_[s] == kFree) {
            slot = s;
            break;
          }
        b = next_produce_++;
        slot_state_[slot] = kFilling;
        slot_batch_[slot] = b;
        ++busy_;
      }
      const int64_t r0 = b * bs_, rows = std::min(bs_, n_ - r0);
      for (size_t k = 0; k < arrays_.size(); ++k) {
        const char* src = static_cast<const char*>(arrays_[k].data_ptr());
        char* dst = static_cast<char*>(slots_[slot][k].data_ptr());
        const size_t rb = row_bytes_[k];
        for (int64_t i = 0; i < rows; ++i) std::memcpy(dst + i * rb, src + order_[r0 + i] * rb, rb);
      }
      {
        std::lock_guard<std::mutex> lk(mu_);
        slot_rows_[slot] = rows;
        slot_state_[slot] = kReady;
        --busy_;
      }
      cv_.notify_all();
    }
  }

  std::vector<torch::Tensor> arrays_;
  std::vector<size_t> row_bytes_;
  int64_t n_ = 0, bs_, nslots_;
  bool shuffle_;
  int64_t seed_;
  bool drop_last_;
  std::vector<std::vector<torch::Tensor>> slots_;
  std::vector<int> slot_state_;
  std::vector<int64_t> slot_batch_, slot_rows_;
  std::vector<int64_t> order_;
  int64_t next_produce_ = 0, next_consume_ = 0, busy_ = 0;
  bool epoch_active_ = false, stop_ = false;
  std::mutex mu_;
  std::condition_variable cv_;
  std::vector<std::thread> workers_;
};

void register_host_runtime(py::module& m);  // host_runtime.cpp

}  // namespace scirs

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "scirs_b200 native host runtime: batch prefetcher, task graph, scans, sort, lock-free ring";
  scirs::register_host_runtime(m);
  py::class_<scirs::BatchPrefetcher>(m, "BatchPrefetcher")
      .def(py::init<std::vector<torch::Tensor>, int64_t, int64_t, int64_t, bool, int64_t, bool, bool>(),
           py::arg("arrays"), py::arg("batch_size"), py::arg("num_slots") = 3, py::arg("num_threads") = 2,
           py::arg("shuffle") = true, py::arg("seed") = 0, py::arg("drop_last") = false, py::arg("pin") = true)
      .def("num_batches", &scirs::BatchPrefetcher::num_batches)
      .def("start_epoch", &scirs::BatchPrefetcher::start_epoch, py::call_guard<py::gil_scoped_release>())
      .def("next", &scirs::BatchPrefetcher::next, py::call_guard<py::gil_scoped_release>())
      .def("release", &scirs::BatchPrefetcher::release);
}
