// Native host-parallel runtime (part of module scirs_b200._data).
//
//  * TaskGraphCore: a DAG of named tasks run by a dataflow scheduler on a
//    pool of native threads. A task becomes ready the moment its last
//    dependency finishes (no level-by-level barrier); a failed task marks
//    every transitive dependent "skipped"; in strict mode the first failure
//    stops new launches. The task bodies are Python callables: a worker
//    takes the interpreter lock only around the call, so bodies that release
//    it (tensor ops, I/O) run concurrently.
//  * parallel_for: indices 0..n-1 handed out through one atomic counter to a
//    set of native threads (dynamic scheduling for uneven work).
//  * scans over contiguous host tensors (sum / prod / min / max, inclusive or
//    exclusive, and a segmented sum): the three-phase blocked algorithm
//    (chunk-local scan in parallel, scan of the chunk totals, carry added in
//    parallel), O(n) work and O(n / T + T) span on T threads.
//  * parallel_sort: stable sort of a 1-D host tensor returning values and
//    indices (chunks sorted in parallel, then rounds of pairwise merges run
//    in parallel), NaN ordered above every number as torch.sort does.
//  * MpmcRing: the bounded multi-producer / multi-consumer lock-free queue
//    of D. Vyukov (one sequence number per cell, producers and consumers
//    each claim a position with a compare-and-swap), holding int64 values;
//    ring_stress drives it from native threads and checks that every value
//    arrives exactly once.
//  * AtomicCounter: a 64-bit counter on std::atomic.
//
// Reference parity: scirs2-core/src/distributed/task_graph.rs:70-613
// (TaskGraph add_task / execute / execute_partial / execution_order /
// execution_levels), parallel_scan.rs:50-427 (prefix sum / scan / min / max /
// segmented sum), par_iter.rs:72-475 (par_map ... par_sort), lock_free.rs:
// 55-496 (lock-free stack / queue / counter); there in Rust on OS threads.
#include <torch/extension.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <deque>
#include <functional>
#include <limits>
#include <memory>
#include <mutex>
#include <numeric>
#include <string>
#include <thread>
#include <type_traits>
#include <unordered_map>
#include <vector>

namespace py = pybind11;

namespace scirs {

namespace {

int resolve_threads(int64_t n_threads, int64_t work_items) {
  int64_t t = n_threads > 0 ? n_threads : std::max(1u, std::thread::hardware_concurrency());
  t = std::min<int64_t>(t, std::max<int64_t>(1, work_items));
  return static_cast<int>(t);
}

// Runs f(tid) on T threads (the caller's thread is tid 0) and joins them.
void run_threads(int T, const std::function<void(int)>& f) {
  std::vector<std::thread> ts;
  ts.reserve(T > 0 ? T - 1 : 0);
  for (int t = 1; t < T; ++t) ts.emplace_back(f, t);
  f(0);
  for (auto& t : ts) t.join();
}

}  // namespace

// ---------------------------------------------------------------------------
// Task graph
// ---------------------------------------------------------------------------

class TaskGraphCore {
 public:
  enum Status : int64_t { kPending = 0, kOk = 1, kFailed = 2, kSkipped = 3, kNotRun = 4 };

  int64_t add_task(const std::string& name, const std::vector<std::string>& deps) {
    TORCH_CHECK(!index_.count(name), "task '", name, "' already exists in the graph");
    std::vector<int64_t> d;
    for (const auto& s : deps) {
      auto it = index_.find(s);
      TORCH_CHECK(it != index_.end(), "dependency '", s, "' of task '", name, "' does not exist in the graph");
      if (std::find(d.begin(), d.end(), it->second) == d.end()) d.push_back(it->second);
    }
    const int64_t id = static_cast<int64_t>(names_.size());
    names_.push_back(name);
    index_[name] = id;
    deps_.push_back(d);
    return id;
  }

  // `task` waits for `dep`; rejected when `task` is already an ancestor of `dep`.
  void add_dependency(const std::string& task, const std::string& dep) {
    const int64_t t = id_of(task), d = id_of(dep);
    TORCH_CHECK(t != d, "a task cannot depend on itself");
    if (std::find(deps_[t].begin(), deps_[t].end(), d) != deps_[t].end()) return;
    // cycle iff t is reachable from d by following dependencies backwards, i.e. d depends on t
    std::vector<char> seen(names_.size(), 0);
    std::vector<int64_t> stack{d};
    while (!stack.empty()) {
      const int64_t u = stack.back();
      stack.pop_back();
      TORCH_CHECK(u != t, "adding dependency '", dep, "' -> '", task, "' would create a cycle");
      if (seen[u]) continue;
      seen[u] = 1;
      for (int64_t v : deps_[u]) stack.push_back(v);
    }
    deps_[t].push_back(d);
  }

  int64_t size() const { return static_cast<int64_t>(names_.size()); }
  const std::vector<std::string>& names() const { return names_; }
  std::vector<int64_t> dependencies(const std::string& name) const { return deps_[id_of(name)]; }

  // Kahn's algorithm; among ready tasks the one added first goes first.
  std::vector<std::string> order() const {
    const size_t n = names_.size();
    std::vector<int64_t> indeg(n, 0);
    auto out = dependents();
    for (size_t i = 0; i < n; ++i) indeg[i] = static_cast<int64_t>(deps_[i].size());
    std::vector<int64_t> ready;
    for (size_t i = 0; i < n; ++i)
      if (indeg[i] == 0) ready.push_back(static_cast<int64_t>(i));
    std::vector<std::string> res;
    while (!ready.empty()) {
      auto it = std::min_element(ready.begin(), ready.end());
      const int64_t u = *it;
      ready.erase(it);
      res.push_back(names_[u]);
      for (int64_t v : out[u])
        if (--indeg[v] == 0) ready.push_back(v);
    }
    return res;
  }

  // level(t) = 0 without dependencies, else 1 + max level of its dependencies.
  std::vector<std::vector<std::string>> levels() const {
    std::vector<int64_t> lv(names_.size(), 0);
    int64_t top = -1;
    for (const auto& nm : order()) {
      const int64_t u = index_.at(nm);
      for (int64_t d : deps_[u]) lv[u] = std::max(lv[u], lv[d] + 1);
      top = std::max(top, lv[u]);
    }
    std::vector<std::vector<std::string>> res(static_cast<size_t>(top + 1));
    for (size_t i = 0; i < names_.size(); ++i) res[lv[i]].push_back(names_[i]);
    return res;
  }

  // Runs callback(task_id) -> bool for every task. Returns the status of each task.
  std::vector<int64_t> run(const py::function& callback, int64_t n_threads, bool partial) {
    const size_t n = names_.size();
    std::vector<int64_t> status(n, kPending);
    if (n == 0) return status;
    const auto out = dependents();
    std::vector<int64_t> indeg(n);
    std::vector<char> bad(n, 0);
    std::deque<int64_t> ready;
    for (size_t i = 0; i < n; ++i) {
      indeg[i] = static_cast<int64_t>(deps_[i].size());
      if (indeg[i] == 0) ready.push_back(static_cast<int64_t>(i));
    }
    std::mutex mu;
    std::condition_variable cv;
    size_t finished = 0;
    int64_t inflight = 0;
    bool abort = false;

    // Called with `mu` held after task u reached a final status.
    auto settle = [&](int64_t u) {
      std::vector<int64_t> stack{u};
      while (!stack.empty()) {
        const int64_t x = stack.back();
        stack.pop_back();
        ++finished;
        for (int64_t v : out[x]) {
          if (status[x] != kOk) bad[v] = 1;
          if (--indeg[v] == 0) {
            if (bad[v]) {
              status[v] = kSkipped;
              stack.push_back(v);
            } else {
              ready.push_back(v);
            }
          }
        }
      }
    };

    auto worker = [&](int) {
      for (;;) {
        int64_t u;
        {
          std::unique_lock<std::mutex> lk(mu);
          cv.wait(lk, [&] { return finished == n || (abort && inflight == 0) || (!abort && !ready.empty()); });
          if (finished == n || abort) return;
          u = ready.front();
          ready.pop_front();
          ++inflight;
        }
        bool ok = false;
        {
          py::gil_scoped_acquire gil;
          try {
            ok = py::bool_(callback(u));  // any truthy return value counts as success
          } catch (py::error_already_set& e) {
            e.discard_as_unraisable(__func__);
            ok = false;
          } catch (const std::exception&) {  // never let an exception leave a worker thread
            ok = false;
          }
        }
        {
          std::lock_guard<std::mutex> lk(mu);
          --inflight;
          status[u] = ok ? kOk : kFailed;
          settle(u);
          if (!ok && !partial) abort = true;
        }
        cv.notify_all();
      }
    };

    {
      py::gil_scoped_release nogil;
      run_threads(resolve_threads(n_threads, static_cast<int64_t>(n)), worker);
    }
    for (auto& s : status)
      if (s == kPending) s = kNotRun;
    return status;
  }

 private:
  int64_t id_of(const std::string& name) const {
    auto it = index_.find(name);
    TORCH_CHECK(it != index_.end(), "no task named '", name, "'");
    return it->second;
  }

  std::vector<std::vector<int64_t>> dependents() const {
    std::vector<std::vector<int64_t>> out(names_.size());
    for (size_t i = 0; i < names_.size(); ++i)
      for (int64_t d : deps_[i]) out[d].push_back(static_cast<int64_t>(i));
    return out;
  }

  std::vector<std::string> names_;
  std::unordered_map<std::string, int64_t> index_;
  std::vector<std::vector<int64_t>> deps_;
};

// callback(i) for i in [0, n), dynamically scheduled over native threads.
void parallel_for(const py::function& callback, int64_t n, int64_t n_threads) {
  if (n <= 0) return;
  std::atomic<int64_t> next{0};
  std::atomic<bool> failed{false};
  auto worker = [&](int) {
    for (;;) {
      const int64_t i = next.fetch_add(1);
      if (i >= n || failed.load()) return;
      py::gil_scoped_acquire gil;
      try {
        callback(i);
      } catch (py::error_already_set& e) {
        e.discard_as_unraisable(__func__);
        failed = true;
      } catch (const std::exception&) {
        failed = true;
      }
    }
  };
  {
    py::gil_scoped_release nogil;
    run_threads(resolve_threads(n_threads, n), worker);
  }
  TORCH_CHECK(!failed.load(), "parallel_for: the callback raised (the exception was reported as unraisable)");
}

// ---------------------------------------------------------------------------
// Scans
// ---------------------------------------------------------------------------

enum ScanOp : int64_t { kSum = 0, kProd = 1, kMin = 2, kMax = 3 };

template <typename T>
struct Op {
  int64_t op;
  T identity() const {
    switch (op) {
      case kSum: return T(0);
      case kProd: return T(1);
      case kMin:
        return std::numeric_limits<T>::has_infinity ? std::numeric_limits<T>::infinity()
                                                     : std::numeric_limits<T>::max();
      default:
        return std::numeric_limits<T>::has_infinity ? -std::numeric_limits<T>::infinity()
                                                     : std::numeric_limits<T>::lowest();
    }
  }
  T operator()(T a, T b) const {
    switch (op) {
      case kSum: return a + b;
      case kProd: return a * b;
      case kMin: return b < a ? b : a;
      default: return b > a ? b : a;
    }
  }
};

// Chunk boundaries [lo, hi) of T near-equal chunks.
inline int64_t chunk_lo(int64_t n, int T, int c) { return n * c / T; }

template <typename T>
void scan_impl(const T* x, T* y, int64_t n, Op<T> op, bool exclusive, int nth) {
  const int Tn = n < 65536 ? 1 : nth;  // small inputs: one thread
  std::vector<T> total(Tn);
  run_threads(Tn, [&](int c) {
    const int64_t lo = chunk_lo(n, Tn, c), hi = chunk_lo(n, Tn, c + 1);
    T acc = op.identity();
    for (int64_t i = lo; i < hi; ++i) {
      acc = op(acc, x[i]);
      y[i] = acc;
    }
    total[c] = acc;
  });
  std::vector<T> carry(Tn, op.identity());
  for (int c = 1; c < Tn; ++c) carry[c] = op(carry[c - 1], total[c - 1]);
  if (Tn > 1)
    run_threads(Tn, [&](int c) {
      if (c == 0) return;
      const int64_t lo = chunk_lo(n, Tn, c), hi = chunk_lo(n, Tn, c + 1);
      for (int64_t i = lo; i < hi; ++i) y[i] = op(carry[c], y[i]);
    });
  if (exclusive && n > 0) {
    std::copy_backward(y, y + n - 1, y + n);
    y[0] = op.identity();
  }
}

torch::Tensor scan(const torch::Tensor& x, int64_t op, bool exclusive, int64_t n_threads) {
  TORCH_CHECK(x.device().is_cpu() && x.dim() == 1, "scan wants a 1-D host tensor");
  TORCH_CHECK(op >= kSum && op <= kMax, "scan op must be 0 (sum), 1 (prod), 2 (min) or 3 (max)");
  auto xc = x.contiguous();
  auto y = torch::empty_like(xc);
  const int64_t n = xc.numel();
  AT_DISPATCH_ALL_TYPES(xc.scalar_type(), "scirs_scan", [&] {
    scan_impl<scalar_t>(xc.data_ptr<scalar_t>(), y.data_ptr<scalar_t>(), n, Op<scalar_t>{op}, exclusive,
                        resolve_threads(n_threads, n));
  });
  return y;
}

// y[i] = x[i] + y[i-1] unless flags[i] (a segment starts at i, y[i] = x[i]).
torch::Tensor segmented_scan_sum(const torch::Tensor& x, const torch::Tensor& flags, int64_t n_threads) {
  TORCH_CHECK(x.device().is_cpu() && x.dim() == 1, "segmented scan wants a 1-D host tensor");
  TORCH_CHECK(flags.numel() == x.numel(), "flags must have one entry per element");
  auto xc = x.contiguous();
  auto fc = flags.to(torch::kBool).contiguous();
  auto y = torch::empty_like(xc);
  const int64_t n = xc.numel();
  const bool* f = fc.data_ptr<bool>();
  AT_DISPATCH_ALL_TYPES(xc.scalar_type(), "scirs_segscan", [&] {
    const scalar_t* xp = xc.data_ptr<scalar_t>();
    scalar_t* yp = y.data_ptr<scalar_t>();
    const int Tn = n < 65536 ? 1 : resolve_threads(n_threads, n);
    std::vector<scalar_t> tail(Tn);  // sum since the chunk's last segment head (or its start)
    std::vector<char> has_head(Tn, 0);
    run_threads(Tn, [&](int c) {
      const int64_t lo = chunk_lo(n, Tn, c), hi = chunk_lo(n, Tn, c + 1);
      scalar_t acc = 0;
      for (int64_t i = lo; i < hi; ++i) {
        if (f[i]) {
          acc = 0;
          has_head[c] = 1;
        }
        acc += xp[i];
        yp[i] = acc;
      }
      tail[c] = acc;
    });
    std::vector<scalar_t> carry(Tn, 0);
    for (int c = 1; c < Tn; ++c) carry[c] = has_head[c - 1] ? tail[c - 1] : carry[c - 1] + tail[c - 1];
    if (Tn > 1)
      run_threads(Tn, [&](int c) {
        if (c == 0) return;
        const int64_t lo = chunk_lo(n, Tn, c), hi = chunk_lo(n, Tn, c + 1);
        for (int64_t i = lo; i < hi && !f[i]; ++i) yp[i] += carry[c];
      });
  });
  return y;
}

// ---------------------------------------------------------------------------
// Stable parallel sort
// ---------------------------------------------------------------------------

template <typename T>
struct Less {
  const T* v;
  bool desc;
  bool operator()(int64_t a, int64_t b) const {
    const T x = v[a], y = v[b];
    if constexpr (std::is_floating_point<T>::value) {
      const bool nx = std::isnan(x), ny = std::isnan(y);
      if (nx || ny) return desc ? (nx && !ny) : (ny && !nx);  // NaN is the largest value
    }
    return desc ? y < x : x < y;
  }
};

std::vector<torch::Tensor> parallel_sort(const torch::Tensor& x, bool descending, int64_t n_threads) {
  TORCH_CHECK(x.device().is_cpu() && x.dim() == 1, "parallel_sort wants a 1-D host tensor");
  auto xc = x.contiguous();
  const int64_t n = xc.numel();
  auto idx = torch::arange(n, torch::TensorOptions().dtype(torch::kLong));
  int64_t* ip = idx.data_ptr<int64_t>();
  AT_DISPATCH_ALL_TYPES(xc.scalar_type(), "scirs_sort", [&] {
    Less<scalar_t> less{xc.data_ptr<scalar_t>(), descending};
    int Tn = n < 32768 ? 1 : resolve_threads(n_threads, n);
    std::vector<int64_t> bounds(Tn + 1);
    for (int c = 0; c <= Tn; ++c) bounds[c] = chunk_lo(n, Tn, c);
    run_threads(Tn, [&](int c) { std::stable_sort(ip + bounds[c], ip + bounds[c + 1], less); });
    // merge neighbouring runs pairwise until one run is left
    while (bounds.size() > 2) {
      const int runs = static_cast<int>(bounds.size()) - 1, pairs = runs / 2;
      run_threads(std::max(1, pairs), [&](int p) {
        if (p >= pairs) return;
        std::inplace_merge(ip + bounds[2 * p], ip + bounds[2 * p + 1], ip + bounds[2 * p + 2], less);
      });
      std::vector<int64_t> nb;
      for (int r = 0; r <= runs; r += 2) nb.push_back(bounds[r]);
      if (nb.back() != bounds.back()) nb.push_back(bounds.back());
      bounds.swap(nb);
    }
  });
  return {xc.index_select(0, idx), idx};
}

// ---------------------------------------------------------------------------
// Lock-free bounded MPMC queue (D. Vyukov's algorithm) and an atomic counter
// ---------------------------------------------------------------------------

class MpmcRing {
 public:
  explicit MpmcRing(int64_t capacity) {
    TORCH_CHECK(capacity >= 2 && (capacity & (capacity - 1)) == 0, "capacity must be a power of two >= 2");
    mask_ = static_cast<size_t>(capacity - 1);
    cells_.reset(new Cell[capacity]);
    for (size_t i = 0; i <= mask_; ++i) cells_[i].seq.store(i, std::memory_order_relaxed);
  }

  bool try_push(int64_t v) {
    size_t pos = enq_.load(std::memory_order_relaxed);
    Cell* c;
    for (;;) {
      c = &cells_[pos & mask_];
      const size_t seq = c->seq.load(std::memory_order_acquire);
      const intptr_t dif = static_cast<intptr_t>(seq) - static_cast<intptr_t>(pos);
      if (dif == 0) {
        if (enq_.compare_exchange_weak(pos, pos + 1, std::memory_order_relaxed)) break;
      } else if (dif < 0) {
        return false;  // full
      } else {
        pos = enq_.load(std::memory_order_relaxed);
      }
    }
    c->val = v;
    c->seq.store(pos + 1, std::memory_order_release);
    return true;
  }

  bool try_pop(int64_t& v) {
    size_t pos = deq_.load(std::memory_order_relaxed);
    Cell* c;
    for (;;) {
      c = &cells_[pos & mask_];
      const size_t seq = c->seq.load(std::memory_order_acquire);
      const intptr_t dif = static_cast<intptr_t>(seq) - static_cast<intptr_t>(pos + 1);
      if (dif == 0) {
        if (deq_.compare_exchange_weak(pos, pos + 1, std::memory_order_relaxed)) break;
      } else if (dif < 0) {
        return false;  // empty
      } else {
        pos = deq_.load(std::memory_order_relaxed);
      }
    }
    v = c->val;
    c->seq.store(pos + mask_ + 1, std::memory_order_release);
    return true;
  }

  py::object pop() {
    int64_t v;
    if (try_pop(v)) return py::int_(v);
    return py::none();
  }

  int64_t size() const {
    const int64_t s = static_cast<int64_t>(enq_.load()) - static_cast<int64_t>(deq_.load());
    return std::max<int64_t>(0, s);
  }
  int64_t capacity() const { return static_cast<int64_t>(mask_ + 1); }

 private:
  struct Cell {
    std::atomic<size_t> seq;
    int64_t val;
  };
  std::unique_ptr<Cell[]> cells_;
  size_t mask_ = 0;
  alignas(64) std::atomic<size_t> enq_{0};
  alignas(64) std::atomic<size_t> deq_{0};
};

// P producer and C consumer threads move P * per_producer distinct values through
// one ring; returns {received, duplicates, missing, timed_out}. Every wait is
// bounded by `timeout_s`.
std::vector<int64_t> ring_stress(int64_t capacity, int64_t producers, int64_t consumers, int64_t per_producer,
                                 double timeout_s) {
  TORCH_CHECK(producers >= 1 && consumers >= 1 && per_producer >= 0, "bad stress sizes");
  MpmcRing ring(capacity);
  const int64_t total = producers * per_producer;
  std::vector<std::atomic<uint8_t>> seen(static_cast<size_t>(total));
  for (auto& s : seen) s.store(0, std::memory_order_relaxed);
  std::atomic<int64_t> received{0}, dup{0};
  std::atomic<bool> timed_out{false};
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
  auto expired = [&] { return std::chrono::steady_clock::now() > deadline; };
  {
    py::gil_scoped_release nogil;
    std::vector<std::thread> ts;
    for (int64_t p = 0; p < producers; ++p)
      ts.emplace_back([&, p] {
        for (int64_t i = 0; i < per_producer; ++i) {
          const int64_t v = p * per_producer + i;
          while (!ring.try_push(v)) {
            if (expired()) {
              timed_out = true;
              return;
            }
            std::this_thread::yield();
          }
        }
      });
    for (int64_t c = 0; c < consumers; ++c)
      ts.emplace_back([&] {
        int64_t v;
        while (received.load() < total) {
          if (ring.try_pop(v)) {
            if (v < 0 || v >= total || seen[v].fetch_add(1) != 0) ++dup;
            ++received;
          } else {
            if (expired()) {
              timed_out = true;
              return;
            }
            std::this_thread::yield();
          }
        }
      });
    for (auto& t : ts) t.join();
  }
  int64_t missing = 0;
  for (auto& s : seen) missing += s.load() == 0;
  return {received.load(), dup.load(), missing, timed_out.load() ? 1 : 0};
}

class AtomicCounter {
 public:
  explicit AtomicCounter(int64_t v) : v_(v) {}
  int64_t increment() { return v_.fetch_add(1) + 1; }
  int64_t decrement() { return v_.fetch_sub(1) - 1; }
  int64_t add(int64_t n) { return v_.fetch_add(n) + n; }
  int64_t get() const { return v_.load(); }
  // (swapped, value seen): the value is replaced only if it equals `expected`
  std::pair<bool, int64_t> compare_and_swap(int64_t expected, int64_t desired) {
    int64_t e = expected;
    const bool ok = v_.compare_exchange_strong(e, desired);
    return {ok, e};
  }
  int64_t reset() { return v_.exchange(0); }

 private:
  std::atomic<int64_t> v_;
};

void register_host_runtime(py::module& m) {
  py::class_<TaskGraphCore>(m, "TaskGraphCore")
      .def(py::init<>())
      .def("add_task", &TaskGraphCore::add_task)
      .def("add_dependency", &TaskGraphCore::add_dependency)
      .def("size", &TaskGraphCore::size)
      .def("names", &TaskGraphCore::names)
      .def("dependencies", &TaskGraphCore::dependencies)
      .def("order", &TaskGraphCore::order)
      .def("levels", &TaskGraphCore::levels)
      .def("run", &TaskGraphCore::run, py::arg("callback"), py::arg("n_threads") = 0, py::arg("partial") = false);
  m.def("parallel_for", &parallel_for, py::arg("callback"), py::arg("n"), py::arg("n_threads") = 0);
  m.def("scan", &scan, py::arg("x"), py::arg("op") = 0, py::arg("exclusive") = false, py::arg("n_threads") = 0,
        py::call_guard<py::gil_scoped_release>());
  m.def("segmented_scan_sum", &segmented_scan_sum, py::arg("x"), py::arg("flags"), py::arg("n_threads") = 0,
        py::call_guard<py::gil_scoped_release>());
  m.def("parallel_sort", &parallel_sort, py::arg("x"), py::arg("descending") = false, py::arg("n_threads") = 0,
        py::call_guard<py::gil_scoped_release>());
  py::class_<MpmcRing>(m, "MpmcRing")
      .def(py::init<int64_t>())
      .def("try_push", &MpmcRing::try_push)
      .def("pop", &MpmcRing::pop)
      .def("size", &MpmcRing::size)
      .def("capacity", &MpmcRing::capacity);
  m.def("ring_stress", &ring_stress, py::arg("capacity"), py::arg("producers"), py::arg("consumers"),
        py::arg("per_producer"), py::arg("timeout_s") = 30.0);
  py::class_<AtomicCounter>(m, "AtomicCounter")
      .def(py::init<int64_t>(), py::arg("initial") = 0)
      .def("increment", &AtomicCounter::increment)
      .def("decrement", &AtomicCounter::decrement)
      .def("add", &AtomicCounter::add)
      .def("get", &AtomicCounter::get)
      .def("compare_and_swap", &AtomicCounter::compare_and_swap)
      .def("reset", &AtomicCounter::reset);
}

}  // namespace scirs
