// Host side of storage-backed embedding tables (the reference's PLE row
// reader, csrc/exl3/ple_read.cpp:323 ple_read_rows, and Engram host fetch,
// csrc/exl3/engram_fetch.cpp:238 FetchState::fetch): rows of a table file are
// read on demand for the token ids of a step.
//
//   RowReader  fixed-size rows of one file, read with pread on a pool of
//              worker threads; a failed read is retried with a 1 ms doubling
//              backoff and, after the last retry, the row is reported failed
//              (the caller poisons it; the row's tokens then fail cleanly).
//              O_DIRECT is optional (aligned bounce buffers).  A test hook
//              fails chosen rows on purpose: faults are injected on the host,
//              never on a device.
//   RowCache   set-associative LRU cache of rows in host memory in front of a
//              RowReader: `fetch` copies hits, reads the misses in one batch,
//              inserts them (evicting the least recently used way of the set)
//              and writes every requested row into a caller buffer (pinned, so
//              the copy to the device that follows is asynchronous).
//              `enqueue` runs the same fetch as a host function on a CUDA
//              stream (cudaLaunchHostFunc): the step's ids are copied to
//              pinned memory, the fetch runs when the stream reaches it, the
//              rows' copy to the device and their dequant follow on the
//              stream, and the host thread never waits.  A job made with
//              `fixed_job` keeps its buffers and row count, so a lookup built
//              from it can be captured in a CUDA graph and replayed (each
//              replay fetches the ids of that replay).
#include <cuda_runtime.h>
#include <fcntl.h>
#include <torch/extension.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <unordered_set>
#include <vector>

namespace b200 {

class RowReader {
 public:
  // Row r is the row_bytes bytes at byte base + r * row_bytes of the file.
  RowReader(const std::string& path, int64_t row_bytes, int64_t num_rows, int threads, int retries, bool o_direct,
            int64_t base = 0)
      : row_bytes_(row_bytes), num_rows_(num_rows), base_(base), retries_(retries), o_direct_(o_direct) {
    if (row_bytes <= 0 || num_rows <= 0) throw std::invalid_argument("row_bytes and num_rows must be positive");
    if (base < 0) throw std::invalid_argument("base must be non-negative");
    fd_ = ::open(path.c_str(), O_RDONLY | (o_direct ? O_DIRECT : 0));
    if (fd_ < 0) throw std::runtime_error("cannot open row table " + path);
    const int n = threads < 1 ? 1 : threads;
    for (int i = 0; i < n; ++i) workers_.emplace_back([this] { worker(); });
  }
  ~RowReader() {
    {
      std::lock_guard<std::mutex> g(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
    if (fd_ >= 0) ::close(fd_);
  }

  int64_t row_bytes() const { return row_bytes_; }
  int64_t num_rows() const { return num_rows_; }

  // Reads rows `ids` into dst (ids.size() x row_bytes); returns 1 per row that failed after all retries.
  std::vector<uint8_t> read(const std::vector<int64_t>& ids, uint8_t* dst) {
    std::vector<uint8_t> failed(ids.size(), 0);
    std::atomic<int64_t> left((int64_t)ids.size());
    std::mutex done_mu;
    std::condition_variable done_cv;
    {
      std::lock_guard<std::mutex> g(mu_);
      for (size_t i = 0; i < ids.size(); ++i) {
        jobs_.push_back([&, i] {
          failed[i] = read_one(ids[i], dst + (int64_t)i * row_bytes_) ? 0 : 1;
          if (--left == 0) {
            std::lock_guard<std::mutex> dg(done_mu);
            done_cv.notify_all();
          }
        });
      }
    }
    cv_.notify_all();
    std::unique_lock<std::mutex> dl(done_mu);
    done_cv.wait(dl, [&] { return left.load() == 0; });
    return failed;
  }

  void fail_rows_for_test(const std::vector<int64_t>& rows) {
    std::lock_guard<std::mutex> g(fail_mu_);
    inject_.clear();
    inject_.insert(rows.begin(), rows.end());
  }

  std::vector<int64_t> stats() const { return {reads_.load(), retries_done_.load(), failures_.load(), bytes_.load()}; }

 private:
  bool read_one(int64_t row, uint8_t* dst) {
    if (row < 0 || row >= num_rows_) {
      ++failures_;
      return false;
    }
    const int64_t off = base_ + row * row_bytes_;
    int delay_us = 1000;
    for (int attempt = 0; attempt <= retries_; ++attempt) {
      if (attempt > 0) {
        ++retries_done_;
        std::this_thread::sleep_for(std::chrono::microseconds(delay_us));
        delay_us *= 2;
      }
      bool injected;
      {
        std::lock_guard<std::mutex> g(fail_mu_);
        injected = inject_.count(row) != 0;
      }
      if (injected) continue;
      if (read_at(off, dst)) {
        ++reads_;
        bytes_ += row_bytes_;
        return true;
      }
    }
    ++failures_;
    return false;
  }

  bool read_at(int64_t off, uint8_t* dst) {
    if (!o_direct_) {
      int64_t done = 0;
      while (done < row_bytes_) {
        const ssize_t r = ::pread(fd_, dst + done, row_bytes_ - done, off + done);
        if (r <= 0) return false;
        done += r;
      }
      return true;
    }
    // O_DIRECT: aligned window around the row, through an aligned bounce buffer
    const int64_t a = 4096, start = off / a * a, end = (off + row_bytes_ + a - 1) / a * a;
    void* buf = nullptr;
    if (posix_memalign(&buf, a, end - start) != 0) return false;
    const ssize_t r = ::pread(fd_, buf, end - start, start);
    const bool ok = r >= (ssize_t)(off + row_bytes_ - start);
    if (ok) std::memcpy(dst, static_cast<uint8_t*>(buf) + (off - start), row_bytes_);
    std::free(buf);
    return ok;
  }

  void worker() {
    for (;;) {
      std::function<void()> job;
      {
        std::unique_lock<std::mutex> l(mu_);
        cv_.wait(l, [&] { return stop_ || !jobs_.empty(); });
        if (stop_ && jobs_.empty()) return;
        job = std::move(jobs_.back());
        jobs_.pop_back();
      }
      job();
    }
  }

  int64_t row_bytes_, num_rows_, base_;
  int retries_;
  bool o_direct_;
  int fd_ = -1;
  std::vector<std::thread> workers_;
  std::vector<std::function<void()>> jobs_;
  std::mutex mu_;
  std::condition_variable cv_;
  bool stop_ = false;
  std::mutex fail_mu_;
  std::unordered_set<int64_t> inject_;
  std::atomic<int64_t> reads_{0}, retries_done_{0}, failures_{0}, bytes_{0};
};

class RowCache {
 public:
  RowCache(std::shared_ptr<RowReader> reader, int64_t capacity_rows, int ways)
      : reader_(std::move(reader)), ways_(ways < 1 ? 1 : ways) {
    sets_ = std::max<int64_t>(1, capacity_rows / ways_);
    const int64_t slots = sets_ * ways_;
    keys_.assign(slots, -1);
    stamp_.assign(slots, 0);
    data_.resize((size_t)slots * reader_->row_bytes());
  }

  ~RowCache() {
    for (Job* j : fixed_jobs_) delete j;
  }

  // Writes rows `ids` into out [n, row_bytes] (uint8, host); returns the failed-row mask.  A negative
  // id (a row the caller does not need, e.g. another rank's) is written as zeros and is not read.
  torch::Tensor fetch(const torch::Tensor& ids, torch::Tensor& out) {
    TORCH_CHECK(ids.scalar_type() == at::kLong && ids.dim() == 1 && !ids.is_cuda(), "ids: host int64 [n]");
    TORCH_CHECK(out.scalar_type() == at::kByte && !out.is_cuda() && out.is_contiguous() && out.size(0) == ids.size(0) &&
                    out.size(1) == reader_->row_bytes(),
                "out: host uint8 [n, row_bytes]");
    auto failed = torch::zeros({ids.size(0)}, torch::dtype(torch::kUInt8));
    fetch_raw(ids.data_ptr<int64_t>(), ids.size(0), out.data_ptr<uint8_t>(), failed.data_ptr<uint8_t>());
    return failed;
  }

  // ---------------------------------------------------------------- stream-ordered fetch
  struct Job {
    RowCache* cache;
    const int64_t* ids;
    int64_t n;
    uint8_t* out;
    uint8_t* failed;
    bool one_shot;
  };

  static void CUDART_CB run_job(void* arg) {
    Job* j = static_cast<Job*>(arg);
    try {
      j->cache->fetch_raw(j->ids, j->n, j->out, j->failed);
    } catch (...) {  // never unwind into the driver: every row of the call fails instead
      std::memset(j->failed, 1, (size_t)j->n);
      ++j->cache->host_errors_;
    }
    if (j->one_shot) delete j;
  }

  // Queue fetch(ids[0:n]) -> out / failed (all pinned host memory, addresses as integers) as a host
  // function on `stream`.  The buffers must stay untouched until the stream has passed the call.
  void enqueue(int64_t stream, int64_t ids, int64_t n, int64_t out, int64_t failed) {
    Job* j = new Job{this, reinterpret_cast<const int64_t*>(ids), n, reinterpret_cast<uint8_t*>(out),
                     reinterpret_cast<uint8_t*>(failed), true};
    const cudaError_t e = cudaLaunchHostFunc(reinterpret_cast<cudaStream_t>(stream), &RowCache::run_job, j);
    if (e != cudaSuccess) {
      delete j;
      TORCH_CHECK(false, "RowCache.enqueue: ", cudaGetErrorString(e));
    }
  }

  // A job with fixed buffers and row count that lives as long as the cache (for graph capture).
  int64_t fixed_job(int64_t ids, int64_t n, int64_t out, int64_t failed) {
    Job* j = new Job{this, reinterpret_cast<const int64_t*>(ids), n, reinterpret_cast<uint8_t*>(out),
                     reinterpret_cast<uint8_t*>(failed), false};
    std::lock_guard<std::mutex> g(mu_);
    fixed_jobs_.push_back(j);
    return (int64_t)(fixed_jobs_.size() - 1);
  }

  void enqueue_job(int64_t stream, int64_t job) {
    Job* j;
    {
      std::lock_guard<std::mutex> g(mu_);
      TORCH_CHECK(job >= 0 && job < (int64_t)fixed_jobs_.size(), "RowCache.enqueue_job: unknown job");
      j = fixed_jobs_[job];
    }
    const cudaError_t e = cudaLaunchHostFunc(reinterpret_cast<cudaStream_t>(stream), &RowCache::run_job, j);
    TORCH_CHECK(e == cudaSuccess, "RowCache.enqueue_job: ", cudaGetErrorString(e));
  }

  int64_t host_errors() const { return host_errors_.load(); }

  void fetch_raw(const int64_t* id, int64_t n, uint8_t* o, uint8_t* f) {
    const int64_t rb = reader_->row_bytes();
    std::memset(f, 0, (size_t)n);
    std::vector<int64_t> miss_rows;
    std::vector<int64_t> miss_idx;
    std::lock_guard<std::mutex> g(mu_);
    for (int64_t i = 0; i < n; ++i) {
      if (id[i] < 0) {
        std::memset(o + i * rb, 0, rb);
        continue;
      }
      const int64_t slot = lookup(id[i]);
      if (slot >= 0) {
        std::memcpy(o + i * rb, &data_[(size_t)slot * rb], rb);
        stamp_[slot] = ++clock_;
        ++hits_;
      } else {
        miss_rows.push_back(id[i]);
        miss_idx.push_back(i);
      }
    }
    if (!miss_rows.empty()) {
      std::vector<uint8_t> buf((size_t)miss_rows.size() * rb);
      std::vector<uint8_t> bad = reader_->read(miss_rows, buf.data());
      for (size_t j = 0; j < miss_rows.size(); ++j) {
        const int64_t i = miss_idx[j];
        std::memcpy(o + i * rb, &buf[j * rb], rb);
        if (bad[j]) {
          f[i] = 1;  // never cached: a later step retries the read
          continue;
        }
        const int64_t slot = victim(miss_rows[j]);
        keys_[slot] = miss_rows[j];
        stamp_[slot] = ++clock_;
        std::memcpy(&data_[(size_t)slot * rb], &buf[j * rb], rb);
        ++misses_;
      }
    }
  }

  std::vector<int64_t> stats() const { return {hits_, misses_}; }

 private:
  int64_t lookup(int64_t row) const {
    const int64_t s = (row % sets_ + sets_) % sets_;
    for (int w = 0; w < ways_; ++w)
      if (keys_[s * ways_ + w] == row) return s * ways_ + w;
    return -1;
  }
  int64_t victim(int64_t row) const {
    const int64_t s = (row % sets_ + sets_) % sets_;
    int64_t best = s * ways_;
    for (int w = 0; w < ways_; ++w) {
      const int64_t slot = s * ways_ + w;
      if (keys_[slot] == row) return slot;  // a concurrent duplicate in the same batch
      if (keys_[slot] < 0) return slot;
      if (stamp_[slot] < stamp_[best]) best = slot;
    }
    return best;
  }

  std::shared_ptr<RowReader> reader_;
  int ways_;
  int64_t sets_;
  std::vector<int64_t> keys_;
  std::vector<uint64_t> stamp_;
  std::vector<uint8_t> data_;
  uint64_t clock_ = 0;
  int64_t hits_ = 0, misses_ = 0;
  std::mutex mu_;
  std::vector<Job*> fixed_jobs_;
  std::atomic<int64_t> host_errors_{0};
};

void register_row_store(pybind11::module_& m) {
  namespace py = pybind11;
  py::class_<RowReader, std::shared_ptr<RowReader>>(m, "RowReader")
      .def(py::init<const std::string&, int64_t, int64_t, int, int, bool, int64_t>(), py::arg("path"),
           py::arg("row_bytes"), py::arg("num_rows"), py::arg("threads") = 8, py::arg("retries") = 3,
           py::arg("o_direct") = false, py::arg("base") = 0)
      .def("read",
           [](RowReader& r, const torch::Tensor& ids, torch::Tensor& out) {
             TORCH_CHECK(ids.scalar_type() == at::kLong && !ids.is_cuda() && out.scalar_type() == at::kByte &&
                             !out.is_cuda() && out.is_contiguous() && out.size(0) == ids.size(0) &&
                             out.size(1) == r.row_bytes(),
                         "RowReader.read: host int64 ids [n], host uint8 out [n, row_bytes]");
             std::vector<int64_t> v(ids.data_ptr<int64_t>(), ids.data_ptr<int64_t>() + ids.size(0));
             std::vector<uint8_t> bad;
             {
               py::gil_scoped_release nogil;
               bad = r.read(v, out.data_ptr<uint8_t>());
             }
             auto t = torch::empty({(int64_t)bad.size()}, torch::dtype(torch::kUInt8));
             std::memcpy(t.data_ptr<uint8_t>(), bad.data(), bad.size());
             return t;
           })
      .def("fail_rows_for_test", &RowReader::fail_rows_for_test)
      .def("stats", &RowReader::stats)
      .def_property_readonly("row_bytes", &RowReader::row_bytes)
      .def_property_readonly("num_rows", &RowReader::num_rows);
  py::class_<RowCache>(m, "RowCache")
      .def(py::init<std::shared_ptr<RowReader>, int64_t, int>(), py::arg("reader"), py::arg("capacity_rows"),
           py::arg("ways") = 8)
      .def("fetch",
           [](RowCache& c, const torch::Tensor& ids, torch::Tensor& out) {
             py::gil_scoped_release nogil;
             return c.fetch(ids, out);
           })
      .def("stats", &RowCache::stats)
      .def("enqueue", &RowCache::enqueue, py::arg("stream"), py::arg("ids"), py::arg("n"), py::arg("out"),
           py::arg("failed"))
      .def("fixed_job", &RowCache::fixed_job, py::arg("ids"), py::arg("n"), py::arg("out"), py::arg("failed"))
      .def("enqueue_job", &RowCache::enqueue_job, py::arg("stream"), py::arg("job"))
      .def("host_errors", &RowCache::host_errors);
}

}  // namespace b200
