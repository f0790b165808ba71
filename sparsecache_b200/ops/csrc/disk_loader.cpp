// Layer-wise KV streaming from disk: file -> pinned staging -> device, one
// layer at a time, with a ready event per layer.
//
// Counterpart of the out-of-tree CacheBlend loader the reference drives
// (README.md:254-282: safetensors on SSD, two pinned buffers, one H2D copy
// per layer with a CUDA event, "disk_sync" vs "disk_async").  Here it is a
// native runtime component: a scheduler thread walks the layers in order;
// for layer l it takes staging buffer l % n_buffers once that buffer's
// previous H2D copy has finished, fills it with a pool of pread() workers
// (every (document, K|V) extent of the layer, in parallel), enqueues the
// copies on its own stream and records the layer's event.  A consumer calls
// wait_layer(l, stream): the host blocks only until layer l's copies are
// enqueued, then the consumer's stream waits on the event, so compute on
// layer l overlaps the reads of layers l+1, l+2, ...
//
// Host mode (device < 0) copies into host memory instead: the same read
// schedule without a GPU (tests, tooling).
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include <cuda_runtime.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

namespace py = pybind11;

namespace sc {

namespace {

struct Extent {
  int file;
  int64_t offset;      // in the file
  int64_t nbytes;
  int64_t dst_offset;  // from the destination base
};

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

double now_ms() {
  using namespace std::chrono;
  return duration<double, std::milli>(steady_clock::now().time_since_epoch()).count();
}

}  // namespace

class LayerwiseKVLoader {
 public:
  LayerwiseKVLoader(int64_t staging_bytes, int n_buffers, int n_threads, int device)
      : staging_bytes_(staging_bytes), n_buffers_(n_buffers), n_threads_(n_threads < 1 ? 1 : n_threads),
        device_(device) {
    if (n_buffers_ < 1 || staging_bytes_ <= 0) throw std::invalid_argument("bad staging geometry");
    if (device_ >= 0) {
      check(cudaSetDevice(device_), "cudaSetDevice");
      check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
    }
    for (int b = 0; b < n_buffers_; ++b) {
      void* p = nullptr;
      if (device_ >= 0) {
        check(cudaHostAlloc(&p, (size_t)staging_bytes_, cudaHostAllocDefault), "cudaHostAlloc");
        cudaEvent_t e;
        check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
        buffer_free_.push_back(e);
      } else {
        p = std::malloc((size_t)staging_bytes_);
        if (p == nullptr) throw std::bad_alloc();
      }
      staging_.push_back(p);
    }
  }

  ~LayerwiseKVLoader() {
    try {
      join();
    } catch (...) {
    }
    for (size_t b = 0; b < staging_.size(); ++b) {
      if (device_ >= 0) {
        cudaFreeHost(staging_[b]);
      } else {
        std::free(staging_[b]);
      }
    }
    for (auto e : buffer_free_) cudaEventDestroy(e);
    for (auto e : layer_ready_) cudaEventDestroy(e);
    if (after_ != nullptr) cudaEventDestroy(after_);
    if (stream_ != nullptr) cudaStreamDestroy(stream_);
    close_files();
  }

  int64_t staging_bytes() const { return staging_bytes_; }

  // Open `paths` (closing the previous request's files) and stream `plan`:
  // plan[l] = extents of the l-th streamed layer as (file, offset, nbytes,
  // dst_offset) rows; dst_base is a device address (host address in host mode).
  // `after_stream`: the copies wait for the work already queued on that stream
  // (e.g. the previous request still reading the destination).
  void start(const std::vector<std::string>& paths, const std::vector<std::vector<std::vector<int64_t>>>& plan,
             int64_t dst_base, int64_t after_stream) {
    join();
    close_files();
    paths_ = paths;
    for (const auto& p : paths_) {
      const int fd = ::open(p.c_str(), O_RDONLY);
      if (fd < 0) {
        close_files();
        throw std::runtime_error("cannot open " + p);
      }
      ::posix_fadvise(fd, 0, 0, POSIX_FADV_SEQUENTIAL);
      fds_.push_back(fd);
    }
    layers_.clear();
    for (const auto& layer : plan) {
      std::vector<Extent> ex;
      int64_t total = 0;
      for (const auto& r : layer) {
        if (r.size() != 4) throw std::invalid_argument("extent rows are (file, offset, nbytes, dst_offset)");
        Extent e{(int)r[0], r[1], r[2], r[3]};
        if (e.file < 0 || e.file >= (int)fds_.size() || e.nbytes < 0) throw std::invalid_argument("bad extent");
        total += e.nbytes;
        ex.push_back(e);
      }
      if (total > staging_bytes_) throw std::invalid_argument("a layer exceeds the staging buffer");
      layers_.push_back(std::move(ex));
    }
    const int L = (int)layers_.size();
    if (device_ >= 0) {
      check(cudaSetDevice(device_), "cudaSetDevice");
      if (after_ == nullptr) check(cudaEventCreateWithFlags(&after_, cudaEventDisableTiming), "cudaEventCreate");
      check(cudaEventRecord(after_, reinterpret_cast<cudaStream_t>(after_stream)), "cudaEventRecord");
      check(cudaStreamWaitEvent(stream_, after_, 0), "cudaStreamWaitEvent");
      while ((int)layer_ready_.size() < L) {
        cudaEvent_t e;
        check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
        layer_ready_.push_back(e);
      }
    }
    {
      std::lock_guard<std::mutex> g(mu_);
      enqueued_ = 0;
      error_.clear();
      read_ms_.assign(L, 0.0);
      bytes_ = 0;
    }
    dst_base_ = dst_base;
    t0_ms_ = now_ms();
    worker_ = std::thread([this] { run(); });
  }

  // Block until layer l's copies are enqueued, then make `stream` wait for them
  // (host mode: until the layer is in the destination).
  void wait_layer(int layer, int64_t stream) {
    std::unique_lock<std::mutex> lk(mu_);
    cv_.wait(lk, [&] { return enqueued_ > layer || !error_.empty(); });
    if (!error_.empty()) throw std::runtime_error(error_);
    lk.unlock();
    if (device_ >= 0)
      check(cudaStreamWaitEvent(reinterpret_cast<cudaStream_t>(stream), layer_ready_[layer], 0),
            "cudaStreamWaitEvent");
  }

  void join() {
    if (worker_.joinable()) worker_.join();
    if (!error_.empty()) {
      std::string e = error_;
      error_.clear();
      throw std::runtime_error(e);
    }
  }

  py::dict stats() {
    std::lock_guard<std::mutex> g(mu_);
    py::dict d;
    d["layers"] = (int)layers_.size();
    d["layers_enqueued"] = enqueued_;
    d["bytes"] = bytes_;
    d["read_ms_per_layer"] = read_ms_;
    d["wall_ms"] = done_ms_ - t0_ms_;
    return d;
  }

 private:
  void close_files() {
    for (int fd : fds_) ::close(fd);
    fds_.clear();
  }

  void fail(const std::string& what) {
    std::lock_guard<std::mutex> g(mu_);
    if (error_.empty()) error_ = what;
    cv_.notify_all();
  }

  // pread the layer's extents into one staging buffer with n_threads workers
  // (extents handed out in order through an atomic index; large extents are
  // read whole, pread loops over short reads).
  void read_layer(const std::vector<Extent>& ex, char* buf, std::vector<int64_t>& buf_off) {
    buf_off.resize(ex.size());
    int64_t o = 0;
    for (size_t i = 0; i < ex.size(); ++i) buf_off[i] = o, o += ex[i].nbytes;
    std::atomic<size_t> next{0};
    std::atomic<bool> bad{false};
    std::string bad_what;
    std::mutex bad_mu;
    auto work = [&] {
      for (size_t i = next++; i < ex.size() && !bad; i = next++) {
        const Extent& e = ex[i];
        int64_t done = 0;
        while (done < e.nbytes) {
          const ssize_t r = ::pread(fds_[e.file], buf + buf_off[i] + done, (size_t)(e.nbytes - done),
                                    (off_t)(e.offset + done));
          if (r <= 0) {
            std::lock_guard<std::mutex> g(bad_mu);
            bad = true;
            bad_what = "short read of " + paths_[e.file];
            return;
          }
          done += r;
        }
      }
    };
    const int n = std::min<int>(n_threads_, (int)ex.size());
    std::vector<std::thread> pool;
    for (int t = 1; t < n; ++t) pool.emplace_back(work);
    work();
    for (auto& t : pool) t.join();
    if (bad) throw std::runtime_error(bad_what);
  }

  void run() {
    try {
      if (device_ >= 0) check(cudaSetDevice(device_), "cudaSetDevice");
      std::vector<int64_t> buf_off;
      for (int l = 0; l < (int)layers_.size(); ++l) {
        const int b = l % n_buffers_;
        // the buffer's previous copies must have left it (double buffering)
        if (device_ >= 0 && l >= n_buffers_) check(cudaEventSynchronize(buffer_free_[b]), "cudaEventSynchronize");
        char* buf = static_cast<char*>(staging_[b]);
        const double t = now_ms();
        read_layer(layers_[l], buf, buf_off);
        const double dt = now_ms() - t;
        int64_t nb = 0;
        for (size_t i = 0; i < layers_[l].size(); ++i) {
          const Extent& e = layers_[l][i];
          nb += e.nbytes;
          char* dst = reinterpret_cast<char*>(dst_base_) + e.dst_offset;
          if (device_ >= 0) {
            check(cudaMemcpyAsync(dst, buf + buf_off[i], (size_t)e.nbytes, cudaMemcpyHostToDevice, stream_),
                  "cudaMemcpyAsync");
          } else {
            std::memcpy(dst, buf + buf_off[i], (size_t)e.nbytes);
          }
        }
        if (device_ >= 0) {
          check(cudaEventRecord(layer_ready_[l], stream_), "cudaEventRecord");
          check(cudaEventRecord(buffer_free_[b], stream_), "cudaEventRecord");
        }
        std::lock_guard<std::mutex> g(mu_);
        read_ms_[l] = dt;
        bytes_ += nb;
        enqueued_ = l + 1;
        cv_.notify_all();
      }
      if (device_ >= 0) check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
      done_ms_ = now_ms();
    } catch (const std::exception& e) {
      done_ms_ = now_ms();
      fail(e.what());
    }
  }

  std::vector<std::string> paths_;
  std::vector<int> fds_;
  int64_t staging_bytes_;
  int n_buffers_, n_threads_, device_;
  cudaStream_t stream_ = nullptr;
  cudaEvent_t after_ = nullptr;
  std::vector<void*> staging_;
  std::vector<cudaEvent_t> buffer_free_, layer_ready_;
  std::vector<std::vector<Extent>> layers_;
  int64_t dst_base_ = 0;
  std::thread worker_;
  std::mutex mu_;
  std::condition_variable cv_;
  int enqueued_ = 0;
  std::string error_;
  std::vector<double> read_ms_;
  int64_t bytes_ = 0;
  double t0_ms_ = 0, done_ms_ = 0;
};

void register_disk_loader(py::module& m) {
  py::class_<LayerwiseKVLoader>(m, "LayerwiseKVLoader")
      .def(py::init<int64_t, int, int, int>(), py::arg("staging_bytes"), py::arg("n_buffers") = 2,
           py::arg("n_threads") = 4, py::arg("device") = -1)
      .def("start", &LayerwiseKVLoader::start, py::arg("paths"), py::arg("plan"), py::arg("dst_base"),
           py::arg("after_stream") = 0)
      .def_property_readonly("staging_bytes", &LayerwiseKVLoader::staging_bytes)
      .def("wait_layer", &LayerwiseKVLoader::wait_layer, py::arg("layer"), py::arg("stream") = 0,
           py::call_guard<py::gil_scoped_release>())
      .def("join", &LayerwiseKVLoader::join, py::call_guard<py::gil_scoped_release>())
      .def("stats", &LayerwiseKVLoader::stats);
}

}  // namespace sc
