// Host-side tranche packing: gather token ranges of a [rows, T, D] KV tensor
// into one contiguous [rows, W, D] block with a pool of threads.
//
// Counterpart of the reference's pinned tranche packing (the P/D pipeline's
// per-stage CPU gather of token ranges into a pinned buffer, done there as a
// PyTorch concatenation followed by a copy into pinned memory): one pass,
// straight into the destination (normally pinned host memory, which the copy
// engine then moves to the device in one transfer per stage).  Rows are
// split evenly over the threads; each row copies its ranges back to back.
#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <torch/extension.h>

namespace py = pybind11;

namespace sc {

namespace {

// Copies ranges [starts[i], ends[i]) of every row of src ([rows, T, D], row-major)
// into dst ([rows, W, D]) back to back, W = sum of the range widths.
void pack_token_ranges(const torch::Tensor& src, const std::vector<int64_t>& starts,
                       const std::vector<int64_t>& ends, torch::Tensor& dst, int64_t n_threads) {
  TORCH_CHECK(src.device().is_cpu() && dst.device().is_cpu(), "pack_token_ranges works on host tensors");
  TORCH_CHECK(src.is_contiguous() && dst.is_contiguous(), "pack_token_ranges needs contiguous tensors");
  TORCH_CHECK(src.dim() == 3 && dst.dim() == 3, "src and dst are [rows, tokens, D]");
  TORCH_CHECK(src.scalar_type() == dst.scalar_type(), "src and dst dtypes differ");
  TORCH_CHECK(starts.size() == ends.size(), "one end per start");
  const int64_t rows = src.size(0), T = src.size(1), D = src.size(2);
  TORCH_CHECK(dst.size(0) == rows && dst.size(2) == D, "dst rows / head dim differ from src");
  int64_t width = 0;
  for (size_t i = 0; i < starts.size(); ++i) {
    TORCH_CHECK(0 <= starts[i] && starts[i] <= ends[i] && ends[i] <= T, "range outside the source tokens");
    width += ends[i] - starts[i];
  }
  TORCH_CHECK(dst.size(1) == width, "dst token count differs from the sum of the ranges");
  const int64_t token_bytes = D * (int64_t)src.element_size();
  const char* s = static_cast<const char*>(src.data_ptr());
  char* d = static_cast<char*>(dst.data_ptr());
  const int64_t nt = std::max<int64_t>(1, std::min<int64_t>(n_threads, rows));
  auto work = [&](int64_t r0, int64_t r1) {
    for (int64_t r = r0; r < r1; ++r) {
      const char* srow = s + r * T * token_bytes;
      char* drow = d + r * width * token_bytes;
      int64_t at = 0;
      for (size_t i = 0; i < starts.size(); ++i) {
        const int64_t n = ends[i] - starts[i];
        std::memcpy(drow + at * token_bytes, srow + starts[i] * token_bytes, (size_t)(n * token_bytes));
        at += n;
      }
    }
  };
  if (nt == 1) {
    work(0, rows);
    return;
  }
  std::vector<std::thread> pool;
  pool.reserve(nt);
  for (int64_t t = 0; t < nt; ++t) {
    const int64_t r0 = rows * t / nt, r1 = rows * (t + 1) / nt;
    pool.emplace_back(work, r0, r1);
  }
  for (auto& th : pool) th.join();
}

}  // namespace

void register_host_pack(py::module& m) {
  m.def("pack_token_ranges", &pack_token_ranges, py::arg("src"), py::arg("starts"), py::arg("ends"),
        py::arg("dst"), py::arg("n_threads") = 8, py::call_guard<py::gil_scoped_release>());
}

}  // namespace sc
