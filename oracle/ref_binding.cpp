// Python binding for the REFERENCE's own implementation, compiled from its sources where they lie
// (csrc/checks.cpp, csrc/sequential.cpp, csrc/{naive,coalesced,vectorized,load_only}.cu of
// Yu-TingLee/int4-GEMV-cuda) by oracle/build_ref.py into oracle/_ref/. TEST INFRASTRUCTURE ONLY:
// it pins the oracle (tests/golden/make_golden.py), is the second GPU oracle in the parity tests
// and is the reference arm of bench.py. The module name differs from the product's int4gemv_ops
// so both can be loaded in one process.
//
// The only thing added here is sequential_threads: it splits the output rows into slices and runs
// the reference's own int4gemv::sequential (csrc/sequential.cpp:11) on each slice in its own
// thread. Rows are independent in that loop, so the result is bit-identical to one call.
#include <torch/extension.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "w4a16.h"

namespace {

at::Tensor sequential_threads(const at::Tensor& x, const at::Tensor& qweight,
                              const at::Tensor& scales, const at::Tensor& zeros,
                              int64_t group_size, int64_t threads) {
  const int64_t n = qweight.size(0);
  threads = std::max<int64_t>(1, std::min<int64_t>(threads, n));
  if (threads == 1) {
    return int4gemv::sequential(x, qweight, scales, zeros, group_size);
  }
  std::vector<at::Tensor> parts(threads);
  std::vector<std::thread> pool;
  pool.reserve(threads);
  for (int64_t t = 0; t < threads; ++t) {
    const int64_t r0 = n * t / threads;
    const int64_t r1 = n * (t + 1) / threads;
    pool.emplace_back([&, t, r0, r1] {
      parts[t] = int4gemv::sequential(x, qweight.narrow(0, r0, r1 - r0).contiguous(),
                                      scales.narrow(0, r0, r1 - r0).contiguous(),
                                      zeros.narrow(0, r0, r1 - r0).contiguous(), group_size);
    });
  }
  {
    py::gil_scoped_release release;
    for (auto& th : pool) th.join();
  }
  return at::cat(parts, 1);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("sequential", &int4gemv::sequential, py::arg("x"), py::arg("qweight"), py::arg("scales"),
        py::arg("zeros"), py::arg("group_size"));
  m.def("sequential_threads", &sequential_threads, py::arg("x"), py::arg("qweight"),
        py::arg("scales"), py::arg("zeros"), py::arg("group_size"), py::arg("threads"));
  m.def("naive", &int4gemv::naive, py::arg("x"), py::arg("qweight"), py::arg("scales"),
        py::arg("zeros"), py::arg("group_size"));
  m.def("coalesced", &int4gemv::coalesced, py::arg("x"), py::arg("qweight"), py::arg("scales"),
        py::arg("zeros"), py::arg("group_size"));
  m.def("vectorized", &int4gemv::vectorized, py::arg("x"), py::arg("qweight"), py::arg("scales"),
        py::arg("zeros"), py::arg("group_size"), py::arg("threads_per_block") = 128,
        py::arg("rows_per_warp") = 2);
  m.def("load_only", &int4gemv::load_only, py::arg("x"), py::arg("qweight"), py::arg("scales"),
        py::arg("zeros"), py::arg("group_size"), py::arg("threads_per_block") = 128,
        py::arg("rows_per_warp") = 2);
  m.def(
      "check_inputs",
      [](const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales,
         const at::Tensor& zeros, int64_t group_size, bool cuda) {
        int4gemv::check_inputs("check", x, qweight, scales, zeros, group_size,
                               cuda ? c10::DeviceType::CUDA : c10::DeviceType::CPU);
      },
      py::arg("x"), py::arg("qweight"), py::arg("scales"), py::arg("zeros"),
      py::arg("group_size"), py::arg("cuda") = false);
}
