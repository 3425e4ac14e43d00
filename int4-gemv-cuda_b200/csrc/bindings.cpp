// The torch binding: the Python module int4gemv_ops with the reference's eight functions, names,
// argument names and defaults (csrc/bindings.cpp:20-41 of Yu-TingLee/int4-GEMV-cuda), plus the
// B200 fast path and the packed-format helpers. Each function checks its tensors (checks.cpp),
// allocates the output through torch's caching allocator on the input's device, and calls the
// torch-free C ABI (include/int4gemv_b200.h) on torch's current stream. Nothing synchronises.
#include <ATen/Parallel.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>

#include <vector>

#include "int4gemv_b200.h"
#include "int4gemv_torch.h"

namespace int4gemv {
namespace {

// Defaults from the reference's block sweep (csrc/bindings.cpp:8-12).
constexpr int64_t kDefaultThreadsPerBlock = 128;
constexpr int64_t kDefaultRowsPerWarp = 2;

void check_status(int status) { TORCH_CHECK(status == INT4GEMV_OK, int4gemv_last_error()); }

void* stream_of(const at::Tensor& t) {
  return static_cast<void*>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

using CudaGemv = int (*)(void*, const void*, const void*, const void*, const void*, int64_t,
                         int64_t, int64_t, int64_t, void*);

at::Tensor run_gemv(const char* name, CudaGemv fn, const at::Tensor& x, const at::Tensor& qweight,
                    const at::Tensor& scales, const at::Tensor& zeros, int64_t group_size) {
  check_inputs(name, x, qweight, scales, zeros, group_size, c10::DeviceType::CUDA);
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor y = x.new_empty({x.size(0), qweight.size(0)});
  check_status(fn(y.data_ptr(), x.data_ptr(), qweight.data_ptr(), scales.data_ptr(),
                  zeros.data_ptr(), x.size(0), qweight.size(0), x.size(1), group_size,
                  stream_of(x)));
  return y;
}

KernelInfo info_of(const char* kernel, int64_t m, int64_t threads, int64_t rows_per_warp) {
  int64_t v[6] = {};
  check_status(int4gemv_kernel_info(kernel, m, threads, rows_per_warp, v));
  return {{"registers", v[0]},       {"local_bytes", v[1]},
          {"threads_per_block", v[2]}, {"max_threads_per_block", v[3]},
          {"blocks_per_sm", v[4]},   {"warps_per_sm", v[5]}};
}

}  // namespace

at::Tensor sequential(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales,
                      const at::Tensor& zeros, int64_t group_size) {
  check_inputs("sequential", x, qweight, scales, zeros, group_size, c10::DeviceType::CPU);
  at::Tensor y = x.new_empty({x.size(0), qweight.size(0)});
  check_status(int4gemv_sequential(y.data_ptr(), x.data_ptr(), qweight.data_ptr(),
                                   scales.data_ptr(), zeros.data_ptr(), x.size(0),
                                   qweight.size(0), x.size(1), group_size,
                                   at::get_num_threads()));
  return y;
}

at::Tensor naive(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales,
                 const at::Tensor& zeros, int64_t group_size) {
  return run_gemv("naive", &int4gemv_naive, x, qweight, scales, zeros, group_size);
}

at::Tensor coalesced(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales,
                     const at::Tensor& zeros, int64_t group_size) {
  return run_gemv("coalesced", &int4gemv_coalesced, x, qweight, scales, zeros, group_size);
}

at::Tensor vectorized(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales,
                      const at::Tensor& zeros, int64_t group_size, int64_t threads_per_block,
                      int64_t rows_per_warp) {
  check_inputs("vectorized", x, qweight, scales, zeros, group_size, c10::DeviceType::CUDA);
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor y = x.new_empty({x.size(0), qweight.size(0)});
  check_status(int4gemv_vectorized(y.data_ptr(), x.data_ptr(), qweight.data_ptr(),
                                   scales.data_ptr(), zeros.data_ptr(), x.size(0),
                                   qweight.size(0), x.size(1), group_size, threads_per_block,
                                   rows_per_warp, stream_of(x)));
  return y;
}

at::Tensor load_only(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales,
                     const at::Tensor& zeros, int64_t group_size, int64_t threads_per_block,
                     int64_t rows_per_warp) {
  check_inputs("load_only", x, qweight, scales, zeros, group_size, c10::DeviceType::CUDA);
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor out = qweight.new_empty({qweight.size(0)});
  check_status(int4gemv_load_only(out.data_ptr(), x.data_ptr(), qweight.data_ptr(),
                                  scales.data_ptr(), zeros.data_ptr(), x.size(0),
                                  qweight.size(0), x.size(1), group_size, threads_per_block,
                                  rows_per_warp, stream_of(x)));
  return out;
}

KernelInfo naive_info(int64_t m) { return info_of("naive", m, 0, 1); }
KernelInfo coalesced_info(int64_t m) { return info_of("coalesced", m, 0, 1); }
KernelInfo vectorized_info(int64_t m, int64_t threads_per_block, int64_t rows_per_warp) {
  return info_of("vectorized", m, threads_per_block, rows_per_warp);
}
KernelInfo w4a16_info(int64_t m) { return info_of("w4a16", m, 0, 1); }

at::Tensor w4a16(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales,
                 const at::Tensor& zeros, int64_t group_size) {
  check_inputs("w4a16", x, qweight, scales, zeros, group_size, c10::DeviceType::CUDA);
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t m = x.size(0), n = qweight.size(0), k = x.size(1);
  at::Tensor y = x.new_empty({m, n});
  const int64_t ws_bytes = int4gemv_w4a16_workspace_size(m, n, k, group_size);
  at::Tensor ws;
  if (ws_bytes > 0) ws = at::empty({ws_bytes}, x.options().dtype(at::kByte));
  check_status(int4gemv_w4a16(y.data_ptr(), x.data_ptr(), qweight.data_ptr(), scales.data_ptr(),
                              zeros.data_ptr(), m, n, k, group_size,
                              ws_bytes > 0 ? ws.data_ptr() : nullptr, ws_bytes, stream_of(x)));
  return y;
}

at::Tensor w4a16_with(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales,
                      const at::Tensor& zeros, int64_t group_size, const std::string& kernel) {
  check_inputs("w4a16", x, qweight, scales, zeros, group_size, c10::DeviceType::CUDA);
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor y = x.new_empty({x.size(0), qweight.size(0)});
  check_status(int4gemv_w4a16_kernel(kernel.c_str(), y.data_ptr(), x.data_ptr(),
                                     qweight.data_ptr(), scales.data_ptr(), zeros.data_ptr(),
                                     x.size(0), qweight.size(0), x.size(1), group_size,
                                     stream_of(x)));
  return y;
}

std::string w4a16_kernel(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales,
                         const at::Tensor& zeros, int64_t group_size) {
  check_inputs("w4a16", x, qweight, scales, zeros, group_size, c10::DeviceType::CUDA);
  return int4gemv_w4a16_kernel_name(x.data_ptr(), qweight.data_ptr(), scales.data_ptr(),
                                    zeros.data_ptr(), x.size(0), qweight.size(0), x.size(1),
                                    group_size);
}

at::Tensor w4a16_silu_mul(const at::Tensor& x, const at::Tensor& qweight,
                          const at::Tensor& scales, const at::Tensor& zeros, int64_t group_size) {
  check_inputs("w4a16_silu_mul", x, qweight, scales, zeros, group_size, c10::DeviceType::CUDA);
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t m = x.size(0), n = qweight.size(0), k = x.size(1);
  TORCH_CHECK(n % 2 == 0, "w4a16_silu_mul: qweight must hold gate and up rows in pairs, got ", n,
              " rows");
  at::Tensor y = x.new_empty({m, n / 2});
  check_status(int4gemv_w4a16_silu_mul(y.data_ptr(), x.data_ptr(), qweight.data_ptr(),
                                       scales.data_ptr(), zeros.data_ptr(), m, n, k, group_size,
                                       stream_of(x)));
  return y;
}

at::Tensor w4a16_f32(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales,
                     const at::Tensor& zeros, int64_t group_size) {
  check_inputs("w4a16_f32", x, qweight, scales, zeros, group_size, c10::DeviceType::CUDA);
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t m = x.size(0), n = qweight.size(0), k = x.size(1);
  at::Tensor y = at::empty({m, n}, x.options().dtype(at::kFloat));
  check_status(int4gemv_w4a16_f32(y.data_ptr(), x.data_ptr(), qweight.data_ptr(),
                                  scales.data_ptr(), zeros.data_ptr(), m, n, k, group_size,
                                  stream_of(x)));
  return y;
}

std::vector<at::Tensor> w4a16_grouped(const at::Tensor& x, const at::Tensor& qweight,
                                      const at::Tensor& scales, const at::Tensor& zeros,
                                      int64_t group_size, const std::vector<int64_t>& sizes) {
  check_inputs("w4a16_grouped", x, qweight, scales, zeros, group_size, c10::DeviceType::CUDA);
  TORCH_CHECK(!sizes.empty() && sizes.size() <= INT4GEMV_MAX_GROUP, "w4a16_grouped: between 1 and ",
              INT4GEMV_MAX_GROUP, " matrices, got ", sizes.size());
  int64_t total = 0;
  for (int64_t n : sizes) {
    TORCH_CHECK(n >= 0, "w4a16_grouped: negative matrix size ", n);
    total += n;
  }
  TORCH_CHECK(total == qweight.size(0), "w4a16_grouped: sizes add up to ", total,
              " rows, the stacked qweight has ", qweight.size(0));
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t m = x.size(0);
  std::vector<at::Tensor> ys;
  std::vector<void*> ptrs;
  for (int64_t n : sizes) {
    ys.push_back(x.new_empty({m, n}));
    ptrs.push_back(ys.back().data_ptr());
  }
  check_status(int4gemv_w4a16_grouped(static_cast<int>(sizes.size()), ptrs.data(), sizes.data(),
                                      x.data_ptr(), qweight.data_ptr(), scales.data_ptr(),
                                      zeros.data_ptr(), m, x.size(1), group_size, stream_of(x)));
  return ys;
}

at::Tensor w4a16_bias_residual(const at::Tensor& x, const at::Tensor& qweight,
                               const at::Tensor& scales, const at::Tensor& zeros,
                               int64_t group_size, const c10::optional<at::Tensor>& bias,
                               const c10::optional<at::Tensor>& residual) {
  check_inputs("w4a16_bias_residual", x, qweight, scales, zeros, group_size, c10::DeviceType::CUDA);
  const int64_t m = x.size(0), n = qweight.size(0), k = x.size(1);
  const void* bias_ptr = nullptr;
  const void* res_ptr = nullptr;
  if (bias.has_value()) {
    const at::Tensor& b = *bias;
    TORCH_CHECK(b.scalar_type() == at::kHalf && b.dim() == 1 && b.size(0) == n && b.is_contiguous() &&
                    b.device() == x.device(),
                "w4a16_bias_residual: bias must be a contiguous float16 [", n, "] tensor on x's device");
    bias_ptr = b.data_ptr();
  }
  if (residual.has_value()) {
    const at::Tensor& r = *residual;
    TORCH_CHECK(r.scalar_type() == at::kHalf && r.dim() == 2 && r.size(0) == m && r.size(1) == n &&
                    r.is_contiguous() && r.device() == x.device(),
                "w4a16_bias_residual: residual must be a contiguous float16 [", m, ", ", n,
                "] tensor on x's device");
    res_ptr = r.data_ptr();
  }
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor y = x.new_empty({m, n});
  check_status(int4gemv_w4a16_bias_residual(y.data_ptr(), x.data_ptr(), qweight.data_ptr(),
                                            scales.data_ptr(), zeros.data_ptr(), bias_ptr, res_ptr,
                                            m, n, k, group_size, stream_of(x)));
  return y;
}

at::Tensor unpack(const at::Tensor& qweight) {
  TORCH_CHECK(qweight.scalar_type() == at::kInt && qweight.dim() == 2 && qweight.is_contiguous() &&
                  qweight.is_cuda(),
              "unpack: expected a contiguous 2-D int32 CUDA qweight");
  const c10::cuda::CUDAGuard guard(qweight.device());
  at::Tensor q = qweight.new_empty({qweight.size(0), qweight.size(1) * 8});
  check_status(int4gemv_unpack(q.data_ptr(), qweight.data_ptr(), qweight.size(0),
                               qweight.size(1) * 8, stream_of(qweight)));
  return q;
}

at::Tensor dequantize(const at::Tensor& qweight, const at::Tensor& scales, const at::Tensor& zeros,
                      int64_t group_size) {
  // Same checks as the GEMV, with an empty x of the right K standing in for the activations.
  const int64_t k = qweight.dim() == 2 ? qweight.size(1) * 8 : 0;
  const at::Tensor x = at::empty({0, k}, scales.options().dtype(at::kHalf));
  check_inputs("dequantize", x, qweight, scales, zeros, group_size, c10::DeviceType::CUDA);
  const c10::cuda::CUDAGuard guard(qweight.device());
  at::Tensor w = at::empty({qweight.size(0), k}, scales.options().dtype(at::kFloat));
  check_status(int4gemv_dequantize(w.data_ptr(), qweight.data_ptr(), scales.data_ptr(),
                                   zeros.data_ptr(), qweight.size(0), k, group_size,
                                   stream_of(qweight)));
  return w;
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> quantize(const at::Tensor& w, int64_t group_size) {
  TORCH_CHECK(w.dim() == 2 && w.is_cuda() && w.is_contiguous(),
              "quantize: expected a contiguous 2-D CUDA tensor w");
  int dtype;
  switch (w.scalar_type()) {
    case at::kFloat: dtype = INT4GEMV_DTYPE_F32; break;
    case at::kHalf: dtype = INT4GEMV_DTYPE_F16; break;
    case at::kBFloat16: dtype = INT4GEMV_DTYPE_BF16; break;
    default: TORCH_CHECK(false, "quantize: w must be float32, float16 or bfloat16, got ", w.scalar_type());
  }
  const int64_t n = w.size(0), k = w.size(1);
  TORCH_CHECK(group_size > 0 && group_size % 8 == 0 && k % group_size == 0, "quantize: group_size ",
              group_size, " must be a positive multiple of 8 dividing K = ", k);
  const c10::cuda::CUDAGuard guard(w.device());
  at::Tensor qweight = at::empty({n, k / 8}, w.options().dtype(at::kInt));
  at::Tensor scales = at::empty({n, k / group_size}, w.options().dtype(at::kHalf));
  at::Tensor zeros = at::empty({n, k / group_size}, w.options().dtype(at::kHalf));
  check_status(int4gemv_quantize(qweight.data_ptr(), scales.data_ptr(), zeros.data_ptr(),
                                 w.data_ptr(), dtype, n, k, group_size, stream_of(w)));
  return {qweight, scales, zeros};
}

at::Tensor pack(const at::Tensor& q) {
  TORCH_CHECK(q.scalar_type() == at::kInt && q.dim() == 2 && q.is_contiguous() && q.is_cuda(),
              "pack: expected a contiguous 2-D int32 CUDA q");
  TORCH_CHECK(q.size(1) % 8 == 0, "pack: K = ", q.size(1), " must be a multiple of 8");
  const c10::cuda::CUDAGuard guard(q.device());
  at::Tensor qweight = q.new_empty({q.size(0), q.size(1) / 8});
  check_status(int4gemv_pack(qweight.data_ptr(), q.data_ptr(), q.size(0), q.size(1), stream_of(q)));
  return qweight;
}

namespace {
void check_ck(const char* name, const at::Tensor& t, at::ScalarType dtype, int64_t rows,
              int64_t cols, const char* what, const at::Tensor& like) {
  TORCH_CHECK(t.scalar_type() == dtype && t.dim() == 2 && t.size(0) == rows && t.size(1) == cols &&
                  t.is_contiguous() && t.device() == like.device(),
              name, ": ", what, " must be a contiguous ", c10::toString(dtype), " [", rows, ", ", cols,
              "] tensor on the device of qweight, got ", t.scalar_type(), " ", t.sizes());
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> repack_outputs(const at::Tensor& like, int64_t n,
                                                              int64_t k, int64_t group_size) {
  return {at::empty({n, k / 8}, like.options().dtype(at::kInt)),
          at::empty({n, k / group_size}, like.options().dtype(at::kHalf)),
          at::empty({n, k / group_size}, like.options().dtype(at::kHalf))};
}
}  // namespace

std::tuple<at::Tensor, at::Tensor, at::Tensor> repack_awq(const at::Tensor& qweight,
                                                         const at::Tensor& qzeros,
                                                         const at::Tensor& scales,
                                                         int64_t group_size) {
  const char* name = "repack_awq";
  TORCH_CHECK(qweight.dim() == 2 && qweight.is_cuda(), name, ": qweight must be a 2-D CUDA tensor");
  TORCH_CHECK(group_size > 0 && qweight.size(0) % group_size == 0, name, ": group_size ",
              group_size, " must divide K = ", qweight.size(0));
  const int64_t k = qweight.size(0), n = qweight.size(1) * 8;
  check_ck(name, qweight, at::kInt, k, n / 8, "qweight", qweight);
  check_ck(name, qzeros, at::kInt, k / group_size, n / 8, "qzeros", qweight);
  check_ck(name, scales, at::kHalf, k / group_size, n, "scales", qweight);
  const c10::cuda::CUDAGuard guard(qweight.device());
  auto out = repack_outputs(qweight, n, k, group_size);
  check_status(int4gemv_repack_awq(std::get<0>(out).data_ptr(), std::get<1>(out).data_ptr(),
                                   std::get<2>(out).data_ptr(), qweight.data_ptr(),
                                   qzeros.data_ptr(), scales.data_ptr(), n, k, group_size,
                                   stream_of(qweight)));
  return out;
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> repack_gptq(const at::Tensor& qweight,
                                                          const at::Tensor& qzeros,
                                                          const at::Tensor& scales,
                                                          int64_t group_size, int64_t zero_offset) {
  const char* name = "repack_gptq";
  TORCH_CHECK(qweight.dim() == 2 && qweight.is_cuda(), name, ": qweight must be a 2-D CUDA tensor");
  const int64_t k = qweight.size(0) * 8, n = qweight.size(1);
  TORCH_CHECK(group_size > 0 && k % group_size == 0, name, ": group_size ", group_size,
              " must divide K = ", k);
  TORCH_CHECK(n % 8 == 0, name, ": N = ", n, " must be a multiple of 8 (packed zero points)");
  check_ck(name, qweight, at::kInt, k / 8, n, "qweight", qweight);
  check_ck(name, qzeros, at::kInt, k / group_size, n / 8, "qzeros", qweight);
  check_ck(name, scales, at::kHalf, k / group_size, n, "scales", qweight);
  const c10::cuda::CUDAGuard guard(qweight.device());
  auto out = repack_outputs(qweight, n, k, group_size);
  check_status(int4gemv_repack_gptq(std::get<0>(out).data_ptr(), std::get<1>(out).data_ptr(),
                                    std::get<2>(out).data_ptr(), qweight.data_ptr(),
                                    qzeros.data_ptr(), scales.data_ptr(),
                                    static_cast<int>(zero_offset), n, k, group_size,
                                    stream_of(qweight)));
  return out;
}

}  // namespace int4gemv

PYBIND11_MODULE(int4gemv_ops, m) {
  using int4gemv::kDefaultRowsPerWarp;
  using int4gemv::kDefaultThreadsPerBlock;
  m.def("sequential", &int4gemv::sequential, py::arg("x"), py::arg("qweight"), py::arg("scales"),
        py::arg("zeros"), py::arg("group_size"));
  m.def("naive", &int4gemv::naive, py::arg("x"), py::arg("qweight"), py::arg("scales"),
        py::arg("zeros"), py::arg("group_size"));
  m.def("coalesced", &int4gemv::coalesced, py::arg("x"), py::arg("qweight"), py::arg("scales"),
        py::arg("zeros"), py::arg("group_size"));
  m.def("vectorized", &int4gemv::vectorized, py::arg("x"), py::arg("qweight"), py::arg("scales"),
        py::arg("zeros"), py::arg("group_size"),
        py::arg("threads_per_block") = kDefaultThreadsPerBlock,
        py::arg("rows_per_warp") = kDefaultRowsPerWarp);
  m.def("load_only", &int4gemv::load_only, py::arg("x"), py::arg("qweight"), py::arg("scales"),
        py::arg("zeros"), py::arg("group_size"),
        py::arg("threads_per_block") = kDefaultThreadsPerBlock,
        py::arg("rows_per_warp") = kDefaultRowsPerWarp);
  m.def("naive_info", &int4gemv::naive_info, py::arg("m"));
  m.def("coalesced_info", &int4gemv::coalesced_info, py::arg("m"));
  m.def("vectorized_info", &int4gemv::vectorized_info, py::arg("m"),
        py::arg("threads_per_block") = kDefaultThreadsPerBlock,
        py::arg("rows_per_warp") = kDefaultRowsPerWarp);

  m.def("w4a16", &int4gemv::w4a16, py::arg("x"), py::arg("qweight"), py::arg("scales"),
        py::arg("zeros"), py::arg("group_size"));
  m.def("w4a16_info", &int4gemv::w4a16_info, py::arg("m"));
  m.def("w4a16_silu_mul", &int4gemv::w4a16_silu_mul, py::arg("x"), py::arg("qweight"),
        py::arg("scales"), py::arg("zeros"), py::arg("group_size"));
  m.def("w4a16_f32", &int4gemv::w4a16_f32, py::arg("x"), py::arg("qweight"), py::arg("scales"),
        py::arg("zeros"), py::arg("group_size") = 128);
  m.def("w4a16_with", &int4gemv::w4a16_with, py::arg("x"), py::arg("qweight"), py::arg("scales"),
        py::arg("zeros"), py::arg("group_size"), py::arg("kernel"));
  m.def("w4a16_kernel", &int4gemv::w4a16_kernel, py::arg("x"), py::arg("qweight"),
        py::arg("scales"), py::arg("zeros"), py::arg("group_size"));
  m.def("w4a16_grouped", &int4gemv::w4a16_grouped, py::arg("x"), py::arg("qweight"),
        py::arg("scales"), py::arg("zeros"), py::arg("group_size"), py::arg("sizes"));
  m.def("w4a16_bias_residual", &int4gemv::w4a16_bias_residual, py::arg("x"), py::arg("qweight"),
        py::arg("scales"), py::arg("zeros"), py::arg("group_size"), py::arg("bias") = py::none(),
        py::arg("residual") = py::none());
  m.def("unpack", &int4gemv::unpack, py::arg("qweight"));
  m.def("dequantize", &int4gemv::dequantize, py::arg("qweight"), py::arg("scales"),
        py::arg("zeros"), py::arg("group_size"));
  m.def("quantize", &int4gemv::quantize, py::arg("w"), py::arg("group_size") = 128);
  m.def("repack_awq", &int4gemv::repack_awq, py::arg("qweight"), py::arg("qzeros"),
        py::arg("scales"), py::arg("group_size"));
  m.def("repack_gptq", &int4gemv::repack_gptq, py::arg("qweight"), py::arg("qzeros"),
        py::arg("scales"), py::arg("group_size"), py::arg("zero_offset") = 1);
  m.def("pack", &int4gemv::pack, py::arg("q"));
  m.def(
      "check_inputs",
      [](const char* name, const at::Tensor& x, const at::Tensor& qweight,
         const at::Tensor& scales, const at::Tensor& zeros, int64_t group_size, bool cuda) {
        int4gemv::check_inputs(name, x, qweight, scales, zeros, group_size,
                               cuda ? c10::DeviceType::CUDA : c10::DeviceType::CPU);
      },
      py::arg("name"), py::arg("x"), py::arg("qweight"), py::arg("scales"), py::arg("zeros"),
      py::arg("group_size"), py::arg("cuda"));
}
