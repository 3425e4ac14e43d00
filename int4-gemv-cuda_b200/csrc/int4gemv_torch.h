// C++ / torch API of the library: the reference's operator declarations (csrc/w4a16.h:17-54 of
// Yu-TingLee/int4-GEMV-cuda), same namespace, names and signatures, so C++ callers of the
// reference link against this instead. Plus the B200 fast path and the packed-format helpers.
//
// y = x @ dequant(W).T, w = (q - z) * s, every group_size weights along K sharing one s and z:
//   x        [M, K]          fp16
//   qweight  [N, K / 8]      int32, eight 4-bit q per word, lowest bits first
//   scales   [N, K / group]  fp16
//   zeros    [N, K / group]  fp16
// Returns y [M, N] fp16 (empty if M or N is 0). Wrong dtypes, shapes or devices throw c10::Error.
#pragma once

#include <ATen/core/Tensor.h>
#include <c10/core/DeviceType.h>
#include <c10/util/Optional.h>

#include <cstdint>
#include <map>
#include <string>
#include <tuple>
#include <vector>

namespace int4gemv {

using KernelInfo = std::map<std::string, int64_t>;

// CPU path, bit-identical to the reference's sequential (csrc/w4a16.h:23).
at::Tensor sequential(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales,
                      const at::Tensor& zeros, int64_t group_size);

// One thread per output row (csrc/w4a16.h:27-29).
at::Tensor naive(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales,
                 const at::Tensor& zeros, int64_t group_size);
KernelInfo naive_info(int64_t m);

// One warp per output row (csrc/w4a16.h:32-34).
at::Tensor coalesced(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales,
                     const at::Tensor& zeros, int64_t group_size);
KernelInfo coalesced_info(int64_t m);

// rows_per_warp (1, 2, 4) rows per warp, 16-byte loads (csrc/w4a16.h:38-41).
at::Tensor vectorized(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales,
                      const at::Tensor& zeros, int64_t group_size, int64_t threads_per_block,
                      int64_t rows_per_warp);
KernelInfo vectorized_info(int64_t m, int64_t threads_per_block, int64_t rows_per_warp);

// vectorized's loads without the math, M = 1 (csrc/w4a16.h:45-47).
at::Tensor load_only(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales,
                     const at::Tensor& zeros, int64_t group_size, int64_t threads_per_block,
                     int64_t rows_per_warp);

// Shared input checks, same conditions and messages as csrc/checks.cpp:9-44.
void check_inputs(const char* name, const at::Tensor& x, const at::Tensor& qweight,
                  const at::Tensor& scales, const at::Tensor& zeros, int64_t group_size,
                  c10::DeviceType device);

// The B200 fast path (no counterpart in the reference): the best kernel for the shape.
at::Tensor w4a16(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales,
                 const at::Tensor& zeros, int64_t group_size);
KernelInfo w4a16_info(int64_t m);
// One named kernel ("tcgen05", "mma_pipeline", "vectorized", "coalesced", "naive"), for tests.
at::Tensor w4a16_with(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales,
                      const at::Tensor& zeros, int64_t group_size, const std::string& kernel);
std::string w4a16_kernel(const at::Tensor& x, const at::Tensor& qweight, const at::Tensor& scales,
                         const at::Tensor& zeros, int64_t group_size);

// Fused gate / up projection: the rows of qweight, scales and zeros are gate and up rows
// interleaved (quant.interleave_rows); returns silu(x @ gate^T) * (x @ up^T), [M, N / 2] fp16.
at::Tensor w4a16_silu_mul(const at::Tensor& x, const at::Tensor& qweight,
                          const at::Tensor& scales, const at::Tensor& zeros, int64_t group_size);

// Several matrices sharing x, their packed weights stacked by rows (sizes[i] rows each): one
// launch, one output [M, sizes[i]] per matrix.
std::vector<at::Tensor> w4a16_grouped(const at::Tensor& x, const at::Tensor& qweight,
                                      const at::Tensor& scales, const at::Tensor& zeros,
                                      int64_t group_size, const std::vector<int64_t>& sizes);

// x @ W^T + bias + residual with both additions fused into the GEMV's store (each optional;
// bias [N], residual [M, N], float16), rounded to fp16 once.
at::Tensor w4a16_bias_residual(const at::Tensor& x, const at::Tensor& qweight,
                               const at::Tensor& scales, const at::Tensor& zeros,
                               int64_t group_size, const c10::optional<at::Tensor>& bias,
                               const c10::optional<at::Tensor>& residual);

// Bit-exact device versions of int4gemv/quant.py:40-53.
at::Tensor unpack(const at::Tensor& qweight);
at::Tensor dequantize(const at::Tensor& qweight, const at::Tensor& scales, const at::Tensor& zeros,
                      int64_t group_size);

// Bit-exact device versions of int4gemv/quant.py:14-37 for finite weights: w [N, K] fp32, fp16
// or bf16 (CUDA, contiguous) -> (qweight, scales, zeros); q [N, K] int32 -> qweight.
std::tuple<at::Tensor, at::Tensor, at::Tensor> quantize(const at::Tensor& w, int64_t group_size);
at::Tensor pack(const at::Tensor& q);

// AWQ / GPTQ checkpoint tensors (CUDA, contiguous) -> (qweight, scales, zeros) of this layout.
// zero_offset: 1 for GPTQ's original format (stored z - 1), 0 for gptq_v2.
std::tuple<at::Tensor, at::Tensor, at::Tensor> repack_awq(const at::Tensor& qweight,
                                                         const at::Tensor& qzeros,
                                                         const at::Tensor& scales,
                                                         int64_t group_size);
std::tuple<at::Tensor, at::Tensor, at::Tensor> repack_gptq(const at::Tensor& qweight,
                                                          const at::Tensor& qzeros,
                                                          const at::Tensor& scales,
                                                          int64_t group_size, int64_t zero_offset);

}  // namespace int4gemv
