// Input checks of the torch API. The conditions and messages are the operator's contract and are
// kept identical to the reference (csrc/checks.cpp:9-44 of Yu-TingLee/int4-GEMV-cuda), so code
// that matches on the reference's error text keeps working.
#include <c10/util/Exception.h>

#include <array>
#include <limits>

#include "int4gemv_torch.h"

namespace int4gemv {

void check_inputs(const char* name, const at::Tensor& x, const at::Tensor& qweight,
                  const at::Tensor& scales, const at::Tensor& zeros, int64_t group_size,
                  c10::DeviceType device) {
  const bool dtypes_ok = x.scalar_type() == at::kHalf && qweight.scalar_type() == at::kInt &&
                         scales.scalar_type() == at::kHalf && zeros.scalar_type() == at::kHalf;
  TORCH_CHECK(dtypes_ok, name, ": expected fp16 x, int32 qweight, fp16 scales and zeros, got ",
              x.scalar_type(), ", ", qweight.scalar_type(), ", ", scales.scalar_type(), ", ",
              zeros.scalar_type());
  const std::array<const at::Tensor*, 4> all = {&x, &qweight, &scales, &zeros};
  bool two_d = true;
  for (const at::Tensor* t : all) two_d = two_d && t->dim() == 2;
  TORCH_CHECK(two_d, name, ": expected 2-D inputs");

  const int64_t m = x.size(0);
  const int64_t k = x.size(1);
  const int64_t n = qweight.size(0);
  constexpr int64_t int_max = std::numeric_limits<int>::max();  // kernels index with int
  TORCH_CHECK(m <= int_max && n <= int_max && k <= int_max, name, ": M = ", m, ", N = ", n,
              ", K = ", k, " must each fit in int");
  TORCH_CHECK(group_size > 0 && group_size % 8 == 0 && k % group_size == 0, name, ": group_size ",
              group_size, " must be a positive multiple of 8 dividing K = ", k);
  TORCH_CHECK(qweight.size(1) * 8 == k, name, ": qweight of shape ", qweight.sizes(),
              " does not pack K = ", k);
  const int64_t groups = k / group_size;
  TORCH_CHECK(scales.size(0) == n && scales.size(1) == groups && zeros.sizes() == scales.sizes(),
              name, ": scales ", scales.sizes(), " and zeros ", zeros.sizes(), " must be [", n,
              ", ", groups, "]");
  bool contiguous = true;
  for (const at::Tensor* t : all) contiguous = contiguous && t->is_contiguous();
  TORCH_CHECK(contiguous, name, ": inputs must be contiguous");
  for (const at::Tensor* t : all) {
    TORCH_CHECK(t->device().type() == device && t->device() == x.device(), name,
                ": expected all inputs on one ", device, " device, got ", x.device(), " and ",
                t->device());
  }
}

}  // namespace int4gemv
