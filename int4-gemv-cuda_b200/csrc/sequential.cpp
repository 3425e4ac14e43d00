// The CPU path of the operator (replaces int4gemv::sequential, csrc/sequential.cpp:11-54 of the
// reference). The fp32 arithmetic follows the same order as the reference, so the result is
// bit-identical: per output row and group, dequantise group_size weights as (q - z) * s, take the
// fp32 dot product with each row of x left to right, add it to the row's running sum; round the
// sum to fp16 at the end. Output rows are independent, so they are spread over host threads
// without changing any result. Must be compiled without FMA contraction or fast-math.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace i4 {
namespace {

inline float half_bits_to_float(uint16_t bits) {
  _Float16 h;
  std::memcpy(&h, &bits, sizeof h);
  return static_cast<float>(h);
}

inline uint16_t float_to_half_bits(float f) {
  const _Float16 h = static_cast<_Float16>(f);  // round to nearest even
  uint16_t bits;
  std::memcpy(&bits, &h, sizeof bits);
  return bits;
}

void rows_range(uint16_t* y, const float* xf, const uint32_t* q, const uint16_t* s,
                const uint16_t* z, int64_t m, int64_t n, int64_t k, int64_t group,
                int64_t row_begin, int64_t row_end) {
  const int64_t groups = k / group;
  const int64_t words = k / 8;
  std::vector<float> w(group);
  std::vector<float> acc(m);
  for (int64_t row = row_begin; row < row_end; ++row) {
    std::fill(acc.begin(), acc.end(), 0.0f);
    for (int64_t g = 0; g < groups; ++g) {
      const float sc = half_bits_to_float(s[row * groups + g]);
      const float zp = half_bits_to_float(z[row * groups + g]);
      const uint32_t* qg = q + row * words + g * (group / 8);
      for (int64_t i = 0; i < group; ++i) {
        const uint32_t nib = (qg[i >> 3] >> (4 * (i & 7))) & 0xFu;
        w[i] = (static_cast<float>(nib) - zp) * sc;
      }
      for (int64_t r = 0; r < m; ++r) {
        const float* xg = xf + r * k + g * group;
        float dot = 0.0f;
        for (int64_t i = 0; i < group; ++i) dot += xg[i] * w[i];
        acc[r] += dot;
      }
    }
    for (int64_t r = 0; r < m; ++r) y[r * n + row] = float_to_half_bits(acc[r]);
  }
}

}  // namespace

void sequential_cpu(uint16_t* y, const uint16_t* x, const uint32_t* q, const uint16_t* s,
                    const uint16_t* z, int64_t m, int64_t n, int64_t k, int64_t group,
                    int64_t threads) {
  std::vector<float> xf(static_cast<size_t>(m * k));
  for (int64_t i = 0; i < m * k; ++i) xf[i] = half_bits_to_float(x[i]);
  if (threads <= 0) threads = std::max(1u, std::thread::hardware_concurrency());
  threads = std::max<int64_t>(1, std::min<int64_t>(threads, n));
  if (threads == 1) {
    rows_range(y, xf.data(), q, s, z, m, n, k, group, 0, n);
    return;
  }
  std::vector<std::thread> pool;
  pool.reserve(threads);
  for (int64_t t = 0; t < threads; ++t) {
    pool.emplace_back(rows_range, y, xf.data(), q, s, z, m, n, k, group, n * t / threads,
                      n * (t + 1) / threads);
  }
  for (auto& th : pool) th.join();
}

}  // namespace i4
