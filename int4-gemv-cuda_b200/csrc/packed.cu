// Device versions of the packed-format helpers of int4gemv/quant.py (reference), bit-exact:
//   unpack      q[n, 8w + j] = (qweight[n, w] >> 4j) & 0xF              (quant.py:40-44)
//   dequantize  w = (float(q) - float(z)) * float(s), one IEEE rounding
//               per operation, no FMA contraction                        (quant.py:47-53)
// Plus y = bias + residual, the K = 0 case of the fused bias / residual GEMV epilogue.
// One thread per packed word; the word's eight outputs are written as two 16-byte (unpack) or
// two 32-byte (dequantize) vectors. Grid-stride loops sized to a multiple of the SM count.
#include "common.cuh"
#include "kernels.h"

namespace i4 {
namespace {

constexpr int kThreads = 256;

__global__ void unpack_kernel(int4* __restrict__ q, const uint32_t* __restrict__ qw,
                              int64_t words) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < words;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t w = qw[i];
    q[2 * i] = make_int4(w & 0xF, (w >> 4) & 0xF, (w >> 8) & 0xF, (w >> 12) & 0xF);
    q[2 * i + 1] = make_int4((w >> 16) & 0xF, (w >> 20) & 0xF, (w >> 24) & 0xF, w >> 28);
  }
}

__global__ void dequantize_kernel(float4* __restrict__ out, const uint32_t* __restrict__ qw,
                                  const half* __restrict__ s, const half* __restrict__ z,
                                  int64_t words, int64_t words_per_row, int64_t groups,
                                  int64_t words_per_group) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < words;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / words_per_row;
    const int64_t grp = (i % words_per_row) / words_per_group;
    const float sc = __half2float(s[row * groups + grp]);
    const float zp = __half2float(z[row * groups + grp]);
    const uint32_t w = qw[i];
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[j] = __fmul_rn(__fsub_rn(static_cast<float>((w >> (4 * j)) & 0xFu), zp), sc);
    }
    out[2 * i] = make_float4(v[0], v[1], v[2], v[3]);
    out[2 * i + 1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

__global__ void bias_residual_kernel(GemvArgs a) {
  const int64_t total = static_cast<int64_t>(a.m) * a.n;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int m = static_cast<int>(i / a.n);
    const int r = static_cast<int>(i - static_cast<int64_t>(m) * a.n);
    a.y[i] = store_value(a, m, r, 0.0f);
  }
}

int grid_for(int64_t items) {
  const int64_t blocks = (items + kThreads - 1) / kThreads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  return static_cast<int>(blocks < cap ? blocks : cap);
}

}  // namespace

cudaError_t launch_unpack(int32_t* q, const uint32_t* qweight, int64_t n, int64_t k,
                          cudaStream_t stream) {
  const int64_t words = n * (k / 8);
  if (words == 0) return cudaSuccess;
  unpack_kernel<<<grid_for(words), kThreads, 0, stream>>>(reinterpret_cast<int4*>(q), qweight,
                                                           words);
  return cudaGetLastError();
}

cudaError_t launch_dequantize(float* w, const uint32_t* qweight, const half* s, const half* z,
                              int64_t n, int64_t k, int64_t group, cudaStream_t stream) {
  const int64_t words = n * (k / 8);
  if (words == 0) return cudaSuccess;
  dequantize_kernel<<<grid_for(words), kThreads, 0, stream>>>(reinterpret_cast<float4*>(w),
                                                               qweight, s, z, words, k / 8,
                                                               k / group, group / 8);
  return cudaGetLastError();
}

cudaError_t launch_bias_residual(const GemvArgs& a, cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(a.m) * a.n;
  if (total == 0) return cudaSuccess;
  bias_residual_kernel<<<grid_for(total), kThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace i4
