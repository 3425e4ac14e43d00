// Repacking of AWQ and GPTQ 4-bit checkpoints into this library's layout (qweight [N, K/8] int32
// with weight k of row n in bits 4 (k % 8) of word k / 8; scales and zeros [N, K/g] fp16), on the
// device. Pure bit movement, exact.
//
// Checkpoint layouts (the packers of AutoAWQ and AutoGPTQ, as restated by vLLM 0.22's
// quantization/utils/quant_utils.py awq_pack / gptq_pack / pack_cols):
//   AWQ   qweight [K, N/8]:   nibble i of word (k, c) = q[k, 8c + kAwqOrder[i]], order 0 2 4 6 1 3 5 7
//         qzeros  [K/g, N/8]: the same packing of z [K/g, N]
//         scales  [K/g, N] fp16
//   GPTQ  qweight [K/8, N]:   nibble i of word (r, n) = q[8r + i, n]
//         qzeros  [K/g, N/8]: nibble i of word (gi, c) = z[gi, 8c + i] - zero_offset
//         (zero_offset 1 in the original "gptq" format, which stores z - 1; 0 in "gptq_v2")
//         scales  [K/g, N] fp16
// Dequantisation is (q - z) * s in all three layouts, so the values carry over unchanged.
//
// Kernels: the AWQ qweight is an 8 x 8 nibble transpose per (8 k, 8 n) block, done through a
// shared-memory tile of 64 k x 256 n so that both the loads (rows of N/8 words) and the stores
// (rows of K/8 words) are coalesced. The GPTQ qweight is already k-packed: a 32-bit word
// transpose [K/8, N] -> [N, K/8] through a padded 32 x 32 tile. Scales and zeros: one thread per
// (group, n), reading along n.
#include "common.cuh"
#include "kernels.h"

namespace i4 {
namespace {

// Nibble position of column j (0..7) in an AWQ word: the inverse of the order 0 2 4 6 1 3 5 7.
__host__ __device__ constexpr int awq_pos(int j) { return (j & 1) * 4 + (j >> 1); }

constexpr int kTileK = 64;        // k rows per AWQ tile (8 output words per n)
constexpr int kTileC = 32;        // input words per k row per tile (256 columns n)
constexpr int kOutPad = 8 * kTileC + 8;  // words per output-tile k-word row, padded

__global__ void __launch_bounds__(256) awq_qweight_kernel(uint32_t* __restrict__ out,
                                                          const uint32_t* __restrict__ in,
                                                          int k, int n) {
  __shared__ uint32_t tin[kTileK][kTileC];
  __shared__ uint32_t tout[8 * kOutPad];  // [k word 0..7][n 0..255], + n / 32 padding
  const int tid = threadIdx.x;
  const int in_words = n / 8, out_words = k / 8;
  const int k0 = blockIdx.y * kTileK, c0 = blockIdx.x * kTileC;
#pragma unroll
  for (int r = 0; r < kTileK / 8; ++r) {
    const int row = r * 8 + (tid >> 5), col = tid & 31;
    const bool in_range = k0 + row < k && c0 + col < in_words;
    tin[row][col] = in_range ? in[static_cast<int64_t>(k0 + row) * in_words + c0 + col] : 0u;
  }
  __syncthreads();
  {
    const int kb = tid >> 5, cb = tid & 31;
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = tin[8 * kb + i][cb];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint32_t o = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) o |= ((w[i] >> (4 * awq_pos(j))) & 0xFu) << (4 * i);
      const int nl = 8 * cb + j;
      tout[kb * kOutPad + nl + (nl >> 5)] = o;
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int idx = r * 256 + tid;
    const int nl = idx >> 3, kbl = idx & 7;
    const int nn = 8 * c0 + nl, kw = k0 / 8 + kbl;
    if (nn < n && kw < out_words) {
      out[static_cast<int64_t>(nn) * out_words + kw] = tout[kbl * kOutPad + nl + (nl >> 5)];
    }
  }
}

// out [cols, rows] = in [rows, cols]^T for 32-bit words.
__global__ void __launch_bounds__(256) transpose_words_kernel(uint32_t* __restrict__ out,
                                                              const uint32_t* __restrict__ in,
                                                              int rows, int cols) {
  __shared__ uint32_t tile[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const int r = r0 + ty + i, c = c0 + tx;
    if (r < rows && c < cols) tile[ty + i][tx] = in[static_cast<int64_t>(r) * cols + c];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const int c = c0 + ty + i, r = r0 + tx;
    if (c < cols && r < rows) out[static_cast<int64_t>(c) * rows + r] = tile[tx][ty + i];
  }
}

// scales_out [n, G] = scales_in [G, n]^T; zeros_out [n, G] = nibble of qzeros [G, n / 8] + offset.
template <bool kAwq>
__global__ void __launch_bounds__(256) zeros_scales_kernel(half* __restrict__ s_out,
                                                           half* __restrict__ z_out,
                                                           const half* __restrict__ s_in,
                                                           const uint32_t* __restrict__ qz,
                                                           int groups, int n, int zero_offset) {
  const int64_t total = static_cast<int64_t>(groups) * n;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int gi = static_cast<int>(i / n);
    const int nn = static_cast<int>(i - static_cast<int64_t>(gi) * n);
    const uint32_t word = qz[static_cast<int64_t>(gi) * (n / 8) + nn / 8];
    const int pos = kAwq ? awq_pos(nn & 7) : (nn & 7);
    const int z = static_cast<int>((word >> (4 * pos)) & 0xFu) + zero_offset;
    const int64_t o = static_cast<int64_t>(nn) * groups + gi;
    s_out[o] = s_in[i];
    z_out[o] = __int2half_rn(z);
  }
}

int grid_for(int64_t threads) {
  const int64_t blocks = (threads + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  return static_cast<int>(blocks < cap ? blocks : cap);
}

}  // namespace

cudaError_t launch_repack(bool awq, uint32_t* qweight, half* scales, half* zeros,
                          const uint32_t* ck_qweight, const uint32_t* ck_qzeros,
                          const half* ck_scales, int64_t n, int64_t k, int64_t group,
                          int zero_offset, cudaStream_t stream) {
  if (n == 0 || k == 0) return cudaSuccess;
  const int ni = static_cast<int>(n), ki = static_cast<int>(k);
  if (awq) {
    const dim3 grid(static_cast<unsigned>((n / 8 + kTileC - 1) / kTileC),
                    static_cast<unsigned>((k + kTileK - 1) / kTileK));
    awq_qweight_kernel<<<grid, 256, 0, stream>>>(qweight, ck_qweight, ki, ni);
  } else {
    const int rows = ki / 8;  // [K/8, N] -> [N, K/8]
    const dim3 grid(static_cast<unsigned>((n + 31) / 32), static_cast<unsigned>((rows + 31) / 32));
    transpose_words_kernel<<<grid, 256, 0, stream>>>(qweight, ck_qweight, rows, ni);
  }
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  const int groups = static_cast<int>(k / group);
  const int grid = grid_for(static_cast<int64_t>(groups) * n);
  if (awq) {
    zeros_scales_kernel<true><<<grid, 256, 0, stream>>>(scales, zeros, ck_scales, ck_qzeros,
                                                         groups, ni, zero_offset);
  } else {
    zeros_scales_kernel<false><<<grid, 256, 0, stream>>>(scales, zeros, ck_scales, ck_qzeros,
                                                          groups, ni, zero_offset);
  }
  return cudaGetLastError();
}

}  // namespace i4
