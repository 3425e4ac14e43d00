// SIMT (CUDA-core) kernels behind the reference's operator names: naive (one thread per output
// row), coalesced (one warp per output row) and vectorized (rows_per_warp rows per warp, 16-byte
// loads), plus load_only, the vectorized load pattern without the math.
//
// The mapping of each operator is part of its documented contract (csrc/w4a16.h:26-47 of the
// reference); the code is written for sm_100a:
//   - naive and coalesced keep the reference's exact fp32 arithmetic per weight
//     (w = (q - z) * s, then an fp32 FMA with x), so their results track csrc/sequential.cpp;
//   - vectorized unpacks nibbles with one LOP3 per pair into fp16 1024 + q (exact), converts to
//     fp32 and applies the zero point once per 32-weight chunk:
//         sum_k (q_k - z) s x_k = s * (sum_k (1024 + q_k) x_k - (1024 + z) sum_k x_k)
//     which is exact algebra; the fp32 rounding it adds is far below the 1e-2 tolerance.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "kernels.h"

namespace i4 {
namespace {

constexpr int kNaiveThreads = 128;
constexpr int kCoalescedWarps = 4;

// Rows m0 .. m0 + TM - 1 of x; rows past m repeat row m - 1 and are never stored.
template <int TM>
__device__ __forceinline__ void tile_rows(const half* (&rows)[TM], const half* x, int m, int m0,
                                          int k) {
#pragma unroll
  for (int i = 0; i < TM; ++i) rows[i] = x + static_cast<int64_t>(min(m0 + i, m - 1)) * k;
}

template <int TM>
__device__ __forceinline__ void store_tile(const GemvArgs& a, const float (&acc)[TM], int m0,
                                           int row) {
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    if (m0 + i < a.m) {
      if (a.epilogue == kStoreF32) {  // the fp32 row sums (int4gemv_w4a16_f32)
        reinterpret_cast<float*>(a.y)[static_cast<int64_t>(m0 + i) * a.n + row] = acc[i];
      } else {
        a.y[static_cast<int64_t>(m0 + i) * a.n + row] = store_value(a, m0 + i, row, acc[i]);
      }
    }
  }
}

// ---- naive: thread r computes y[m0 .. m0 + TM), row r ------------------------------------------

template <int TM>
__global__ void __launch_bounds__(kNaiveThreads) naive_kernel(GemvArgs a) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= a.n) return;
  const int m0 = blockIdx.y * TM;
  const int words = a.k / 8;
  const int groups = a.k / a.group;
  const uint32_t* qrow = a.q + static_cast<int64_t>(row) * words;
  const half* srow = a.s + static_cast<int64_t>(row) * groups;
  const half* zrow = a.z + static_cast<int64_t>(row) * groups;
  const half* xr[TM];
  tile_rows(xr, a.x, a.m, m0, a.k);

  float acc[TM] = {};
  const int words_per_group = a.group / 8;
  for (int g = 0; g < groups; ++g) {
    const float s = __half2float(srow[g]);
    const float z = __half2float(zrow[g]);
    for (int w = g * words_per_group; w < (g + 1) * words_per_group; ++w) {
      const uint32_t word = qrow[w];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float wt = __fmul_rn(__fsub_rn(static_cast<float>((word >> (4 * j)) & 0xFu), z), s);
#pragma unroll
        for (int i = 0; i < TM; ++i) acc[i] = fmaf(__half2float(xr[i][8 * w + j]), wt, acc[i]);
      }
    }
  }
  store_tile(a, acc, m0, row);
}

// ---- coalesced: warp per row, lanes stride the row's words -------------------------------------

template <int TM>
__global__ void __launch_bounds__(kCoalescedWarps * kWarp) coalesced_kernel(GemvArgs a) {
  const int lane = threadIdx.x % kWarp;
  const int row = blockIdx.x * kCoalescedWarps + threadIdx.x / kWarp;
  if (row >= a.n) return;  // whole warps leave; nothing below synchronises the block
  const int m0 = blockIdx.y * TM;
  const int words = a.k / 8;
  const int groups = a.k / a.group;
  const uint32_t* qrow = a.q + static_cast<int64_t>(row) * words;
  const half* srow = a.s + static_cast<int64_t>(row) * groups;
  const half* zrow = a.z + static_cast<int64_t>(row) * groups;
  const half* xr[TM];
  tile_rows(xr, a.x, a.m, m0, a.k);

  float acc[TM] = {};
  for (int w = lane; w < words; w += kWarp) {
    const uint32_t word = qrow[w];
    const int g = (8 * w) / a.group;
    const float s = __half2float(srow[g]);
    const float z = __half2float(zrow[g]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float wt = __fmul_rn(__fsub_rn(static_cast<float>((word >> (4 * j)) & 0xFu), z), s);
#pragma unroll
      for (int i = 0; i < TM; ++i) acc[i] = fmaf(__half2float(xr[i][8 * w + j]), wt, acc[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < TM; ++i) acc[i] = warp_sum(acc[i]);
  if (lane == 0) store_tile(a, acc, m0, row);
}

// ---- vectorized: RPW rows per warp, lane-strided 16-byte chunks of 32 weights ------------------

template <int TM, int RPW>
__global__ void vectorized_kernel(GemvArgs a) {
  const int lane = threadIdx.x % kWarp;
  const int warps = blockDim.x / kWarp;
  const int row0 = (blockIdx.x * warps + threadIdx.x / kWarp) * RPW;
  if (row0 >= a.n) return;
  const int m0 = blockIdx.y * TM;
  const int chunks = a.k / 32;
  const int groups = a.k / a.group;

  const uint4* qrow[RPW];
  const half* srow[RPW];
  const half* zrow[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int64_t row = min(row0 + r, a.n - 1);
    qrow[r] = reinterpret_cast<const uint4*>(a.q + row * (a.k / 8));
    srow[r] = a.s + row * groups;
    zrow[r] = a.z + row * groups;
  }
  const half* xr[TM];
  tile_rows(xr, a.x, a.m, m0, a.k);

  float acc[RPW][TM] = {};
  for (int c = lane; c < chunks; c += kWarp) {
    uint4 packed[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) packed[r] = ld_stream_v4(qrow[r] + c);
    const int g = (32 * c) / a.group;
    float s[RPW], z1024[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      s[r] = __half2float(srow[r][g]);
      z1024[r] = 1024.0f + __half2float(zrow[r][g]);
    }
    float part[RPW][TM] = {};
    float xsum[TM] = {};
#pragma unroll
    for (int word = 0; word < 4; ++word) {
      // qf[r][j] = 1024 + q_j of this word, j = 0..7.
      float qf[RPW][8];
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        uint32_t h[4];
        unpack_pairs((&packed[r].x)[word], h);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = half2_bits_to_float2(h[j]);
          qf[r][j] = f.x;
          qf[r][j + 4] = f.y;
        }
      }
#pragma unroll
      for (int i = 0; i < TM; ++i) {
        const uint4 xv = *reinterpret_cast<const uint4*>(xr[i] + 32 * c + 8 * word);
        float xf[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = half2_bits_to_float2((&xv.x)[j]);
          xf[2 * j] = f.x;
          xf[2 * j + 1] = f.y;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          xsum[i] += xf[j];
#pragma unroll
          for (int r = 0; r < RPW; ++r) part[r][i] = fmaf(xf[j], qf[r][j], part[r][i]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
#pragma unroll
      for (int i = 0; i < TM; ++i) {
        acc[r][i] = fmaf(s[r], fmaf(-z1024[r], xsum[i], part[r][i]), acc[r][i]);
      }
    }
  }

#pragma unroll
  for (int r = 0; r < RPW; ++r) {
#pragma unroll
    for (int i = 0; i < TM; ++i) acc[r][i] = warp_sum(acc[r][i]);
  }
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      if (row0 + r < a.n) store_tile(a, acc[r], m0, row0 + r);
    }
  }
}

// ---- load_only: vectorized's loads at M = 1, XOR-folded per row --------------------------------

template <int RPW>
__global__ void load_only_kernel(uint32_t* out, GemvArgs a) {
  const int lane = threadIdx.x % kWarp;
  const int warps = blockDim.x / kWarp;
  const int row0 = (blockIdx.x * warps + threadIdx.x / kWarp) * RPW;
  if (row0 >= a.n) return;
  const int chunks = a.k / 32;
  const int groups = a.k / a.group;
  uint32_t acc[RPW] = {};
  for (int c = lane; c < chunks; c += kWarp) {
    uint4 packed[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int64_t row = min(row0 + r, a.n - 1);
      packed[r] = ld_stream_v4(reinterpret_cast<const uint4*>(a.q + row * (a.k / 8)) + c);
    }
    uint32_t xbits = 0;
#pragma unroll
    for (int word = 0; word < 4; ++word) {
      const uint4 xv = *reinterpret_cast<const uint4*>(a.x + 32 * c + 8 * word);
      xbits ^= xv.x ^ xv.y ^ xv.z ^ xv.w;
    }
    // A scale and zero pair is folded in once per group: by the chunk that starts the group.
    const bool first_of_group = (32 * c) % a.group == 0;
    const int g = (32 * c) / a.group;
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      const int64_t row = min(row0 + r, a.n - 1);
      acc[r] ^= packed[r].x ^ packed[r].y ^ packed[r].z ^ packed[r].w ^ xbits;
      if (first_of_group) {
        acc[r] ^= static_cast<uint32_t>(__half_as_ushort(a.s[row * groups + g])) ^
                  static_cast<uint32_t>(__half_as_ushort(a.z[row * groups + g]));
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const uint32_t v = warp_xor(acc[r]);
    if (lane == 0 && row0 + r < a.n) out[row0 + r] = v;
  }
}

// ---- dispatch -----------------------------------------------------------------------------------

template <typename F>
cudaError_t with_tile_m(int m, F&& f) {
  if (m <= 1) return f.template operator()<1>();
  if (m == 2) return f.template operator()<2>();
  if (m <= 4) return f.template operator()<4>();
  return f.template operator()<8>();
}

template <typename F>
cudaError_t with_rows_per_warp(int rpw, F&& f) {
  switch (rpw) {
    case 1:
      return f.template operator()<1>();
    case 2:
      return f.template operator()<2>();
    case 4:
      return f.template operator()<4>();
    default:
      return cudaErrorInvalidValue;
  }
}

dim3 tiled_grid(int blocks_x, int m, int tm) { return dim3(blocks_x, (m + tm - 1) / tm); }

template <typename Kernel>
cudaError_t attrs_of(Kernel kernel, int threads, KernelAttrs* out) {
  cudaFuncAttributes fa;
  cudaError_t err = cudaFuncGetAttributes(&fa, kernel);
  if (err != cudaSuccess) return err;
  int blocks = 0;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, threads, 0);
  if (err != cudaSuccess) return err;
  out->registers = fa.numRegs;
  out->local_bytes = static_cast<int>(fa.localSizeBytes);
  out->max_threads_per_block = fa.maxThreadsPerBlock;
  out->blocks_per_sm = blocks;
  out->threads_per_block = threads;
  return cudaSuccess;
}

}  // namespace

cudaError_t launch_naive(const GemvArgs& a, cudaStream_t stream) {
  return with_tile_m(a.m, [&]<int TM>() {
    naive_kernel<TM><<<tiled_grid((a.n + kNaiveThreads - 1) / kNaiveThreads, a.m, TM),
                       kNaiveThreads, 0, stream>>>(a);
    return cudaGetLastError();
  });
}

cudaError_t launch_coalesced(const GemvArgs& a, cudaStream_t stream) {
  return with_tile_m(a.m, [&]<int TM>() {
    coalesced_kernel<TM><<<tiled_grid((a.n + kCoalescedWarps - 1) / kCoalescedWarps, a.m, TM),
                           kCoalescedWarps * kWarp, 0, stream>>>(a);
    return cudaGetLastError();
  });
}

cudaError_t launch_vectorized(const GemvArgs& a, int threads, int rpw, cudaStream_t stream) {
  return with_rows_per_warp(rpw, [&]<int RPW>() {
    return with_tile_m(a.m, [&]<int TM>() {
      const int rows_per_block = threads / kWarp * RPW;
      vectorized_kernel<TM, RPW><<<tiled_grid((a.n + rows_per_block - 1) / rows_per_block, a.m, TM),
                                   threads, 0, stream>>>(a);
      return cudaGetLastError();
    });
  });
}

cudaError_t launch_load_only(uint32_t* out, const GemvArgs& a, int threads, int rpw,
                             cudaStream_t stream) {
  return with_rows_per_warp(rpw, [&]<int RPW>() {
    const int rows_per_block = threads / kWarp * RPW;
    load_only_kernel<RPW><<<(a.n + rows_per_block - 1) / rows_per_block, threads, 0, stream>>>(out,
                                                                                              a);
    return cudaGetLastError();
  });
}

cudaError_t vectorized_max_threads(int m, int rpw, int* max_threads) {
  return with_rows_per_warp(rpw, [&]<int RPW>() {
    return with_tile_m(m, [&]<int TM>() {
      cudaFuncAttributes fa;
      const cudaError_t err = cudaFuncGetAttributes(&fa, vectorized_kernel<TM, RPW>);
      if (err == cudaSuccess) *max_threads = fa.maxThreadsPerBlock;
      return err;
    });
  });
}

cudaError_t simt_attrs(const char* kernel, int m, int threads, int rpw, KernelAttrs* out) {
  if (std::strcmp(kernel, "naive") == 0) {
    return with_tile_m(m, [&]<int TM>() { return attrs_of(naive_kernel<TM>, kNaiveThreads, out); });
  }
  if (std::strcmp(kernel, "coalesced") == 0) {
    return with_tile_m(
        m, [&]<int TM>() { return attrs_of(coalesced_kernel<TM>, kCoalescedWarps * kWarp, out); });
  }
  if (std::strcmp(kernel, "vectorized") == 0) {
    return with_rows_per_warp(rpw, [&]<int RPW>() {
      return with_tile_m(
          m, [&]<int TM>() { return attrs_of(vectorized_kernel<TM, RPW>, threads, out); });
    });
  }
  return cudaErrorInvalidValue;
}

}  // namespace i4
