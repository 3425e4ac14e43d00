// Round-to-nearest group quantisation and packing on the device, bit-exact with the reference's
// int4gemv/quant.py:14-37 for finite inputs:
//
//   per group of `group` weights along K (quant.py:21-29):
//     lo = min(min(w), 0), hi = max(max(w), 0)
//     s  = fp16(max((hi - lo) / 15, 1e-6))           the fp16-rounded scale, used as fp32 below
//     z  = clamp(rint(-lo / s), 0, 15)               rint = round half to even (torch.round)
//     q  = clamp(rint(w / s + z), 0, 15)
//   pack (quant.py:32-37): word = sum_j q[8w + j] << 4j, modulo 2^32 (so out-of-range q wrap the
//   same way the reference's int64 sum does after its cast to int32).
//
// Every fp32 operation is one IEEE operation rounded to nearest even (__fsub_rn, __fdiv_rn,
// __fadd_rn: no contraction, no approximate division), which is what torch's CPU and CUDA
// elementwise kernels compute. The sign of a zero zero-point follows the first minimal element of
// the group in k order (lo = -0.0 gives z = +0.0, lo = +0.0 gives z = -0.0), as a sequential scan
// does; ties of min are therefore broken by position in the reductions below.
//
// Mapping. Each thread owns one packed word: it loads the word's 8 weights (32 B of fp32 or 16 B
// of fp16 / bf16, one or two vector loads), so a warp reads 1 KB (512 B) of contiguous weights and
// writes 128 B of contiguous words. When a group spans a power-of-two number of words <= 32, the
// group's threads are an aligned segment of one warp and reduce min / max with xor shuffles inside
// the segment; other group sizes take one warp per group with a loop over the group's words.
// The path is HBM-bound: per weight it reads 4 (or 2) bytes and writes 0.5 + 4 / group bytes.
#include "common.cuh"
#include "kernels.h"

#include <cuda_bf16.h>

namespace i4 {
namespace {

constexpr int kThreads = 256;

// The 8 weights of one packed word, widened to fp32 (exact for fp16 and bf16).
template <int DT>
__device__ __forceinline__ void load8(const void* w, int64_t word, float (&v)[8]) {
  if constexpr (DT == kWeightF32) {
    const float4* p = static_cast<const float4*>(w) + 2 * word;
    const float4 a = __ldcs(p), b = __ldcs(p + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 r = __ldcs(static_cast<const uint4*>(w) + word);
    const uint32_t u[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (DT == kWeightF16) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u[i]));
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      } else {
        v[2 * i] = __uint_as_float(u[i] << 16);
        v[2 * i + 1] = __uint_as_float(u[i] & 0xFFFF0000u);
      }
    }
  }
}

// Running minimum with its position: a later element replaces the minimum only when strictly
// smaller, or equal (+0 / -0) and earlier in k.
struct MinPos {
  float v;
  int pos;
};

__device__ __forceinline__ void take_min(MinPos& a, float v, int pos) {
  if (v < a.v || (v == a.v && pos < a.pos)) {
    a.v = v;
    a.pos = pos;
  }
}

// Min (with position) and max over the 8 weights of one word; `pos0` = position of v[0].
__device__ __forceinline__ void scan8(const float (&v)[8], int pos0, MinPos& lo, float& hi) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    take_min(lo, v[j], pos0 + j);
    hi = fmaxf(hi, v[j]);
  }
}

// Reduction over the lanes of an aligned segment of `width` lanes (a power of two <= 32).
__device__ __forceinline__ void segment_reduce(MinPos& lo, float& hi, int width) {
  for (int off = width >> 1; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, lo.v, off);
    const int op = __shfl_xor_sync(0xffffffffu, lo.pos, off);
    take_min(lo, ov, op);
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, off));
  }
}

struct GroupParams {
  float s;  // fp16-rounded scale, as fp32
  float z;  // zero point 0..15 (possibly -0.0)
  half s_h, z_h;
};

__device__ __forceinline__ GroupParams group_params(float lo, float hi) {
  if (lo > 0.0f) lo = 0.0f;
  if (hi < 0.0f) hi = 0.0f;
  float s = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
  if (s < 1e-6f) s = 1e-6f;
  GroupParams g;
  g.s_h = __float2half_rn(s);
  g.s = __half2float(g.s_h);
  float z = rintf(__fdiv_rn(-lo, g.s));
  if (z < 0.0f) z = 0.0f;
  if (z > 15.0f) z = 15.0f;
  g.z = z;
  g.z_h = __float2half_rn(z);
  return g;
}

__device__ __forceinline__ uint32_t quantize_word(const float (&v)[8], const GroupParams& g) {
  uint32_t word = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float q = rintf(__fadd_rn(__fdiv_rn(v[j], g.s), g.z));
    if (q < 0.0f) q = 0.0f;
    if (q > 15.0f) q = 15.0f;
    word |= static_cast<uint32_t>(q) << (4 * j);
  }
  return word;
}

// Groups of `width` words, width a power of two <= 32: segments of one warp. Warp-uniform loop
// over chunks of 32 words; lanes past the end compute on clamped data and store nothing (segments
// never straddle the end because the word count is a multiple of width).
template <int DT>
__global__ void __launch_bounds__(kThreads) quantize_segment_kernel(
    uint32_t* __restrict__ qw, half* __restrict__ s, half* __restrict__ z,
    const void* __restrict__ w, int64_t words, int width) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int seg_lane = lane & (width - 1);
  for (int64_t base = warp * 32; base < words; base += warps * 32) {
    const int64_t i = base + lane;
    const bool live = i < words;
    float v[8];
    load8<DT>(w, live ? i : words - 1, v);
    MinPos lo{v[0], 8 * seg_lane};
    float hi = v[0];
    scan8(v, 8 * seg_lane, lo, hi);
    segment_reduce(lo, hi, width);
    const GroupParams g = group_params(lo.v, hi);
    if (!live) continue;
    qw[i] = quantize_word(v, g);
    if (seg_lane == 0) {
      const int64_t grp = i / width;
      s[grp] = g.s_h;
      z[grp] = g.z_h;
    }
  }
}

// Any group size (a multiple of 8): one warp per group, lanes stride over the group's words.
template <int DT>
__global__ void __launch_bounds__(kThreads) quantize_group_kernel(
    uint32_t* __restrict__ qw, half* __restrict__ s, half* __restrict__ z,
    const void* __restrict__ w, int64_t groups, int width) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t grp = warp; grp < groups; grp += warps) {
    const int64_t first = grp * width;
    MinPos lo{INFINITY, 0x7fffffff};
    float hi = -INFINITY;
    for (int j = lane; j < width; j += 32) {
      float v[8];
      load8<DT>(w, first + j, v);
      scan8(v, 8 * j, lo, hi);
    }
    segment_reduce(lo, hi, 32);
    const GroupParams g = group_params(lo.v, hi);
    for (int j = lane; j < width; j += 32) {
      float v[8];
      load8<DT>(w, first + j, v);
      qw[first + j] = quantize_word(v, g);
    }
    if (lane == 0) {
      s[grp] = g.s_h;
      z[grp] = g.z_h;
    }
  }
}

// pack: one thread per word, 8 int32 in (two 16-byte loads), one word out.
__global__ void __launch_bounds__(kThreads) pack_kernel(uint32_t* __restrict__ qw,
                                                        const int4* __restrict__ q,
                                                        int64_t words) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < words;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int4 a = __ldcs(q + 2 * i), b = __ldcs(q + 2 * i + 1);
    const uint32_t v[8] = {static_cast<uint32_t>(a.x), static_cast<uint32_t>(a.y),
                           static_cast<uint32_t>(a.z), static_cast<uint32_t>(a.w),
                           static_cast<uint32_t>(b.x), static_cast<uint32_t>(b.y),
                           static_cast<uint32_t>(b.z), static_cast<uint32_t>(b.w)};
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) word += v[j] << (4 * j);
    qw[i] = word;
  }
}

int grid_for(int64_t threads) {
  const int64_t blocks = (threads + kThreads - 1) / kThreads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  return static_cast<int>(blocks < cap ? blocks : cap);
}

template <int DT>
cudaError_t launch_quantize_t(uint32_t* qweight, half* s, half* z, const void* w, int64_t n,
                              int64_t k, int64_t group, cudaStream_t stream) {
  const int64_t words = n * (k / 8);
  const int width = static_cast<int>(group / 8);
  if ((width & (width - 1)) == 0 && width <= 32) {
    quantize_segment_kernel<DT><<<grid_for(words), kThreads, 0, stream>>>(qweight, s, z, w,
                                                                           words, width);
  } else {
    const int64_t groups = n * (k / group);
    quantize_group_kernel<DT><<<grid_for(groups * 32), kThreads, 0, stream>>>(qweight, s, z, w,
                                                                               groups, width);
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_quantize(uint32_t* qweight, half* scales, half* zeros, const void* w,
                            int dtype, int64_t n, int64_t k, int64_t group, cudaStream_t stream) {
  if (n * k == 0) return cudaSuccess;
  switch (dtype) {
    case kWeightF32:
      return launch_quantize_t<kWeightF32>(qweight, scales, zeros, w, n, k, group, stream);
    case kWeightF16:
      return launch_quantize_t<kWeightF16>(qweight, scales, zeros, w, n, k, group, stream);
    case kWeightBF16:
      return launch_quantize_t<kWeightBF16>(qweight, scales, zeros, w, n, k, group, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_pack(uint32_t* qweight, const int32_t* q, int64_t n, int64_t k,
                        cudaStream_t stream) {
  const int64_t words = n * (k / 8);
  if (words == 0) return cudaSuccess;
  pack_kernel<<<grid_for(words), kThreads, 0, stream>>>(qweight, reinterpret_cast<const int4*>(q),
                                                        words);
  return cudaGetLastError();
}

}  // namespace i4
