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
// The reference computes each of these as one IEEE fp32 operation rounded to nearest even; the
// group parameters here do the same (__fsub_rn, __fdiv_rn: no contraction, no approximate
// division). For q, w / s is first estimated as w * (1 / s) (one correctly rounded reciprocal per
// group, then a fused multiply-add with z), which can only round differently from the reference
// when the value lies within 1e-5 of a half-integer; any word with a weight within 1e-4 of one is
// recomputed with IEEE division (quantize_word). The sign of a zero zero-point follows the first
// minimal element of the group in k order (lo = -0.0 gives z = +0.0, lo = +0.0 gives z = -0.0),
// as a sequential scan does (first_zero_key).
//
// Mapping. Each thread owns two consecutive packed words (16 weights: 64 B of fp32 or 32 B of
// fp16 / bf16), so a warp reads 2 KB (1 KB) of contiguous weights and writes 256 B of words. When
// a group spans a power-of-two number of words <= 64, its threads are an aligned segment of one
// warp and reduce min / max with xor shuffles inside the segment; other group sizes take one warp
// per group with a loop over the group's words. The path is HBM-bound: per weight it reads 4 (or
// 2) bytes and writes 0.5 + 4 / group bytes.
#include "common.cuh"
#include "kernels.h"

#include <cuda_bf16.h>

#include <climits>

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

// Min and max over a thread's weights; the position of the first zero matters only when the
// group's minimum is a zero (see first_zero_key).
template <int N>
__device__ __forceinline__ void min_max(const float (&v)[N][8], float& lo, float& hi) {
#pragma unroll
  for (int t = 0; t < N; ++t)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      lo = fminf(lo, v[t][j]);
      hi = fmaxf(hi, v[t][j]);
    }
}

// 2 * (position in the group of the thread's first zero weight) + its sign bit, or INT_MAX.
// `pos0` = position of v[0][0]. The smallest key over the group gives the sign that a sequential
// scan (which keeps the first of equal minima) leaves in lo.
template <int N>
__device__ __forceinline__ int first_zero_key(const float (&v)[N][8], int pos0) {
#pragma unroll
  for (int t = 0; t < N; ++t)
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (v[t][j] == 0.0f) return 2 * (pos0 + 8 * t + j) + (__float_as_uint(v[t][j]) >> 31);
    }
  return INT_MAX;
}

// Reduction over an aligned segment of `width` lanes (a power of two <= 32).
__device__ __forceinline__ void segment_min_max(float& lo, float& hi, int width) {
  for (int off = width >> 1; off > 0; off >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, off));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, off));
  }
}

__device__ __forceinline__ int segment_min(int key, int width) {
  for (int off = width >> 1; off > 0; off >>= 1) key = min(key, __shfl_xor_sync(0xffffffffu, key, off));
  return key;
}

struct GroupParams {
  float s;  // fp16-rounded scale, as fp32
  float r;  // 1 / s, correctly rounded: the estimate of w / s is w * r
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
  g.r = __frcp_rn(g.s);
  float z = rintf(__fdiv_rn(-lo, g.s));
  if (z < 0.0f) z = 0.0f;
  if (z > 15.0f) z = 15.0f;
  g.z = z;
  g.z_h = __float2half_rn(z);
  return g;
}

// q = clamp(rint(fl(fl(w / s) + z)), 0, 15) with IEEE division: the reference's arithmetic.
__device__ __forceinline__ uint32_t quantize_word_exact(const float (&v)[8], const GroupParams& g) {
  uint32_t word = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float q = rintf(__fadd_rn(__fdiv_rn(v[j], g.s), g.z));
    q = fminf(fmaxf(q, 0.0f), 15.0f);
    word |= static_cast<uint32_t>(q) << (4 * j);
  }
  return word;
}

// Adding 1.5 * 2^23 to c in [0, 15] rounds it to an integer, half to even, held in the low
// mantissa bits: bits = 0x4B400000 + rint(c).
constexpr float kRoundMagic = 12582912.0f;
__host__ __device__ constexpr uint32_t magic_sum() {
  uint32_t s = 0;
  for (int j = 0; j < 8; ++j) s += 0x4B400000u << (4 * j);
  return s;
}

// The same word from the estimate t = fma(w, 1 / s, z). For every weight of the group |w / s| < 16
// (also when s rounds to an fp16 subnormal) and z <= 15, so the estimate and the reference's
// fl(fl(w / s) + z) are both within 3e-6 of the exact value. Clamping before rounding gives the
// same q as rounding before clamping (0 and 15 are integers), so they can round differently only
// when the clamped estimate lies within 1e-5 of a half-integer; a word with any weight within 1e-4
// of one is recomputed exactly. Packing: sum_j bits_j << 4j minus the magic's share, one integer
// multiply-add per weight.
__device__ __forceinline__ uint32_t quantize_word(const float (&v)[8], const GroupParams& g) {
  uint32_t acc = 0;
  float dmax = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float c = fminf(fmaxf(fmaf(v[j], g.r, g.z), 0.0f), 15.0f);
    const float m = __fadd_rn(c, kRoundMagic);
    dmax = fmaxf(dmax, fabsf(__fsub_rn(c, __fsub_rn(m, kRoundMagic))));
    acc += __float_as_uint(m) << (4 * j);
  }
  if (dmax > 0.4999f) return quantize_word_exact(v, g);
  constexpr uint32_t kMagicSum = magic_sum();
  return acc - kMagicSum;
}

// Groups of `width` lanes x WPT words (width a power of two <= 32): aligned segments of one warp.
// Warp-uniform loop over chunks of 32 WPT words; lanes past the end compute on clamped data and
// store nothing (segments never straddle the end because the word count is a multiple of a
// group's words).
template <int DT, int WPT>
__global__ void __launch_bounds__(kThreads) quantize_segment_kernel(
    uint32_t* __restrict__ qw, half* __restrict__ s, half* __restrict__ z,
    const void* __restrict__ w, int64_t words, int width) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int seg_lane = lane & (width - 1);
  for (int64_t base = warp * 32 * WPT; base < words; base += warps * 32 * WPT) {
    const int64_t i0 = base + lane * WPT;
    const bool live = i0 < words;
    float v[WPT][8];
#pragma unroll
    for (int t = 0; t < WPT; ++t) load8<DT>(w, live ? i0 + t : words - WPT + t, v[t]);
    float lo = v[0][0], hi = v[0][0];
    min_max(v, lo, hi);
    segment_min_max(lo, hi, width);
    if (lo == 0.0f) {  // uniform over the segment
      const int key = segment_min(first_zero_key(v, 8 * WPT * seg_lane), width);
      lo = (key & 1) ? -0.0f : 0.0f;
    }
    const GroupParams g = group_params(lo, hi);
    if (!live) continue;
    if constexpr (WPT == 2) {
      *reinterpret_cast<uint2*>(qw + i0) = make_uint2(quantize_word(v[0], g),
                                                      quantize_word(v[1], g));
    } else {
      qw[i0] = quantize_word(v[0], g);
    }
    if (seg_lane == 0) {
      const int64_t grp = i0 / (static_cast<int64_t>(width) * WPT);
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
    float lo = INFINITY, hi = -INFINITY;
    for (int j = lane; j < width; j += 32) {
      float v[1][8];
      load8<DT>(w, first + j, v[0]);
      min_max(v, lo, hi);
    }
    segment_min_max(lo, hi, 32);
    if (lo == 0.0f) {
      int key = INT_MAX;
      for (int j = lane; j < width; j += 32) {
        float v[1][8];
        load8<DT>(w, first + j, v[0]);
        key = min(key, first_zero_key(v, 8 * j));
      }
      lo = (segment_min(key, 32) & 1) ? -0.0f : 0.0f;
    }
    const GroupParams g = group_params(lo, hi);
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
  const int gw = static_cast<int>(group / 8);  // words per group
  const bool pow2 = (gw & (gw - 1)) == 0;
  if (pow2 && gw >= 2 && gw <= 64) {  // two words per thread, gw / 2 lanes per group
    quantize_segment_kernel<DT, 2><<<grid_for(words / 2), kThreads, 0, stream>>>(
        qweight, s, z, w, words, gw / 2);
  } else if (gw == 1) {
    quantize_segment_kernel<DT, 1><<<grid_for(words), kThreads, 0, stream>>>(qweight, s, z, w,
                                                                              words, 1);
  } else {
    const int64_t groups = n * (k / group);
    quantize_group_kernel<DT><<<grid_for(groups * 32), kThreads, 0, stream>>>(qweight, s, z, w,
                                                                               groups, gw);
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
