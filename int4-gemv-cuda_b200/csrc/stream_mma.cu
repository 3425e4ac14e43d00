// The B200 fast path for M <= 32: TMA tile stream of the packed weights + warp-level tensor-core
// MMAs (mma.sync m16n8k16, f16 x f16 -> f32) on the nibbles unpacked in registers.
//
// Why warp MMAs at small M. Per packed 32-bit word (8 weights) a thread spends one shift and four
// LOP3s to turn the nibbles into the A fragments of two m16n8k16 MMAs (the magic-number trick:
// 1024 + q and 1024 + 16 q in fp16, exact), and each MMA covers 256 weights x 8 rows of x. That
// is about 6 warp instructions per 256 weights, flat in M up to 8 and + 2 MMAs per 8 more rows of
// x, far below what streaming 4-bit weights at HBM speed leaves per SM. A 128-row tcgen05 MMA
// has a fixed issue cost per 16 k that makes it the slower choice at M <= 32.
//
// Work split. One CTA per SM (grid = SMs), with at most 113 KB of shared memory when it fits, so
// the next GEMV in the stream (launched with programmatic stream serialization) becomes resident
// beside it and starts streaming its own weights while this one drains. CTA c owns rows
// [4 u0, 4 u1), an equal share of 4-row units. Its rows are taken in k-panels (all of K when x
// fits) x blocks of 32 rows x stages of 8 items (an item = 128 weights = one group).
//
// Warps. One producer warp (weight_stream.cuh) fills a ring of stages with 2-D TMA tiles. Eight
// consumer warps split each stage: warp w takes rows 16 (w % 2) .. + 15 of the block and items
// 2 (w / 2), 2 (w / 2) + 1. MMA row g (and g + 8) is block row rho(g) = (g >> 1) | ((g & 1) << 2)
// (and + 8), so the 8 threads of one shared-memory phase read two rows whose 128-byte swizzle
// puts their 16-byte granules in different banks.
//
// x. Per panel the consumers copy x into shared memory, each 8-weight block permuted to
// [x0, x4, x1/16, x5/16, x2, x6, x3/16, x7/16] (matching the unpacked A halves) and laid out so
// that the B fragment a thread needs for word j of an item is one 16-byte load, conflict-free:
//     xs[m][item][j][c][8 halves], row stride = panel bytes + 64.
// The same pass builds corr[item][m] = (1024 * sum of the B values, sum of the x they stand for),
// so for each (row, item) the MMA result D gives
//     sum_k (q_k - z) s x_k = s * (D - 1024 sum_k b_k - z sum_k x_k).
// The weights are bit-exact; the arithmetic is fp32 accumulation of exact fp16 products.
//
// Results. Each warp keeps per-row fp32 partials for its items; at the end of a block they go to
// shared memory, and after the last block the four item-pair partials of each output are added
// in a fixed order, so results are deterministic. Every mbarrier wait is bounded; on timeout the
// kernel records a status word and runs to completion without writing y.
#include <algorithm>
#include <mutex>

#include "weight_stream.cuh"

namespace i4 {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * kWarp;
constexpr int kThreads = kConsumerThreads + kWarp;
constexpr int kMaxStages = 8;
constexpr int kCoResident = 113 * 1024;  // leaves room for the next kernel's CTA on the SM
constexpr int kSmemLimit = 227 * 1024;
constexpr int kConsumerBarrier = 1;
constexpr int kMaxM = 32;

struct MmaPlan {
  int ctas;
  int units;        // 4-row units in N
  int rows_cap;     // rows of the largest CTA share
  int steps;        // stages per row: K / 1024
  int panel_steps;  // stages per k-panel
  int xs_stride;    // bytes per row of x in the panel buffer
  int mc;           // columns of the corr table: M rounded up to even
  int stages;
  int off_xs, off_corr, off_red, off_stage, smem_bytes;
  int strict;       // 1: read the weights only after griddepcontrol.wait
  int* status;
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, __half2 f) {
  __half2 h;
  memcpy(&h, &a, 4);
  h = __hmul2(h, f);
  uint32_t r;
  memcpy(&r, &h, 4);
  return r;
}

__device__ __forceinline__ float half_lo(uint32_t v) {
  return __half2float(__ushort_as_half(static_cast<uint16_t>(v & 0xFFFFu)));
}
__device__ __forceinline__ float half_hi(uint32_t v) {
  return __half2float(__ushort_as_half(static_cast<uint16_t>(v >> 16)));
}

// Copies x[:, k0 : k0 + pk] into the permuted panel layout and builds the corr table.
__device__ __forceinline__ void load_x_panel(const GemvArgs& a, const MmaPlan& p, int k0, int pk,
                                             unsigned char* xs, float2* corr, int tid) {
  const __half2 sixteenth = __float2half2_rn(0.0625f);
  const int blocks8 = pk / 8;         // 8-weight blocks per row of x in this panel
  const int count = a.m * blocks8;    // a multiple of 16: sixteen lanes share one (m, item)
  for (int base = 0; base < count; base += kConsumerThreads) {
    const int idx = base + tid;
    const bool active = idx < count;
    float bsum = 0.0f, xsum = 0.0f;
    int m = 0, b = 0;
    if (active) {
      m = idx / blocks8;
      b = idx - m * blocks8;
      const uint4 v = *reinterpret_cast<const uint4*>(a.x + static_cast<int64_t>(m) * a.k + k0 + 8 * b);
      uint4 o;
      o.x = prmt(v.x, v.z, 0x5410);                          // x0, x4
      o.y = hmul2_bits(prmt(v.x, v.z, 0x7632), sixteenth);   // x1/16, x5/16
      o.z = prmt(v.y, v.w, 0x5410);                          // x2, x6
      o.w = hmul2_bits(prmt(v.y, v.w, 0x7632), sixteenth);   // x3/16, x7/16
      const int item = b >> 4, w = b & 15;
      *reinterpret_cast<uint4*>(xs + m * p.xs_stride + item * 256 + ((w & 3) * 4 + (w >> 2)) * 16) = o;
      const float ones = (half_lo(o.x) + half_hi(o.x)) + (half_lo(o.z) + half_hi(o.z));
      const float sixteenths = (half_lo(o.y) + half_hi(o.y)) + (half_lo(o.w) + half_hi(o.w));
      bsum = ones + sixteenths;
      xsum = ones + 16.0f * sixteenths;
    }
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) {
      bsum += __shfl_xor_sync(0xffffffffu, bsum, off);
      xsum += __shfl_xor_sync(0xffffffffu, xsum, off);
    }
    if (active && (b & 15) == 0) corr[(b >> 4) * p.mc + m] = make_float2(1024.0f * bsum, xsum);
  }
}

// At M <= 8, two CTAs' worth of registers per SM: this kernel's and the next one's. Larger M
// needs the registers for its extra accumulators.
template <int MT>
__global__ void __launch_bounds__(kThreads, MT == 1 ? 2 : 1)
    stream_mma_kernel(GemvArgs a, MmaPlan p, const __grid_constant__ WeightMaps maps) {
  extern __shared__ __align__(1024) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  unsigned char* xs = smem + p.off_xs;
  float2* corr = reinterpret_cast<float2*>(smem + p.off_corr);
  float* red = reinterpret_cast<float*>(smem + p.off_red);
  unsigned char* stages = smem + p.off_stage;

  const int tid = threadIdx.x;
  const int warp = tid / kWarp;
  const int lane = tid % kWarp;

  const int u0 = static_cast<int>(static_cast<int64_t>(blockIdx.x) * p.units / p.ctas);
  const int u1 = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * p.units / p.ctas);
  const int row_begin = 4 * u0;
  const int rows = min(4 * u1, a.n) - row_begin;
  const int blocks = (rows + kBlockRows - 1) / kBlockRows;

  if (tid == kConsumerThreads) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) launch_dependents();  // the next GEMV may become resident beside this CTA

  if (warp == kConsumerWarps) {
    if (p.strict) grid_dependency_wait();
    produce_weight_stages(maps, row_begin, rows, p.steps, p.panel_steps, stages, p.stages, full,
                          empty, p.status);
    return;
  }

  // ---------------- consumers ----------------
  const int g = lane >> 2;
  const int c = lane & 3;
  const int tile = warp & 1;
  const int pair = warp >> 1;
  const int r_lo = 16 * tile + ((g >> 1) | ((g & 1) << 2));  // block rows of MMA rows g, g + 8
  const int r_hi = r_lo + 8;
  grid_dependency_wait();  // x may be the previous kernel's output; y is written below

  bool ok = true;
  int sit = 0;  // stages consumed
  for (int p0 = 0; p0 < p.steps; p0 += p.panel_steps) {
    const int psteps = min(p.panel_steps, p.steps - p0);
    if (p0 > 0) named_barrier(kConsumerBarrier, kConsumerThreads);  // done with the last panel
    load_x_panel(a, p, p0 * kItemsPerStage * kItemK, psteps * kItemsPerStage * kItemK, xs, corr,
                 tid);
    named_barrier(kConsumerBarrier, kConsumerThreads);

    for (int blk = 0; blk < blocks; ++blk) {
      const int rows_b = min(kBlockRows, rows - blk * kBlockRows);
      const bool active = 16 * tile < rows_b;
      float acc[2][MT][2];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) acc[h][mt][0] = acc[h][mt][1] = 0.0f;

      for (int j = 0; j < psteps; ++j, ++sit) {
        const int slot = sit % p.stages;
        if (ok && !mbar_wait_bounded(&full[slot], (sit / p.stages) & 1)) {
          ok = false;
          atomicExch(p.status, kStatusFullBarrierTimeout);
        }
        const unsigned char* st = stages + slot * kStageBytes;
        uint4 aw[2][2];
        uint32_t s2[2], z2[2];  // scales / zeros of the warp's two items, rows r_lo and r_hi
        if (active) {
#pragma unroll
          for (int ii = 0; ii < 2; ++ii) {
            aw[ii][0] = stage_words(st, r_lo, 2 * pair + ii, c);
            aw[ii][1] = stage_words(st, r_hi, 2 * pair + ii, c);
          }
          const unsigned char* sp = st + kStageQBytes + 4 * pair;
          s2[0] = *reinterpret_cast<const uint32_t*>(sp + r_lo * kSzRowBytes);
          s2[1] = *reinterpret_cast<const uint32_t*>(sp + r_hi * kSzRowBytes);
          z2[0] = *reinterpret_cast<const uint32_t*>(sp + (kBlockRows + r_lo) * kSzRowBytes);
          z2[1] = *reinterpret_cast<const uint32_t*>(sp + (kBlockRows + r_hi) * kSzRowBytes);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);  // the stage may be refilled
        if (!active) continue;

#pragma unroll(MT == 1 ? 2 : 1)
        for (int ii = 0; ii < 2; ++ii) {
          const int item_p = j * kItemsPerStage + 2 * pair + ii;  // item within the panel
          float d[MT][2][4];
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int ch = 0; ch < 2; ++ch)
#pragma unroll
              for (int e = 0; e < 4; ++e) d[mt][ch][e] = 0.0f;
          // Selects rather than indexing, so a rolled loop keeps aw in registers.
          const uint4 al = ii == 0 ? aw[0][0] : aw[1][0];
          const uint4 ah = ii == 0 ? aw[0][1] : aw[1][1];
          const uint32_t wl[4] = {al.x, al.y, al.z, al.w};
          const uint32_t wh[4] = {ah.x, ah.y, ah.z, ah.w};
#pragma unroll
          for (int jw = 0; jw < 4; ++jw) {
            uint32_t hl[4], hh[4];
            unpack_x16(wl[jw], hl);
            unpack_x16(wh[jw], hh);
            const uint32_t a0[4] = {hl[0], hh[0], hl[1], hh[1]};
            const uint32_t a1[4] = {hl[2], hh[2], hl[3], hh[3]};
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              const int m = g + 8 * mt;
              uint4 xb = make_uint4(0, 0, 0, 0);
              if (m < a.m) {
                xb = *reinterpret_cast<const uint4*>(xs + m * p.xs_stride + item_p * 256 +
                                                     (jw * 4 + c) * 16);
              }
              mma_16816(d[mt][jw & 1], a0, xb.x, xb.y);
              mma_16816(d[mt][jw & 1], a1, xb.z, xb.w);
            }
          }
          const float s_lo = ii ? half_hi(s2[0]) : half_lo(s2[0]);
          const float s_hi = ii ? half_hi(s2[1]) : half_lo(s2[1]);
          const float z_lo = ii ? half_hi(z2[0]) : half_lo(z2[0]);
          const float z_hi = ii ? half_hi(z2[1]) : half_lo(z2[1]);
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const int m0 = 8 * mt + 2 * c;
            const float4 cr = *reinterpret_cast<const float4*>(corr + item_p * p.mc +
                                                               (m0 < a.m ? m0 : 0));
            const float d0 = d[mt][0][0] + d[mt][1][0], d1 = d[mt][0][1] + d[mt][1][1];
            const float d2 = d[mt][0][2] + d[mt][1][2], d3 = d[mt][0][3] + d[mt][1][3];
            acc[0][mt][0] = fmaf(s_lo, fmaf(-z_lo, cr.y, d0 - cr.x), acc[0][mt][0]);
            acc[0][mt][1] = fmaf(s_lo, fmaf(-z_lo, cr.w, d1 - cr.z), acc[0][mt][1]);
            acc[1][mt][0] = fmaf(s_hi, fmaf(-z_hi, cr.y, d2 - cr.x), acc[1][mt][0]);
            acc[1][mt][1] = fmaf(s_hi, fmaf(-z_hi, cr.w, d3 - cr.z), acc[1][mt][1]);
          }
        }
      }
      // Block end: this warp's partials of (rows r_lo / r_hi, columns 8 mt + 2 c + e).
      if (active) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = h ? r_hi : r_lo;
          if (r >= rows_b) continue;
          float* dst = red + (pair * p.rows_cap + blk * kBlockRows + r) * a.m;
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int m = 8 * mt + 2 * c + e;
              if (m < a.m) dst[m] = p0 == 0 ? acc[h][mt][e] : dst[m] + acc[h][mt][e];
            }
          }
        }
      }
    }
  }

  // ---- add the four item-pair partials of every output in a fixed order; store fp16 ----------
  named_barrier(kConsumerBarrier, kConsumerThreads);
  for (int o = tid; o < rows * a.m; o += kConsumerThreads) {
    const int m = o / rows;
    const int r = o - m * rows;
    float sum = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) sum += red[(q * p.rows_cap + r) * a.m + m];
    if (ok) a.y[static_cast<int64_t>(m) * a.n + row_begin + r] = __float2half_rn(sum);
  }
}

int tile_count(int m) { return (m + 7) / 8; }

// Lays out shared memory for `panel_steps` stages per panel; true if it fits `limit` with at
// least `min_stages` stages.
bool plan_smem(const GemvArgs& a, MmaPlan* p, int limit, int min_stages) {
  const int pk = p->panel_steps * kItemsPerStage * kItemK;
  p->xs_stride = pk * 2 + 64;
  int64_t off = 1024;  // mbarriers
  p->off_xs = static_cast<int>(off);
  off += static_cast<int64_t>(a.m) * p->xs_stride;
  off = (off + 15) / 16 * 16;
  p->off_corr = static_cast<int>(off);
  off += static_cast<int64_t>(pk / kItemK) * p->mc * 8;
  p->off_red = static_cast<int>(off);
  off += static_cast<int64_t>(4) * p->rows_cap * a.m * 4;
  off = (off + 1023) / 1024 * 1024;
  p->off_stage = static_cast<int>(off);
  if (off > limit) return false;
  const int64_t stages = std::min<int64_t>((limit - off) / kStageBytes, kMaxStages);
  if (stages < min_stages) return false;
  p->stages = static_cast<int>(stages);
  p->smem_bytes = static_cast<int>(off + stages * kStageBytes);
  return true;
}

bool make_plan(const GemvArgs& a, MmaPlan* p, const char** why) {
  auto fail = [&](const char* reason) {
    if (why) *why = reason;
    return false;
  };
  if (a.m < 1 || a.m > kMaxM) return fail("M must be in [1, 32]");
  if (!weight_stream_supported(a, why)) return false;
  if (reinterpret_cast<uintptr_t>(a.x) % 16) return fail("x must be 16-byte aligned");
  p->units = (a.n + 3) / 4;
  p->ctas = std::min(sm_count(), p->units);
  p->rows_cap = 4 * ((p->units + p->ctas - 1) / p->ctas);
  p->steps = a.k / (kItemK * kItemsPerStage);
  p->mc = (a.m + 1) & ~1;
  // Prefer room for the next kernel's CTA, then fewer k-panels.
  const int limits[3] = {kCoResident, kSmemLimit, kSmemLimit};
  const int min_stages[3] = {4, 4, 3};
  for (int t = 0; t < 3; ++t) {
    for (int panels = 1; panels <= p->steps; ++panels) {
      p->panel_steps = (p->steps + panels - 1) / panels;
      if (plan_smem(a, p, limits[t], min_stages[t])) {
        p->strict = 0;
        return true;
      }
    }
  }
  return fail("x does not fit in shared memory");
}

std::once_flag g_attr_once[4][64];

template <int MT>
cudaError_t ensure_smem_attr() {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  cudaError_t result = cudaSuccess;
  std::call_once(g_attr_once[MT - 1][dev & 63], [&] {
    result = cudaFuncSetAttribute(stream_mma_kernel<MT>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
  });
  return result;
}

template <typename F>
cudaError_t with_mt(int m, F&& f) {
  switch (tile_count(m)) {
    case 1:
      return f.template operator()<1>();
    case 2:
      return f.template operator()<2>();
    case 3:
      return f.template operator()<3>();
    default:
      return f.template operator()<4>();
  }
}

}  // namespace

bool stream_mma_supported(const GemvArgs& a, const char** why) {
  MmaPlan p;
  return make_plan(a, &p, why);
}

cudaError_t launch_stream_mma(const GemvArgs& a, cudaStream_t stream, bool strict) {
  MmaPlan p;
  if (!make_plan(a, &p, nullptr)) return cudaErrorInvalidValue;
  p.strict = strict ? 1 : 0;
  p.status = device_status_word();
  if (!p.status) return cudaErrorInvalidSymbol;
  WeightMaps maps;
  const cudaError_t merr = weight_maps_for(a, &maps);
  if (merr != cudaSuccess) return merr;
  return with_mt(a.m, [&]<int MT>() {
    cudaError_t err = ensure_smem_attr<MT>();
    if (err != cudaSuccess) return err;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.ctas);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = p.smem_bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, stream_mma_kernel<MT>, a, p, maps);
  });
}

cudaError_t stream_mma_attrs(int m, KernelAttrs* out) {
  return with_mt(m < 1 ? 1 : m, [&]<int MT>() {
    cudaFuncAttributes fa;
    cudaError_t err = cudaFuncGetAttributes(&fa, stream_mma_kernel<MT>);
    if (err != cudaSuccess) return err;
    out->registers = fa.numRegs;
    out->local_bytes = static_cast<int>(fa.localSizeBytes);
    out->max_threads_per_block = fa.maxThreadsPerBlock;
    out->blocks_per_sm = 1;  // plus, when it fits in 113 KB, the next kernel's CTA
    out->threads_per_block = kThreads;
    return cudaSuccess;
  });
}

}  // namespace i4
