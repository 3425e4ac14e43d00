// The B200 fast path for M <= 32: TMA tile stream of the packed weights + warp-level tensor-core
// MMAs (mma.sync m16n8k16, f16 x f16 -> f32) on the nibbles unpacked in registers.
//
// Why warp MMAs at small M. Per packed 32-bit word (8 weights) a thread spends one shift and four
// LOP3s to turn the nibbles into fp16 A-fragment registers (the magic-number trick: 1024 + q and
// 1024 + 16 q, exact); one m16n8k16 MMA then covers 256 weights. A 128-row tcgen05 MMA has a
// fixed issue cost per 16 k that makes it the slower choice at M <= 32 (measured).
//
// Work split. One CTA per SM (grid = SMs) using the SM's shared memory for a deep ring of stages.
// CTA c owns rows [4 u0, 4 u1), an equal share of 4-row units. Its rows are taken in k-panels
// (all of K when x fits) x blocks of 32 rows x stages of 8 items (an item = 128 weights = one
// group). A producer warp fills the ring with 2-D TMA tiles (weight_stream.cuh) and, right after
// the dependency on the previous kernel in the stream resolves, copies each panel of x into
// shared memory with a bulk copy ahead of the remaining weight tiles, so x does not queue behind
// them. Eight consumer warps split each stage.
//
// Narrow path (M <= 4, MP = 2 or 4 rows of x per item in the 8 MMA columns). The eight MMA
// columns hold 8 / MP different items x MP rows of x: both k-slot pairs of thread c (2c, 2c+1 and
// 2c+8, 2c+9) take two adjacent words of one item, and its B values are non-zero only in that
// item's columns. So an MMA still covers 256 weights, but scales are applied once per stage
// instead of once per item. Warp w takes MMA rows 16 (w % 2) .. + 15 of the block and word
// quarter q = w / 2 of every item (rotated by thread, below); the item's correction is applied by
// the q = 0 warp.
//
// Wide path (5 <= M <= 32: MT = ceil(M / 8) tiles of 8 rows of x). Warp w takes rows 16 (w % 2)
// .. + 15 and items 2 (w / 2), 2 (w / 2) + 1; each item's MMAs accumulate from zero, and its
// scale and correction are applied per item.
//
// Both paths: MMA row g (and g + 8) is block row mma_row(g) (and + 8), and in the narrow path the
// word quarter a thread reads is rotated by its k-slot group, so the sixteen-byte loads of one
// shared-memory phase hit distinct banks under the 128-byte swizzle. Each panel of x is permuted
// in shared memory, each 8-weight block to [x0, x4, x1/16, x5/16, x2, x6, x3/16, x7/16]
// (matching the unpacked A halves), and laid out so that one 16-byte load gives a thread its B
// register pairs for two MMAs; lanes whose B values are zero read a zeroed block instead. The
// same pass builds corr[item][m] = (1024 * sum of the B values, sum of the x they stand for), so
// for each (row, item)
//     sum_k (q_k - z) s x_k = s * (D - 1024 sum_k b_k - z sum_k x_k).
// The weights are bit-exact; the arithmetic is fp32 accumulation of exact fp16 products.
//
// Results. Per-thread fp32 partials go to shared memory at the end of each block; after the last
// block the partials of each output are added in a fixed order, so results are deterministic.
// Every mbarrier wait is bounded; on timeout the kernel records a status word and runs to
// completion without writing y.
#include <algorithm>
#include <mutex>

#include "exchange.cuh"
#include "weight_stream.cuh"

namespace i4 {
namespace {

constexpr int kMaxStages = 12;
constexpr int kSmemLimit = 227 * 1024;
constexpr int kConsumerBarrier = 1;
constexpr int kMaxM = 32;
constexpr int kNarrowItemBytes = 272;  // one item of one x row, narrow layout (256 + 16 pad)
constexpr int kZeroBytes = 2048;       // zeroed block read by lanes whose B values are zero
constexpr int kPreStages = 2;          // weight stages issued before the dependency wait

// mbarriers at the start of shared memory
constexpr int kBarFull = 0;                   // [kMaxStages] stage landed
constexpr int kBarEmpty = kMaxStages;         // [kMaxStages] stage consumed (8 warps)
constexpr int kBarXFull = 2 * kMaxStages;     // x panel landed
constexpr int kBarXEmpty = 2 * kMaxStages + 1;  // x panel permuted: its raw buffer is free

struct MmaPlan {
  int ctas;
  int units;        // 4-row units in N
  int rows_cap;     // rows of the largest CTA share
  int steps;        // stages per row: K / 1024
  int panel_steps;  // stages per k-panel
  int xs_stride;    // bytes per row of x in the permuted panel buffer
  int mc;           // columns of the corr table: M rounded up to even
  int stages;
  int pre_stages;   // weight stages the producer issues before the dependency wait
  int off_xr, off_xs, off_corr, off_red, off_stage, smem_bytes;
  int strict;       // 1: read the weights only after griddepcontrol.wait
  int* status;
  // Wide path with a workspace: x permuted once per call by stream_mma_xprep_kernel; panel pi is
  // xslot bytes at xpre + pi * xslot (the xs rows, then the corr table), copied into xr.
  const unsigned char* xpre;
  int xslot;
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

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// MMA row g -> block row: the two rows of one shared-memory phase (g = 2p, 2p + 1) differ in
// bit 1, which the 128-byte swizzle turns into different banks.
__device__ __forceinline__ int mma_row(int g) {
  return (g & 4) | ((g & 1) << 1) | ((g >> 1) & 1);
}

// x0..x7 (one 8-weight block) -> the B halves matching unpack_x16: (x0, x4), (x1/16, x5/16),
// (x2, x6), (x3/16, x7/16); adds the block's B values to bsum and the x they stand for to xsum.
__device__ __forceinline__ uint4 permute_block(const uint4& v, float& bsum, float& xsum) {
  const __half2 sixteenth = __float2half2_rn(0.0625f);
  uint4 o;
  o.x = prmt(v.x, v.z, 0x5410);
  o.y = hmul2_bits(prmt(v.x, v.z, 0x7632), sixteenth);
  o.z = prmt(v.y, v.w, 0x5410);
  o.w = hmul2_bits(prmt(v.y, v.w, 0x7632), sixteenth);
  const float ones = (half_lo(o.x) + half_hi(o.x)) + (half_lo(o.z) + half_hi(o.z));
  const float sixteenths = (half_lo(o.y) + half_hi(o.y)) + (half_lo(o.w) + half_hi(o.w));
  bsum += ones + sixteenths;
  xsum += ones + 16.0f * sixteenths;
  return o;
}

// Permutes the raw x panel xr[m][pk] (as landed) into the consumers' layout and builds the corr
// table. Each thread takes two adjacent words (16 weights) of one row of x; eight threads cover
// an item. Narrow layout: xs[m][item][word pair t][half h][word 2t + i][2 halves]: the 16 bytes
// at (t, h) are the B registers (word 2t, word 2t+1) of MMAs 2h and 2h + 1. Wide layout:
// xs[m][item][j][c][8 halves] for word 4 c + j, item stride 256.
template <bool NARROW, int kConsumerThreads>
__device__ __forceinline__ void permute_x_panel(const GemvArgs& a, const MmaPlan& p, int pk,
                                                const unsigned char* xr, int xr_stride,
                                                unsigned char* xs, float2* corr, int tid) {
  const int pairs = pk / 16;        // word pairs per row of x in this panel
  const int count = a.m * pairs;    // a multiple of 8: eight lanes share one (m, item)
  for (int base = 0; base < count; base += kConsumerThreads) {
    const int idx = base + tid;
    const bool active = idx < count;
    float bsum = 0.0f, xsum = 0.0f;
    int m = 0, v = 0;
    if (active) {
      m = idx / pairs;
      v = idx - m * pairs;
      const uint4* src =
          reinterpret_cast<const uint4*>(xr + (static_cast<int64_t>(m) * xr_stride + 16 * v) * 2);
      const uint4 o0 = permute_block(src[0], bsum, xsum);
      const uint4 o1 = permute_block(src[1], bsum, xsum);
      const int item = v >> 3, t = v & 7;
      unsigned char* row = xs + m * p.xs_stride;
      if (NARROW) {
        uint4* dst = reinterpret_cast<uint4*>(row + item * kNarrowItemBytes + t * 32);
        dst[0] = make_uint4(o0.x, o1.x, o0.y, o1.y);
        dst[1] = make_uint4(o0.z, o1.z, o0.w, o1.w);
      } else {
        const int w0 = 2 * t, w1 = 2 * t + 1;
        *reinterpret_cast<uint4*>(row + item * 256 + ((w0 & 3) * 4 + (w0 >> 2)) * 16) = o0;
        *reinterpret_cast<uint4*>(row + item * 256 + ((w1 & 3) * 4 + (w1 >> 2)) * 16) = o1;
      }
    }
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) {
      bsum += __shfl_xor_sync(0xffffffffu, bsum, off);
      xsum += __shfl_xor_sync(0xffffffffu, xsum, off);
    }
    if (active && (v & 7) == 0) corr[(v >> 3) * p.mc + m] = make_float2(1024.0f * bsum, xsum);
  }
}

// The same panel from a workspace slot already permuted by stream_mma_xprep_kernel (landed in the
// raw x buffer): the xs rows and the corr table, copied 16 bytes at a time.
template <int kThreads>
__device__ __forceinline__ void copy_x_slot(const unsigned char* slot, int x_bytes, int corr_bytes,
                                            unsigned char* xs, float2* corr, int tid) {
  const uint4* sx = reinterpret_cast<const uint4*>(slot);
  uint4* dx = reinterpret_cast<uint4*>(xs);
  for (int i = tid; i < x_bytes / 16; i += kThreads) dx[i] = sx[i];
  const uint4* sc = reinterpret_cast<const uint4*>(slot + x_bytes);
  uint4* dc = reinterpret_cast<uint4*>(corr);
  for (int i = tid; i < corr_bytes / 16; i += kThreads) dc[i] = sc[i];
}

// Permutes x once per call for the wide path: block pi writes into workspace slot pi exactly what
// permute_x_panel writes into a CTA's shared memory for k-panel pi (the xs rows, then the corr
// table), so the GEMV's CTAs copy it instead of each permuting all of x.
constexpr int kXprepThreads = 256;

__global__ void __launch_bounds__(kXprepThreads)
    stream_mma_xprep_kernel(GemvArgs a, MmaPlan p, unsigned char* ws) {
  // The GEMV (launched with programmatic serialization) may start its weight stream now; it
  // reads the workspace only after its dependency wait, i.e. after this grid has completed.
  if (threadIdx.x == 0) launch_dependents();
  const int pi = blockIdx.x;
  const int p0 = pi * p.panel_steps;
  const int pk = min(p.panel_steps, p.steps - p0) * kItemsPerStage * kItemK;
  unsigned char* slot = ws + static_cast<int64_t>(pi) * p.xslot;
  const half* x0 = a.x + static_cast<int64_t>(p0) * kItemsPerStage * kItemK;
  permute_x_panel<false, kXprepThreads>(
      a, p, pk, reinterpret_cast<const unsigned char*>(x0), a.k, slot,
      reinterpret_cast<float2*>(slot + static_cast<int64_t>(a.m) * p.xs_stride), threadIdx.x);
}

// The consumers' side of the stage ring (slot and phase kept incrementally: no division).
struct StageRing {
  uint64_t* full;
  int stages;
  int* status;
  bool ok;
  int slot;
  uint32_t phase;
  // Waits (bounded) for the next stage to land; returns its buffer index.
  __device__ __forceinline__ int next() {
    const int s = slot;
    if (ok && !mbar_wait_bounded(&full[s], phase)) {
      ok = false;
      atomicExch(status, kStatusFullBarrierTimeout);
    }
    if (++slot == stages) {
      slot = 0;
      phase ^= 1u;
    }
    return s;
  }
};

// ---- producer ----------------------------------------------------------------------------------
__device__ __forceinline__ void issue_x_panel(const GemvArgs& a, int k0, int pk, unsigned char* xr,
                                              uint64_t* xfull, uint64_t policy, int lane) {
  if (lane == 0) mbar_arrive_expect_tx(xfull, static_cast<uint32_t>(a.m * pk * 2));
  __syncwarp();
  for (int m = lane; m < a.m; m += kWarp) {
    bulk_g2s(xr + static_cast<int64_t>(m) * pk * 2, a.x + static_cast<int64_t>(m) * a.k + k0,
             static_cast<uint32_t>(pk * 2), xfull, policy);
  }
}

// Copies workspace slot pi (the permuted x panel and its corr table) into the raw x buffer.
__device__ __forceinline__ void issue_x_slot(const MmaPlan& p, int pi, unsigned char* xr,
                                             uint64_t* xfull, uint64_t policy, int lane) {
  if (lane == 0) {
    mbar_arrive_expect_tx(xfull, static_cast<uint32_t>(p.xslot));
    bulk_g2s(xr, p.xpre + static_cast<int64_t>(pi) * p.xslot, static_cast<uint32_t>(p.xslot),
             xfull, policy);
  }
  __syncwarp();
}

// Streams the CTA's weights (panel by panel, block by block, stage by stage) and, per panel, its
// raw x (or, with a workspace, its pre-permuted x slot). The first p.pre_stages weight stages go out before the dependency wait (unless strict);
// x for panel 0 right after it, ahead of the remaining weight stages.
__device__ __forceinline__ void produce(const GemvArgs& a, const MmaPlan& p, const WeightMaps& maps,
                                        int row_begin, int rows, unsigned char* smem) {
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint64_t* full = bars + kBarFull;
  uint64_t* empty = bars + kBarEmpty;
  unsigned char* stages = smem + p.off_stage;
  unsigned char* xr = smem + p.off_xr;
  const int lane = threadIdx.x % kWarp;
  const uint64_t wpolicy = l2_evict_first_policy();
  const uint64_t xpolicy = l2_evict_last_policy();
  const int blocks = (rows + kBlockRows - 1) / kBlockRows;
  const int pre = p.strict ? 0 : p.pre_stages;  // < the stages of panel 0
  if (p.strict) grid_dependency_wait();
  bool x0_sent = false;
  if (pre == 0) {
    if (!p.strict) grid_dependency_wait();
    if (p.xpre) {
      issue_x_slot(p, 0, xr, &bars[kBarXFull], xpolicy, lane);
    } else {
      issue_x_panel(a, 0, min(p.panel_steps, p.steps) * kItemsPerStage * kItemK, xr,
                    &bars[kBarXFull], xpolicy, lane);
    }
    x0_sent = true;
  }
  bool ok = true;
  int it = 0, slot = 0, use = 0;
  for (int pi = 0, p0 = 0; p0 < p.steps; ++pi, p0 += p.panel_steps) {
    const int p1 = min(p.steps, p0 + p.panel_steps);
    if (pi > 0) {
      if (ok && !mbar_wait_bounded(&bars[kBarXEmpty], (pi - 1) & 1)) {
        ok = false;
        if (lane == 0) atomicExch(p.status, kStatusEmptyBarrierTimeout);
      }
      if (ok && p.xpre) {
        issue_x_slot(p, pi, xr, &bars[kBarXFull], xpolicy, lane);
      } else if (ok) {
        issue_x_panel(a, p0 * kItemsPerStage * kItemK, (p1 - p0) * kItemsPerStage * kItemK, xr,
                      &bars[kBarXFull], xpolicy, lane);
      }
    }
    for (int blk = 0; blk < blocks; ++blk) {
      const int rows4 = (min(kBlockRows, rows - blk * kBlockRows) + 3) & ~3;
      LaneBox b;
      const bool has_box = lane_box(maps, lane, rows4, row_begin + blk * kBlockRows, &b);
      for (int j = p0; j < p1; ++j, ++it) {
        if (!x0_sent && it == pre) {
          grid_dependency_wait();
          if (p.xpre) {
            issue_x_slot(p, 0, xr, &bars[kBarXFull], xpolicy, lane);
          } else {
            issue_x_panel(a, 0, (p1 - p0) * kItemsPerStage * kItemK, xr, &bars[kBarXFull],
                          xpolicy, lane);
          }
          x0_sent = true;
        }
        if (ok && use > 0 && !mbar_wait_bounded(&empty[slot], (use - 1) & 1)) {
          ok = false;
          if (lane == 0) atomicExch(p.status, kStatusEmptyBarrierTimeout);
        }
        if (ok) {
          issue_stage(b, has_box, j, rows4, stages + slot * kStageBytes, &full[slot], wpolicy,
                      lane);
        }
        if (++slot == p.stages) {
          slot = 0;
          ++use;
        }
      }
    }
  }
  // Do not leave while copies into this CTA's shared memory may be in flight: the last weight
  // stages and the last x panel.
  if (ok) {
    for (int back = 1; back <= min(it, p.stages); ++back) {
      const int j = it - back;
      if (!mbar_wait_bounded(&full[j % p.stages], (j / p.stages) & 1)) break;
    }
    const int panels = (p.steps + p.panel_steps - 1) / p.panel_steps;
    mbar_wait_bounded(&bars[kBarXFull], (panels - 1) & 1);
  }
}

// ---- narrow path ---------------------------------------------------------------------------------
// MP = 2 or 4. A stage's work per 16-row tile is four rounds j = 0..3 over four word quarters. In
// round j thread (g, c) processes words w and w + 1 (k-slot pairs 2c, 2c+1 and 2c+8, 2c+9) of one
// item, rows r_lo and r_hi:
//   MP = 2: item c + 4 (j / 2), w = 4 qc + 2 (j % 2); accumulator columns 2 c + m.
//   MP = 4: item 4 (c / 2) + j, w = 4 qc + 2 (c % 2); accumulator columns 4 (c / 2) + m.
// qc = (q + c / 2) % 4 is the thread's rotated word quarter. D sets (one accumulator set per
// group of items): MP = 2: j / 2, MP = 4: j. With NR = 2 rounds per warp, warps w and w + 8 share
// a (tile, quarter) and take rounds 0, 1 and 2, 3 (hs = w / 8). Every load offset below is a
// per-thread base plus a compile-time constant.
template <int MP, int NR>
struct NarrowThread {
  static constexpr int kSets = MP == 4 ? NR : NR / 2;  // D sets per warp and stage
  int c, q, hs;
  int r_lo, r_hi;
  int item0;       // stage item of the thread's D set 0 (epilogue columns 2 c, 2 c + 1)
  int a_base;      // stage offset of the A granule of (the first item, row r_lo)
  int a_base_odd;  // MP 4: the same for the odd round (granule half flipped)
  int b_base;      // x offset of the lane's B values in the stage's first item, or of the zeros
  int b_step;      // x bytes per stage for lanes with B values, 0 for the others

  __device__ __forceinline__ void init(int warp, int lane, int m_rows, int xs_stride,
                                       int zero_rel) {
    const int g = lane >> 2;
    c = lane & 3;
    q = (warp >> 1) & 3;
    hs = NR == 4 ? 0 : warp >> 3;
    const int qc = (q + (c >> 1)) & 3;
    r_lo = 16 * (warp & 1) + mma_row(g);
    r_hi = r_lo + 8;
    const int r7 = r_lo & 7;
    bool on;
    if (MP == 4) {
      // items 4 (c / 2) + NR hs + round
      const int row_off = r_lo * 128 + 8 * (c & 1) + ((c >> 1) * 2 + (NR / 2) * hs) * kChunkBytes;
      a_base = row_off + ((qc ^ r7) * 16);
      a_base_odd = row_off + (((4 + qc) ^ r7) * 16);
      const int m = g & 3;
      on = (g >> 2) == (c >> 1) && m < m_rows;
      item0 = 4 * (c >> 1) + NR * hs;
      b_base = m * xs_stride + (4 * (c >> 1) + NR * hs) * kNarrowItemBytes +
               (2 * qc + (c & 1)) * 32;
    } else {
      // items c + 4 (hs + round / 2)
      a_base = ((c >> 1) + 2 * hs) * kChunkBytes + r_lo * 128 + ((((c & 1) * 4 + qc) ^ r7) * 16);
      a_base_odd = 0;
      const int m = g & 1;
      on = (g >> 1) == c && m < m_rows;
      item0 = c + 4 * hs;
      b_base = m * xs_stride + (c + 4 * hs) * kNarrowItemBytes + 2 * qc * 32;
    }
    if (!on) b_base = zero_rel;
    b_step = on ? kItemsPerStage * kNarrowItemBytes : 0;
  }
  // Stage offset of A load i (MP 2: item sel i; MP 4: round i) of row h.
  __device__ __forceinline__ int a_off(int i, int h) const {
    if (MP == 4) return ((i & 1) ? a_base_odd : a_base) + (i >> 1) * kChunkBytes + h * 1024;
    return a_base + i * 2 * kChunkBytes + h * 1024;
  }
  // Offset of the B loads of round j (half h: MMAs 2h, 2h + 1) from the lane's stage base.
  __device__ __forceinline__ static constexpr int b_off(int j, int h) {
    return MP == 2 ? (j >> 1) * 4 * kNarrowItemBytes + (j & 1) * 32 + 16 * h
                   : j * kNarrowItemBytes + 16 * h;
  }
  __device__ __forceinline__ int col_m(int e) const { return (2 * c + e) % MP; }
  // Stage item of the thread's accumulator columns in D set `set`.
  __device__ __forceinline__ int col_item(int set) const {
    return MP == 2 ? item0 + 4 * set : item0 + set;
  }
};

// Raw fp16 scale (or zero) bits of the thread's epilogue items (col_item(set)) for one row of a
// landed stage.
template <int MP, int NR>
struct SzBits {
  static constexpr int kSets = NarrowThread<MP, NR>::kSets;
  uint32_t w[2];
  __device__ __forceinline__ void load(const unsigned char* row_base, int item0) {
    if (MP == 2) {
#pragma unroll
      for (int s = 0; s < kSets; ++s) {
        w[s] = *reinterpret_cast<const uint16_t*>(row_base + 2 * (item0 + 4 * s));
      }
    } else if (kSets == 2) {
      w[0] = *reinterpret_cast<const uint32_t*>(row_base + 2 * item0);
    } else {
      const uint2 v = *reinterpret_cast<const uint2*>(row_base + 2 * item0);
      w[0] = v.x;
      w[1] = v.y;
    }
  }
  __device__ __forceinline__ float get(int set) const {
    if (MP == 2) return half_lo(w[set]);
    return (set & 1) ? half_hi(w[set >> 1]) : half_lo(w[set >> 1]);
  }
};

// One landed stage's operands in registers: the A words, scales and zeros of the warp's share.
template <int MP, int NR>
struct NarrowRegs {
  uint4 wa[2][2];              // MP 2: [item sel][row] = the 4 words of the granule
  uint2 wb[4][2];              // MP 4: [round][row] = words w, w + 1
  SzBits<MP, NR> sb[2], zb[2];  // [row]
};

template <int MP>
__host__ __device__ constexpr int narrow_acc() {  // accumulator chains per D set
  return MP == 4 ? 2 : 1;
}

// Loads the warp's share of a landed stage into registers and releases the stage.
template <int MP, int NR>
__device__ __forceinline__ void narrow_load(const NarrowThread<MP, NR>& t, const unsigned char* st,
                                            NarrowRegs<MP, NR>& r, uint64_t* empty_bar,
                                            uint32_t* scratch, int lane) {
  if (MP == 4) {
#pragma unroll
    for (int j = 0; j < NR; ++j)
#pragma unroll
      for (int h = 0; h < 2; ++h) r.wb[j][h] = *reinterpret_cast<const uint2*>(st + t.a_off(j, h));
  } else {
#pragma unroll
    for (int i = 0; i < NR / 2; ++i)
#pragma unroll
      for (int h = 0; h < 2; ++h) r.wa[i][h] = *reinterpret_cast<const uint4*>(st + t.a_off(i, h));
  }
  const unsigned char* sp = st + kStageQBytes;
  const unsigned char* zp = sp + kBlockRows * kSzRowBytes;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int row = h ? t.r_hi : t.r_lo;
    r.sb[h].load(sp + row * kSzRowBytes, t.item0);
    if (t.q == 0) r.zb[h].load(zp + row * kSzRowBytes, t.item0);
  }
  // release only once every load above has returned (see stage_reads_done)
  constexpr int kSets = NarrowThread<MP, NR>::kSets;
  constexpr int kWords = MP == 2 ? kSets : (kSets == 2 ? 1 : 2);  // SzBits words loaded
  uint32_t folded = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    if (MP == 4) {
#pragma unroll
      for (int j = 0; j < NR; ++j) folded ^= r.wb[j][h].x ^ r.wb[j][h].y;
    } else {
#pragma unroll
      for (int i = 0; i < NR / 2; ++i) folded ^= fold4(r.wa[i][h]);
    }
#pragma unroll
    for (int w = 0; w < kWords; ++w) {
      folded ^= r.sb[h].w[w];
      if (t.q == 0) folded ^= r.zb[h].w[w];
    }
  }
  stage_reads_done(folded, scratch, lane);
  __syncwarp();
  if (lane == 0) mbar_arrive(empty_bar);  // the stage may be refilled
}

// The stage's 4 NR MMAs. Accumulators: MP 2: one chain per set; MP 4: [set][hh % 2]. The first MMA
// into each chain starts it (C = 0). A single chain per set measured fastest for MP 2: the other
// warps and the overlapped loads of the next stage hide its latency.
template <int MP, int NR>
__device__ __forceinline__ void narrow_mma(const NarrowRegs<MP, NR>& r, const unsigned char* xb,
                                           float (&d)[NarrowThread<MP, NR>::kSets]
                                                     [narrow_acc<MP>()][4]) {
  constexpr int kAcc = narrow_acc<MP>();
#pragma unroll
  for (int j = 0; j < NR; ++j) {
    uint32_t w0r0, w0r1, w1r0, w1r1;  // words w, w + 1 of rows r_lo, r_hi
    if (MP == 2) {
      const int w = 2 * (j & 1);
      w0r0 = word_of(r.wa[j >> 1][0], w);
      w0r1 = word_of(r.wa[j >> 1][1], w);
      w1r0 = word_of(r.wa[j >> 1][0], w + 1);
      w1r1 = word_of(r.wa[j >> 1][1], w + 1);
    } else {
      w0r0 = r.wb[j][0].x;
      w0r1 = r.wb[j][1].x;
      w1r0 = r.wb[j][0].y;
      w1r1 = r.wb[j][1].y;
    }
    // The nibble unpacking of unpack_x16, one MMA operand quad at a time: the four LOP3s that make
    // an MMA's A registers come right before it, so each lands where the MMA reads it.
    const uint32_t lo[4] = {w0r0, w0r1, w1r0, w1r1};
    const uint32_t hi[4] = {w0r0 >> 8, w0r1 >> 8, w1r0 >> 8, w1r1 >> 8};
    const uint4 bx0 = *reinterpret_cast<const uint4*>(xb + NarrowThread<MP, NR>::b_off(j, 0));
    const uint4 bx1 = *reinterpret_cast<const uint4*>(xb + NarrowThread<MP, NR>::b_off(j, 1));
    const int set = MP == 2 ? (j >> 1) : j;
#pragma unroll
    for (int hh = 0; hh < 4; ++hh) {
      uint32_t afr[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) afr[i] = magic_f16(hh < 2 ? lo[i] : hi[i], hh & 1);
      const uint4& bx = hh < 2 ? bx0 : bx1;
      const uint32_t b0 = (hh & 1) ? bx.z : bx.x;
      const uint32_t b1 = (hh & 1) ? bx.w : bx.y;
      const bool first = MP == 2 ? ((j & 1) == 0 && hh == 0) : hh < 2;
      if (first) {
        mma_16816_first(d[set][hh % kAcc], afr, b0, b1);
      } else {
        mma_16816(d[set][hh % kAcc], afr, b0, b1);
      }
    }
  }
}

// Scale (and, in the q == 0 warps, the group correction) of the stage's D sets into
// acc[row lo / hi][e]. kCorr and the x row count are compile-time where the kernel instance
// allows, so the epilogue has no selects.
template <int MP, int NR, bool kCorr>
__device__ __forceinline__ void narrow_epilogue_impl(const NarrowThread<MP, NR>& t,
                                                     const NarrowRegs<MP, NR>& r,
                                                     const float (&d)[NarrowThread<MP, NR>::kSets]
                                                                     [narrow_acc<MP>()][4],
                                                     const float2* corr_stage, int mc, int m_rows,
                                                     float (&acc)[2][2]) {
  constexpr int kSets = NarrowThread<MP, NR>::kSets;
  constexpr int kAcc = narrow_acc<MP>();
#pragma unroll
  for (int set = 0; set < kSets; ++set) {
    float dsum[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float v = d[set][0][e];
#pragma unroll
      for (int i = 1; i < kAcc; ++i) v += d[set][i][e];
      dsum[e] = v;
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int m = t.col_m(e);
      if (m >= m_rows) continue;
      if (kCorr) {
        const float2 cr = corr_stage[t.col_item(set) * mc + m];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float v = dsum[2 * h + e] - fmaf(r.zb[h].get(set), cr.y, cr.x);
          acc[h][e] = fmaf(r.sb[h].get(set), v, acc[h][e]);
        }
      } else {
#pragma unroll
        for (int h = 0; h < 2; ++h) acc[h][e] = fmaf(r.sb[h].get(set), dsum[2 * h + e], acc[h][e]);
      }
    }
  }
}

template <int MP, int NR>
__device__ __forceinline__ void narrow_epilogue(const NarrowThread<MP, NR>& t,
                                                const NarrowRegs<MP, NR>& r,
                                                const float (&d)[NarrowThread<MP, NR>::kSets]
                                                                [narrow_acc<MP>()][4],
                                                const float2* corr_stage, int mc, int m_rows,
                                                float (&acc)[2][2]) {
  if (t.q == 0) {  // warp-uniform
    narrow_epilogue_impl<MP, NR, true>(t, r, d, corr_stage, mc, m_rows, acc);
  } else {
    narrow_epilogue_impl<MP, NR, false>(t, r, d, corr_stage, mc, m_rows, acc);
  }
}

// ---- wide path: one stage of one warp -----------------------------------------------------------
// The warp takes NI items (item0, item0 + 1, ...) of its 16-row tile.
template <int MT, int NI>
__device__ __forceinline__ void wide_stage(const unsigned char* st, const unsigned char* xs,
                                           const float2* corr, int xs_stride, int mc, int m_rows,
                                           int j_panel, int item0, int g, int c, int r_lo,
                                           int r_hi, float (&acc)[2][MT][2], uint64_t* empty_bar,
                                           uint32_t* scratch, int lane) {
  uint4 aw[NI][2];
  uint32_t sz[NI][2];  // scale bits | zero bits << 16 of item item0 + ii, rows r_lo and r_hi
  uint32_t folded = 0;
#pragma unroll
  for (int ii = 0; ii < NI; ++ii) {
    aw[ii][0] = stage_words(st, r_lo, item0 + ii, c);
    aw[ii][1] = stage_words(st, r_hi, item0 + ii, c);
    sz[ii][0] = stage_sz(st, r_lo, item0 + ii);
    sz[ii][1] = stage_sz(st, r_hi, item0 + ii);
    folded ^= fold4(aw[ii][0]) ^ fold4(aw[ii][1]) ^ sz[ii][0] ^ sz[ii][1];
  }
  // release only once every load above has returned (see stage_reads_done)
  stage_reads_done(folded, scratch, lane);
  __syncwarp();
  if (lane == 0) mbar_arrive(empty_bar);  // the stage may be refilled

#pragma unroll(MT == 1 ? NI : 1)
  for (int ii = 0; ii < NI; ++ii) {
    const int item_p = j_panel * kItemsPerStage + item0 + ii;  // item within the panel
    // [tile][jw % 2][a0 / a1]: consecutive MMAs never share an accumulator.
    float d[MT][2][2][4];
    // Selects rather than indexing, so a rolled loop keeps aw in registers.
    const uint4 al = ii == 0 ? aw[0][0] : aw[NI - 1][0];
    const uint4 ah = ii == 0 ? aw[0][1] : aw[NI - 1][1];
#pragma unroll
    for (int jw = 0; jw < 4; ++jw) {
      uint32_t hl[4], hh[4];
      unpack_x16(word_of(al, jw), hl);
      unpack_x16(word_of(ah, jw), hh);
      const uint32_t a0[4] = {hl[0], hh[0], hl[1], hh[1]};
      const uint32_t a1[4] = {hl[2], hh[2], hl[3], hh[3]};
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int m = g + 8 * mt;
        uint4 xb = make_uint4(0, 0, 0, 0);
        if (m < m_rows) {
          xb = *reinterpret_cast<const uint4*>(xs + m * xs_stride + item_p * 256 +
                                               (jw * 4 + c) * 16);
        }
        if (jw < 2) {
          mma_16816_first(d[mt][jw & 1][0], a0, xb.x, xb.y);
          mma_16816_first(d[mt][jw & 1][1], a1, xb.z, xb.w);
        } else {
          mma_16816(d[mt][jw & 1][0], a0, xb.x, xb.y);
          mma_16816(d[mt][jw & 1][1], a1, xb.z, xb.w);
        }
      }
    }
    const uint32_t szl = ii == 0 ? sz[0][0] : sz[NI - 1][0];
    const uint32_t szh = ii == 0 ? sz[0][1] : sz[NI - 1][1];
    const float s_lo = half_lo(szl), z_lo = half_hi(szl);
    const float s_hi = half_lo(szh), z_hi = half_hi(szh);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int m0 = 8 * mt + 2 * c;
      const float4 cr =
          *reinterpret_cast<const float4*>(corr + item_p * mc + (m0 < m_rows ? m0 : 0));
      float dd[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        dd[e] = (d[mt][0][0][e] + d[mt][0][1][e]) + (d[mt][1][0][e] + d[mt][1][1][e]);
      }
      acc[0][mt][0] = fmaf(s_lo, fmaf(-z_lo, cr.y, dd[0] - cr.x), acc[0][mt][0]);
      acc[0][mt][1] = fmaf(s_lo, fmaf(-z_lo, cr.w, dd[1] - cr.z), acc[0][mt][1]);
      acc[1][mt][0] = fmaf(s_hi, fmaf(-z_hi, cr.y, dd[2] - cr.x), acc[1][mt][0]);
      acc[1][mt][1] = fmaf(s_hi, fmaf(-z_hi, cr.w, dd[3] - cr.z), acc[1][mt][1]);
    }
  }
}

// MP: M rounded up to 2 or 4 (narrow path) or 8 (wide path, MT tiles of 8 rows of x). MC: M when
// the instance serves a single M (else 0: read at run time). CW: consumer warps, 8 or 16. With 16 (17 warps, at most 5 per SM sub-partition) a thread may use
// 96 registers, so the sub-partition's 16384 registers hold them; with 8 (3 per sub-partition),
// 168. Measured on B200: M = 1 is fastest with 8 consumer warps, 2 <= M <= 8 with 16.
template <int MP, int MT, int CW, int MC>
__global__ void __maxnreg__(CW == 16 ? 96 : 168)
    stream_mma_kernel(GemvArgs a, MmaPlan p, const __grid_constant__ WeightMaps maps,
                      const __grid_constant__ EpilogueExtra ex) {
  const PeerSet& peers = ex.peers;
  constexpr bool kNarrow = MP < 8;
  const int m_rows = MC > 0 ? MC : a.m;  // rows of x: compile-time where the instance has one M
  constexpr int kCW = CW;
  constexpr int kConsumerThreads = kCW * kWarp;
  constexpr int kThreads = kConsumerThreads + kWarp;
  constexpr int kSplit = kCW / 8;      // warps sharing one (tile, word quarter or item pair)
  constexpr int kNR = 4 / kSplit;      // narrow: rounds per warp and stage
  constexpr int kNI = 2 / kSplit;      // wide: items per warp and stage
  constexpr int kRedCols = 8;          // narrow path: accumulator columns per row
  extern __shared__ __align__(1024) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint64_t* full = bars + kBarFull;
  uint64_t* empty = bars + kBarEmpty;
  unsigned char* zero = smem + 1024;
  uint32_t* scratch = reinterpret_cast<uint32_t*>(smem + 512);  // see stage_reads_done
  const unsigned char* xr = smem + p.off_xr;
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
      mbar_init(&empty[s], kCW);
    }
    mbar_init(&bars[kBarXFull], 1);
    mbar_init(&bars[kBarXEmpty], 1);
    fence_mbar_init();
  }
  for (int i = tid; i < kZeroBytes / 16; i += kThreads) {
    reinterpret_cast<uint4*>(zero)[i] = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  if (tid == 0) launch_dependents();  // the next GEMV may launch as SMs free up

  if (warp == kCW) {
    produce(a, p, maps, row_begin, rows, smem);
    return;
  }

  // ---------------- consumers ----------------
  const int tile = warp & 1;
  const int g = lane >> 2, c = lane & 3;
  const int group = (warp >> 1) & 3;  // word quarter (narrow) or item pair (wide)
  const int hs = warp >> 3;           // which half of the group's work, when split
  const int src = hs * 4 + group;     // partial-sum source of this warp
  const int r_lo = 16 * tile + mma_row(g);
  const int r_hi = r_lo + 8;
  NarrowThread<kNarrow ? MP : 2, kNR> nt;
  if constexpr (kNarrow) nt.init(warp, lane, m_rows, p.xs_stride, static_cast<int>(zero - xs));

  StageRing in{full, p.stages, p.status, true, 0, 0u};
  for (int pi = 0, p0 = 0; p0 < p.steps; ++pi, p0 += p.panel_steps) {
    const int psteps = min(p.panel_steps, p.steps - p0);
    if (pi > 0) named_barrier(kConsumerBarrier, kConsumerThreads);  // done with the last panel
    if (in.ok && !mbar_wait_bounded(&bars[kBarXFull], pi & 1)) {
      in.ok = false;
      atomicExch(p.status, kStatusFullBarrierTimeout);
    }
    if (!kNarrow && p.xpre) {
      copy_x_slot<kConsumerThreads>(xr, a.m * p.xs_stride, psteps * kItemsPerStage * p.mc * 8,
                                    xs, corr, tid);
    } else {
      const int pk = psteps * kItemsPerStage * kItemK;
      permute_x_panel<kNarrow, kConsumerThreads>(a, p, pk, xr, pk, xs, corr, tid);
    }
    named_barrier(kConsumerBarrier, kConsumerThreads);
    if (tid == 0) mbar_arrive(&bars[kBarXEmpty]);  // the raw x buffer may be refilled

    for (int blk = 0; blk < blocks; ++blk) {
      const int rows_b = min(kBlockRows, rows - blk * kBlockRows);
      const bool active = 16 * tile < rows_b;
      if constexpr (kNarrow) {
        float acc[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
        if (!active) {
          for (int j = 0; j < psteps; ++j) {
            const int slot = in.next();
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
          }
        } else {
          // Software pipeline, two stages per iteration with alternating register sets: the MMAs
          // of stage j are issued, then stage j + 1 is waited for and loaded, then stage j's
          // epilogue runs, so the MMA latency overlaps the wait and the loads.
          using Regs = NarrowRegs<MP, kNR>;
          using Acc = float[NarrowThread<MP, kNR>::kSets][narrow_acc<MP>()][4];
          Regs ra, rb;
          int slot = in.next();
          narrow_load(nt, stages + slot * kStageBytes, ra, &empty[slot], scratch, lane);
          for (int j = 0; j < psteps; j += 2) {
            Acc d;
            narrow_mma(ra, xs + nt.b_base + j * nt.b_step, d);
            if (j + 1 < psteps) {
              slot = in.next();
              narrow_load(nt, stages + slot * kStageBytes, rb, &empty[slot], scratch, lane);
            }
            narrow_epilogue(nt, ra, d, corr + j * kItemsPerStage * p.mc, p.mc, m_rows, acc);
            if (j + 1 >= psteps) break;
            narrow_mma(rb, xs + nt.b_base + (j + 1) * nt.b_step, d);
            if (j + 2 < psteps) {
              slot = in.next();
              narrow_load(nt, stages + slot * kStageBytes, ra, &empty[slot], scratch, lane);
            }
            narrow_epilogue(nt, rb, d, corr + (j + 1) * kItemsPerStage * p.mc, p.mc, m_rows, acc);
          }
        }
        if (active) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int r = h ? r_hi : r_lo;
            if (r >= rows_b) continue;
            float* dst = red + (src * p.rows_cap + blk * kBlockRows + r) * kRedCols + 2 * c;
#pragma unroll
            for (int e = 0; e < 2; ++e) dst[e] = pi == 0 ? acc[h][e] : dst[e] + acc[h][e];
          }
        }
      } else {
        float acc[2][MT][2];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) acc[h][mt][0] = acc[h][mt][1] = 0.0f;
        for (int j = 0; j < psteps; ++j) {
          const int slot = in.next();
          if (!active) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            continue;
          }
          wide_stage<MT, kNI>(stages + slot * kStageBytes, xs, corr, p.xs_stride, p.mc, a.m, j,
                              2 * group + hs, g, c, r_lo, r_hi, acc, &empty[slot], scratch,
                              lane);
        }
        if (active) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int r = h ? r_hi : r_lo;
            if (r >= rows_b) continue;
            float* dst = red + (src * p.rows_cap + blk * kBlockRows + r) * a.m;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int m = 8 * mt + 2 * c + e;
                if (m < a.m) dst[m] = pi == 0 ? acc[h][mt][e] : dst[m] + acc[h][mt][e];
              }
            }
          }
        }
      }
    }
  }

  // ---- add the partials of every output in a fixed order; store fp16 -------------------------
  named_barrier(kConsumerBarrier, kConsumerThreads);
  auto row_sum = [&](int r, int m) {
    float sum = 0.0f;
    if constexpr (kNarrow) {
#pragma unroll
      for (int q = 0; q < 4 * kSplit; ++q)
#pragma unroll
        for (int f = 0; f < 8 / MP; ++f) sum += red[(q * p.rows_cap + r) * kRedCols + f * MP + m];
    } else {
#pragma unroll
      for (int q = 0; q < 4 * kSplit; ++q) sum += red[(q * p.rows_cap + r) * a.m + m];
    }
    return sum;
  };
  if (a.epilogue == kSiluMul) {
    // Row pairs (gate 2i, up 2i + 1) never straddle CTAs: shares are whole 4-row units.
    const int pairs = rows / 2;
    for (int o = tid; o < pairs * a.m; o += kConsumerThreads) {
      const int m = o / pairs;
      const int i = o - m * pairs;
      const float gate = row_sum(2 * i, m);
      const float up = row_sum(2 * i + 1, m);
      const float silu = gate / (1.0f + __expf(-gate));
      if (in.ok) {
        a.y[static_cast<int64_t>(m) * (a.n / 2) + row_begin / 2 + i] = __float2half_rn(silu * up);
      }
    }
  } else if (a.epilogue == kGroupedY) {
    // Stacked matrices: row r of this CTA belongs to the matrix whose row range holds it.
    const GroupOut& go = ex.groups;
    for (int o = tid; o < rows * a.m; o += kConsumerThreads) {
      const int m = o / rows;
      const int row = row_begin + o - m * rows;
      int gi = 0;
      while (gi + 1 < go.count && row >= go.row_end[gi]) ++gi;
      const int base = gi ? go.row_end[gi - 1] : 0;
      const int ng = go.row_end[gi] - base;
      const float sum = row_sum(row - row_begin, m);
      if (in.ok) go.y[gi][static_cast<int64_t>(m) * ng + row - base] = __float2half_rn(sum);
    }
  } else if (a.epilogue == kGatherPeers) {
    // This rank's columns of y, each as a tagged word (fp16 bits, call number), into every other
    // rank's gather buffer and straight into this rank's y. The rows this CTA then copies into y
    // are the same row range of every other rank's shard: the words its counterpart CTAs write;
    // each is read once its tag shows this call.
    const unsigned epoch = exchange_epoch(peers);
    named_barrier(kConsumerBarrier, kConsumerThreads);  // every thread has read the call number
    for (int o = tid; o < rows * a.m; o += kConsumerThreads) {
      const int m = o / rows;
      const int r = o - m * rows;
      const unsigned h = __half_as_ushort(__float2half_rn(row_sum(r, m)));
      const int64_t at = static_cast<int64_t>(m) * peers.n_total + peers.col0 + row_begin + r;
      for (int q = 0; q < peers.world; ++q) {
        if (q == peers.rank) {
          if (in.ok) a.y[at] = __ushort_as_half(static_cast<unsigned short>(h));
        } else {
          st_tagged(exchange_words(peers, q, epoch) + at, h, epoch);
        }
      }
    }
    const unsigned long long* buf = exchange_words(peers, peers.rank, epoch);
    bool live = true;
    for (int o = tid; o < peers.world * rows * a.m; o += kConsumerThreads) {
      const int q = o / (rows * a.m);
      if (q == peers.rank) continue;  // this rank's own rows went to y above
      const int rem = o - q * rows * a.m;
      const int m = rem / rows;
      const int r = rem - m * rows;
      const int64_t at = static_cast<int64_t>(m) * peers.n_total + q * a.n + row_begin + r;
      const unsigned h = exchange_read(buf + at, epoch, &live, p.status);
      if (in.ok) a.y[at] = __ushort_as_half(static_cast<unsigned short>(h));
    }
    exchange_done(peers, epoch, tid);
  } else if (a.epilogue == kReducePeers) {
    // This rank's fp32 partial sums, as tagged words, into slot `rank` of every other rank's
    // receive buffer; then the sum of the ranks' partials for this CTA's rows in rank order (the
    // same on every rank, so all ranks hold bit-identical y), each other rank's read once its tag
    // shows this call, this rank's own taken from the same fixed-order sum in shared memory.
    const unsigned epoch = exchange_epoch(peers);
    named_barrier(kConsumerBarrier, kConsumerThreads);  // every thread has read the call number
    const int64_t slot = static_cast<int64_t>(a.m) * a.n;
    for (int o = tid; o < rows * a.m; o += kConsumerThreads) {
      const int m = o / rows;
      const int r = o - m * rows;
      const unsigned bits = __float_as_uint(row_sum(r, m));
      const int64_t at = peers.rank * slot + static_cast<int64_t>(m) * a.n + row_begin + r;
      for (int q = 0; q < peers.world; ++q) {
        if (q != peers.rank) st_tagged(exchange_words(peers, q, epoch) + at, bits, epoch);
      }
    }
    const unsigned long long* mine = exchange_words(peers, peers.rank, epoch);
    bool live = true;
    for (int o = tid; o < rows * a.m; o += kConsumerThreads) {
      const int m = o / rows;
      const int r = o - m * rows;
      const int64_t at = static_cast<int64_t>(m) * a.n + row_begin + r;
      float total = 0.0f;
      for (int q = 0; q < peers.world; ++q) {
        total += q == peers.rank
                     ? row_sum(r, m)
                     : __uint_as_float(exchange_read(mine + q * slot + at, epoch, &live, p.status));
      }
      if (in.ok) a.y[at] = store_value(a, m, row_begin + r, total);
    }
    exchange_done(peers, epoch, tid);
  } else if (a.epilogue == kStoreF32) {
    float* yf = reinterpret_cast<float*>(a.y);
    for (int o = tid; o < rows * a.m; o += kConsumerThreads) {
      const int m = o / rows;
      const int r = o - m * rows;
      const float sum = row_sum(r, m);
      if (in.ok) yf[static_cast<int64_t>(m) * a.n + row_begin + r] = sum;
    }
  } else {
    for (int o = tid; o < rows * a.m; o += kConsumerThreads) {
      const int m = o / rows;
      const int r = o - m * rows;
      const float sum = row_sum(r, m);
      if (in.ok) {
        a.y[static_cast<int64_t>(m) * a.n + row_begin + r] = store_value(a, m, row_begin + r, sum);
      }
    }
  }
}

int pad_of(int m) { return m <= 2 ? 2 : m <= 4 ? 4 : 8; }

int consumer_warps_for(int m) { return m == 1 || m > 8 ? 8 : 16; }

// Lays out shared memory for `panel_steps` stages per panel; true if it fits with at least
// `min_stages` stages.
bool plan_smem(const GemvArgs& a, MmaPlan* p, int min_stages, bool xpre) {
  const bool narrow = pad_of(a.m) < 8;
  const int pk = p->panel_steps * kItemsPerStage * kItemK;
  const int items = pk / kItemK;
  p->xs_stride = narrow ? (items * kNarrowItemBytes + 127) / 128 * 128 + 16 : pk * 2 + 64;
  // A workspace slot: the permuted panel's xs rows, then its corr table (16-byte multiples).
  const int64_t xslot =
      static_cast<int64_t>(a.m) * p->xs_stride + static_cast<int64_t>(items) * p->mc * 8;
  p->xslot = xpre ? static_cast<int>(xslot) : 0;
  int64_t off = 1024 + kZeroBytes;  // mbarriers, zeros
  p->off_xr = static_cast<int>(off);
  off += xpre ? xslot : static_cast<int64_t>(a.m) * pk * 2;
  p->off_xs = static_cast<int>(off);
  off += static_cast<int64_t>(a.m) * p->xs_stride;
  off = (off + 15) / 16 * 16;
  p->off_corr = static_cast<int>(off);
  off += static_cast<int64_t>(items) * p->mc * 8;
  p->off_red = static_cast<int>(off);
  const int sources = 4 * (consumer_warps_for(a.m) / 8);  // partial sums per output row
  off += static_cast<int64_t>(sources) * p->rows_cap * (narrow ? 8 : a.m) * 4;
  off = (off + 1023) / 1024 * 1024;
  p->off_stage = static_cast<int>(off);
  if (off > kSmemLimit) return false;
  const int64_t stages = std::min<int64_t>((kSmemLimit - off) / kStageBytes, kMaxStages);
  if (stages < min_stages) return false;
  p->stages = static_cast<int>(stages);
  p->smem_bytes = static_cast<int>(off + stages * kStageBytes);
  p->pre_stages = std::min({kPreStages, p->panel_steps - 1, p->stages});
  return true;
}

bool make_plan(const GemvArgs& a, MmaPlan* p, const char** why, bool xpre = false) {
  auto fail = [&](const char* reason) {
    if (why) *why = reason;
    return false;
  };
  if (a.m < 1 || a.m > kMaxM) return fail("M must be in [1, 32]");
  if (!weight_stream_supported(a, why)) return false;
  if (reinterpret_cast<uintptr_t>(a.x) % 16) return fail("x must be 16-byte aligned");
  if (a.epilogue == kSiluMul && a.n % 2) return fail("gate/up rows must come in pairs (N even)");
  p->units = (a.n + 3) / 4;
  p->ctas = std::min(sm_count(), p->units);
  p->rows_cap = 4 * ((p->units + p->ctas - 1) / p->ctas);
  p->steps = a.k / (kItemK * kItemsPerStage);
  p->mc = (a.m + 1) & ~1;
  p->strict = 0;
  p->xpre = nullptr;
  xpre = xpre && pad_of(a.m) == 8;  // the wide path only
  // Fewest k-panels that leave a deep ring; then accept a shallower one.
  for (const int min_stages : {8, 4, 3}) {
    for (int panels = 1; panels <= p->steps; ++panels) {
      p->panel_steps = (p->steps + panels - 1) / panels;
      if (plan_smem(a, p, min_stages, xpre)) return true;
    }
  }
  return fail("x does not fit in shared memory");
}

// Kernel instances (MP, MT, CW) for M = 1, 2, 3..4, 5..8, 9..16, 17..24, 25..32.
template <typename F>
cudaError_t with_shape(int m, F&& f) {
  if (m <= 1) return f.template operator()<2, 1, 8, 1>();
  if (m <= 2) return f.template operator()<2, 1, 16, 2>();
  if (m <= 4) return f.template operator()<4, 1, 16, 0>();
  if (m <= 8) return f.template operator()<8, 1, 16, 0>();
  if (m <= 16) return f.template operator()<8, 2, 8, 0>();
  if (m <= 24) return f.template operator()<8, 3, 8, 0>();
  return f.template operator()<8, 4, 8, 0>();
}

int shape_index(int m) {
  return m <= 1 ? 0 : m <= 2 ? 1 : m <= 4 ? 2 : m <= 8 ? 3 : m <= 16 ? 4 : m <= 24 ? 5 : 6;
}

std::once_flag g_attr_once[7][64];

}  // namespace

bool stream_mma_supported(const GemvArgs& a, const char** why) {
  MmaPlan p;
  return make_plan(a, &p, why);
}

int64_t stream_mma_workspace_bytes(const GemvArgs& a) {
  MmaPlan p;
  if (a.epilogue != kStoreY || !make_plan(a, &p, nullptr, true) || p.xslot == 0) return 0;
  const int64_t panels = (p.steps + p.panel_steps - 1) / p.panel_steps;
  return panels * p.xslot;
}

cudaError_t launch_stream_mma(const GemvArgs& a, cudaStream_t stream, bool strict,
                              const PeerSet* peers, const GroupOut* groups, void* workspace,
                              int64_t workspace_bytes) {
  MmaPlan p;
  // With a large enough workspace the wide path takes x permuted once by the pre-kernel.
  const int64_t ws_need = workspace ? stream_mma_workspace_bytes(a) : 0;
  const bool xpre = ws_need > 0 && workspace_bytes >= ws_need;
  if (!make_plan(a, &p, nullptr, xpre)) return cudaErrorInvalidValue;
  if (xpre) p.xpre = static_cast<const unsigned char*>(workspace);
  const bool exchange = a.epilogue == kGatherPeers || a.epilogue == kReducePeers;
  if (exchange != (peers != nullptr)) return cudaErrorInvalidValue;
  if ((a.epilogue == kGroupedY) != (groups != nullptr)) return cudaErrorInvalidValue;
  EpilogueExtra ex{};
  if (peers) ex.peers = *peers;
  if (groups) ex.groups = *groups;
  p.strict = strict ? 1 : 0;
  p.status = device_status_word();
  if (!p.status) return cudaErrorInvalidSymbol;
  WeightMaps maps;
  const cudaError_t merr = weight_maps_for(a, &maps);
  if (merr != cudaSuccess) return merr;
  int dev = 0;
  const cudaError_t derr = cudaGetDevice(&dev);
  if (derr != cudaSuccess) return derr;
  if (xpre) {
    const int panels = (p.steps + p.panel_steps - 1) / p.panel_steps;
    stream_mma_xprep_kernel<<<panels, kXprepThreads, 0, stream>>>(
        a, p, static_cast<unsigned char*>(workspace));
    const cudaError_t perr = cudaGetLastError();
    if (perr != cudaSuccess) return perr;
  }
  return with_shape(a.m, [&]<int MP, int MT, int CW, int MC>() {
    cudaError_t result = cudaSuccess;
    std::call_once(g_attr_once[shape_index(a.m)][dev & 63], [&] {
      result = cudaFuncSetAttribute(stream_mma_kernel<MP, MT, CW, MC>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    });
    if (result != cudaSuccess) return result;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.ctas);
    cfg.blockDim = dim3((CW + 1) * kWarp);
    cfg.dynamicSmemBytes = p.smem_bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, stream_mma_kernel<MP, MT, CW, MC>, a, p, maps, ex);
  });
}

// Occupancy is reported for the shared memory the kernel uses at N = K = 8192.
cudaError_t stream_mma_attrs(int m, KernelAttrs* out) {
  const int mm = m < 1 ? 1 : m > kMaxM ? kMaxM : m;
  return with_shape(mm, [&]<int MP, int MT, int CW, int MC>() {
    cudaFuncAttributes fa;
    cudaError_t err = cudaFuncGetAttributes(&fa, stream_mma_kernel<MP, MT, CW, MC>);
    if (err != cudaSuccess) return err;
    err = cudaFuncSetAttribute(stream_mma_kernel<MP, MT, CW, MC>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (err != cudaSuccess) return err;
    GemvArgs a{};
    a.m = mm;
    a.n = a.k = 8192;
    a.group = kItemK;
    MmaPlan p;
    int blocks = 0;
    if (make_plan(a, &p, nullptr)) {
      err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
          &blocks, stream_mma_kernel<MP, MT, CW, MC>, (CW + 1) * kWarp, p.smem_bytes);
      if (err != cudaSuccess) return err;
    }
    out->registers = fa.numRegs;
    out->local_bytes = static_cast<int>(fa.localSizeBytes);
    out->max_threads_per_block = fa.maxThreadsPerBlock;
    out->blocks_per_sm = blocks;
    out->threads_per_block = (CW + 1) * kWarp;
    return cudaSuccess;
  });
}

}  // namespace i4
