// tcgen05 W4A16 GEMV for 1 <= M <= 64 (dispatched for 9 <= M <= 64): the weights dequantized into
// tensor memory, one fp32 accumulator per 128-row tile held in TMEM across the whole of a CTA's
// share of K.
//
// Why tcgen05 here. One kind::f16 MMA (M = 128, K = 16) covers 2048 weights whatever N is, up to
// N = 64 rows of x, while the warp MMA (m16n8k16) count grows with every 8 rows of x. Measured on
// B200 inside this pipeline an MMA costs about 100-120 cycles (its B operand moves every
// instruction, the stage commits, and the dequant warps' TMEM stores share the tensor memory with
// the MMA's A reads; alone, with a fixed B, it is 47 cycles), so the warp MMA stays ahead up to
// M = 8 and this kernel is ahead from M = 10 on.
//
// Tiles and work split. The weight rows are cut into tiles of 128 (the 128 TMEM lanes) and K into
// stages of 256 weights (two quantisation groups). The (tile, stage) units, tile-major, are split
// into one contiguous range per CTA (grid = SMs), so every CTA streams the same number of weight
// bytes to within one stage. A CTA's range covers the end of one tile, any whole tiles, and the
// start of another; a tile that several CTAs share is finished by the last of them to arrive,
// which adds all the partial sums in CTA order (deterministic) and stores y.
//
// Roles (18 warps, one CTA per SM):
//   producer (1 warp)  2-D TMA tiles of each stage into a ring in shared memory: 128 rows x 128
//                      packed bytes (128-byte swizzle) plus the scales and zeros of the stage's
//                      8-group window (128 rows x 8 fp16 each, the TMA's smallest aligned box).
//   dequant (8 warps)  warp w owns TMEM lanes 32 (w % 4) .. + 31 (one weight row per thread) and
//                      group w / 4 of the stage: 16 packed words -> 128 fp16 weights
//                          (1024 + q) - 1024 = q exactly, then w = q s + (-z s) (one fma)
//                      with the magic-number unpack (x16 for odd nibble pairs, matched by x / 16
//                      in B), stored to the stage's A buffer in TMEM (tcgen05.st).
//   x (4 warps)        copy the stage's slice of x (M rows x 256) into shared memory with
//                      cp.async several stages ahead (the load path: x does not queue behind the
//                      weight tiles in the TMA engine), then permute it into a B buffer, per
//                      8-weight block [x0, x4, x1/16, x5/16, x2, x6, x3/16, x7/16] to match the A
//                      halves, in the canonical no-swizzle K-major layout; rows M .. NX-1 stay 0.
//   MMA (1 thread)     16 tcgen05.mma (M = 128, N = NX, K = 16) per stage into the tile's
//                      accumulator (two TMEM buffers, so one tile's epilogue overlaps the next
//                      tile's MMAs); one tcgen05.commit per stage frees its A and B buffers.
//   epilogue (4 warps) reads each finished accumulator (tcgen05.ld), stores y or the partial sums,
//                      and finishes shared tiles.
//
// Numerics: each weight is (q - z) s in fp16 (q exact, z s rounded once, the fma rounded once),
// products with x exact in the tensor core, fp32 accumulation. Within the 1e-2 relative tolerance
// of the reference's fp32 oracle, not bit-exact.
//
// Launch overlap: programmatic stream serialization like the other fast kernels. The producer
// reads weights, scales and zeros before griddepcontrol.wait unless strict; x is read, and y, the
// partial sums and the tile counters are touched, only after it. Every mbarrier wait is bounded;
// after a timeout the kernel records a status word, stops waiting, still takes part in the tile
// counting (so the counters stay consistent for later calls) and stores no y.
#include <algorithm>
#include <mutex>
#include <vector>

#include "tcgen05.cuh"
#include "weight_stream.cuh"

namespace i4 {

// Split-K partial sums (two slots per CTA: its first and its last tile) and per-tile arrival
// counts. Static, so no call allocates; the counters start at zero when the module loads and the
// CTA that finishes a tile sets its counter back to zero.
constexpr int kTdMaxCtas = 160;
constexpr int kTdMaxM = 64;
constexpr int kTdMaxTiles = 4096;
__device__ __align__(256) float g_td_partials[kTdMaxCtas * 2 * kTdMaxM * 128];
__device__ unsigned g_td_arrivals[kTdMaxTiles];

namespace {

constexpr int kTdTileRows = 128;
constexpr int kTdStageK = 256;                      // weights per row per stage (2 groups)
constexpr int kTdQBytes = kTdTileRows * 128;        // packed words of a stage
constexpr int kTdSzBytes = kTdTileRows * 8 * 2;     // scales (or zeros) of an 8-group window
constexpr int kTdStageBytes = kTdQBytes + 2 * kTdSzBytes;  // 20480
constexpr int kTdBRowBytes = kTdStageK * 2;         // one row of x per stage, fp16
constexpr int kTdXRowBytes = kTdBRowBytes + 16;     // raw x row in shared memory, padded
constexpr int kTdDqWarps = 8;
constexpr int kTdProducerWarp = 8;
constexpr int kTdMmaWarp = 9;
constexpr int kTdXWarp0 = 10;
constexpr int kTdXWarps = 4;
constexpr int kTdEpiWarp0 = 14;
constexpr int kTdEpiWarps = 4;
constexpr int kTdThreads = (kTdEpiWarp0 + kTdEpiWarps) * kWarp;  // 576
constexpr int kTdAStages = 3;                       // A buffers in TMEM, 128 columns each
constexpr int kTdDCol = kTdAStages * 128;           // first accumulator column (2 x NX follow)
constexpr int kTdTmemCols = 512;
constexpr int kTdMaxQStages = 6;                    // weight stages in flight per CTA
constexpr int kTdMaxBStages = 3;
constexpr int kTdMaxXStages = 6;                    // cp.async groups in flight per x thread
constexpr int kTdSmemLimit = 227 * 1024;
constexpr int kTdXBarrier = 2;
constexpr int kTdEpiBarrier = 3;
constexpr int kStatusTdTimeout = 6;

// mbarriers (8 bytes each) at the start of shared memory
constexpr int kBarQFull = 0;                           // [6] stage landed (1 arrival + bytes)
constexpr int kBarQEmpty = kBarQFull + kTdMaxQStages;  // [6] stage read (8 dequant warps)
constexpr int kBarBFull = kBarQEmpty + kTdMaxQStages;  // [3] B written (128 x threads)
constexpr int kBarAFull = kBarBFull + kTdMaxBStages;   // [3] A written (256 dequant threads)
constexpr int kBarUnit = kBarAFull + kTdAStages;       // [3] unit's MMAs done: A and B free
constexpr int kBarDFull = kBarUnit + kTdAStages;       // [2] accumulator complete (commit)
constexpr int kBarDEmpty = kBarDFull + 2;              // [2] accumulator read (128 threads)
constexpr int kBarDone = kBarDEmpty + 2;               // every MMA complete (commit)
constexpr int kTdTmemSlot = 8 * (kBarDone + 1);
constexpr int kTdFlagOff = kTdTmemSlot + 16;
constexpr int kTdScratchOff = 512;                     // 32 words, see stage_reads_done
constexpr int kTdHeader = 1024;
static_assert(kTdFlagOff + 16 <= kTdScratchOff, "shared-memory header");

struct TdMaps {
  CUtensorMap q;  // qweight as uint8 [N][K / 2], box 128 x 128 rows, 128-byte swizzle
  CUtensorMap s;  // scales as uint16 [N][K / 128], box 8 x 128 rows
  CUtensorMap z;  // zeros, same
};

struct TdPlan {
  int ctas;
  int tiles;     // ceil(N / 128)
  int spt;       // stages per tile: K / 256
  int units;     // tiles * spt
  int qstages, bstages, xstages;
  int xslot;     // bytes of one raw x stage: M rows of kTdXRowBytes, rounded up to 128
  int off_x, off_b, off_q, smem_bytes;
  int strict;    // 1: read the weights only after griddepcontrol.wait
  int* status;
  float* partials;
  unsigned* arrivals;
};

__device__ __forceinline__ uint32_t f16x2_add(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t f16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// One packed word -> four A registers in unpack_x16's order, dequantized: (q - z) s for the
// (1024 + q) halves, 16 (q - z) s for the (1024 + 16 q) halves.
__device__ __forceinline__ void dequant_word(uint32_t w, uint32_t s2, uint32_t c1, uint32_t c16,
                                             uint32_t* out) {
  uint32_t h[4];
  unpack_x16(w, h);
  constexpr uint32_t kMinus1024 = 0xE400E400u;
  out[0] = f16x2_fma(f16x2_add(h[0], kMinus1024), s2, c1);
  out[1] = f16x2_fma(f16x2_add(h[1], kMinus1024), s2, c16);
  out[2] = f16x2_fma(f16x2_add(h[2], kMinus1024), s2, c1);
  out[3] = f16x2_fma(f16x2_add(h[3], kMinus1024), s2, c16);
}

__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y,
                                       uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tma_2d_hint(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// 16-byte asynchronous copy global -> shared on the load path (cp.async, cached in L2 only).
__device__ __forceinline__ void cp_async_16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// Waits until at most n of this thread's cp.async groups are pending (n = 0..7).
__device__ __forceinline__ void cp_async_wait_pending(int n) {
  switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
    case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
    case 6: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 7;" ::: "memory"); break;
  }
}

// First unit of CTA c.
__device__ __forceinline__ int unit_begin(const TdPlan& p, int c) {
  return static_cast<int>(static_cast<int64_t>(c) * p.units / p.ctas);
}
// The CTA whose range holds unit u.
__device__ __forceinline__ int cta_of_unit(const TdPlan& p, int u) {
  return static_cast<int>((static_cast<int64_t>(u + 1) * p.ctas + p.units - 1) / p.units) - 1;
}

__device__ __forceinline__ bool td_wait(uint64_t* bar, uint32_t parity, bool& ok, int* status) {
  if (!ok) return false;
  if (!mbar_wait_bounded(bar, parity)) {
    ok = false;
    atomicExch(status, kStatusTdTimeout);
    return false;
  }
  return true;
}

__device__ __forceinline__ void td_store(const GemvArgs& a, int m, int row, float v) {
  if (a.epilogue == kStoreF32) {
    reinterpret_cast<float*>(a.y)[static_cast<int64_t>(m) * a.n + row] = v;
  } else {
    a.y[static_cast<int64_t>(m) * a.n + row] = store_value(a, m, row, v);
  }
}

template <int NX>
__global__ void __launch_bounds__(kTdThreads, 1)
    tc_dequant_kernel(GemvArgs a, TdPlan p, const __grid_constant__ TdMaps maps) {
  extern __shared__ __align__(1024) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kTdTmemSlot);
  volatile int* last_flag = reinterpret_cast<volatile int*>(smem + kTdFlagOff);
  uint32_t* scratch = reinterpret_cast<uint32_t*>(smem + kTdScratchOff);
  unsigned char* xsm = smem + p.off_x;
  unsigned char* bsm = smem + p.off_b;
  unsigned char* qsm = smem + p.off_q;
  constexpr int kNb = NX / 8;  // core-matrix columns of B
  constexpr int kBStageBytes = NX * kTdBRowBytes;

  const int tid = threadIdx.x;
  const int warp = tid / kWarp;
  const int lane = tid % kWarp;
  const int u0 = unit_begin(p, blockIdx.x);
  const int u1 = unit_begin(p, blockIdx.x + 1);
  const int t_first = u0 / p.spt;
  const int t_last = (u1 - 1) / p.spt;

  if (tid == 0) {
    for (int s = 0; s < p.qstages; ++s) {
      mbar_init(&bars[kBarQFull + s], 1);
      mbar_init(&bars[kBarQEmpty + s], kTdDqWarps);
    }
    for (int s = 0; s < p.bstages; ++s) mbar_init(&bars[kBarBFull + s], kTdXWarps * kWarp);
    for (int s = 0; s < kTdAStages; ++s) {
      mbar_init(&bars[kBarAFull + s], kTdDqWarps * kWarp);
      mbar_init(&bars[kBarUnit + s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[kBarDFull + s], 1);
      mbar_init(&bars[kBarDEmpty + s], kTdEpiWarps * kWarp);
    }
    mbar_init(&bars[kBarDone], 1);
    fence_mbar_init();
  }
  if (warp == kTdMmaWarp) tmem_alloc(tmem_slot, kTdTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) launch_dependents();

  bool ok = true;
  if (warp < kTdDqWarps) {
    // ---------------- dequant warps ----------------
    const int quarter = warp & 3;
    const int grp = warp >> 2;  // group of the stage
    const int rl = 32 * quarter + lane;
    const uint32_t lane_field = static_cast<uint32_t>(32 * quarter) << 16;
    int qs = 0, as = 0;
    uint32_t qph = 0, aph = 0;
    int i = 0;
    for (int u = u0; u < u1; ++u, ++i) {
      td_wait(&bars[kBarQFull + qs], qph, ok, p.status);
      const unsigned char* st = qsm + qs * kTdStageBytes;
      uint32_t w[16];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 v = *reinterpret_cast<const uint4*>(st + rl * 128 +
                                                        ((((grp << 2) | c) ^ (rl & 7)) << 4));
        w[4 * c + 0] = v.x;
        w[4 * c + 1] = v.y;
        w[4 * c + 2] = v.z;
        w[4 * c + 3] = v.w;
      }
      const int g8 = (2 * (u % p.spt) + grp) & 7;
      const uint32_t sb = *reinterpret_cast<const uint16_t*>(st + kTdQBytes + rl * 16 + g8 * 2);
      const uint32_t zb =
          *reinterpret_cast<const uint16_t*>(st + kTdQBytes + kTdSzBytes + rl * 16 + g8 * 2);
      {
        // release only once every load above has returned (see stage_reads_done)
        uint32_t folded = sb ^ (zb << 16);
#pragma unroll
        for (int j = 0; j < 16; ++j) folded ^= w[j];
        stage_reads_done(folded, scratch, lane);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kBarQEmpty + qs]);
      if (++qs == p.qstages) {
        qs = 0;
        qph ^= 1u;
      }

      const float sf = __half2float(__ushort_as_half(static_cast<uint16_t>(sb)));
      const float zf = __half2float(__ushort_as_half(static_cast<uint16_t>(zb)));
      const __half nzs = __float2half_rn(-zf * sf);
      const uint32_t c1 = static_cast<uint32_t>(__half_as_ushort(nzs)) * 0x10001u;
      const uint32_t c16 =
          static_cast<uint32_t>(__half_as_ushort(__hmul(nzs, __ushort_as_half(0x4C00)))) *
          0x10001u;  // 16 * (-z s), exact
      const uint32_t s2 = sb * 0x10001u;

      // A buffer `as` was last read by the MMAs of unit i - 3 (phase (i - 3) / 3 of its barrier).
      if (i >= kTdAStages) td_wait(&bars[kBarUnit + as], aph ^ 1u, ok, p.status);
      tc_fence_after();
      const uint32_t a_addr = tmem + lane_field + as * 128 + grp * 64;
#pragma unroll
      for (int c4 = 0; c4 < 4; ++c4) {
        uint32_t v[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) dequant_word(w[4 * c4 + j], s2, c1, c16, &v[4 * j]);
        tmem_st16(a_addr + 16 * c4, v);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars[kBarAFull + as]);
      if (++as == kTdAStages) {
        as = 0;
        aph ^= 1u;
      }
    }
  } else if (warp == kTdProducerWarp) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t policy = l2_evict_first_policy();
      if (p.strict) grid_dependency_wait();
      int qs = 0;
      uint32_t qph = 0;
      int i = 0;
      for (int u = u0; u < u1; ++u, ++i) {
        if (i >= p.qstages && !td_wait(&bars[kBarQEmpty + qs], qph ^ 1u, ok, p.status)) break;
        const int t = u / p.spt;
        const int j = u % p.spt;
        unsigned char* st = qsm + qs * kTdStageBytes;
        uint64_t* full = &bars[kBarQFull + qs];
        mbar_arrive_expect_tx(full, kTdStageBytes);
        tma_2d_hint(st, &maps.q, j * 128, t * kTdTileRows, full, policy);
        tma_2d(st + kTdQBytes, &maps.s, (j >> 2) * 8, t * kTdTileRows, full);
        tma_2d(st + kTdQBytes + kTdSzBytes, &maps.z, (j >> 2) * 8, t * kTdTileRows, full);
        if (++qs == p.qstages) {
          qs = 0;
          qph ^= 1u;
        }
      }
      // Do not leave while copies into this CTA's shared memory may be in flight.
      if (ok) {
        for (int back = 1; back <= min(i, p.qstages); ++back) {
          const int k = i - back;
          if (!mbar_wait_bounded(&bars[kBarQFull + k % p.qstages], (k / p.qstages) & 1)) break;
        }
      }
    }
    __syncwarp();
  } else if (warp == kTdMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t kIdesc = idesc_f16_f32(kTdTileRows, NX);
      const uint32_t b_base = smem_addr(bsm);
      int as = 0, bs = 0;
      uint32_t aph = 0, bph = 0;
      bool issued = false;
      for (int t = t_first; t <= t_last && ok; ++t) {
        const int r = t - t_first;
        const int ub = max(u0, t * p.spt);
        const int ue = min(u1, (t + 1) * p.spt);
        const uint32_t d_addr = tmem + kTdDCol + (r & 1) * NX;
        if (r >= 2 && !td_wait(&bars[kBarDEmpty + (r & 1)], ((r - 2) >> 1) & 1, ok, p.status))
          break;
        for (int u = ub; u < ue; ++u) {
          if (!td_wait(&bars[kBarAFull + as], aph, ok, p.status)) break;
          if (!td_wait(&bars[kBarBFull + bs], bph, ok, p.status)) break;
          tc_fence_after();
          const uint32_t a_addr = tmem + as * 128;
          const uint32_t b_addr = b_base + bs * kBStageBytes;
#pragma unroll
          for (int kk = 0; kk < kTdStageK / 16; ++kk) {
            const uint64_t bdesc = smem_desc(b_addr + 2 * kk * kNb * 128, kNb * 128, 128);
            mma_f16(d_addr, a_addr + 8 * kk, bdesc, kIdesc, u != ub || kk != 0);
          }
          mma_commit(&bars[kBarUnit + as]);  // one commit frees the unit's A and B buffers
          issued = true;
          if (++as == kTdAStages) {
            as = 0;
            aph ^= 1u;
          }
          if (++bs == p.bstages) {
            bs = 0;
            bph ^= 1u;
          }
        }
        if (ok) mma_commit(&bars[kBarDFull + (r & 1)]);
      }
      if (issued) {
        mma_commit(&bars[kBarDone]);
        mbar_wait_bounded(&bars[kBarDone], 0);
      }
    }
    __syncwarp();
  } else if (warp < kTdEpiWarp0) {
    // ---------------- x warps ----------------
    // Each thread copies its own 16-byte blocks of x xstages units ahead and later permutes
    // exactly those blocks into the B buffer, so no thread reads another's copies. Block (m, kc)
    // of a raw stage is at m * kTdXRowBytes + 16 kc (rows padded by 16 bytes, so eight rows of one
    // k-chunk hit eight different banks); lane = (m % 8) + 8 (kc % 4), so one warp store fills
    // four whole 128-byte rows of B.
    const int xt = tid - kTdXWarp0 * kWarp;
    const int xw = xt / kWarp;
    grid_dependency_wait();  // x may be the previous kernel's output
    const int n_units = u1 - u0;
    const int tasks = ((a.m + 7) >> 3) * 8;
    const int lm = lane & 7;
    const int lk = lane >> 3;
    auto copy_x = [&](int i) {  // this thread's blocks of unit u0 + i into raw slot i % xstages
      if (i < n_units) {
        unsigned char* dst = xsm + (i % p.xstages) * p.xslot;
        const half* src = a.x + ((u0 + i) % p.spt) * kTdStageK;
        for (int t0 = xw; t0 < tasks; t0 += kTdXWarps) {
          const int m = (t0 >> 3) * 8 + lm;
          const int kc = (t0 & 7) * 4 + lk;
          if (m < a.m) {
            cp_async_16(dst + m * kTdXRowBytes + kc * 16,
                        src + static_cast<int64_t>(m) * a.k + 8 * kc);
          }
        }
      }
      cp_async_commit();  // one group per unit, empty or not, so the counts stay uniform
    };
    for (int i = 0; i < p.xstages; ++i) copy_x(i);
    for (int o = xt * 16; o < p.bstages * kBStageBytes; o += kTdXWarps * kWarp * 16) {
      *reinterpret_cast<uint4*>(bsm + o) = make_uint4(0, 0, 0, 0);
    }
    named_barrier(kTdXBarrier, kTdXWarps * kWarp);
    int bs = 0;
    for (int i = 0; i < n_units; ++i) {
      cp_async_wait_pending(p.xstages - 1);  // this thread's blocks of unit i have landed
      if (i >= p.bstages) {
        // B buffer bs was last read by the MMAs of unit j = i - bstages, whose commit completes
        // phase j / 3 of unit barrier j % 3. That barrier is never two phases ahead of this wait
        // (its next phase needs B of a later unit) and unit j - 3 was waited for earlier.
        const int j = i - p.bstages;
        td_wait(&bars[kBarUnit + j % kTdAStages], (j / kTdAStages) & 1, ok, p.status);
      }
      const unsigned char* raw = xsm + (i % p.xstages) * p.xslot;
      unsigned char* bst = bsm + bs * kBStageBytes;
      for (int t0 = xw; t0 < tasks; t0 += kTdXWarps) {
        const int m = (t0 >> 3) * 8 + lm;
        const int kc = (t0 & 7) * 4 + lk;
        if (m < a.m) {
          const uint4 v = *reinterpret_cast<const uint4*>(raw + m * kTdXRowBytes + kc * 16);
          *reinterpret_cast<uint4*>(bst + (kc * kNb + (m >> 3)) * 128 + (m & 7) * 16) =
              permute_x8(v);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // B visible to the MMAs
      mbar_arrive(&bars[kBarBFull + bs]);
      copy_x(i + p.xstages);  // the slot's blocks were consumed by the stores above
      if (++bs == p.bstages) bs = 0;
    }
    cp_async_wait_pending(0);  // nothing in flight into shared memory at exit
  } else {
    // ---------------- epilogue warps ----------------
    const int quarter = warp & 3;
    const int et = tid - kTdEpiWarp0 * kWarp;
    const int rl = 32 * quarter + lane;
    const uint32_t lane_field = static_cast<uint32_t>(32 * quarter) << 16;
    grid_dependency_wait();  // y, the partial sums and the counters of the previous call
    for (int t = t_first; t <= t_last; ++t) {
      const int r = t - t_first;
      const int db = r & 1;
      const bool have = td_wait(&bars[kBarDFull + db], (r >> 1) & 1, ok, p.status);
      tc_fence_after();
      const int row = t * kTdTileRows + rl;
      const bool valid = row < a.n;
      const int c_lo = cta_of_unit(p, t * p.spt);
      const int c_hi = cta_of_unit(p, min((t + 1) * p.spt, p.units) - 1);
      const int slot = t == t_first ? 0 : 1;
      float* mine = p.partials + (static_cast<int64_t>(blockIdx.x) * 2 + slot) * a.m * 128;
#pragma unroll
      for (int c16 = 0; c16 < NX / 16; ++c16) {
        if (c16 * 16 < a.m) {
          uint32_t d[16];
          tmem_ld16(tmem + lane_field + kTdDCol + db * NX + 16 * c16, d);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int m = c16 * 16 + e;
            if (m < a.m) {
              const float v = __uint_as_float(d[e]);
              if (c_lo == c_hi) {
                if (valid && have) td_store(a, m, row, v);
              } else {
                mine[m * 128 + rl] = v;
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&bars[kBarDEmpty + db]);
      if (c_lo != c_hi) {
        __threadfence();
        named_barrier(kTdEpiBarrier, kTdEpiWarps * kWarp);
        if (et == 0) {
          const unsigned before = atomicAdd(&p.arrivals[t], 1u);
          const int last = before == static_cast<unsigned>(c_hi - c_lo);
          if (last) atomicExch(&p.arrivals[t], 0u);
          *last_flag = last;
        }
        named_barrier(kTdEpiBarrier, kTdEpiWarps * kWarp);
        if (*last_flag) {
          __threadfence();
          const bool store = valid && *reinterpret_cast<volatile int*>(p.status) == 0;
          // c_lo's range may start in an earlier tile (then this is its last tile, slot 1); every
          // later contributor starts in this tile (slot 0).
          const int lo_slot = unit_begin(p, c_lo) / p.spt == t ? 0 : 1;
          // Eight outputs at a time, the partials of up to four contributors loaded together
          // (one round trip to L2 instead of one per contributor), then added in CTA order.
          for (int m0 = 0; m0 < a.m; m0 += 8) {
            float sum[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) sum[e] = 0.0f;
            for (int c0 = c_lo; c0 <= c_hi; c0 += 4) {
              float v[4][8];
#pragma unroll
              for (int ci = 0; ci < 4; ++ci) {
                const int c = c0 + ci;
                const int cs = c == c_lo ? lo_slot : 0;
                const float* src =
                    p.partials + ((static_cast<int64_t>(c) * 2 + cs) * a.m + m0) * 128 + rl;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  v[ci][e] = c <= c_hi && m0 + e < a.m ? __ldcg(src + e * 128) : 0.0f;
                }
              }
#pragma unroll
              for (int ci = 0; ci < 4; ++ci) {
                if (c0 + ci <= c_hi) {
#pragma unroll
                  for (int e = 0; e < 8; ++e) sum[e] += v[ci][e];
                }
              }
            }
            if (store) {
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                if (m0 + e < a.m) td_store(a, m0 + e, row, sum[e]);
              }
            }
          }
        }
        named_barrier(kTdEpiBarrier, kTdEpiWarps * kWarp);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kTdMmaWarp) tmem_dealloc(tmem, kTdTmemCols);
}

int td_nx(int m) { return (m + 15) / 16 * 16; }

bool td_plan(const GemvArgs& a, TdPlan* p, const char** why) {
  auto fail = [&](const char* reason) {
    if (why) *why = reason;
    return false;
  };
  if (a.m < 1 || a.m > kTdMaxM) return fail("M must be in [1, 64]");
  if (a.group != kItemK) return fail("group_size must be 128");
  if (a.k < 1024 || a.k % 1024 != 0) return fail("K must be a positive multiple of 1024");
  if (a.epilogue != kStoreY && a.epilogue != kStoreF32)
    return fail("only plain stores (fp16 y or fp32 row sums)");
  if (reinterpret_cast<uintptr_t>(a.q) % 16 || reinterpret_cast<uintptr_t>(a.x) % 16 ||
      reinterpret_cast<uintptr_t>(a.s) % 16 || reinterpret_cast<uintptr_t>(a.z) % 16)
    return fail("x, qweight, scales and zeros must be 16-byte aligned");
  const int64_t tiles = (static_cast<int64_t>(a.n) + kTdTileRows - 1) / kTdTileRows;
  if (tiles > kTdMaxTiles) return fail("N must be at most 524288");
  p->tiles = static_cast<int>(tiles);
  p->spt = a.k / kTdStageK;
  const int64_t units = tiles * p->spt;
  if (units > (1LL << 30)) return fail("too many stages");
  p->units = static_cast<int>(units);
  p->ctas = std::min({sm_count(), p->units, kTdMaxCtas});
  if (p->ctas < 1) return fail("no SMs");
  const int nx = td_nx(a.m);
  // Deepest rings that leave at least four weight stages: raw x, then B, give way first.
  p->xslot = (a.m * kTdXRowBytes + 127) / 128 * 128;
  for (int xst = kTdMaxXStages, bst = kTdMaxBStages;;) {
    p->xstages = xst;
    p->bstages = bst;
    p->off_x = kTdHeader;
    p->off_b = p->off_x + xst * p->xslot;
    const int64_t b_end = p->off_b + static_cast<int64_t>(bst) * nx * kTdBRowBytes;
    p->off_q = static_cast<int>((b_end + 1023) / 1024 * 1024);
    const int64_t qstages =
        std::min<int64_t>((kTdSmemLimit - p->off_q) / kTdStageBytes, kTdMaxQStages);
    if (qstages >= 4 || (xst == 2 && bst == 2)) {
      if (qstages < 2) return fail("shared memory");
      p->qstages = static_cast<int>(qstages);
      break;
    }
    if (xst > 2) {
      --xst;
    } else {
      --bst;
    }
  }
  p->smem_bytes = static_cast<int>(p->off_q + static_cast<int64_t>(p->qstages) * kTdStageBytes);
  p->strict = 0;
  p->status = nullptr;
  p->partials = nullptr;
  p->arrivals = nullptr;
  return true;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 td_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      f = nullptr;
    }
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}

struct TdMapEntry {
  int dev;
  const void* q;
  const void* s;
  const void* z;
  int n, k;
  TdMaps maps;
};
std::mutex g_td_mu;
std::vector<TdMapEntry> g_td_maps;  // most recently used first
constexpr size_t kTdMapCache = 64;

cudaError_t td_maps_for(const GemvArgs& a, TdMaps* out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  std::lock_guard<std::mutex> lock(g_td_mu);
  for (size_t i = 0; i < g_td_maps.size(); ++i) {
    const TdMapEntry& e = g_td_maps[i];
    if (e.dev == dev && e.q == a.q && e.s == a.s && e.z == a.z && e.n == a.n && e.k == a.k) {
      *out = e.maps;
      if (i != 0) std::swap(g_td_maps[i], g_td_maps[0]);
      return cudaSuccess;
    }
  }
  auto encode = td_encode_fn();
  if (!encode) return cudaErrorNotSupported;
  TdMapEntry e{dev, a.q, a.s, a.z, a.n, a.k, {}};
  const cuuint32_t estr[2] = {1, 1};
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(a.k / 2), static_cast<cuuint64_t>(a.n)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.k / 2)};
  const cuuint32_t box[2] = {128, kTdTileRows};
  if (encode(&e.maps.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint32_t*>(a.q), dims,
             strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
    return cudaErrorInvalidValue;
  }
  const int groups = a.k / a.group;
  const cuuint64_t sdims[2] = {static_cast<cuuint64_t>(groups), static_cast<cuuint64_t>(a.n)};
  const cuuint64_t sstrides[1] = {static_cast<cuuint64_t>(groups) * 2};
  const cuuint32_t sbox[2] = {8, kTdTileRows};
  for (int which = 0; which < 2; ++which) {
    if (encode(which == 0 ? &e.maps.s : &e.maps.z, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2,
               const_cast<half*>(which == 0 ? a.s : a.z), sdims, sstrides, sbox, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      return cudaErrorInvalidValue;
    }
  }
  g_td_maps.insert(g_td_maps.begin(), e);
  if (g_td_maps.size() > kTdMapCache) g_td_maps.pop_back();
  *out = e.maps;
  return cudaSuccess;
}

// The static partial sums and counters of the current device (looked up once per device).
cudaError_t td_scratch(float** partials, unsigned** arrivals) {
  static std::mutex mu;
  static void* part[64] = {};
  static void* arr[64] = {};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!part[dev]) {
    void* pp = nullptr;
    void* ap = nullptr;
    err = cudaGetSymbolAddress(&pp, g_td_partials);
    if (err != cudaSuccess) return err;
    err = cudaGetSymbolAddress(&ap, g_td_arrivals);
    if (err != cudaSuccess) return err;
    part[dev] = pp;
    arr[dev] = ap;
  }
  *partials = static_cast<float*>(part[dev]);
  *arrivals = static_cast<unsigned*>(arr[dev]);
  return cudaSuccess;
}

// Calls of this kernel share the device's partial sums and counters, so two of them must not run
// at the same time. Calls in one stream are ordered (each touches them only after its dependency
// wait); before a call in another stream than the last one, that stream waits for an event
// recorded after the last call. Streams being captured into a graph are left alone.
struct TdOrder {
  std::mutex mu;
  bool has[64] = {};
  cudaStream_t last[64] = {};
  cudaEvent_t done[64] = {};
};
TdOrder g_td_order;

bool stream_capturing(cudaStream_t stream) {
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &st) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return st != cudaStreamCaptureStatusNone;
}

template <typename F>
cudaError_t with_td_nx(int m, F&& f) {
  switch (td_nx(m)) {
    case 16:
      return f.template operator()<16>();
    case 32:
      return f.template operator()<32>();
    case 48:
      return f.template operator()<48>();
    default:
      return f.template operator()<64>();
  }
}

std::once_flag g_td_attr_once[4][64];

}  // namespace

bool tc_dequant_supported(const GemvArgs& a, const char** why) {
  TdPlan p;
  return td_plan(a, &p, why);
}

cudaError_t launch_tc_dequant(const GemvArgs& a, cudaStream_t stream, bool strict) {
  TdPlan p;
  if (!td_plan(a, &p, nullptr)) return cudaErrorInvalidValue;
  p.strict = strict ? 1 : 0;
  p.status = device_status_word();
  if (!p.status) return cudaErrorInvalidSymbol;
  cudaError_t err = td_scratch(&p.partials, &p.arrivals);
  if (err != cudaSuccess) return err;
  TdMaps maps;
  err = td_maps_for(a, &maps);
  if (err != cudaSuccess) return err;
  int dev = 0;
  err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  const bool capturing = stream_capturing(stream);
  std::lock_guard<std::mutex> lock(g_td_order.mu);
  if (!capturing) {
    if (!g_td_order.done[dev]) {
      err = cudaEventCreateWithFlags(&g_td_order.done[dev], cudaEventDisableTiming);
      if (err != cudaSuccess) return err;
    }
    if (g_td_order.has[dev] && g_td_order.last[dev] != stream) {
      err = cudaStreamWaitEvent(stream, g_td_order.done[dev], 0);
      if (err != cudaSuccess) return err;
    }
  }
  err = with_td_nx(a.m, [&]<int NX>() {
    cudaError_t result = cudaSuccess;
    std::call_once(g_td_attr_once[NX / 16 - 1][dev & 63], [&] {
      result = cudaFuncSetAttribute(tc_dequant_kernel<NX>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kTdSmemLimit);
    });
    if (result != cudaSuccess) return result;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.ctas);
    cfg.blockDim = dim3(kTdThreads);
    cfg.dynamicSmemBytes = p.smem_bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, tc_dequant_kernel<NX>, a, p, maps);
  });
  if (err != cudaSuccess || capturing) return err;
  err = cudaEventRecord(g_td_order.done[dev], stream);
  if (err != cudaSuccess) return err;
  g_td_order.has[dev] = true;
  g_td_order.last[dev] = stream;
  return cudaSuccess;
}

cudaError_t tc_dequant_attrs(int m, KernelAttrs* out) {
  const int mm = m < 1 ? 1 : m > kTdMaxM ? kTdMaxM : m;
  return with_td_nx(mm, [&]<int NX>() {
    cudaFuncAttributes fa;
    cudaError_t err = cudaFuncGetAttributes(&fa, tc_dequant_kernel<NX>);
    if (err != cudaSuccess) return err;
    out->registers = fa.numRegs;
    out->local_bytes = static_cast<int>(fa.localSizeBytes);
    out->max_threads_per_block = fa.maxThreadsPerBlock;
    out->blocks_per_sm = 1;
    out->threads_per_block = kTdThreads;
    return cudaSuccess;
  });
}

}  // namespace i4
