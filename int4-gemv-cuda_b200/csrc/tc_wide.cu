// tcgen05 W4A16 GEMV for 1 <= M <= 64 with the weights as the MMA's N operand: one kind::f16 MMA
// (M = 128 lanes of x, N = 256 weight rows, K = 16) covers 4096 weights, twice what an MMA with
// the weights as its 128-row A operand covers, so a CTA issues half the MMAs for its share.
//
// Operands. A = x: the rows of x (M of them, padded to a multiple of 8) in the canonical
// no-swizzle K-major layout in shared memory, copied there as they are (16-byte blocks of 8
// consecutive k) by cp.async; the MMA reads 128 rows, and the rows past M hold whatever follows
// in shared memory: they only feed accumulator lanes past M, which nobody reads. B = the
// dequantised weights, fp16, written by the dequant warps into the same layout (256 rows x 64 k
// per stage). D = fp32 in TMEM: lane m = row m of x, column n = weight row n of the tile, two
// accumulators of 256 columns (one tile's epilogue overlaps the next tile's MMAs).
//
// Tiles and work split. Weight rows in tiles of 256, K in stages of 64 (half a quantisation
// group); the (tile, stage) units, tile-major, are split into one contiguous range per CTA
// (grid = SMs). A tile that several CTAs share is finished by the last of them to arrive, which
// adds all the partial sums in CTA order (deterministic) and stores y.
//
// Roles (26 warps, one CTA per SM):
//   producer (1 warp)  2-D TMA tiles: each stage's packed words (256 rows x 32 bytes) into a
//                      ring, and the scales and zeros of each 8-group window (256 rows x 8 fp16
//                      each, the TMA's smallest aligned box) with the stage that starts it, into
//                      one of two window slots.
//   dequant (16 warps) thread (row n, half h) turns 4 packed words (k 32 h .. 32 h + 31 of the
//                      stage) into 32 fp16 weights in natural k order:
//                          byte b of the word -> (1024 + q_2b, 1024 + 16 q_2b+1)  (PRMT + LOP3)
//                          -> (q_2b, q_2b+1) exactly (one fma with (1, 1/16), (-1024, -64))
//                          -> w = q s + (-z s)        (one fma, -z s rounded once)
//                      and stores them into the stage's B buffer.
//   x (4 warps)        cp.async of the stage's x blocks into an x ring several stages ahead.
//   MMA (1 thread)     4 tcgen05.mma per stage into the tile's accumulator; one tcgen05.commit
//                      per stage frees its x and B buffers.
//   epilogue (4 warps) reads each finished accumulator (tcgen05.ld; the warp of TMEM lanes 0-31
//                      holds rows 0-31 of x), stores y or the partial sums, finishes shared tiles.
//
// Numerics: each weight is (q - z) s in fp16 (q exact, z s rounded once, the fma rounded once),
// products with x exact in the tensor core, fp32 accumulation: within the 1e-2 relative tolerance
// of the reference's fp32 oracle, not bit-exact.
//
// Launch overlap: programmatic stream serialization. The producer reads weights, scales and
// zeros before griddepcontrol.wait unless strict; x is read, and y, the partial sums and the tile
// counters are touched, only after it. Every mbarrier wait is bounded; after a timeout the kernel
// records a status word, stops waiting, still takes part in the tile counting and stores no y.
#include <algorithm>
#include <mutex>
#include <vector>

#include "tcgen05.cuh"
#include "weight_stream.cuh"

namespace i4 {

constexpr int kTwMaxCtas = 160;
constexpr int kTwMaxM = 64;
constexpr int kTwMaxTiles = 4096;
constexpr int kTwTileRows = 256;
// Split-K partial sums (two slots per CTA: its first and its last tile) and per-tile arrival
// counts, static so no call allocates; the CTA that finishes a tile sets its counter back to zero.
__device__ __align__(256) float g_tw_partials[kTwMaxCtas * 2 * kTwMaxM * kTwTileRows];
__device__ unsigned g_tw_arrivals[kTwMaxTiles];

namespace {

constexpr int kTwStageK = 64;                           // weights per row per stage
constexpr int kTwQBytes = kTwTileRows * kTwStageK / 2;  // 8192: packed words of a stage
constexpr int kTwSzBytes = kTwTileRows * 8 * 2;         // 4096: scales (or zeros) of 8 groups
constexpr int kTwWindowStages = 8 * kItemK / kTwStageK;  // 16 stages share a window
constexpr int kTwBBytes = kTwTileRows * kTwStageK * 2;  // 32768: fp16 weights of a stage
constexpr int kTwBLbo = kTwTileRows / 8 * 128;          // bytes between k-adjacent core matrices
constexpr int kTwDqWarps = 16;
constexpr int kTwProducerWarp = 16;
constexpr int kTwMmaWarp = 17;
constexpr int kTwXWarp0 = 18;
constexpr int kTwXWarps = 4;
constexpr int kTwEpiWarp0 = 22;
constexpr int kTwEpiWarps = 4;
constexpr int kTwThreads = (kTwEpiWarp0 + kTwEpiWarps) * kWarp;  // 832
constexpr int kTwTmemCols = 512;
constexpr int kTwMaxQStages = 8;
constexpr int kTwMaxBStages = 4;
constexpr int kTwMaxXStages = 8;
constexpr int kTwSmemLimit = 227 * 1024;
constexpr int kTwEpiBarrier = 3;
constexpr int kStatusTwTimeout = 6;

// mbarriers (8 bytes each) at the start of shared memory
constexpr int kBarQFull = 0;                              // [8] stage landed (1 arrival + bytes)
constexpr int kBarQEmpty = kBarQFull + kTwMaxQStages;     // [8] stage read (16 dequant warps)
constexpr int kBarXFull = kBarQEmpty + kTwMaxQStages;     // [8] x copied (4 x warps)
constexpr int kBarUnit = kBarXFull + kTwMaxXStages;       // [8] unit's MMAs done (commit)
constexpr int kBarBFull = kBarUnit + kTwMaxXStages;       // [4] B written (16 dequant warps)
constexpr int kBarDFull = kBarBFull + kTwMaxBStages;      // [2] accumulator complete (commit)
constexpr int kBarDEmpty = kBarDFull + 2;                 // [2] accumulator read (128 threads)
constexpr int kBarDone = kBarDEmpty + 2;                  // every MMA complete (commit)
constexpr int kTwTmemSlot = (8 * (kBarDone + 1) + 15) / 16 * 16;
constexpr int kTwFlagOff = kTwTmemSlot + 16;
constexpr int kTwScratchOff = 512;                        // 32 words, see stage_reads_done
constexpr int kTwHeader = 1024;
static_assert(kTwFlagOff + 16 <= kTwScratchOff, "shared-memory header");

struct TwMaps {
  CUtensorMap q;  // qweight as uint8 [N][K / 2], box 32 x 256 rows
  CUtensorMap s;  // scales as uint16 [N][K / 128], box 8 x 256 rows
  CUtensorMap z;  // zeros, same
};

struct TwPlan {
  int ctas;
  int tiles;     // ceil(N / 256)
  int spt;       // stages per tile: K / 64
  int units;     // tiles * spt
  int qstages, bstages, xstages;
  int m8;        // rows of x rounded up to 8
  int xslot;     // bytes of one x stage: m8 x 128
  int off_x, off_b, off_q, off_sz, smem_bytes;
  int strict;    // 1: read the weights only after griddepcontrol.wait
  int* status;
  float* partials;
  unsigned* arrivals;
};

__device__ __forceinline__ uint32_t f16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// One packed word (q0..q7, q_j in bits 4j..4j+3) -> four registers (w0, w1), (w2, w3), (w4, w5),
// (w6, w7) with w = (q - z) s: byte b copied to both halves (PRMT), its low nibble into the low
// half's mantissa and its high nibble into bits 4..7 of the high half's (LOP3 with 0x6400) give
// (1024 + q_2b, 1024 + 16 q_2b+1); one fma with (1, 1/16) and (-1024, -64) gives (q_2b, q_2b+1)
// exactly; a second, q s + c with c = -z s, gives the weights.
__device__ __forceinline__ void dequant_word_natural(uint32_t w, uint32_t s2, uint32_t c2,
                                                     uint32_t* out) {
  constexpr uint32_t kScale = 0x2C003C00u;   // (1, 1/16)
  constexpr uint32_t kOffset = 0xD400E400u;  // (-1024, -64)
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    uint32_t t, h;
    asm("prmt.b32 %0, %1, %1, %2;" : "=r"(t) : "r"(w), "r"(0x1111u * b));
    asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(h) : "r"(t), "r"(0x00F0000Fu), "r"(0x64006400u));
    out[b] = f16x2_fma(f16x2_fma(h, kScale, kOffset), s2, c2);
  }
}

// D (TMEM, f32) = A (shared memory, f16) x B (shared memory, f16) [+ D], M = 128, K = 16.
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
}

__device__ __forceinline__ void tw_tma_2d(void* dst, const CUtensorMap* map, int x, int y,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tw_tma_2d_hint(void* dst, const CUtensorMap* map, int x, int y,
                                               uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// 16-byte asynchronous copy global -> shared on the load path (cp.async, cached in L2 only).
__device__ __forceinline__ void tw_cp_async_16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void tw_cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// Waits until at most n of this thread's cp.async groups are pending (n = 0..7).
__device__ __forceinline__ void tw_cp_async_wait_pending(int n) {
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
__device__ __forceinline__ int tw_unit_begin(const TwPlan& p, int c) {
  return static_cast<int>(static_cast<int64_t>(c) * p.units / p.ctas);
}
// The CTA whose range holds unit u.
__device__ __forceinline__ int tw_cta_of_unit(const TwPlan& p, int u) {
  return static_cast<int>((static_cast<int64_t>(u + 1) * p.ctas + p.units - 1) / p.units) - 1;
}

__device__ __forceinline__ bool tw_wait(uint64_t* bar, uint32_t parity, bool& ok, int* status) {
  if (!ok) return false;
  if (!mbar_wait_bounded_suspend(bar, parity)) {
    ok = false;
    atomicExch(status, kStatusTwTimeout);
    return false;
  }
  return true;
}

__device__ __forceinline__ void tw_store(const GemvArgs& a, int m, int row, float v) {
  if (a.epilogue == kStoreF32) {
    reinterpret_cast<float*>(a.y)[static_cast<int64_t>(m) * a.n + row] = v;
  } else {
    a.y[static_cast<int64_t>(m) * a.n + row] = store_value(a, m, row, v);
  }
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  uint32_t u;
  memcpy(&u, &h, 4);
  return u;
}

__global__ void __launch_bounds__(kTwThreads, 1)
    tc_wide_kernel(GemvArgs a, TwPlan p, const __grid_constant__ TwMaps maps) {
  extern __shared__ __align__(1024) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kTwTmemSlot);
  volatile int* last_flag = reinterpret_cast<volatile int*>(smem + kTwFlagOff);
  uint32_t* scratch = reinterpret_cast<uint32_t*>(smem + kTwScratchOff);
  unsigned char* xsm = smem + p.off_x;
  unsigned char* bsm = smem + p.off_b;
  unsigned char* qsm = smem + p.off_q;
  unsigned char* szsm = smem + p.off_sz;

  const int tid = threadIdx.x;
  const int warp = tid / kWarp;
  const int lane = tid % kWarp;
  const int u0 = tw_unit_begin(p, blockIdx.x);
  const int u1 = tw_unit_begin(p, blockIdx.x + 1);
  const int n_units = u1 - u0;
  const int t_first = u0 / p.spt;
  const int t_last = (u1 - 1) / p.spt;

  if (tid == 0) {
    for (int s = 0; s < p.qstages; ++s) {
      mbar_init(&bars[kBarQFull + s], 1);
      mbar_init(&bars[kBarQEmpty + s], kTwDqWarps);
    }
    for (int s = 0; s < p.xstages; ++s) {
      mbar_init(&bars[kBarXFull + s], kTwXWarps);
      mbar_init(&bars[kBarUnit + s], 1);
    }
    for (int s = 0; s < p.bstages; ++s) mbar_init(&bars[kBarBFull + s], kTwDqWarps);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[kBarDFull + s], 1);
      mbar_init(&bars[kBarDEmpty + s], kTwEpiWarps * kWarp);
    }
    mbar_init(&bars[kBarDone], 1);
    fence_mbar_init();
  }
  if (warp == kTwMmaWarp) tmem_alloc(tmem_slot, kTwTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) launch_dependents();

  bool ok = true;
  if (warp < kTwDqWarps) {
    // ---------------- dequant warps ----------------
    const int n = tid & (kTwTileRows - 1);  // weight row of the tile
    const int h = tid / kTwTileRows;        // k 32 h .. 32 h + 31 of the stage
    // Ring slots and phases kept incrementally (no division per unit).
    int qs = 0;
    uint32_t qph = 0;
    int wc = -1;              // window counter, as the producer keeps it
    int j = u0 % p.spt;       // stage of unit i within its tile
    int b = 0;                // B buffer of unit i
    int vs = 0;               // unit barrier of unit i - bstages, and its phase
    uint32_t vph = 0;
    for (int i = 0; i < n_units; ++i) {
      if (i == 0 || j % kTwWindowStages == 0) ++wc;
      tw_wait(&bars[kBarQFull + qs], qph, ok, p.status);
      const uint4 v = *reinterpret_cast<const uint4*>(qsm + qs * kTwQBytes + n * 32 + h * 16);
      const unsigned char* sz = szsm + (wc & 1) * (2 * kTwSzBytes) + n * 16 + ((j >> 1) & 7) * 2;
      const uint32_t sb = *reinterpret_cast<const uint16_t*>(sz);
      const uint32_t zb = *reinterpret_cast<const uint16_t*>(sz + kTwSzBytes);
      // release only once every load above has returned (see stage_reads_done)
      stage_reads_done(fold4(v) ^ sb ^ (zb << 16), scratch, lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kBarQEmpty + qs]);
      if (++qs == p.qstages) {
        qs = 0;
        qph ^= 1u;
      }

      const float sf = __half2float(__ushort_as_half(static_cast<uint16_t>(sb)));
      const float zf = __half2float(__ushort_as_half(static_cast<uint16_t>(zb)));
      const uint32_t c2 = static_cast<uint32_t>(__half_as_ushort(__float2half_rn(-zf * sf))) *
                          0x10001u;
      const uint32_t s2 = sb * 0x10001u;
      uint32_t o[16];
      dequant_word_natural(v.x, s2, c2, &o[0]);
      dequant_word_natural(v.y, s2, c2, &o[4]);
      dequant_word_natural(v.z, s2, c2, &o[8]);
      dequant_word_natural(v.w, s2, c2, &o[12]);

      // B buffer b was last read by the MMAs of unit i - bstages (unit barrier
      // (i - bstages) % xstages; xstages >= bstages keeps its phase exact, see the plan).
      if (i >= p.bstages) {
        tw_wait(&bars[kBarUnit + vs], vph, ok, p.status);
        if (++vs == p.xstages) {
          vs = 0;
          vph ^= 1u;
        }
      }
      unsigned char* dst = bsm + b * kTwBBytes + (n >> 3) * 128 + (n & 7) * 16;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        *reinterpret_cast<uint4*>(dst + (4 * h + c) * kTwBLbo) =
            make_uint4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // B visible to the MMAs
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kBarBFull + b]);
      if (++b == p.bstages) b = 0;
      if (++j == p.spt) j = 0;
    }
  } else if (warp == kTwProducerWarp) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t policy = l2_evict_first_policy();
      if (p.strict) grid_dependency_wait();
      int qs = 0;
      uint32_t qph = 0;
      int wc = -1;
      int t = u0 / p.spt;
      int j = u0 % p.spt;
      int i = 0;
      for (; i < n_units; ++i) {
        const bool new_window = i == 0 || j % kTwWindowStages == 0;
        if (new_window) ++wc;
        if (i >= p.qstages && !tw_wait(&bars[kBarQEmpty + qs], qph ^ 1u, ok, p.status)) break;
        uint64_t* full = &bars[kBarQFull + qs];
        mbar_arrive_expect_tx(full, kTwQBytes + (new_window ? 2 * kTwSzBytes : 0));
        tw_tma_2d_hint(qsm + qs * kTwQBytes, &maps.q, j * (kTwStageK / 2), t * kTwTileRows, full,
                       policy);
        if (new_window) {
          // Window slot wc & 1 last held window wc - 2, whose stages the dequant warps have all
          // released: the empty wait above covers stage i - qstages, inside window wc - 1
          // (a whole window of 16 stages, more than the ring holds).
          unsigned char* sz = szsm + (wc & 1) * (2 * kTwSzBytes);
          const int gx = (j / kTwWindowStages) * 8;
          tw_tma_2d(sz, &maps.s, gx, t * kTwTileRows, full);
          tw_tma_2d(sz + kTwSzBytes, &maps.z, gx, t * kTwTileRows, full);
        }
        if (++qs == p.qstages) {
          qs = 0;
          qph ^= 1u;
        }
        if (++j == p.spt) {
          j = 0;
          ++t;
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
  } else if (warp == kTwMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t kIdesc = idesc_f16_f32(128, kTwTileRows);
      const uint32_t x_base = smem_addr(xsm);
      const uint32_t b_base = smem_addr(bsm);
      const uint32_t lbo_a = static_cast<uint32_t>(p.m8) * 16;
      int xs = 0, bs = 0;
      uint32_t xph = 0, bph = 0;
      bool issued = false;
      for (int t = t_first; t <= t_last && ok; ++t) {
        const int r = t - t_first;
        const int ub = max(u0, t * p.spt);
        const int ue = min(u1, (t + 1) * p.spt);
        const uint32_t d_addr = tmem + (r & 1) * kTwTileRows;
        if (r >= 2 && !tw_wait(&bars[kBarDEmpty + (r & 1)], ((r - 2) >> 1) & 1, ok, p.status))
          break;
        for (int u = ub; u < ue; ++u) {
          if (!tw_wait(&bars[kBarXFull + xs], xph, ok, p.status)) break;
          if (!tw_wait(&bars[kBarBFull + bs], bph, ok, p.status)) break;
          tc_fence_after();
          const uint32_t a_addr = x_base + xs * p.xslot;
          const uint32_t b_addr = b_base + bs * kTwBBytes;
#pragma unroll
          for (int kk = 0; kk < kTwStageK / 16; ++kk) {
            const uint64_t adesc = smem_desc(a_addr + 2 * kk * lbo_a, lbo_a, 128);
            const uint64_t bdesc = smem_desc(b_addr + 2 * kk * kTwBLbo, kTwBLbo, 128);
            mma_f16_ss(d_addr, adesc, bdesc, kIdesc, u != ub || kk != 0);
          }
          mma_commit(&bars[kBarUnit + xs]);  // frees the unit's x and B buffers
          issued = true;
          if (++xs == p.xstages) {
            xs = 0;
            xph ^= 1u;
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
  } else if (warp < kTwEpiWarp0) {
    // ---------------- x warps ----------------
    // Thread xt copies 16-byte blocks (row m, chunk kc) of a unit's x into its x slot at
    // kc * m8 * 16 + m * 16 (the K-major core-matrix layout), `look` units ahead of the unit it
    // hands to the MMA. A unit is handed over (each x warp arrives once) as soon as this thread's
    // copies of it have landed, before waiting for the slot of the unit `look` ahead, so the MMA
    // of unit i + 1 never waits for more than the MMAs of unit i - 3 to complete.
    const int xt = tid - kTwXWarp0 * kWarp;
    grid_dependency_wait();  // x may be the previous kernel's output
    const int look = p.xstages - 3;
    const int blocks = a.m * 8;
    const int lbo_a = p.m8 * 16;
    int jn = u0 % p.spt;  // stage (within its tile) and x slot of the next unit to copy
    int sn = 0;
    auto issue = [&]() {  // copies the next unit, units in order
      unsigned char* dst = xsm + sn * p.xslot;
      const half* src = a.x + jn * kTwStageK;
      for (int b = xt; b < blocks; b += kTwXWarps * kWarp) {
        const int m = b >> 3;
        const int kc = b & 7;
        tw_cp_async_16(dst + kc * lbo_a + m * 16, src + static_cast<int64_t>(m) * a.k + 8 * kc);
      }
      if (++sn == p.xstages) sn = 0;
      if (++jn == p.spt) jn = 0;
    };
    for (int i = 0; i < look; ++i) {
      if (i < n_units) issue();
      tw_cp_async_commit();  // one group per unit, empty or not, so the counts stay uniform
    }
    int hs = 0;  // x slot of the unit handed over
    int vs = 0;  // unit barrier of unit i + look - xstages, and its phase
    uint32_t vph = 0;
    for (int i = 0; i < n_units; ++i) {
      tw_cp_async_wait_pending(look - 1);  // this thread's blocks of unit i have landed
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // x visible to the MMAs
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kBarXFull + hs]);
      if (++hs == p.xstages) hs = 0;
      const int nx = i + look;
      if (nx < n_units) {
        // the next unit's slot was last read by the MMAs of unit nx - xstages = i - 3
        if (nx >= p.xstages) {
          tw_wait(&bars[kBarUnit + vs], vph, ok, p.status);
          if (++vs == p.xstages) {
            vs = 0;
            vph ^= 1u;
          }
        }
        issue();
      }
      tw_cp_async_commit();
    }
    tw_cp_async_wait_pending(0);  // nothing in flight into shared memory at exit
  } else {
    // ---------------- epilogue warps ----------------
    const int quarter = warp & 3;
    const int et = tid - kTwEpiWarp0 * kWarp;
    const int m = 32 * quarter + lane;  // row of x in this lane of the accumulator
    const uint32_t lane_field = static_cast<uint32_t>(32 * quarter) << 16;
    const bool rows_here = 32 * quarter < a.m;  // uniform over the warp
    const bool vec_y = a.epilogue == kStoreY && !a.bias && !a.residual && a.n % 8 == 0 &&
                       reinterpret_cast<uintptr_t>(a.y) % 16 == 0;
    grid_dependency_wait();  // y, the partial sums and the counters of the previous call
    for (int t = t_first; t <= t_last; ++t) {
      const int r = t - t_first;
      const int db = r & 1;
      const bool have = tw_wait(&bars[kBarDFull + db], (r >> 1) & 1, ok, p.status);
      tc_fence_after();
      const int row0 = t * kTwTileRows;
      const int c_lo = tw_cta_of_unit(p, t * p.spt);
      const int c_hi = tw_cta_of_unit(p, min((t + 1) * p.spt, p.units) - 1);
      const int slot = t == t_first ? 0 : 1;
      float* mine = p.partials + (static_cast<int64_t>(blockIdx.x) * 2 + slot) * a.m * kTwTileRows;
      if (rows_here) {
        for (int c = 0; c < kTwTileRows / 16; ++c) {
          uint32_t d[16];
          tmem_ld16(tmem + lane_field + db * kTwTileRows + 16 * c, d);
          tmem_wait_ld();
          if (m < a.m) {
            const int rr = row0 + 16 * c;
            if (c_lo == c_hi) {
              if (have) {
                if (vec_y && rr + 16 <= a.n) {
                  uint4* dst = reinterpret_cast<uint4*>(a.y + static_cast<int64_t>(m) * a.n + rr);
#pragma unroll
                  for (int e = 0; e < 2; ++e) {
                    dst[e] = make_uint4(
                        pack_half2(__uint_as_float(d[8 * e]), __uint_as_float(d[8 * e + 1])),
                        pack_half2(__uint_as_float(d[8 * e + 2]), __uint_as_float(d[8 * e + 3])),
                        pack_half2(__uint_as_float(d[8 * e + 4]), __uint_as_float(d[8 * e + 5])),
                        pack_half2(__uint_as_float(d[8 * e + 6]), __uint_as_float(d[8 * e + 7])));
                  }
                } else {
#pragma unroll
                  for (int e = 0; e < 16; ++e) {
                    if (rr + e < a.n) tw_store(a, m, rr + e, __uint_as_float(d[e]));
                  }
                }
              }
            } else {
              float4* dst = reinterpret_cast<float4*>(mine + m * kTwTileRows + 16 * c);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                dst[e] = make_float4(__uint_as_float(d[4 * e]), __uint_as_float(d[4 * e + 1]),
                                     __uint_as_float(d[4 * e + 2]), __uint_as_float(d[4 * e + 3]));
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&bars[kBarDEmpty + db]);
      if (c_lo != c_hi) {
        __threadfence();
        named_barrier(kTwEpiBarrier, kTwEpiWarps * kWarp);
        if (et == 0) {
          const unsigned before = atomicAdd(&p.arrivals[t], 1u);
          const int last = before == static_cast<unsigned>(c_hi - c_lo);
          if (last) atomicExch(&p.arrivals[t], 0u);
          *last_flag = last;
        }
        named_barrier(kTwEpiBarrier, kTwEpiWarps * kWarp);
        if (*last_flag) {
          __threadfence();
          const bool store = *reinterpret_cast<volatile int*>(p.status) == 0;
          // c_lo's range may start in an earlier tile (then this is its last tile, slot 1); every
          // later contributor starts in this tile (slot 0).
          const int lo_slot = tw_unit_begin(p, c_lo) / p.spt == t ? 0 : 1;
          constexpr int kChunks = kTwTileRows / 8;
          // Eight outputs per task; the partials of up to eight contributors loaded together (one
          // round trip to L2 per eight), then added in CTA order.
          for (int task = et; task < a.m * kChunks; task += kTwEpiWarps * kWarp) {
            const int mm = task / kChunks;
            const int c8 = task - mm * kChunks;
            float sum[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) sum[e] = 0.0f;
            for (int c0 = c_lo; c0 <= c_hi; c0 += 8) {
              float4 v[8][2];
#pragma unroll
              for (int ci = 0; ci < 8; ++ci) {
                const int c = c0 + ci;
                const int cs = c == c_lo ? lo_slot : 0;
                const float4* src = reinterpret_cast<const float4*>(
                    p.partials + ((static_cast<int64_t>(c) * 2 + cs) * a.m + mm) * kTwTileRows +
                    8 * c8);
                const bool here = c <= c_hi;
                v[ci][0] = here ? __ldcg(src) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                v[ci][1] = here ? __ldcg(src + 1) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
              }
#pragma unroll
              for (int ci = 0; ci < 8; ++ci) {
                if (c0 + ci <= c_hi) {
                  sum[0] += v[ci][0].x;
                  sum[1] += v[ci][0].y;
                  sum[2] += v[ci][0].z;
                  sum[3] += v[ci][0].w;
                  sum[4] += v[ci][1].x;
                  sum[5] += v[ci][1].y;
                  sum[6] += v[ci][1].z;
                  sum[7] += v[ci][1].w;
                }
              }
            }
            if (store) {
              const int rr = row0 + 8 * c8;
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                if (rr + e < a.n) tw_store(a, mm, rr + e, sum[e]);
              }
            }
          }
        }
        named_barrier(kTwEpiBarrier, kTwEpiWarps * kWarp);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kTwMmaWarp) tmem_dealloc(tmem, kTwTmemCols);
}

bool tw_plan(const GemvArgs& a, TwPlan* p, const char** why) {
  auto fail = [&](const char* reason) {
    if (why) *why = reason;
    return false;
  };
  if (a.m < 1 || a.m > kTwMaxM) return fail("M must be in [1, 64]");
  if (a.group != kItemK) return fail("group_size must be 128");
  if (a.k < 1024 || a.k % 1024 != 0) return fail("K must be a positive multiple of 1024");
  if (a.epilogue != kStoreY && a.epilogue != kStoreF32)
    return fail("only plain stores (fp16 y or fp32 row sums)");
  if (reinterpret_cast<uintptr_t>(a.q) % 16 || reinterpret_cast<uintptr_t>(a.x) % 16 ||
      reinterpret_cast<uintptr_t>(a.s) % 16 || reinterpret_cast<uintptr_t>(a.z) % 16)
    return fail("x, qweight, scales and zeros must be 16-byte aligned");
  const int64_t tiles = (static_cast<int64_t>(a.n) + kTwTileRows - 1) / kTwTileRows;
  if (tiles > kTwMaxTiles) return fail("N must be at most 1048576");
  p->tiles = static_cast<int>(tiles);
  p->spt = a.k / kTwStageK;
  const int64_t units = tiles * p->spt;
  if (units > (1LL << 30)) return fail("too many stages");
  p->units = static_cast<int>(units);
  p->ctas = std::min({sm_count(), p->units, kTwMaxCtas});
  if (p->ctas < 1) return fail("no SMs");
  p->m8 = (a.m + 7) / 8 * 8;
  p->xslot = p->m8 * 128;
  // The MMA reads 128 rows of x from each x slot: up to 2 KB past the last one, which the B
  // buffers that follow cover. Four B buffers, an x ring of 6 (5 for M > 32: xstages >= bstages
  // keeps the unit barriers' phases exact), and the deepest q ring (up to 8 stages) that fits.
  p->bstages = 4;
  p->xstages = a.m <= 32 ? kTwMaxXStages - 2 : 5;
  p->off_x = kTwHeader;
  p->off_b = (p->off_x + p->xstages * p->xslot + 1023) / 1024 * 1024;
  p->off_sz = p->off_b + p->bstages * kTwBBytes;
  p->off_q = p->off_sz + 2 * 2 * kTwSzBytes;
  const int64_t qstages =
      std::min<int64_t>((kTwSmemLimit - p->off_q) / kTwQBytes, kTwMaxQStages);
  if (qstages < 4) return fail("shared memory");
  p->qstages = static_cast<int>(qstages);
  p->smem_bytes = p->off_q + p->qstages * kTwQBytes;
  p->strict = 0;
  p->status = nullptr;
  p->partials = nullptr;
  p->arrivals = nullptr;
  return true;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tw_encode_fn() {
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

struct TwMapEntry {
  int dev;
  const void* q;
  const void* s;
  const void* z;
  int n, k;
  TwMaps maps;
};
std::mutex g_tw_mu;
std::vector<TwMapEntry> g_tw_maps;  // most recently used first
constexpr size_t kTwMapCache = 64;

cudaError_t tw_maps_for(const GemvArgs& a, TwMaps* out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  std::lock_guard<std::mutex> lock(g_tw_mu);
  for (size_t i = 0; i < g_tw_maps.size(); ++i) {
    const TwMapEntry& e = g_tw_maps[i];
    if (e.dev == dev && e.q == a.q && e.s == a.s && e.z == a.z && e.n == a.n && e.k == a.k) {
      *out = e.maps;
      if (i != 0) std::swap(g_tw_maps[i], g_tw_maps[0]);
      return cudaSuccess;
    }
  }
  auto encode = tw_encode_fn();
  if (!encode) return cudaErrorNotSupported;
  TwMapEntry e{dev, a.q, a.s, a.z, a.n, a.k, {}};
  const cuuint32_t estr[2] = {1, 1};
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(a.k / 2), static_cast<cuuint64_t>(a.n)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.k / 2)};
  const cuuint32_t box[2] = {kTwStageK / 2, kTwTileRows};
  if (encode(&e.maps.q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint32_t*>(a.q), dims,
             strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
    return cudaErrorInvalidValue;
  }
  const int groups = a.k / a.group;
  const cuuint64_t sdims[2] = {static_cast<cuuint64_t>(groups), static_cast<cuuint64_t>(a.n)};
  const cuuint64_t sstrides[1] = {static_cast<cuuint64_t>(groups) * 2};
  const cuuint32_t sbox[2] = {8, kTwTileRows};
  for (int which = 0; which < 2; ++which) {
    if (encode(which == 0 ? &e.maps.s : &e.maps.z, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2,
               const_cast<half*>(which == 0 ? a.s : a.z), sdims, sstrides, sbox, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      return cudaErrorInvalidValue;
    }
  }
  g_tw_maps.insert(g_tw_maps.begin(), e);
  if (g_tw_maps.size() > kTwMapCache) g_tw_maps.pop_back();
  *out = e.maps;
  return cudaSuccess;
}

// The static partial sums and counters of the current device (looked up once per device).
cudaError_t tw_scratch(float** partials, unsigned** arrivals) {
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
    err = cudaGetSymbolAddress(&pp, g_tw_partials);
    if (err != cudaSuccess) return err;
    err = cudaGetSymbolAddress(&ap, g_tw_arrivals);
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
struct TwOrder {
  std::mutex mu;
  bool has[64] = {};
  cudaStream_t last[64] = {};
  cudaEvent_t done[64] = {};
};
TwOrder g_tw_order;

bool tw_stream_capturing(cudaStream_t stream) {
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &st) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return st != cudaStreamCaptureStatusNone;
}

std::once_flag g_tw_attr_once[64];

}  // namespace

bool tc_wide_supported(const GemvArgs& a, const char** why) {
  TwPlan p;
  return tw_plan(a, &p, why);
}

cudaError_t launch_tc_wide(const GemvArgs& a, cudaStream_t stream, bool strict) {
  TwPlan p;
  if (!tw_plan(a, &p, nullptr)) return cudaErrorInvalidValue;
  p.strict = strict ? 1 : 0;
  p.status = device_status_word();
  if (!p.status) return cudaErrorInvalidSymbol;
  cudaError_t err = tw_scratch(&p.partials, &p.arrivals);
  if (err != cudaSuccess) return err;
  TwMaps maps;
  err = tw_maps_for(a, &maps);
  if (err != cudaSuccess) return err;
  int dev = 0;
  err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  const bool capturing = tw_stream_capturing(stream);
  std::lock_guard<std::mutex> lock(g_tw_order.mu);
  if (!capturing) {
    if (!g_tw_order.done[dev]) {
      err = cudaEventCreateWithFlags(&g_tw_order.done[dev], cudaEventDisableTiming);
      if (err != cudaSuccess) return err;
    }
    if (g_tw_order.has[dev] && g_tw_order.last[dev] != stream) {
      err = cudaStreamWaitEvent(stream, g_tw_order.done[dev], 0);
      if (err != cudaSuccess) return err;
    }
  }
  cudaError_t result = cudaSuccess;
  std::call_once(g_tw_attr_once[dev & 63], [&] {
    result = cudaFuncSetAttribute(tc_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  kTwSmemLimit);
  });
  if (result != cudaSuccess) return result;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.ctas);
  cfg.blockDim = dim3(kTwThreads);
  cfg.dynamicSmemBytes = p.smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  err = cudaLaunchKernelEx(&cfg, tc_wide_kernel, a, p, maps);
  if (err != cudaSuccess || capturing) return err;
  err = cudaEventRecord(g_tw_order.done[dev], stream);
  if (err != cudaSuccess) return err;
  g_tw_order.has[dev] = true;
  g_tw_order.last[dev] = stream;
  return cudaSuccess;
}

cudaError_t tc_wide_attrs(int m, KernelAttrs* out) {
  (void)m;
  cudaFuncAttributes fa;
  cudaError_t err = cudaFuncGetAttributes(&fa, tc_wide_kernel);
  if (err != cudaSuccess) return err;
  out->registers = fa.numRegs;
  out->local_bytes = static_cast<int>(fa.localSizeBytes);
  out->max_threads_per_block = fa.maxThreadsPerBlock;
  out->blocks_per_sm = 1;
  out->threads_per_block = kTwThreads;
  return cudaSuccess;
}

}  // namespace i4
