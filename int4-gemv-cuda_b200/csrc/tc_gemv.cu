// The B200 fast path for M <= 8: a TMA-fed tcgen05 (5th-generation tensor core) W4A16 GEMV.
//
// Work split. Two CTAs per SM (grid = 2 x SMs). CTA c owns output rows [4 u0, 4 u1), an equal
// share of 4-row units, so every CTA streams the same number of weight bytes to within 4 rows.
// A CTA takes its rows in blocks of up to 32 and each row in stages of 8 items of 128 weights
// (512 contiguous packed bytes).
//
// Memory side. A producer warp streams every stage (rows x 512 bytes) with 2-D TMA tile copies
// (cp.async.bulk.tensor, boxes of 32/16/8/4 rows x 128 bytes so a CTA never fetches rows it does
// not own, completion counted in bytes on an mbarrier) into a ring of shared-memory buffers in the
// 128-byte swizzled layout, so sixteen-byte loads by 32 threads of 32 different rows hit 32
// different banks. (One 1-D bulk copy per row and stage, 512 bytes each, streams at less than half
// the bandwidth of these tiles on B200.) The stage's scales and zeros (8 groups x rows) come in
// the same way, as two more tiles per box.
//
// Math side. One warpgroup (128 threads = the 128 lanes of TMEM). Thread l of warp q owns row l of
// the block and every item i with i % 4 == q. Per item it unpacks the 16 packed words with one
// shift and four LOP3s each into fp16 1024 + q / 1024 + 16 q (exact) and stores them into its TMEM
// lane: the A operand of tcgen05.mma (M = 128, K = 16, f16 x f16 -> f32). Once all 128 lanes have
// stored (a relaxed mbarrier arrival, so no thread waits for its own loads), one thread issues the
// item's eight MMAs against x in shared memory (the B operand) and commits them to an mbarrier.
// One item later each thread reads its accumulator back (tcgen05.ld) and applies the group's
// scale and zero in fp32:
//     sum_k (q_k - z) s x_k = s * (D - 1024 sum_k b_k - z sum_k x_k)
// (b_k are the B operands; the two sums over x come from a per-CTA table). B holds one column per
// (quarter q, row m of x): x of the items i = 4t + q, each 8-weight block permuted to
// [x0, x4, x1/16, x5/16, x2, x6, x3/16, x7/16] to match the A operand, in the canonical no-swizzle
// K-major layout (8x16-byte core matrices). A and D are double-buffered in TMEM (256 columns per
// CTA, so two CTAs fit an SM), so unpacking one item overlaps the MMAs of the previous one.
//
// Launch overlap. The kernel is launched with programmatic stream serialization and triggers its
// dependents early, so the next GEMV in the stream becomes resident while this one finishes and
// starts streaming its weights. Everything that may have been produced by the previous kernel in
// the stream (x) is read, and y is written, only after griddepcontrol.wait. Weights, scales and
// zeros are read before it unless the caller asks for strict ordering.
//
// The four quarters' partial sums per row meet in shared memory and are added in a fixed order,
// so results are deterministic. Every mbarrier wait is bounded; on timeout the kernel records a
// status word, stops issuing work without leaving a barrier unmatched, and still frees its TMEM.
#include <algorithm>
#include <mutex>

#include "tcgen05.cuh"
#include "weight_stream.cuh"

namespace i4 {
namespace {

constexpr int kConsumerWarps = 4;  // one warpgroup: TMEM lanes 0..127
constexpr int kThreads = (kConsumerWarps + 1) * kWarp;
constexpr int kTmemCols = 256;
constexpr int kMaxStages = 6;
constexpr int kTwoPerSm = 113 * 1024;  // shared memory that still fits two CTAs per SM
constexpr int kSmemLimit = 227 * 1024;
constexpr int kStatusMmaTimeout = 4;
constexpr int kStatusLoadTimeout = 5;
constexpr int kConsumerBarrier = 1;

// mbarrier slots (8 bytes each) at the start of shared memory
constexpr int kBarFull = 0;                    // [kMaxStages] stage landed (bytes)
constexpr int kBarEmpty = kMaxStages;          // [kMaxStages] stage consumed (4 warps)
constexpr int kBarMma = 2 * kMaxStages;        // [2] MMAs of buffer b done (commit)
constexpr int kBarA = 2 * kMaxStages + 2;      // [2] A operand of buffer b written (128 lanes)
constexpr int kTmemSlot = 8 * (2 * kMaxStages + 4);
constexpr int kScratchOff = 512;  // 32 words, see stage_reads_done

struct TcPlan {
  int ctas;
  int units;        // 4-row units in N
  int nb;           // 8-column core-matrix groups in B
  int n_mma;        // MMA N
  uint32_t idesc;
  uint32_t lbo, sbo;  // B descriptor strides (bytes)
  int rows_cap;     // max rows per CTA
  int stages;
  int off_b, off_corr, off_red, off_stage, smem_bytes;
  int strict;       // 1: read weights only after griddepcontrol.wait
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

template <int MT>
__global__ void __launch_bounds__(kThreads, 2)
    tc_gemv_kernel(GemvArgs a, TcPlan p, const __grid_constant__ WeightMaps maps) {
  extern __shared__ __align__(1024) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kTmemSlot);
  unsigned char* bsm = smem + p.off_b;
  float2* corr = reinterpret_cast<float2*>(smem + p.off_corr);
  float* red = reinterpret_cast<float*>(smem + p.off_red);
  unsigned char* stages = smem + p.off_stage;

  const int tid = threadIdx.x;
  const int warp = tid / kWarp;
  const int lane = tid % kWarp;
  const int items_row = a.k / kItemK;
  const int steps = items_row / kItemsPerStage;  // stages per 32-row block

  const int u0 = static_cast<int>(static_cast<int64_t>(blockIdx.x) * p.units / p.ctas);
  const int u1 = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * p.units / p.ctas);
  const int row_begin = 4 * u0;
  const int rows = min(4 * u1, a.n) - row_begin;
  const int blocks = (rows + kBlockRows - 1) / kBlockRows;

  if (tid == kConsumerWarps * kWarp) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&bars[kBarFull + s], 1);
      mbar_init(&bars[kBarEmpty + s], kConsumerWarps);
    }
    mbar_init(&bars[kBarMma + 0], 1);
    mbar_init(&bars[kBarMma + 1], 1);
    mbar_init(&bars[kBarA + 0], 128);
    mbar_init(&bars[kBarA + 1], 128);
    fence_mbar_init();
  }
  if (warp == 0) {
    // TMEM before the dependents trigger: a next-kernel CTA must never hold TMEM this CTA needs.
    tmem_alloc(tmem_slot, kTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0) launch_dependents();  // the next GEMV may become resident as SMs free up

  if (warp == kConsumerWarps) {
    // ---------------- producer warp ----------------
    if (p.strict) grid_dependency_wait();
    produce_weight_stages(maps, row_begin, rows, steps, steps, stages, p.stages, &bars[kBarFull],
                          &bars[kBarEmpty], p.status);
    return;
  }

  // ---------------- consumer warpgroup ----------------
  const int quarter = warp;  // TMEM lanes 32 q .. 32 q + 31
  grid_dependency_wait();  // x may be the previous kernel's output

  // B operand: for item-step t and quarter q, column n = q MT + m holds x[m] of item 4 t + q.
  {
    const __half2 sixteenth = __float2half2_rn(0.0625f);
    const int ncols = p.nb * 8;
    const int kc_count = (items_row / 4) * (kItemK / 8);
    for (int idx = tid; idx < kc_count * ncols; idx += kConsumerWarps * kWarp) {
      const int kc = idx / ncols;
      const int n = idx % ncols;
      const int q = n / MT;
      const int m = n % MT;
      uint4 o = make_uint4(0, 0, 0, 0);
      if (q < 4 && m < a.m) {
        const int t = kc / (kItemK / 8);
        const int k0 = (4 * t + q) * kItemK + 8 * (kc % (kItemK / 8));
        const uint4 v =
            *reinterpret_cast<const uint4*>(a.x + static_cast<int64_t>(m) * a.k + k0);
        o.x = prmt(v.x, v.z, 0x5410);
        o.y = hmul2_bits(prmt(v.x, v.z, 0x7632), sixteenth);
        o.z = prmt(v.y, v.w, 0x5410);
        o.w = hmul2_bits(prmt(v.y, v.w, 0x7632), sixteenth);
      }
      *reinterpret_cast<uint4*>(bsm + (kc * p.nb + n / 8) * 128 + 16 * (n % 8)) = o;
    }
  }
  named_barrier(kConsumerBarrier, kConsumerWarps * kWarp);
  // corr[m][i] = (1024 * sum of the B operands of item i, sum of the x values they stand for);
  // one warp per entry, fixed reduction order.
  for (int idx = warp; idx < a.m * items_row; idx += kConsumerWarps) {
    const int m = idx / items_row;
    const int item = idx % items_row;
    const int kc0 = (item / 4) * (kItemK / 8);
    const int n = (item % 4) * MT + m;
    float bsum = 0.0f, xsum = 0.0f;
    if (lane < kItemK / 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(bsm + ((kc0 + lane) * p.nb + n / 8) * 128 +
                                                      16 * (n % 8));
      const float2 p0 = half2_bits_to_float2(v.x), p1 = half2_bits_to_float2(v.y);
      const float2 p2 = half2_bits_to_float2(v.z), p3 = half2_bits_to_float2(v.w);
      const float ones = (p0.x + p0.y) + (p2.x + p2.y);
      const float sixteenths = (p1.x + p1.y) + (p3.x + p3.y);
      bsum = ones + sixteenths;
      xsum = ones + 16.0f * sixteenths;
    }
    bsum = warp_sum(bsum);
    xsum = warp_sum(xsum);
    if (lane == 0) corr[idx] = make_float2(1024.0f * bsum, xsum);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // B visible to the tensor core
  tc_fence_before();
  named_barrier(kConsumerBarrier, kConsumerWarps * kWarp);
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  bool ok = true;

  const uint32_t lane_addr = static_cast<uint32_t>(32 * quarter) << 16;
  const uint32_t b_base = smem_addr(bsm);
  const bool issuer = tid == 0;

  float yacc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) yacc[m] = 0.0f;

  // Epilogue of item-step `it` (buffer it & 1): scale, zero, accumulate; park at block end.
  auto epilogue = [&](int it, int item, int row_local, bool valid, bool block_end, uint32_t sz) {
    const int buf = it & 1;
    if (ok && !mbar_wait_bounded(&bars[kBarMma + buf], (it >> 1) & 1)) {
      ok = false;
      atomicExch(p.status, kStatusMmaTimeout);
    }
    tc_fence_after();
    float d[MT];
    tmem_ld<MT>(tmem + lane_addr + 128 + buf * p.n_mma + quarter * MT, d);
    const float sc = __half2float(__ushort_as_half(static_cast<uint16_t>(sz & 0xFFFF)));
    const float zp = __half2float(__ushort_as_half(static_cast<uint16_t>(sz >> 16)));
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const float2 cr = corr[min(m, a.m - 1) * items_row + item];
      yacc[m] = fmaf(sc, fmaf(-zp, cr.y, d[m] - cr.x), yacc[m]);
    }
    if (block_end) {
      if (valid) {
#pragma unroll
        for (int m = 0; m < MT; ++m) red[(quarter * p.rows_cap + row_local) * MT + m] = yacc[m];
      }
#pragma unroll
      for (int m = 0; m < MT; ++m) yacc[m] = 0.0f;
    }
  };

  int it = 0;  // item-steps issued by this CTA
  int prev_item = 0, prev_row = 0;
  bool prev_valid = false, prev_end = false;
  uint32_t prev_sz = 0;
  int sit = 0;  // stages consumed
  for (int blk = 0; blk < blocks; ++blk) {
    const int rows_b = min(kBlockRows, rows - blk * kBlockRows);
    const int row_local = blk * kBlockRows + lane;
    const bool valid = lane < rows_b;
    for (int j = 0; j < steps; ++j, ++sit) {
      const int slot = sit % p.stages;
      if (ok && !mbar_wait_bounded(&bars[kBarFull + slot], (sit / p.stages) & 1)) {
        ok = false;
        atomicExch(p.status, kStatusLoadTimeout);
      }
      // This thread's two items of the stage: 4 t + quarter, t = 0, 1. Item i of the stage is
      // 16-byte granules (i % 2) * 4 + c of column chunk i / 2; the swizzle XORs the granule with
      // the row's index mod 8.
      uint32_t qw[2][16];
      const unsigned char* rowp = stages + slot * kStageBytes + lane * 128;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int item_s = 4 * t + quarter;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int granule = ((item_s & 1) * 4 + c) ^ (lane & 7);
          const uint4 v = *reinterpret_cast<const uint4*>(rowp + (item_s >> 1) * kChunkBytes +
                                                          granule * 16);
          qw[t][4 * c + 0] = v.x;
          qw[t][4 * c + 1] = v.y;
          qw[t][4 * c + 2] = v.z;
          qw[t][4 * c + 3] = v.w;
        }
      }
      // Scale and zero of the two items (row-major [row][8 groups] in the stage).
      uint32_t szw[2];
      {
        const uint16_t* ss = reinterpret_cast<const uint16_t*>(stages + slot * kStageBytes +
                                                               kStageQBytes) +
                             lane * kItemsPerStage;
        const uint16_t* zz = ss + kBlockRows * kItemsPerStage;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          szw[t] = static_cast<uint32_t>(ss[4 * t + quarter]) |
                   (static_cast<uint32_t>(zz[4 * t + quarter]) << 16);
        }
      }
      {
        // release only once every load above has returned (see stage_reads_done)
        uint32_t folded = szw[0] ^ szw[1];
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int w = 0; w < 16; ++w) folded ^= qw[t][w];
        stage_reads_done(folded, reinterpret_cast<uint32_t*>(smem + kScratchOff), lane);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kBarEmpty + slot]);  // stage may be refilled

#pragma unroll
      for (int t = 0; t < 2; ++t, ++it) {
        const int buf = it & 1;
        const int tstep = 2 * j + t;           // item-step within the row
        const int item = 4 * tstep + quarter;  // this thread's item (= group)
        const uint32_t a_addr = tmem + lane_addr + buf * (kItemK / 2);
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint32_t v[16];
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            uint32_t h[4];
            unpack_x16(qw[t][4 * c4 + w], h);
            v[4 * w + 0] = h[0];
            v[4 * w + 1] = h[1];
            v[4 * w + 2] = h[2];
            v[4 * w + 3] = h[3];
          }
          tmem_st16(a_addr + 16 * c4, v);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive_relaxed(&bars[kBarA + buf]);
        if (issuer && ok && !mbar_wait_bounded(&bars[kBarA + buf], (it >> 1) & 1)) {
          ok = false;
          atomicExch(p.status, kStatusMmaTimeout);
        }
        if (issuer && ok) {
          tc_fence_after();
          const uint32_t d_addr = tmem + 128 + buf * p.n_mma;
          const uint32_t a_base = tmem + buf * (kItemK / 2);
          const uint32_t b_step = b_base + tstep * (kItemK / 8) * p.nb * 128;
#pragma unroll
          for (int kk = 0; kk < kItemK / 16; ++kk) {
            const uint64_t bdesc = smem_desc(b_step + 2 * kk * p.nb * 128, p.lbo, p.sbo);
            mma_f16(d_addr, a_base + 8 * kk, bdesc, p.idesc, kk > 0);
          }
          mma_commit(&bars[kBarMma + buf]);
        }
        if (it > 0) epilogue(it - 1, prev_item, prev_row, prev_valid, prev_end, prev_sz);
        prev_sz = szw[t];
        prev_item = item;
        prev_row = row_local;
        prev_valid = valid;
        prev_end = (j == steps - 1) && (t == 1);
      }
    }
  }
  if (it > 0) epilogue(it - 1, prev_item, prev_row, prev_valid, prev_end, prev_sz);

  // ---- add the four quarters of every (row, row of x) in a fixed order and store fp16 ---------
  tc_fence_before();
  named_barrier(kConsumerBarrier, kConsumerWarps * kWarp);
  for (int o = tid; o < rows * a.m; o += kConsumerWarps * kWarp) {
    const int r = o % rows;
    const int m = o / rows;
    float sum = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) sum += red[(q * p.rows_cap + r) * MT + m];
    if (ok) {
      a.y[static_cast<int64_t>(m) * a.n + row_begin + r] = store_value(a, m, row_begin + r, sum);
    }
  }
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

int round_up(int v, int m) { return (v + m - 1) / m * m; }

int tile_m(int m) { return m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : 8; }

bool plan_smem(const GemvArgs& a, TcPlan* p, int limit, int min_stages);

bool make_plan(const GemvArgs& a, TcPlan* p, const char** why) {
  auto fail = [&](const char* reason) {
    if (why) *why = reason;
    return false;
  };
  if (a.m < 1 || a.m > 8) return fail("M must be in [1, 8]");
  if (a.group != kItemK) return fail("group_size must be 128");
  if (a.k % (kItemK * kItemsPerStage) != 0) return fail("K must be a multiple of 1024");
  if (reinterpret_cast<uintptr_t>(a.q) % 16 || reinterpret_cast<uintptr_t>(a.x) % 16 ||
      reinterpret_cast<uintptr_t>(a.s) % 16 || reinterpret_cast<uintptr_t>(a.z) % 16)
    return fail("x, qweight, scales and zeros must be 16-byte aligned");
  const int mt = tile_m(a.m);
  p->nb = (4 * mt + 7) / 8;
  p->n_mma = std::max(16, round_up(4 * mt, 16));
  if (128 + 2 * p->n_mma > kTmemCols) return fail("TMEM budget");
  p->lbo = static_cast<uint32_t>(p->nb * 128);
  p->sbo = p->nb * 8 >= p->n_mma ? 128u : 0u;  // N = 16 over 8 stored columns: alias them
  p->idesc = (1u << 4) | (static_cast<uint32_t>(p->n_mma >> 3) << 17) | ((128u >> 4) << 24);
  p->units = (a.n + 3) / 4;
  // Two CTAs per SM when x, the tables and >= 3 stages fit in half the shared memory.
  p->ctas = std::min(2 * sm_count(), p->units);
  p->rows_cap = 4 * ((p->units + p->ctas - 1) / p->ctas);
  if (!plan_smem(a, p, kTwoPerSm, 3)) {
    p->ctas = std::min(sm_count(), p->units);
    p->rows_cap = 4 * ((p->units + p->ctas - 1) / p->ctas);
    if (!plan_smem(a, p, kSmemLimit, 2)) return fail("x does not fit in shared memory");
  }
  p->strict = 0;
  return true;
}

// Lays out shared memory for the plan; true if it fits `limit` with at least `min_stages` stages.
bool plan_smem(const GemvArgs& a, TcPlan* p, int limit, int min_stages) {
  const int mt = tile_m(a.m);
  const int items_row = a.k / kItemK;
  const int64_t b_bytes = static_cast<int64_t>(items_row / 4) * (kItemK / 8) * p->nb * 128;
  int64_t off = 1024;
  p->off_b = static_cast<int>(off);
  off = (off + b_bytes + 127) / 128 * 128;
  p->off_corr = static_cast<int>(off);
  off = (off + static_cast<int64_t>(a.m) * items_row * 8 + 127) / 128 * 128;
  p->off_red = static_cast<int>(off);
  off = (off + static_cast<int64_t>(4) * p->rows_cap * mt * 4 + 1023) / 1024 * 1024;
  p->off_stage = static_cast<int>(off);
  const int64_t stages = std::min<int64_t>((limit - off) / kStageBytes, kMaxStages);
  if (off > limit || stages < min_stages) return false;
  p->stages = static_cast<int>(stages);
  p->smem_bytes = static_cast<int>(off + stages * kStageBytes);
  return true;
}

std::once_flag g_tc_attr_once[4][64];

template <int MT>
cudaError_t ensure_smem_attr() {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  constexpr int variant = MT == 1 ? 0 : MT == 2 ? 1 : MT == 4 ? 2 : 3;
  cudaError_t result = cudaSuccess;
  std::call_once(g_tc_attr_once[variant][dev & 63], [&] {
    result = cudaFuncSetAttribute(tc_gemv_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  kSmemLimit);
  });
  return result;
}

template <typename F>
cudaError_t with_mt(int m, F&& f) {
  switch (tile_m(m)) {
    case 1:
      return f.template operator()<1>();
    case 2:
      return f.template operator()<2>();
    case 4:
      return f.template operator()<4>();
    default:
      return f.template operator()<8>();
  }
}

}  // namespace

bool tc_gemv_supported(const GemvArgs& a, const char** why) {
  TcPlan p;
  return make_plan(a, &p, why);
}

cudaError_t launch_tc_gemv(const GemvArgs& a, cudaStream_t stream, bool strict) {
  TcPlan p;
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
    return cudaLaunchKernelEx(&cfg, tc_gemv_kernel<MT>, a, p, maps);
  });
}

cudaError_t tc_gemv_attrs(int m, KernelAttrs* out) {
  return with_mt(m, [&]<int MT>() {
    cudaFuncAttributes fa;
    cudaError_t err = cudaFuncGetAttributes(&fa, tc_gemv_kernel<MT>);
    if (err != cudaSuccess) return err;
    out->registers = fa.numRegs;
    out->local_bytes = static_cast<int>(fa.localSizeBytes);
    out->max_threads_per_block = fa.maxThreadsPerBlock;
    out->blocks_per_sm = 2;  // when x, the tables and the stages fit in half the SM
    out->threads_per_block = kThreads;
    return cudaSuccess;
  });
}

}  // namespace i4
