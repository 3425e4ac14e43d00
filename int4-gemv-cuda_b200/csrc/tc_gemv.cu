// The B200 fast path for M <= 8: a tcgen05 (5th-generation tensor core) W4A16 GEMV.
//
// Mapping. One CTA per SM, two warpgroups. The CTA owns output rows [c N / P, (c + 1) N / P) (the
// same number of weight bytes per SM, within a row). Its rows are cut into blocks of 32 and K into
// S = 4 or 8 equal slices; a task is (block, four consecutive slices) and the warpgroups take the
// tasks in turn. Inside a task one thread owns one (row, slice): TMEM lane 32 q + l is row l of the
// block in slice 4 h + q, where q is the warp's quarter of the warpgroup. So every lane of the
// 128-lane MMA does useful work even when a CTA owns only 28 or 56 rows.
//
// Per 128-weight step ("item") a thread
//   1. has its 64 packed bytes (two 256-bit loads issued four items ahead, L1 bypassed) and its
//      scale / zero,
//   2. unpacks each 32-bit word with one shift and four LOP3s into fp16 1024 + q / 1024 + 16 q
//      (exact) and stores the 64 fp16 pairs into its TMEM lane (the MMA's A operand),
//   3. after a warpgroup barrier, one thread issues eight tcgen05.mma (M = 128, N = 16..64, K = 16,
//      f16 x f16 -> f32) against x in shared memory (the B operand) and commits to an mbarrier,
//   4. one item later the thread reads its accumulator column(s) back with tcgen05.ld and applies
//      the group's scale and zero in fp32:
//          sum_k (q_k - z) s x_k = s * (D - 1024 sum_k b_k - z sum_k x_k)
//      (b_k are the B operands; both sums over x come from a per-CTA table).
// The B operand holds, for every slice s and row m of x, the column n = s MT + m: x of that slice,
// each 8-weight block permuted to [x0, x4, x1/16, x5/16, x2, x6, x3/16, x7/16] to match the unpacked
// A operand, in the canonical no-swizzle K-major layout (8x16-byte core matrices). A lane of quarter
// q reads only its own slice's column of D. The A and D buffers are double-buffered per warpgroup
// in TMEM (the CTA allocates all 512 columns), so unpacking item i+1 overlaps the MMAs of item i.
//
// Partial sums per (row, slice) meet in shared memory and are added in a fixed order (so results
// are deterministic) before the fp16 store. Every mbarrier wait is bounded; on timeout the kernel
// records a status word, stops issuing work without leaving a barrier unmatched, and still frees
// its TMEM.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace i4 {

namespace {

constexpr int kWarpgroups = 2;  // mbarriers: 4 per warpgroup in the first 64 bytes
constexpr int kThreads = kWarpgroups * 128;
constexpr int kTmemCols = 512;
constexpr int kItemK = 128;        // weights per row per item (= one TMEM A buffer of 64 columns)
constexpr int kPrefetch = 4;       // items of packed weights in flight per thread
constexpr int kSmemLimit = 227 * 1024;
constexpr int kStatusMmaTimeout = 4;

struct TcPlan {
  int ctas;
  int slices;       // S
  int items_slice;  // items per slice = K / 128 / S
  int nb;           // 8-column core-matrix groups in B
  int n_mma;        // MMA N
  uint32_t idesc;
  uint32_t lbo, sbo;  // B descriptor strides (bytes)
  int rows_cap;     // max rows per CTA rounded up to 32
  int group_shift;  // group_size = 128 << group_shift
  int off_b, off_corr, off_red, smem_bytes;
  int* status;      // device status word (int4gemv_device_status)
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

// 32 bytes, read once: skip L1.
__device__ __forceinline__ void ld_stream_v8(const void* p, uint32_t (&r)[8]) {
  asm volatile(
      "ld.global.nc.L1::no_allocate.v8.u32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "l"(p));
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

template <int MT>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float (&v)[MT]) {
  uint32_t r[MT];
  if constexpr (MT == 1) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r[0]) : "r"(taddr));
  } else if constexpr (MT == 2) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];"
                 : "=r"(r[0]), "=r"(r[1])
                 : "r"(taddr));
  } else if constexpr (MT == 4) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
  } else {
    static_assert(MT == 8, "MT must be 1, 2, 4 or 8");
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7])
        : "r"(taddr));
  }
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < MT; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}

// Shared-memory matrix descriptor, no swizzle, K-major (sm_100 format, version 1).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFF) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32) | (static_cast<uint64_t>(1) << 46);
}

template <int MT>
__global__ void __launch_bounds__(kThreads, 1) tc_gemv_kernel(GemvArgs a, TcPlan p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  // [0, 64): mbarriers, per warpgroup 2 "MMAs done" and 2 "A operand written"; [64, 68): TMEM
  // base address
  uint64_t* mbar = reinterpret_cast<uint64_t*>(smem);
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(smem + 64);
  unsigned char* bsm = smem + p.off_b;
  float2* corr = reinterpret_cast<float2*>(smem + p.off_corr);
  float* red = reinterpret_cast<float*>(smem + p.off_red);

  const int tid = threadIdx.x;
  const int warp = tid / kWarp;
  const int lane = tid % kWarp;
  const int wg = warp / 4;
  const int quarter = warp % 4;
  const int groups = a.k / a.group;
  const int items_row = a.k / kItemK;
  const int slice_k = a.k / p.slices;

  if (warp == 0) {
    asm volatile(
        "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
            smem_addr(tmem_base_slot)),
        "r"(kTmemCols)
        : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int w = 0; w < kWarpgroups; ++w) {
      mbar_init(&mbar[4 * w + 0], 1);    // MMAs of buffer 0 done (tcgen05.commit)
      mbar_init(&mbar[4 * w + 1], 1);    // MMAs of buffer 1 done
      mbar_init(&mbar[4 * w + 2], 128);  // A operand of buffer 0 written by all 128 lanes
      mbar_init(&mbar[4 * w + 3], 128);  // A operand of buffer 1 written
    }
    fence_mbar_init();
  }

  // ---- B operand: x, permuted per 8-weight block, one column per (slice, row of x) -------------
  {
    const __half2 sixteenth = __float2half2_rn(0.0625f);
    const int ncols = p.nb * 8;
    const int kc_count = slice_k / 8;
    for (int idx = tid; idx < kc_count * ncols; idx += kThreads) {
      const int kc = idx / ncols;
      const int n = idx % ncols;
      const int s = n / MT;
      const int m = n % MT;
      uint4 o = make_uint4(0, 0, 0, 0);
      if (s < p.slices && m < a.m) {
        const uint4 v = *reinterpret_cast<const uint4*>(
            a.x + static_cast<int64_t>(m) * a.k + s * slice_k + 8 * kc);
        o.x = prmt(v.x, v.z, 0x5410);
        o.y = hmul2_bits(prmt(v.x, v.z, 0x7632), sixteenth);
        o.z = prmt(v.y, v.w, 0x5410);
        o.w = hmul2_bits(prmt(v.y, v.w, 0x7632), sixteenth);
      }
      *reinterpret_cast<uint4*>(bsm + (kc * p.nb + n / 8) * 128 + 16 * (n % 8)) = o;
    }
  }
  __syncthreads();
  // corr[m][g] = (1024 * sum of B operands, sum of the x values they stand for), per 128 weights;
  // one warp per entry, fixed reduction order.
  for (int idx = warp; idx < a.m * items_row; idx += kThreads / kWarp) {
    const int m = idx / items_row;
    const int item = idx % items_row;
    const int s = item / p.items_slice;
    const int kc0 = (item % p.items_slice) * (kItemK / 8);
    const int n = s * MT + m;
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
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_base_slot;

  // ---- work list of this warpgroup ----------------------------------------------------------
  const int row_begin = static_cast<int>(static_cast<int64_t>(blockIdx.x) * a.n / p.ctas);
  const int row_end = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * a.n / p.ctas);
  const int rows = row_end - row_begin;
  const int blocks = (rows + 31) / 32;
  const int quads = p.slices / 4;
  const int tasks = blocks * quads;
  const int my_tasks = tasks > wg ? (tasks - wg + kWarpgroups - 1) / kWarpgroups : 0;
  const int items = my_tasks * p.items_slice;

  const uint32_t lane_addr = static_cast<uint32_t>(32 * quarter) << 16;
  const uint32_t a_col0 = static_cast<uint32_t>(wg * 2) * (kItemK / 2);
  const uint32_t d_col0 = 256u + static_cast<uint32_t>(wg * 2) * p.n_mma;
  uint64_t* bar = mbar + 4 * wg;        // bar[buf]: MMAs done
  uint64_t* a_ready = mbar + 4 * wg + 2;  // a_ready[buf]: A operand complete
  const uint32_t b_base = smem_addr(bsm);
  const bool issuer = (tid % 128) == 0;
  const int64_t row_bytes = a.k / 2;

  // The warpgroup's items in order: task tl covers block (t / quads), slices (t % quads) * 4 + q
  // with t = wg + tl * kWarpgroups; an item is one 128-weight step of the thread's slice. Cursors
  // advance by one item without divisions (quads is 1 or 2).
  const int quad_shift = quads == 2 ? 1 : 0;
  const int gshift = p.group_shift;  // group = 128 << gshift
  int ld_task = 0, ld_j = 0, ld_rl = 0, ld_sl = 0;
  bool ld_valid = false;
  const unsigned char* ld_src = nullptr;
  const half* ld_s = nullptr;
  const half* ld_z = nullptr;
  auto start_task = [&](int tl) {
    const int t = wg + tl * kWarpgroups;
    const int blk = t >> quad_shift;
    ld_sl = (t & (quads - 1)) * 4 + quarter;
    ld_rl = 32 * blk + lane;
    ld_valid = ld_rl < rows;
    const int64_t row = row_begin + (ld_valid ? ld_rl : 0);
    const int item0 = ld_sl * p.items_slice;
    ld_src = reinterpret_cast<const unsigned char*>(a.q) + row * row_bytes + item0 * (kItemK / 2);
    ld_s = a.s + row * groups + (item0 >> gshift);
    ld_z = a.z + row * groups + (item0 >> gshift);
  };
  if (my_tasks > 0) start_task(0);

  uint32_t qbuf[kPrefetch][16];
  uint32_t szbuf[kPrefetch];  // scale bits | zero bits << 16
  int meta_j[kPrefetch];      // item within the slice
  int meta_sl[kPrefetch];     // slice
  int meta_rl[kPrefetch];     // row within the CTA (or -1 for a lane past the last row)

  // Loads the loader cursor's item into `slot`, then advances the cursor.
  auto issue_load = [&](int slot) {
    if (ld_task >= my_tasks) return;
    if (ld_valid) {
      uint32_t lo[8], hi[8];
      ld_stream_v8(ld_src, lo);
      ld_stream_v8(ld_src + 32, hi);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        qbuf[slot][j] = lo[j];
        qbuf[slot][8 + j] = hi[j];
      }
      const int gi = ((ld_sl * p.items_slice + ld_j) >> gshift) -
                     ((ld_sl * p.items_slice) >> gshift);
      szbuf[slot] = static_cast<uint32_t>(__half_as_ushort(ld_s[gi])) |
                    (static_cast<uint32_t>(__half_as_ushort(ld_z[gi])) << 16);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) qbuf[slot][j] = 0;
      szbuf[slot] = 0;
    }
    meta_j[slot] = ld_j;
    meta_sl[slot] = ld_sl;
    meta_rl[slot] = ld_valid ? ld_rl : -1;
    ld_src += kItemK / 2;
    if (++ld_j == p.items_slice) {
      ld_j = 0;
      if (++ld_task < my_tasks) start_task(ld_task);
    }
  };

  float yacc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) yacc[m] = 0.0f;
  bool ok = true;

  // Epilogue of an item whose MMAs were committed to bar[buf] (use `use`): scale, zero,
  // accumulate; park the partial sum at the end of a task.
  auto epilogue = [&](int buf, int use, int j, int sl, int rl, uint32_t sz) {
    if (ok && !mbar_wait_bounded(&bar[buf], use & 1)) {
      ok = false;
      atomicExch(p.status, kStatusMmaTimeout);
    }
    tc_fence_after();
    float d[MT];
    tmem_ld<MT>(tmem + lane_addr + d_col0 + buf * p.n_mma + sl * MT, d);
    const float sc = __half2float(__ushort_as_half(static_cast<uint16_t>(sz & 0xFFFF)));
    const float zp = __half2float(__ushort_as_half(static_cast<uint16_t>(sz >> 16)));
    const int ir = sl * p.items_slice + j;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const float2 cr = corr[min(m, a.m - 1) * items_row + ir];
      yacc[m] = fmaf(sc, fmaf(-zp, cr.y, d[m] - cr.x), yacc[m]);
    }
    if (j == p.items_slice - 1) {
      if (rl >= 0) {
#pragma unroll
        for (int m = 0; m < MT; ++m) red[(sl * p.rows_cap + rl) * MT + m] = yacc[m];
      }
#pragma unroll
      for (int m = 0; m < MT; ++m) yacc[m] = 0.0f;
    }
  };

#pragma unroll
  for (int i = 0; i < kPrefetch; ++i) issue_load(i);

  uint32_t prev_sz = 0;
  int prev_j = 0, prev_sl = 0, prev_rl = -1;
  for (int base = 0; base < items; base += kPrefetch) {
#pragma unroll
    for (int u = 0; u < kPrefetch; ++u) {
      const int it = base + u;
      if (it < items) {
        const int buf = it & 1;
        // 2. unpack into this lane's TMEM row (A operand, 64 columns = 128 weights)
        const uint32_t a_addr = tmem + lane_addr + a_col0 + buf * (kItemK / 2);
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          uint32_t v[16];
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            uint32_t h[4];
            unpack_x16(qbuf[u][4 * c4 + w], h);
            v[4 * w + 0] = h[0];
            v[4 * w + 1] = h[1];
            v[4 * w + 2] = h[2];
            v[4 * w + 3] = h[3];
          }
          tmem_st16(a_addr + 16 * c4, v);
        }
        const uint32_t sz = szbuf[u];
        const int cur_j = meta_j[u], cur_sl = meta_sl[u], cur_rl = meta_rl[u];
        issue_load(u);
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        tc_fence_before();
        // Relaxed arrival: a bar.sync here would first wait for this thread's prefetch loads.
        asm volatile("mbarrier.arrive.relaxed.cta.shared::cta.b64 _, [%0];" ::"r"(
                         smem_addr(&a_ready[buf]))
                     : "memory");
        // 3. one thread issues the item's 8 MMAs once all 128 lanes wrote their A rows
        if (issuer && ok && !mbar_wait_bounded(&a_ready[buf], (it >> 1) & 1)) {
          ok = false;
          atomicExch(p.status, kStatusMmaTimeout);
        }
        if (issuer && ok) {
          tc_fence_after();
          const uint32_t d_addr = tmem + d_col0 + buf * p.n_mma;
          const uint32_t a_base = tmem + a_col0 + buf * (kItemK / 2);
          const uint32_t b_item = b_base + cur_j * (kItemK / 8) * p.nb * 128;
#pragma unroll
          for (int j = 0; j < kItemK / 16; ++j) {
            const uint64_t bdesc = smem_desc(b_item + 2 * j * p.nb * 128, p.lbo, p.sbo);
            mma_f16(d_addr, a_base + 8 * j, bdesc, p.idesc, j > 0);
          }
          mma_commit(&bar[buf]);
        }
        // 4. epilogue of the previous item (its MMAs had a whole item of time to finish)
        if (it > 0) epilogue((it - 1) & 1, (it - 1) >> 1, prev_j, prev_sl, prev_rl, prev_sz);
        prev_sz = sz;
        prev_j = cur_j;
        prev_sl = cur_sl;
        prev_rl = cur_rl;
      }
    }
  }
  if (items > 0) epilogue((items - 1) & 1, (items - 1) >> 1, prev_j, prev_sl, prev_rl, prev_sz);

  // ---- add the slices of every (row, column of x) in a fixed order and store fp16 ---------------
  tc_fence_before();
  __syncthreads();
  for (int o = tid; o < rows * a.m; o += kThreads) {
    const int r = o % rows;
    const int m = o / rows;
    float sum = 0.0f;
    for (int s = 0; s < p.slices; ++s) sum += red[(s * p.rows_cap + r) * MT + m];
    if (ok) a.y[static_cast<int64_t>(m) * a.n + row_begin + r] = __float2half_rn(sum);
  }
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

int round_up(int v, int m) { return (v + m - 1) / m * m; }

int tile_m(int m) { return m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : 8; }

bool make_plan(const GemvArgs& a, TcPlan* p, const char** why) {
  auto fail = [&](const char* reason) {
    if (why) *why = reason;
    return false;
  };
  if (a.m < 1 || a.m > 8) return fail("M must be in [1, 8]");
  if (a.group % kItemK != 0) return fail("group_size must be a multiple of 128");
  p->group_shift = 0;
  while ((kItemK << p->group_shift) < a.group) ++p->group_shift;
  if ((kItemK << p->group_shift) != a.group) return fail("group_size must be 128 times a power of 2");
  if (reinterpret_cast<uintptr_t>(a.q) % 32 != 0) return fail("qweight must be 32-byte aligned");
  if (reinterpret_cast<uintptr_t>(a.x) % 16 != 0) return fail("x must be 16-byte aligned");
  const int items_row = a.k / kItemK;
  const int mt = tile_m(a.m);
  int slices = 0;
  for (int s : {8, 4}) {
    if (items_row % s == 0 && s * mt <= 64) {
      slices = s;
      break;
    }
  }
  if (!slices) return fail("K / 128 must be a multiple of 4");
  p->slices = slices;
  p->items_slice = items_row / slices;
  p->nb = (slices * mt + 7) / 8;
  p->n_mma = std::max(16, round_up(slices * mt, 16));
  if (2 * kWarpgroups * p->n_mma + 2 * kWarpgroups * (kItemK / 2) > kTmemCols)
    return fail("TMEM budget");
  p->lbo = static_cast<uint32_t>(p->nb * 128);
  p->sbo = p->nb * 8 >= p->n_mma ? 128u : (p->nb == 1 ? 0u : 128u);
  if (p->nb * 8 < p->n_mma && p->nb != 1) return fail("B column padding");
  p->idesc = (1u << 4) | (static_cast<uint32_t>(p->n_mma >> 3) << 17) | ((128u >> 4) << 24);
  p->ctas = std::min(sm_count(), a.n);
  const int rows_max = (a.n + p->ctas - 1) / p->ctas;
  p->rows_cap = round_up(rows_max, 32);
  const int64_t b_bytes = static_cast<int64_t>(a.k / slices / 8) * p->nb * 128;
  p->off_b = 1024;
  p->off_corr = static_cast<int>(round_up(static_cast<int>(std::min<int64_t>(b_bytes, kSmemLimit)) + p->off_b, 128));
  p->off_red = round_up(p->off_corr + a.m * items_row * 8, 128);
  const int64_t end = static_cast<int64_t>(p->off_red) +
                      static_cast<int64_t>(slices) * p->rows_cap * mt * 4;
  if (b_bytes > kSmemLimit || end > kSmemLimit) return fail("x does not fit in shared memory");
  // At least half of the SM's shared memory, so two CTAs never share an SM (each takes all of
  // TMEM).
  p->smem_bytes = static_cast<int>(std::max<int64_t>(end, 120 * 1024));
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

cudaError_t launch_tc_gemv(const GemvArgs& a, cudaStream_t stream) {
  TcPlan p;
  if (!make_plan(a, &p, nullptr)) return cudaErrorInvalidValue;
  p.status = device_status_word();
  if (!p.status) return cudaErrorInvalidSymbol;
  return with_mt(a.m, [&]<int MT>() {
    cudaError_t err = ensure_smem_attr<MT>();
    if (err != cudaSuccess) return err;
    tc_gemv_kernel<MT><<<p.ctas, kThreads, p.smem_bytes, stream>>>(a, p);
    return cudaGetLastError();
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
    out->blocks_per_sm = 1;
    out->threads_per_block = kThreads;
    return cudaSuccess;
  });
}

}  // namespace i4
