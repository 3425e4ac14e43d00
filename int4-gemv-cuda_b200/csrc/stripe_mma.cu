// The B200 fast path for M <= 8: stripes of 32 rows x 2048 weights streamed by TMA into a ring of
// shared-memory stages, and warp-level tensor-core MMAs (mma.sync m16n8k16, f16 x f16 -> f32) on
// the nibbles unpacked in registers.
//
// Memory side. One CTA per SM; CTA c owns rows [4 u0, 4 u1), an equal share of 4-row units. Its
// rows are taken in blocks of up to 32, each block in stripes of 2048 weights along K. A stripe is
// one 2-D TMA tile of the packed weights (32 rows x 1 KB, no swizzle) plus two tiles of its scales
// and zeros (32 rows x 16 groups), 34 KB in all; blocks of fewer rows use boxes of 16 / 8 / 4 rows,
// so a CTA never fetches a row it does not own. On B200 these 1 KB-wide tiles stream a W4A16
// matrix about 20 % faster than 128-byte-wide ones (measured). The ring holds three stripes
// (about 100 KB per SM), and unless the caller asks for strict ordering the producer warp issues
// the whole ring before griddepcontrol.wait: while the previous kernel in the stream finishes, the
// weights of this call are already on their way.
//
// x. Right after the dependency wait every consumer thread loads its share of x with 16-byte loads
// (one round trip), permutes each 8-weight block to the order of the unpacked A halves,
// [x0, x4, x1/16, x5/16, x2, x6, x3/16, x7/16], and stores it with per-item (128-weight) padding so
// the B loads of different items hit different banks. The same pass builds two small tables:
// bq[item][granule][m] = the sum of the B values of each 4-word granule, and xs[item][m] = the sum
// of the item's x.
//
// Math side. Sixteen consumer warps. For M <= 2 warp w takes items 4 (w % 4) .. + 3 of every
// stripe and one word granule (4 words) of each; lane (g, c) takes item 4 (w % 4) + c ("narrow"
// layout: the eight MMA columns are four items x two rows of x, and lane c's k-slots hold its own
// item's words, so one MMA covers 256 weights of four different groups), granule (w / 4 + c / 2)
// % 4 (rotated so the 16-byte loads of one shared-memory phase hit distinct banks), and rows g,
// g + 8, 16 + g, 24 + g of the block. For M = 3 or 4 the eight columns are two items x four rows
// of x: lanes c and c ^ 1 share item 2 (w % 8) + c / 2, each with its own granule 2 (w / 8) + c % 2;
// for M = 5..8 one item x eight rows: warp w takes item w, lane c its granule c. Either way an MMA
// still covers 256 weights, so M = 8 costs the MMAs of M = 1.
//
// K-panels. When x for all of K does not fit beside the ring (M = 8 at K = 8192 would need 139 KB),
// the CTA takes K in 2, 4, ... panels: it permutes the panel's x, runs all its row blocks over the
// panel's stripes (the producer streams in the same order), and each warp adds its partials to the
// earlier panels' in panel order. Per packed word one shift and four LOP3s give the fp16 A halves 1024 + q
// and 1024 + 16 q exactly; the B registers of a word are reused for both 16-row tiles. Each tile's
// low-half MMA chain starts from C = -1024 * (sum of the B values of the granule), which removes
// the magic-number offset inside the tensor core, so after the stripe the accumulators hold
// sum_k q_k x_k per (row, item) and the stripe epilogue is one scale multiply-add per row:
//     sum_k (q_k - z) s x_k = s * (sum_k q_k x_k - z * sum_k x_k),
// the z term added by the granule-0 warps only. The weights are bit-exact; the arithmetic is
// fp32 accumulation of exact fp16 products.
//
// Results. After a block the four item lanes of each row are added with two shuffles and each
// warp writes one partial per (row, m) to shared memory; after the last block the sixteen
// partials of every output are added in a fixed order, so results are deterministic. Every
// mbarrier wait is bounded; on timeout the kernel records a status word and runs to completion
// without writing y.
#include <algorithm>
#include <mutex>
#include <vector>

#include "exchange.cuh"
#include "weight_stream.cuh"

namespace i4 {
namespace {

constexpr int kSxRows = 32;                            // rows per block (tallest box)
constexpr int kSxK = 2048;                             // weights per stripe along K
constexpr int kSxItems = kSxK / kItemK;                // 16 groups per stripe
constexpr int kSxRowBytes = kSxK / 2;                  // 1024 packed bytes per row and stripe
constexpr int kSxQBytes = kSxRows * kSxRowBytes;       // 32 KB
constexpr int kSxMetaRow = kSxItems * 2;               // 32 bytes of scales (or zeros) per row
constexpr int kSxSOff = kSxQBytes;
constexpr int kSxZOff = kSxQBytes + kSxRows * kSxMetaRow;
constexpr int kSxStageBytes = kSxQBytes + 2 * kSxRows * kSxMetaRow;  // 34816
constexpr int kSxTxPerRow = kSxRowBytes + 2 * kSxMetaRow;           // 1088 bytes land per row
constexpr int kSxItemBytes = 272;   // one item of permuted x for one row of x (256 + 16 pad)
// Ring depth. Deeper rings keep more bytes in flight across all SMs, which lengthens every
// request's queueing in the memory system, x's included; three 34 KB stripes per SM measured
// fastest back to back (five: +4 %).
constexpr int kSxMaxStages = 3;
constexpr int kSxMaxConsumers = 16 * kWarp;  // the most consumer threads of any instance
constexpr int kSxSmemLimit = 227 * 1024;
constexpr int kSxMinStages = 3;
constexpr int kSxBarrier = 1;       // named barrier of the consumer warps
constexpr int kSxZeroOff = 1024;    // 512 zero bytes: the B source of lanes without x
constexpr int kSxHeader = 1536;     // mbarriers + zero block

// qweight as [N][K / 8] 32-bit words (boxes of 256 words = one stripe row); scales and zeros as
// [N][K / 128] halves (boxes of 16 groups); each with boxes of 32, 16, 8 and 4 rows.
struct StripeMaps {
  CUtensorMap q[4];
  CUtensorMap s[4];
  CUtensorMap z[4];
};

struct StripePlan {
  int ctas;
  int units;       // 4-row units in N
  int rows_cap;    // rows of the largest CTA share
  int stripes;     // K / 2048
  int items;       // K / 128
  int panels;      // K-panels: x is prepared one panel at a time (stripes split evenly)
  int xs_stride;   // bytes of permuted x per row of x (one panel)
  int stages;
  int off_xs, off_bq, off_xsum, off_red, off_stage, smem_bytes;
  int strict;      // 1: read the weights only after griddepcontrol.wait
  int* status;
};

// The box this lane issues for a block of rows4 rows (a multiple of 4, at most 32): boxes are the
// binary decomposition of rows4 into 32 / 16 / 8 / 4 rows, largest first; lane 3 b + t issues box
// b of tensor t (0 weights, 1 scales, 2 zeros). Returns false if the lane has no box.
struct StripeBox {
  const CUtensorMap* map;
  int dst;    // byte offset in the stage
  int row;    // first row (global)
  int kind;   // 0 weights, 1 scales, 2 zeros
};

__device__ __forceinline__ bool stripe_box(const StripeMaps& maps, int lane, int rows4, int row0,
                                           StripeBox* b) {
  const int box = lane / 3, kind = lane % 3;
  int n = 0, off = 0;
  for (int hi = 0; hi < 4; ++hi) {
    const int h = kSxRows >> hi;
    if (rows4 & h) {
      if (n == box && lane < 12) {
        b->kind = kind;
        b->row = row0 + off;
        b->map = kind == 0 ? &maps.q[hi] : kind == 1 ? &maps.s[hi] : &maps.z[hi];
        b->dst = kind == 0 ? off * kSxRowBytes : (kind == 1 ? kSxSOff : kSxZOff) + off * kSxMetaRow;
        return true;
      }
      ++n;
      off += h;
    }
  }
  return false;
}

__device__ __forceinline__ void issue_stripe(const StripeBox& b, bool has_box, int stripe,
                                             int rows4, unsigned char* stage, uint64_t* full_bar,
                                             uint64_t policy, int lane) {
  if (lane == 0) mbar_arrive_expect_tx(full_bar, static_cast<uint32_t>(rows4 * kSxTxPerRow));
  __syncwarp();
  if (has_box) {
    // x coordinate in elements: 256 words per stripe for the weights, 16 groups for scales/zeros
    const int x = b.kind == 0 ? stripe * (kSxRowBytes / 4) : stripe * kSxItems;
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(stage + b.dst)),
        "l"(b.map), "r"(x), "r"(b.row), "r"(smem_addr(full_bar)), "l"(policy)
        : "memory");
  }
}

// The producer warp: the CTA's K-panels x blocks x stripes through the ring (the consumers' order). Unless strict, the first
// min(stages, total) stripes go out before griddepcontrol.wait. empty[s] expects one arrival per
// consumer warp.
__device__ __forceinline__ void stripe_produce(const StripePlan& p, const StripeMaps& maps,
                                               int row_begin, int rows, unsigned char* smem) {
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kSxMaxStages;
  unsigned char* stages = smem + p.off_stage;
  const int lane = threadIdx.x % kWarp;
  const uint64_t policy = l2_evict_first_policy();
  const int blocks = (rows + kSxRows - 1) / kSxRows;
  const int total = blocks * p.stripes;
  const int pre = p.strict ? 0 : min(p.stages, total);
  if (pre == 0) grid_dependency_wait();
  bool ok = true;
  int it = 0, slot = 0, use = 0;
  for (int pn = 0; pn < p.panels; ++pn) {
    const int j0 = pn * p.stripes / p.panels, j1 = (pn + 1) * p.stripes / p.panels;
    for (int blk = 0; blk < blocks; ++blk) {
      const int rows4 = (min(kSxRows, rows - blk * kSxRows) + 3) & ~3;
      StripeBox b;
      const bool has_box = stripe_box(maps, lane, rows4, row_begin + blk * kSxRows, &b);
      for (int j = j0; j < j1; ++j, ++it) {
        if (it == pre && pre > 0) grid_dependency_wait();
        if (ok && use > 0 && !mbar_wait_bounded(&empty[slot], (use - 1) & 1)) {
          ok = false;
          if (lane == 0) atomicExch(p.status, kStatusEmptyBarrierTimeout);
        }
        if (ok) issue_stripe(b, has_box, j, rows4, stages + slot * kSxStageBytes, &full[slot],
                             policy, lane);
        if (++slot == p.stages) {
          slot = 0;
          ++use;
        }
      }
    }
  }
  if (pre == total) grid_dependency_wait();  // every stripe fit in the ring
  // Do not leave while copies into this CTA's shared memory may be in flight.
  if (ok) {
    for (int back = 1; back <= min(it, p.stages); ++back) {
      const int j = it - back;
      if (!mbar_wait_bounded(&full[j % p.stages], (j / p.stages) & 1)) break;
    }
  }
}

// x of one K-panel (8-weight blocks kw0 .. kw0 + kw_per_m - 1 of every row) -> the permuted B
// layout and the two tables (see the file comment), indexed from the panel's first item. Thread t
// handles blocks 2 t and 2 t + 1 of each 2 x NT-block step; a thread pair covers one 4-word
// granule, eight threads one item. With TS = 8 (the MC = 8 layout, the four lanes of an MMA on the
// four granules of one item) word w of granule g is stored at position w ^ g of the granule, so
// those lanes' 16-byte loads hit distinct banks.
template <int NT, int TS>
__device__ __forceinline__ void stripe_prepare_x(const GemvArgs& a, const StripePlan& p,
                                                 unsigned char* smem, int tid, int kw0,
                                                 int kw_per_m) {
  const int total = a.m * kw_per_m;
  unsigned char* xs = smem + p.off_xs;
  float* bq = reinterpret_cast<float*>(smem + p.off_bq);    // [items][4][TS]
  float* xsum = reinterpret_cast<float*>(smem + p.off_xsum);  // [items][TS]
  for (int base = 0; base < total; base += 4 * NT) {
    // Two steps per round: all four 16-byte loads are in flight together.
    uint4 v[4];
    int idx[2];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      idx[s] = base + s * 2 * NT + 2 * tid;
      if (idx[s] < total) {
        const int m = idx[s] / kw_per_m, kw = idx[s] - m * kw_per_m;
        const uint4* src =
            reinterpret_cast<const uint4*>(a.x + static_cast<int64_t>(m) * a.k) + kw0 + kw;
        v[2 * s] = ld_stream_v4(src);
        v[2 * s + 1] = ld_stream_v4(src + 1);
      }
    }
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      if (base + s * 2 * NT >= total) break;  // uniform over the CTA
      const bool valid = idx[s] < total;
      float bsum = 0.0f, xsm = 0.0f;
      int m = 0, kw = 0;
      if (valid) {
        m = idx[s] / kw_per_m;
        kw = idx[s] - m * kw_per_m;
        const uint4 o0 = permute_x_block(v[2 * s], bsum, xsm);
        const uint4 o1 = permute_x_block(v[2 * s + 1], bsum, xsm);
        unsigned char* item_x = xs + m * p.xs_stride + (kw >> 4) * kSxItemBytes;
        if constexpr (TS == 8) {
          const int gr = (kw >> 2) & 3, w = kw & 3;  // kw is even: words w and w + 1
          reinterpret_cast<uint4*>(item_x + (gr * 4 + (w ^ gr)) * 16)[0] = o0;
          reinterpret_cast<uint4*>(item_x + (gr * 4 + ((w + 1) ^ gr)) * 16)[0] = o1;
        } else {
          reinterpret_cast<uint4*>(item_x + (kw & 15) * 16)[0] = o0;
          reinterpret_cast<uint4*>(item_x + (kw & 15) * 16)[1] = o1;
        }
      }
      bsum += __shfl_xor_sync(0xffffffffu, bsum, 1);  // the granule (4 words) of a thread pair
      xsm += __shfl_xor_sync(0xffffffffu, xsm, 1);
      xsm += __shfl_xor_sync(0xffffffffu, xsm, 2);
      xsm += __shfl_xor_sync(0xffffffffu, xsm, 4);  // the item (16 words) of eight threads
      if (valid) {
        const int item = kw >> 4, gran = (kw >> 2) & 3;
        // the columns of rows a.m .. TS - 1 of x (absent) hold zeros
        if ((tid & 1) == 0) {
          bq[(item * 4 + gran) * TS + m] = -1024.0f * bsum;
          if (m == 0)
            for (int mm = a.m; mm < TS; ++mm) bq[(item * 4 + gran) * TS + mm] = 0.0f;
        }
        if ((tid & 7) == 0) {
          xsum[item * TS + m] = xsm;
          if (m == 0)
            for (int mm = a.m; mm < TS; ++mm) xsum[item * TS + mm] = 0.0f;
        }
      }
    }
  }
}

// One stage's operands of a consumer lane: the A words of its GPW granules in rows g, g + 8
// (tile 0) and 16 + g, 24 + g (tile 1), and those rows' scale (and zero) bits of its item.
template <int GPW>
struct StripeRegs {
  uint4 aw[GPW][2][2];  // [granule][tile][row g / g + 8]
  uint32_t sb[2][2], zb[2][2];
};

// The lane's B registers of one stripe (four words of x per granule in the permuted order), the C
// value that starts its first low-half MMA chain per tile (-1024 x the B sum of its granules, per
// row of x) and the item's x sum.
template <int GPW>
struct StripeX {
  uint4 bx[GPW][4];
  float2 cinit, xsm;
};

template <int GPW, int NT>
__device__ __forceinline__ void stripe_load(const unsigned char* st, const int (&a_off)[GPW],
                                            int s_off, int z_off, bool zero_term,
                                            StripeRegs<GPW>& r) {
#pragma unroll
  for (int t = 0; t < NT; ++t) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = 16 * t + 8 * h;
#pragma unroll
      for (int q = 0; q < GPW; ++q) {
        r.aw[q][t][h] = *reinterpret_cast<const uint4*>(st + a_off[q] + row * kSxRowBytes);
      }
      r.sb[t][h] = *reinterpret_cast<const uint16_t*>(st + s_off + row * kSxMetaRow);
      if (zero_term) r.zb[t][h] = *reinterpret_cast<const uint16_t*>(st + z_off + row * kSxMetaRow);
    }
  }
}

// TS: columns of the tables. With TS = 4 (the MC = 4 layout, one granule per lane) the lane's D
// columns also take the B values of its partner lane (c ^ 1), whose granule is gran ^ 1; m0 is
// the first of the lane's two rows of x.
// TS = 8 (the MC = 8 layout): the D columns take the B values of all four lanes (the item's four
// granules), and word u of the lane's granule sits at position u ^ swz (see stripe_prepare_x).
template <int GPW, int TS>
__device__ __forceinline__ void stripe_load_x(const unsigned char* const (&b_base)[GPW], int b_step,
                                              const float* bq, const float* xsum, int j, int item,
                                              const int (&gran)[GPW], int m0, int swz,
                                              bool zero_term, StripeX<GPW>& x) {
  const int tab = j * kSxItems + item;
  float2 ci = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int q = 0; q < GPW; ++q) {
    const unsigned char* bsrc = b_base[q] + j * b_step;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      x.bx[q][u] = *reinterpret_cast<const uint4*>(bsrc + (TS == 8 ? (u ^ swz) : u) * 16);
    }
    if constexpr (TS == 8) {
#pragma unroll
      for (int g4 = 0; g4 < 4; ++g4) {
        const float2 v = *reinterpret_cast<const float2*>(bq + (tab * 4 + g4) * TS + m0);
        ci.x += v.x;
        ci.y += v.y;
      }
      continue;
    }
    const float2 v = *reinterpret_cast<const float2*>(bq + (tab * 4 + gran[q]) * TS + m0);
    ci.x += v.x;
    ci.y += v.y;
    if constexpr (TS == 4) {
      const float2 w = *reinterpret_cast<const float2*>(bq + (tab * 4 + (gran[q] ^ 1)) * TS + m0);
      ci.x += w.x;
      ci.y += w.y;
    }
  }
  x.cinit = ci;
  x.xsm = zero_term ? *reinterpret_cast<const float2*>(xsum + tab * TS + m0)
                    : make_float2(0.0f, 0.0f);
}

// The stage's 16 GPW MMAs: per tile and granule a low-half and a high-half chain over the
// granule's four words (the first low-half chain started from C = cinit, the others from zero),
// added at the end: d[t] = sum_k q_k x_k for the lane's (rows, item) as the MMA D fragment (rows
// g, g + 8 x columns 2c, 2c + 1).
template <int GPW, int NT>
__device__ __forceinline__ void stripe_mma(const StripeRegs<GPW>& r, const StripeX<GPW>& x,
                                           float (&d)[2][4]) {
  float ch[2][2 * GPW - 1][4];  // the chains other than the first low-half one
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    d[t][0] = d[t][2] = x.cinit.x;
    d[t][1] = d[t][3] = x.cinit.y;
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
#pragma unroll
    for (int q = 0; q < GPW; ++q) {
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        uint32_t hg[4], h8[4];
        unpack_x16(word_of4(r.aw[q][t][0], u), hg);
        unpack_x16(word_of4(r.aw[q][t][1], u), h8);
        const uint32_t alo[4] = {hg[0], h8[0], hg[1], h8[1]};
        const uint32_t ahi[4] = {hg[2], h8[2], hg[3], h8[3]};
        if (q == 0) {
          mma_16816(d[t], alo, x.bx[q][u].x, x.bx[q][u].y);
        } else if (u == 0) {
          mma_16816_first(ch[t][2 * q - 1], alo, x.bx[q][u].x, x.bx[q][u].y);
        } else {
          mma_16816(ch[t][2 * q - 1], alo, x.bx[q][u].x, x.bx[q][u].y);
        }
        if (u == 0) {
          mma_16816_first(ch[t][2 * q], ahi, x.bx[q][u].z, x.bx[q][u].w);
        } else {
          mma_16816(ch[t][2 * q], ahi, x.bx[q][u].z, x.bx[q][u].w);
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
#pragma unroll
      for (int i = 0; i < 2 * GPW - 1; ++i) d[t][e] += ch[t][i][e];
    }
  }
}

// One scale per (row, item) into the row accumulators; the granule-0 warps add the zero term.
// E: the lane's D columns that hold rows of x (1 for M = 1, else 2).
template <int E, int GPW, int NT>
__device__ __forceinline__ void stripe_epilogue(const StripeRegs<GPW>& r, const float (&d)[2][4],
                                                float2 xsm, bool zero_term,
                                                float (&acc)[2][2][E]) {
#pragma unroll
  for (int t = 0; t < NT; ++t) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float s = __half2float(__ushort_as_half(static_cast<uint16_t>(r.sb[t][h])));
      const float z =
          zero_term ? __half2float(__ushort_as_half(static_cast<uint16_t>(r.zb[t][h]))) : 0.0f;
#pragma unroll
      for (int m = 0; m < E; ++m) {
        const float xz = m == 0 ? xsm.x : xsm.y;
        acc[t][h][m] = fmaf(s, fmaf(-z, xz, d[t][2 * h + m]), acc[t][h][m]);
      }
    }
  }
}

// MC: columns per group in the MMA's eight (1 or 2: four groups per MMA; 4 for M = 3 or 4: two
// groups, each over the k-slots of a lane pair). CW: consumer warps, 16 (one 4-word granule per
// lane and stage) or 8 (two; MC <= 2 only); plus one producer warp. LO: the loads-only ceiling of the same stream (no x, no MMA):
// every packed word and, once per (row, group), the scale and zero bits are XOR-folded into one
// 32-bit word per row, written to ((uint32_t*) a.y)[row].
// PN: x in K-panels (p.panels > 1); false compiles the single-panel form.
template <int MC, int CW, bool LO = false, bool PN = false>
__global__ void __launch_bounds__((CW + 1) * kWarp, 1)
    stripe_mma_kernel(GemvArgs a, StripePlan p, const __grid_constant__ StripeMaps maps,
                      const __grid_constant__ PeerSet peers) {
  constexpr int kGPW = 16 / CW;            // granules per lane and stage
  constexpr int kConsumers = CW * kWarp;
  constexpr int kTS = MC <= 2 ? 2 : MC;     // columns of the x tables
  constexpr int kE = MC == 1 ? 1 : 2;       // the lane's D columns that hold rows of x
  static_assert(MC <= 2 || CW == 16, "the MC = 4 and 8 layouts take one granule per lane");
  extern __shared__ __align__(1024) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kSxMaxStages;
  unsigned char* stages = smem + p.off_stage;
  float* red = reinterpret_cast<float*>(smem + p.off_red);  // [CW warps][rows_cap][MC]

  const int tid = threadIdx.x;
  const int warp = tid / kWarp;
  const int lane = tid % kWarp;

  const int u0 = static_cast<int>(static_cast<int64_t>(blockIdx.x) * p.units / p.ctas);
  const int u1 = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * p.units / p.ctas);
  const int row_begin = 4 * u0;
  const int rows = min(4 * u1, a.n) - row_begin;
  const int blocks = (rows + kSxRows - 1) / kSxRows;

  if (tid == kConsumers) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], CW);
    }
    fence_mbar_init();
  }
  for (int i = tid; i < 512 / 16; i += (CW + 1) * kWarp) {
    reinterpret_cast<uint4*>(smem + kSxZeroOff)[i] = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  if (tid == 0) launch_dependents();  // the next GEMV may launch as SMs free up

  if (warp == CW) {
    stripe_produce(p, maps, row_begin, rows, smem);
    return;
  }

  // ---------------- consumers ----------------
  grid_dependency_wait();  // x may come from the previous kernel in the stream

  const int g = lane >> 2, c = lane & 3;
  // MC <= 2: lane c takes item 4 (w % 4) + c (column pair c), granule set w / 4 (kGPW granules);
  //   column g is (item g / 2, row of x g % 2).
  // MC = 4: lanes c and c ^ 1 take item 2 (w % 8) + c / 2 (columns 4 (c / 2) .. + 3), with the
  //   granules 2 (w / 8) + c % 2; column g is (item g / 4, row of x g % 4), and the lane's D
  //   columns 2c, 2c + 1 are rows m0 = 2 (c % 2) and m0 + 1 of its item.
  // MC = 8: warp w takes item w, lane c its granule c; column g is row g of x, and the lane's D
  //   columns are rows m0 = 2c and m0 + 1.
  // A k-slot's word depends on c only (never on g): B column g is supplied by the lanes of row g.
  const int iq = MC == 8 ? warp : MC == 4 ? (warp & 7) : (warp & 3);
  const int wq = MC == 8 ? 0 : MC == 4 ? (warp >> 3) : (warp >> 2);
  const int item = MC == 8 ? iq : MC == 4 ? 2 * iq + (c >> 1) : 4 * iq + c;  // in a stripe
  const bool zero_term = wq == 0;  // the warps holding granule 0 of their items add the zero term
  // the row of x whose B values this lane holds
  const int xm = MC == 8 ? g : MC == 4 ? (g & 3) : g - 2 * c;
  const bool has_x = MC == 8   ? xm < a.m
                     : MC == 4 ? ((g >> 2) == (c >> 1) && xm < a.m)
                               : (xm >= 0 && xm < MC);
  const int m0 = MC == 8 ? 2 * c : MC == 4 ? 2 * (c & 1) : 0;
  const unsigned char* xs = smem + p.off_xs;
  const float* bq = reinterpret_cast<const float*>(smem + p.off_bq);
  const float* xsum = reinterpret_cast<const float*>(smem + p.off_xsum);
  int gran[kGPW], a_off[kGPW];
  const unsigned char* b_base[kGPW];
#pragma unroll
  for (int q = 0; q < kGPW; ++q) {
    // MC <= 2: granules rotated by c / 2 so the 16-byte loads of one shared-memory phase hit
    // distinct banks
    gran[q] = MC == 8 ? c : MC == 4 ? 2 * wq + (c & 1) : (kGPW * wq + q + (c >> 1)) & 3;
    a_off[q] = g * kSxRowBytes + item * 64 + gran[q] * 16;
    b_base[q] = has_x ? xs + xm * p.xs_stride + item * kSxItemBytes + gran[q] * 64
                      : smem + kSxZeroOff;
  }
  const int b_step = has_x ? kSxItems * kSxItemBytes : 0;
  const int s_off = kSxSOff + g * kSxMetaRow + item * 2;
  const int z_off = kSxZOff + g * kSxMetaRow + item * 2;

  // Per stage: wait for it, load the lane's weights, scales and x, issue the MMAs, run the stage
  // epilogue, release the stage. (Loading the next stage's operands during this stage's MMAs was
  // measured slower on B200.)
  StageRingSx ring{full, p.stages, p.status, true, 0, 0u};
  // One block of rows: NT 16-row tiles (2, or 1 when the block has at most 16 rows), a
  // compile-time count so the two tiles' MMAs interleave freely.
  auto run_block = [&]<int NT>(int blk, int rows_b, int j0, int j1, bool accumulate) {
    if constexpr (LO) {
      uint32_t f[2][2] = {{0u, 0u}, {0u, 0u}};  // [tile][row g / g + 8]
      for (int j = j0; j < j1; ++j) {
        const int slot = ring.next();
        StripeRegs<kGPW> r;
        stripe_load<kGPW, NT>(stages + slot * kSxStageBytes, a_off, s_off, z_off, zero_term, r);
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int q = 0; q < kGPW; ++q) f[t][h] ^= fold4(r.aw[q][t][h]);
            if (zero_term) f[t][h] ^= r.sb[t][h] | (r.zb[t][h] << 16);
          }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);  // after the folds: every load has returned
      }
      uint32_t* redu = reinterpret_cast<uint32_t*>(red);
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t v = f[t][h];
          v ^= __shfl_xor_sync(0xffffffffu, v, 1);
          v ^= __shfl_xor_sync(0xffffffffu, v, 2);
          if (c == 0 && 16 * t + 8 * h + g < rows_b) {
            uint32_t* dst = &redu[warp * p.rows_cap + blk * kSxRows + 16 * t + 8 * h + g];
            *dst = accumulate ? *dst ^ v : v;
          }
        }
      return;
    }
    float acc[2][2][kE];  // [tile][row g / g + 8][row of x m0 + e]
#pragma unroll
    for (int t = 0; t < 2; ++t)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int e = 0; e < kE; ++e) acc[t][h][e] = 0.0f;
    for (int j = j0; j < j1; ++j) {
      const int slot = ring.next();
      StripeRegs<kGPW> r;
      stripe_load<kGPW, NT>(stages + slot * kSxStageBytes, a_off, s_off, z_off, zero_term, r);
      StripeX<kGPW> xr;
      stripe_load_x<kGPW, kTS>(b_base, b_step, bq, xsum, j - j0, item, gran, m0, c, zero_term,
                               xr);
      float d[2][4];
      stripe_mma<kGPW, NT>(r, xr, d);
      stripe_epilogue<kE, kGPW, NT>(r, d, xr.xsm, zero_term, acc);
      // Release the stage only after its values have been used: mbarrier.arrive does not wait
      // for shared-memory loads still in flight, and a refill served from L2 can land within a
      // few hundred nanoseconds. (Releasing here measured as fast as releasing right after the
      // loads.)
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);  // the stage may be refilled
    }
    // the items of this warp (four, two for MC = 4, one for MC = 8), then one partial per
    // (row, m) and warp, added to the earlier K-panels' in panel order
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int e = 0; e < kE; ++e) {
          float v = acc[t][h][e];
          if constexpr (MC <= 2) v += __shfl_xor_sync(0xffffffffu, v, 1);
          if constexpr (MC <= 4) v += __shfl_xor_sync(0xffffffffu, v, 2);
          const bool writer = MC == 8 ? true : MC == 4 ? c < 2 : c == 0;
          if (writer && 16 * t + 8 * h + g < rows_b) {
            float* dst = &red[(warp * p.rows_cap + blk * kSxRows + 16 * t + 8 * h + g) * MC + m0 + e];
            *dst = accumulate ? *dst + v : v;
          }
        }
  };
  const int panels = PN ? p.panels : 1;
  for (int pn = 0; pn < panels; ++pn) {
    const int j0 = PN ? pn * p.stripes / p.panels : 0;
    const int j1 = PN ? (pn + 1) * p.stripes / p.panels : p.stripes;
    if constexpr (!LO) {
      if (pn > 0) named_barrier(kSxBarrier, kConsumers);  // the last panel's x is no longer read
      stripe_prepare_x<kConsumers, kTS>(a, p, smem, tid, j0 * (kSxK / 8), (j1 - j0) * (kSxK / 8));
      named_barrier(kSxBarrier, kConsumers);
    }
    for (int blk = 0; blk < blocks; ++blk) {
      const int rows_b = min(kSxRows, rows - blk * kSxRows);
      if (rows_b > 16) {  // uniform over the CTA
        run_block.template operator()<2>(blk, rows_b, j0, j1, PN && pn > 0);
      } else {
        run_block.template operator()<1>(blk, rows_b, j0, j1, PN && pn > 0);
      }
    }
  }

  // ---- add the CW partials of every output in a fixed order; store fp16 ---------------------
  named_barrier(kSxBarrier, kConsumers);
  if constexpr (LO) {
    const uint32_t* redu = reinterpret_cast<const uint32_t*>(red);
    for (int r = tid; r < rows; r += kConsumers) {
      uint32_t v = 0;
#pragma unroll
      for (int w = 0; w < CW; ++w) v ^= redu[w * p.rows_cap + r];
      if (ring.ok) reinterpret_cast<uint32_t*>(a.y)[row_begin + r] = v;
    }
    return;
  }
  auto row_sum = [&](int r, int m) {
    float sum = 0.0f;
#pragma unroll
    for (int w = 0; w < CW; ++w) sum += red[(w * p.rows_cap + r) * MC + m];
    return sum;
  };
  if (a.epilogue == kGatherPeers) {
    // Rows split over ranks: this rank's columns of y, each as a tagged word (fp16 bits, call
    // number), into every other rank's gather buffer and straight into this rank's y; then the
    // same rows of every other rank's shard, each once its tag shows this call.
    const unsigned epoch = exchange_epoch(peers);
    named_barrier(kSxBarrier, kConsumers);  // every thread has read the call number
    for (int o = tid; o < rows * a.m; o += kConsumers) {
      const int m = o / rows;
      const int r = o - m * rows;
      const unsigned h = __half_as_ushort(__float2half_rn(row_sum(r, m)));
      const int64_t at = static_cast<int64_t>(m) * peers.n_total + peers.col0 + row_begin + r;
      for (int q = 0; q < peers.world; ++q) {
        if (q == peers.rank) {
          if (ring.ok) a.y[at] = __ushort_as_half(static_cast<unsigned short>(h));
        } else {
          st_tagged(exchange_words(peers, q, epoch) + at, h, epoch);
        }
      }
    }
    const unsigned long long* buf = exchange_words(peers, peers.rank, epoch);
    bool live = true;
    for (int o = tid; o < peers.world * rows * a.m; o += kConsumers) {
      const int q = o / (rows * a.m);
      if (q == peers.rank) continue;
      const int rem = o - q * rows * a.m;
      const int m = rem / rows;
      const int r = rem - m * rows;
      const int64_t at = static_cast<int64_t>(m) * peers.n_total + q * a.n + row_begin + r;
      const unsigned h = exchange_read(buf + at, epoch, &live, p.status);
      if (ring.ok) a.y[at] = __ushort_as_half(static_cast<unsigned short>(h));
    }
    exchange_done(peers, epoch, tid);
    return;
  }
  if (a.epilogue == kReducePeers) {
    // K split over ranks: this rank's fp32 partial sums, as tagged words, into slot `rank` of
    // every other rank's buffer; then the ranks' partials of this CTA's rows added in rank order
    // (this rank's own from shared memory), the same on every rank.
    const unsigned epoch = exchange_epoch(peers);
    named_barrier(kSxBarrier, kConsumers);  // every thread has read the call number
    const int64_t slot = static_cast<int64_t>(a.m) * a.n;
    for (int o = tid; o < rows * a.m; o += kConsumers) {
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
    for (int o = tid; o < rows * a.m; o += kConsumers) {
      const int m = o / rows;
      const int r = o - m * rows;
      const int64_t at = static_cast<int64_t>(m) * a.n + row_begin + r;
      float total = 0.0f;
      for (int q = 0; q < peers.world; ++q) {
        total += q == peers.rank
                     ? row_sum(r, m)
                     : __uint_as_float(exchange_read(mine + q * slot + at, epoch, &live, p.status));
      }
      if (ring.ok) a.y[at] = store_value(a, m, row_begin + r, total);
    }
    exchange_done(peers, epoch, tid);
    return;
  }
  for (int o = tid; o < rows * a.m; o += kConsumers) {
    const int m = o / rows;
    const int r = o - m * rows;
    const float sum = row_sum(r, m);
    if (ring.ok) {
      a.y[static_cast<int64_t>(m) * a.n + row_begin + r] = store_value(a, m, row_begin + r, sum);
    }
  }
}

// ---- host ---------------------------------------------------------------------------------------

bool stripe_plan(const GemvArgs& a, StripePlan* p, const char** why) {
  auto fail = [&](const char* reason) {
    if (why) *why = reason;
    return false;
  };
  if (a.m < 1 || a.m > 8) return fail("M must be in [1, 8]");
  if (a.group != kItemK) return fail("group_size must be 128");
  if (a.k % kSxK != 0) return fail("K must be a multiple of 2048");
  if (a.epilogue != kStoreY && a.epilogue != kGatherPeers && a.epilogue != kReducePeers)
    return fail("plain stores or the fused exchange only");
  if (reinterpret_cast<uintptr_t>(a.q) % 16 || reinterpret_cast<uintptr_t>(a.s) % 16 ||
      reinterpret_cast<uintptr_t>(a.z) % 16 || reinterpret_cast<uintptr_t>(a.x) % 16) {
    return fail("x, qweight, scales and zeros must be 16-byte aligned");
  }
  p->units = (a.n + 3) / 4;
  p->ctas = std::min(sm_count(), p->units);
  p->rows_cap = 4 * ((p->units + p->ctas - 1) / p->ctas);
  p->stripes = a.k / kSxK;
  p->items = a.k / kItemK;
  const int mc = a.m <= 2 ? a.m : a.m <= 4 ? 4 : 8;  // the kernel's MC
  const int ts = a.m <= 2 ? 2 : mc;                   // columns of the x tables
  // The fewest K-panels (1, 2, 4, ... stripes) whose permuted x, tables and partials leave room
  // for the three-stripe ring.
  for (int panels = 1;; panels *= 2) {
    // (M <= 2 keeps all of x: the single-panel kernels only)
    if (panels > p->stripes || (a.m <= 2 && panels > 1)) {
      return fail("x does not fit in shared memory");
    }
    p->panels = panels;
    const int items = (p->stripes + panels - 1) / panels * kSxItems;  // of the longest panel
    p->xs_stride = items * kSxItemBytes;
    if (mc == 8) p->xs_stride += (64 - p->xs_stride % 128 + 128) % 128;  // rows 64 B apart in banks
    int64_t off = kSxHeader;
    p->off_xs = static_cast<int>(off);
    off += static_cast<int64_t>(a.m) * p->xs_stride;
    p->off_bq = static_cast<int>(off);
    off += static_cast<int64_t>(items) * 4 * ts * 4;
    p->off_xsum = static_cast<int>(off);
    off += static_cast<int64_t>(items) * ts * 4;
    p->off_red = static_cast<int>(off);
    off += static_cast<int64_t>(16) * p->rows_cap * mc * 4;  // partials of up to 16 warps
    off = (off + 1023) / 1024 * 1024;
    p->off_stage = static_cast<int>(off);
    if (off >= kSxSmemLimit) continue;
    const int64_t stages =
        std::min<int64_t>((kSxSmemLimit - off) / kSxStageBytes, kSxMaxStages);
    if (stages < kSxMinStages) continue;
    p->stages = static_cast<int>(stages);
    p->smem_bytes = static_cast<int>(off + stages * kSxStageBytes);
    break;
  }
  p->strict = 0;
  p->status = nullptr;
  return true;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 stripe_encode_fn() {
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

struct StripeMapEntry {
  int dev;
  const void* q;
  const void* s;
  const void* z;
  int n, k;
  StripeMaps maps;
};
std::mutex g_stripe_mu;
std::vector<StripeMapEntry> g_stripe_maps;  // most recently used first
constexpr size_t kStripeMapCache = 64;

cudaError_t stripe_maps_for(const GemvArgs& a, StripeMaps* out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  std::lock_guard<std::mutex> lock(g_stripe_mu);
  for (size_t i = 0; i < g_stripe_maps.size(); ++i) {
    const StripeMapEntry& e = g_stripe_maps[i];
    if (e.dev == dev && e.q == a.q && e.s == a.s && e.z == a.z && e.n == a.n && e.k == a.k) {
      *out = e.maps;
      if (i != 0) std::swap(g_stripe_maps[i], g_stripe_maps[0]);
      return cudaSuccess;
    }
  }
  auto encode = stripe_encode_fn();
  if (!encode) return cudaErrorNotSupported;
  StripeMapEntry e{dev, a.q, a.s, a.z, a.n, a.k, {}};
  const cuuint32_t estr[2] = {1, 1};
  const int groups = a.k / a.group;
  for (int hi = 0; hi < 4; ++hi) {
    const cuuint32_t h = static_cast<cuuint32_t>(kSxRows >> hi);
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(a.k / 8), static_cast<cuuint64_t>(a.n)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.k / 2)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kSxRowBytes / 4), h};
    if (encode(&e.maps.q[hi], CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(a.q), dims,
               strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      return cudaErrorInvalidValue;
    }
    const cuuint64_t sdims[2] = {static_cast<cuuint64_t>(groups), static_cast<cuuint64_t>(a.n)};
    const cuuint64_t sstrides[1] = {static_cast<cuuint64_t>(groups) * 2};
    const cuuint32_t sbox[2] = {static_cast<cuuint32_t>(kSxItems), h};
    for (int which = 0; which < 2; ++which) {
      if (encode(which == 0 ? &e.maps.s[hi] : &e.maps.z[hi], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2,
                 const_cast<half*>(which == 0 ? a.s : a.z), sdims, sstrides, sbox, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                 CU_TENSOR_MAP_L2_PROMOTION_NONE,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
        return cudaErrorInvalidValue;
      }
    }
  }
  g_stripe_maps.insert(g_stripe_maps.begin(), e);
  if (g_stripe_maps.size() > kStripeMapCache) g_stripe_maps.pop_back();
  *out = e.maps;
  return cudaSuccess;
}

#ifndef STRIPE_CW
#define STRIPE_CW 16
#endif
// Kernel instances (rows of x, consumer warps).
template <typename F>
cudaError_t with_stripe_m(int m, int panels, F&& f) {
  if (m <= 1) return f.template operator()<1, STRIPE_CW, false>();
  if (m == 2) return f.template operator()<2, STRIPE_CW, false>();
  if (m <= 4) {
    if (panels > 1) return f.template operator()<4, 16, true>();
    return f.template operator()<4, 16, false>();
  }
  if (panels > 1) return f.template operator()<8, 16, true>();
  return f.template operator()<8, 16, false>();
}

std::once_flag g_stripe_attr_once[8][2][64];

}  // namespace

bool stripe_mma_supported(const GemvArgs& a, const char** why) {
  StripePlan p;
  return stripe_plan(a, &p, why);
}

cudaError_t launch_stripe_mma(const GemvArgs& a, cudaStream_t stream, bool strict,
                              const PeerSet* peers) {
  const bool exchange = a.epilogue == kGatherPeers || a.epilogue == kReducePeers;
  if (exchange != (peers != nullptr)) return cudaErrorInvalidValue;
  PeerSet ps{};
  if (peers) ps = *peers;
  StripePlan p;
  if (!stripe_plan(a, &p, nullptr)) return cudaErrorInvalidValue;
  p.strict = strict ? 1 : 0;
  p.status = device_status_word();
  if (!p.status) return cudaErrorInvalidSymbol;
  StripeMaps maps;
  const cudaError_t merr = stripe_maps_for(a, &maps);
  if (merr != cudaSuccess) return merr;
  int dev = 0;
  const cudaError_t derr = cudaGetDevice(&dev);
  if (derr != cudaSuccess) return derr;
  return with_stripe_m(a.m, p.panels, [&]<int MC, int CW, bool PN>() {
    cudaError_t result = cudaSuccess;
    std::call_once(g_stripe_attr_once[MC - 1][PN ? 1 : 0][dev & 63], [&] {
      result = cudaFuncSetAttribute(stripe_mma_kernel<MC, CW, false, PN>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kSxSmemLimit);
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
    return cudaLaunchKernelEx(&cfg, stripe_mma_kernel<MC, CW, false, PN>, a, p, maps, ps);
  });
}

cudaError_t launch_stripe_load_only(uint32_t* out, const GemvArgs& args, cudaStream_t stream) {
  GemvArgs a = args;
  a.y = reinterpret_cast<half*>(out);
  a.x = nullptr;
  a.m = 1;
  a.epilogue = kStoreY;
  StripePlan p;
  if (!stripe_plan(a, &p, nullptr)) return cudaErrorInvalidValue;
  p.strict = 0;
  p.status = device_status_word();
  if (!p.status) return cudaErrorInvalidSymbol;
  StripeMaps maps;
  const cudaError_t merr = stripe_maps_for(a, &maps);
  if (merr != cudaSuccess) return merr;
  int dev = 0;
  const cudaError_t derr = cudaGetDevice(&dev);
  if (derr != cudaSuccess) return derr;
  static std::once_flag attr_once[64];
  cudaError_t result = cudaSuccess;
  std::call_once(attr_once[dev & 63], [&] {
    result = cudaFuncSetAttribute(stripe_mma_kernel<1, STRIPE_CW, true>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, kSxSmemLimit);
  });
  if (result != cudaSuccess) return result;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.ctas);
  cfg.blockDim = dim3((STRIPE_CW + 1) * kWarp);
  cfg.dynamicSmemBytes = p.smem_bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, stripe_mma_kernel<1, STRIPE_CW, true>, a, p, maps, PeerSet{});
}

cudaError_t stripe_mma_attrs(int m, KernelAttrs* out) {
  const int mm = m < 1 ? 1 : m > 8 ? 8 : m;
  return with_stripe_m(mm, 1, [&]<int MC, int CW, bool PN>() {
    cudaFuncAttributes fa;
    cudaError_t err = cudaFuncGetAttributes(&fa, stripe_mma_kernel<MC, CW, false, PN>);
    if (err != cudaSuccess) return err;
    out->registers = fa.numRegs;
    out->local_bytes = static_cast<int>(fa.localSizeBytes);
    out->max_threads_per_block = fa.maxThreadsPerBlock;
    out->blocks_per_sm = 1;
    out->threads_per_block = (CW + 1) * kWarp;
    return cudaSuccess;
  });
}

}  // namespace i4
