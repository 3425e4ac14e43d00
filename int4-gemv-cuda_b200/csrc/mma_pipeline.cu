// The B200 fast path for small M (1..16): a persistent, warp-specialised W4A16 GEMV.
//
// Work split. One CTA per SM. CTA c owns output rows [c N / P, (c + 1) N / P): every CTA streams
// the same number of weight bytes (within one row), whatever N is, so there is no wave tail. A
// CTA walks its rows in chunks of at most 128 rows and each chunk in k-blocks of KB weights.
//
// Memory side. A producer warp streams each (chunk, k-block) stage into a ring of shared-memory
// buffers with 1-D bulk copies (cp.async.bulk, one per weight row, completion counted on an
// mbarrier in bytes, L2 evict-first since the weights are read once). The stage's scales and zeros
// come in with 4-byte cp.async on the same mbarrier. Rows are padded to a stride of 64 mod 128
// bytes so the consumers' 16-byte shared loads are bank-conflict free.
//
// Math side. Eight consumer warps each own a 16-row tile of the chunk (and, when the chunk has
// fewer than 8 tiles, a subset of the stage's groups). Per packed word a thread does one shift and
// four LOP3s to get fp16 operands 1024 + q or 1024 + 16 q (exact), and feeds them as the A operand
// of mma.sync m16n8k16 (fp32 accumulate); B holds x, one column per row of x (M <= 8 per n-tile).
// Within each 8-weight block x is permuted and the 16x lanes are pre-divided by 16 once per CTA
// (x_perm), so the A operand needs no shuffling. The zero point and the 1024 offset are removed
// in fp32 once per (row, group):
//     sum_k (q_k - z) s x_k = s * (sum_k a_k b_k - 1024 sum_k b_k - z sum_k x_k)
// where a_k b_k are the MMA operands; the two sums over x come from a per-CTA table. This keeps
// the CUDA-core cost near 6 instructions per 8 weights, well inside the issue budget that HBM3e
// bandwidth leaves per byte.
//
// Every mbarrier wait is bounded (about a second); on timeout the kernel records a status word
// (read by int4gemv_device_status), skips the remaining work without leaving any barrier
// unmatched, waits (bounded) for its own bulk copies and returns.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace i4 {

__device__ int g_status;

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * kWarp;
constexpr int kThreads = kConsumerThreads + kWarp;
constexpr int kMaxStages = 8;
constexpr int kMaxChunkRows = 128;
constexpr int kSmemLimit = 227 * 1024;
constexpr int kConsumerBarrier = 1;

struct Plan {
  int ctas;
  int kb;          // weights per row per stage (multiple of 2 * group and of the k-step)
  int num_kb;
  int stages;
  int row_stride;  // bytes per weight row in a stage buffer
  int rows_cap;    // rows per chunk, upper bound
  int sz_per_row;  // scales (and zeros) per row per stage = kb / group
  int stage_bytes;
  int off_xperm, off_corr, off_red, off_stages;
  int smem_bytes;
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

__device__ __forceinline__ float h2f_bits(uint16_t b) { return __half2float(__ushort_as_half(b)); }

constexpr int kStatusBadPlan = 3;

// NT: n-tiles of 8 rows of x (M <= 8 NT). KSW: packed words per thread per k-step; 4 when
// group % 128 == 0 (a thread reads 16 contiguous bytes per row), else 1 (group % 32 == 0).
template <int NT, int KSW>
__global__ void __launch_bounds__(kThreads, 1) mma_pipeline_kernel(GemvArgs a, Plan p) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  half* xperm = reinterpret_cast<half*>(smem + p.off_xperm);
  float2* corr = reinterpret_cast<float2*>(smem + p.off_corr);
  float* red = reinterpret_cast<float*>(smem + p.off_red);
  unsigned char* stages = smem + p.off_stages;

  const int warp = threadIdx.x / kWarp;
  const int lane = threadIdx.x % kWarp;
  const int groups = a.k / a.group;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1 + kWarp);  // producer's expect_tx + one cp.async arrival per lane
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  const int cta = blockIdx.x;
  const int row_begin = static_cast<int>(static_cast<int64_t>(cta) * a.n / p.ctas);
  const int row_end = static_cast<int>(static_cast<int64_t>(cta + 1) * a.n / p.ctas);
  const int rows = row_end - row_begin;
  // Chunks of at most p.rows_cap rows (the host sized the stage buffers for that many).
  const int chunks = (rows + p.rows_cap - 1) / p.rows_cap;
  const int kwords = a.k / 8;

  if (warp == kConsumerWarps) {
    // ---------------- producer warp ----------------
    const uint64_t policy = l2_evict_first_policy();
    bool ok = true;
    int it = 0;
    for (int ci = 0; ci < chunks; ++ci) {
      const int c0 = row_begin + static_cast<int>(static_cast<int64_t>(ci) * rows / chunks);
      const int c1 = row_begin + static_cast<int>(static_cast<int64_t>(ci + 1) * rows / chunks);
      const int crows = c1 - c0;
      if (crows > p.rows_cap && ok) {  // never copy past a stage buffer
        ok = false;
        if (lane == 0) atomicExch(&g_status, kStatusBadPlan);
      }
      for (int kbi = 0; kbi < p.num_kb; ++kbi, ++it) {
        const int slot = it % p.stages;
        const int use = it / p.stages;
        if (ok && use > 0 && !mbar_wait_bounded(&empty[slot], (use - 1) & 1)) {
          ok = false;
          if (lane == 0) atomicExch(&g_status, kStatusEmptyBarrierTimeout);
        }
        if (!ok) continue;
        const int k0 = kbi * p.kb;
        const int klen = min(p.kb, a.k - k0);
        const int ng = klen / a.group;
        unsigned char* st = stages + static_cast<size_t>(slot) * p.stage_bytes;
        half* st_s = reinterpret_cast<half*>(st + p.rows_cap * p.row_stride);
        half* st_z = st_s + p.rows_cap * p.sz_per_row;
        if (lane == 0) mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(crows * (klen / 2)));
        __syncwarp();
        for (int r = lane; r < crows; r += kWarp) {
          const int64_t row = c0 + r;
          bulk_g2s(st + r * p.row_stride,
                   reinterpret_cast<const unsigned char*>(a.q) + row * (a.k / 2) + k0 / 2,
                   static_cast<uint32_t>(klen / 2), &full[slot], policy);
          const half* srow = a.s + row * groups + k0 / a.group;
          const half* zrow = a.z + row * groups + k0 / a.group;
          for (int j = 0; j < ng; j += 2) {
            cp_async_4(st_s + r * p.sz_per_row + j, srow + j);
            cp_async_4(st_z + r * p.sz_per_row + j, zrow + j);
          }
        }
        cp_async_arrive_noinc(&full[slot]);
      }
    }
    // Do not leave while bulk copies into this CTA's shared memory may be in flight.
    if (ok) {
      for (int back = 1; back <= min(it, p.stages); ++back) {
        const int j = it - back;
        if (!mbar_wait_bounded(&full[j % p.stages], (j / p.stages) & 1)) break;
      }
    }
    return;
  }

  // ---------------- consumer warps ----------------
  const int tid = threadIdx.x;
  const int g = lane >> 2;  // row within the mma tile (and row of x for B)
  const int c = lane & 3;   // k-slot pair within the mma tile

  // x_perm: each 8-weight block [x0..x7] becomes [x0, x4, x1/16, x5/16, x2, x6, x3/16, x7/16], the
  // B operands matching unpack_x16's A operands.
  {
    const __half2 sixteenth = __float2half2_rn(0.0625f);
    const int blocks = a.m * kwords;
    for (int b = tid; b < blocks; b += kConsumerThreads) {
      const uint4 v = *reinterpret_cast<const uint4*>(a.x + static_cast<int64_t>(b) * 8);
      uint4 o;
      o.x = prmt(v.x, v.z, 0x5410);
      o.y = hmul2_bits(prmt(v.x, v.z, 0x7632), sixteenth);
      o.z = prmt(v.y, v.w, 0x5410);
      o.w = hmul2_bits(prmt(v.y, v.w, 0x7632), sixteenth);
      *reinterpret_cast<uint4*>(xperm + static_cast<int64_t>(b) * 8) = o;
    }
    named_barrier(kConsumerBarrier, kConsumerThreads);
    // corr[m][grp] = (1024 * sum of B operands, sum of the x values they stand for): one warp
    // per (row of x, group), lanes over 8-weight blocks, fixed shuffle tree (deterministic).
    for (int idx = warp; idx < a.m * groups; idx += kConsumerWarps) {
      const int mrow = idx / groups;
      const int grp = idx % groups;
      const half* blk = xperm + static_cast<int64_t>(mrow) * a.k + grp * a.group;
      float bsum = 0.0f, xsum = 0.0f;
      for (int j = lane; j < a.group / 8; j += kWarp) {
        const uint4 v = *reinterpret_cast<const uint4*>(blk + 8 * j);
        const float2 p0 = half2_bits_to_float2(v.x), p1 = half2_bits_to_float2(v.y);
        const float2 p2 = half2_bits_to_float2(v.z), p3 = half2_bits_to_float2(v.w);
        const float ones = (p0.x + p0.y) + (p2.x + p2.y);
        const float sixteenths = (p1.x + p1.y) + (p3.x + p3.y);
        bsum += ones + sixteenths;
        xsum += ones + 16.0f * sixteenths;
      }
      bsum = warp_sum(bsum);
      xsum = warp_sum(xsum);
      if (lane == 0) corr[idx] = make_float2(1024.0f * bsum, xsum);
    }
    named_barrier(kConsumerBarrier, kConsumerThreads);
  }

  constexpr int kStepK = 32 * KSW;  // weights per row per k-step (4 threads x KSW words x 8)
  bool ok = true;
  int it = 0;
  for (int ci = 0; ci < chunks; ++ci) {
    const int c0 = row_begin + static_cast<int>(static_cast<int64_t>(ci) * rows / chunks);
    const int c1 = row_begin + static_cast<int>(static_cast<int64_t>(ci + 1) * rows / chunks);
    const int crows = c1 - c0;
    if (crows > p.rows_cap) ok = false;  // the producer records the status
    const int tiles_used = (crows + 15) / 16;
    const int T = tiles_used <= 1 ? 1 : tiles_used <= 2 ? 2 : tiles_used <= 4 ? 4 : 8;
    const int tile = warp % T;
    const int sub = warp / T;
    const int nsub = kConsumerWarps / T;
    const bool active = tile < tiles_used;
    const int rowA = 16 * tile + g;  // chunk-local rows of this thread's accumulators
    const int rowB = rowA + 8;

    float yacc[NT][4] = {};
    for (int kbi = 0; kbi < p.num_kb; ++kbi, ++it) {
      const int slot = it % p.stages;
      if (ok && !mbar_wait_bounded(&full[slot], (it / p.stages) & 1)) {
        ok = false;
        atomicExch(&g_status, kStatusFullBarrierTimeout);
      }
      if (ok && active) {
        const int k0 = kbi * p.kb;
        const int klen = min(p.kb, a.k - k0);
        const int ng = klen / a.group;
        const unsigned char* st = stages + static_cast<size_t>(slot) * p.stage_bytes;
        const uint16_t* st_s =
            reinterpret_cast<const uint16_t*>(st + p.rows_cap * p.row_stride);
        const uint16_t* st_z = st_s + p.rows_cap * p.sz_per_row;
        const unsigned char* qa_row = st + rowA * p.row_stride;
        const unsigned char* qb_row = st + rowB * p.row_stride;
        for (int gl = sub; gl < ng; gl += nsub) {
          float accE[NT][4] = {}, accO[NT][4] = {};
          for (int ks = 0; ks < a.group / kStepK; ++ks) {
            const int kk = gl * a.group + ks * kStepK;  // stage-local weight offset of the k-step
            uint32_t qa[KSW], qb[KSW];
            if constexpr (KSW == 4) {
              const uint4 va = *reinterpret_cast<const uint4*>(qa_row + kk / 2 + 16 * c);
              const uint4 vb = *reinterpret_cast<const uint4*>(qb_row + kk / 2 + 16 * c);
              qa[0] = va.x, qa[1] = va.y, qa[2] = va.z, qa[3] = va.w;
              qb[0] = vb.x, qb[1] = vb.y, qb[2] = vb.z, qb[3] = vb.w;
            } else {
              qa[0] = *reinterpret_cast<const uint32_t*>(qa_row + kk / 2 + 4 * c);
              qb[0] = *reinterpret_cast<const uint32_t*>(qb_row + kk / 2 + 4 * c);
            }
#pragma unroll
            for (int i = 0; i < KSW; ++i) {
              uint32_t P[4], Q[4];
              unpack_x16(qa[i], P);
              unpack_x16(qb[i], Q);
              const uint32_t a_lo[4] = {P[0], Q[0], P[1], Q[1]};
              const uint32_t a_hi[4] = {P[2], Q[2], P[3], Q[3]};
              const int kglob = k0 + kk + 8 * (KSW * c + i);
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) {
                const int mrow = g + 8 * nt;
                uint4 b = make_uint4(0, 0, 0, 0);
                if (mrow < a.m) {
                  b = *reinterpret_cast<const uint4*>(xperm + static_cast<int64_t>(mrow) * a.k +
                                                      kglob);
                }
                mma_16816(accE[nt], a_lo, b.x, b.y);
                mma_16816(accO[nt], a_hi, b.z, b.w);
              }
            }
          }
          // Group epilogue: y += s * (acc - 1024 sum b - z sum x), per (row, column of x).
          const int grp = k0 / a.group + gl;
          const float sA = h2f_bits(st_s[rowA * p.sz_per_row + gl]);
          const float zA = h2f_bits(st_z[rowA * p.sz_per_row + gl]);
          const float sB = h2f_bits(st_s[rowB * p.sz_per_row + gl]);
          const float zB = h2f_bits(st_z[rowB * p.sz_per_row + gl]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int col = min(8 * nt + 2 * c + (i & 1), a.m - 1);
              const float2 cr = corr[col * groups + grp];
              const float s = i < 2 ? sA : sB;
              const float z = i < 2 ? zA : zB;
              const float t = fmaf(-z, cr.y, (accE[nt][i] + accO[nt][i]) - cr.x);
              yacc[nt][i] = fmaf(s, t, yacc[nt][i]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }

    // Chunk epilogue: add the warps that share a tile (fixed order) and store fp16.
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      *reinterpret_cast<float4*>(red + ((warp * kWarp + lane) * NT + nt) * 4) =
          make_float4(yacc[nt][0], yacc[nt][1], yacc[nt][2], yacc[nt][3]);
    }
    named_barrier(kConsumerBarrier, kConsumerThreads);
    if (ok) {
      for (int o = tid; o < crows * a.m; o += kConsumerThreads) {
        const int r = o % crows;
        const int mcol = o / crows;
        const int t = r / 16, rr = r % 16;
        const int src_lane = (rr % 8) * 4 + (mcol % 8) / 2;
        const int i = (rr / 8) * 2 + (mcol & 1);
        const int nt = mcol / 8;
        float sum = 0.0f;
        for (int w = t; w < kConsumerWarps; w += T) {
          sum += red[((w * kWarp + src_lane) * NT + nt) * 4 + i];
        }
        a.y[static_cast<int64_t>(mcol) * a.n + c0 + r] = store_value(a, mcol, c0 + r, sum);
      }
    }
    named_barrier(kConsumerBarrier, kConsumerThreads);
  }
}

template <typename F>
cudaError_t with_variant(int m, int group, F&& f) {
  const bool wide = group % 128 == 0;
  if (m <= 8) {
    return wide ? f.template operator()<1, 4>() : f.template operator()<1, 1>();
  }
  return wide ? f.template operator()<2, 4>() : f.template operator()<2, 1>();
}

int round_up(int v, int m) { return (v + m - 1) / m * m; }

bool make_plan(const GemvArgs& a, Plan* p, const char** why) {
  auto fail = [&](const char* reason) {
    if (why) *why = reason;
    return false;
  };
  if (a.m < 1 || a.m > 16) return fail("M must be in [1, 16]");
  if (static_cast<int64_t>(a.m) * a.k * 2 > kSmemLimit) return fail("x does not fit in shared memory");
  if (a.group % 32 != 0) return fail("group_size must be a multiple of 32");
  const int groups = a.k / a.group;
  if (groups % 2 != 0) return fail("K / group_size must be even");
  if (reinterpret_cast<uintptr_t>(a.x) % 16 || reinterpret_cast<uintptr_t>(a.q) % 16)
    return fail("x and qweight must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(a.s) % 4 || reinterpret_cast<uintptr_t>(a.z) % 4)
    return fail("scales and zeros must be 4-byte aligned");
  const int nt = a.m <= 8 ? 1 : 2;
  const int ksw = a.group % 128 == 0 ? 4 : 1;
  const int step = std::max(2 * a.group, 32 * ksw);

  p->ctas = std::min(sm_count(), a.n);
  const int rows_max = (a.n + p->ctas - 1) / p->ctas;
  const int chunks = (rows_max + kMaxChunkRows - 1) / kMaxChunkRows;
  p->rows_cap = round_up((rows_max + chunks - 1) / chunks, 16);

  const int off_bars = 0;
  p->off_xperm = round_up(off_bars + 2 * kMaxStages * 8, 128);
  p->off_corr = round_up(p->off_xperm + a.m * a.k * 2, 128);
  p->off_red = round_up(p->off_corr + a.m * groups * 8, 128);
  p->off_stages = round_up(p->off_red + kConsumerWarps * kWarp * nt * 16, 128);
  const int budget = kSmemLimit - p->off_stages;
  if (budget <= 0) return fail("x does not fit in shared memory");

  // Largest k-block that still leaves >= 4 stages; else the largest with >= 2.
  const int candidates[] = {2048, 1024, 512, 256, 128, 64};
  int best_kb = 0, best_stages = 0;
  for (int want : {4, 2}) {
    for (int kb : candidates) {
      if (kb % step != 0) continue;
      const int kbe = std::min(kb, round_up(a.k, step));
      const int row_stride = round_up(kbe / 2, 128) + 64;
      const int sz = kbe / a.group;
      const int stage = round_up(p->rows_cap * row_stride + 2 * p->rows_cap * sz * 2, 128);
      const int stages = std::min(kMaxStages, budget / stage);
      if (stages >= want) {
        best_kb = kbe;
        best_stages = stages;
        p->row_stride = row_stride;
        p->sz_per_row = sz;
        p->stage_bytes = stage;
        break;
      }
    }
    if (best_kb) break;
  }
  if (!best_kb) return fail("no k-block fits in shared memory");
  p->kb = best_kb;
  p->num_kb = (a.k + best_kb - 1) / best_kb;
  p->stages = best_stages;
  p->smem_bytes = p->off_stages + best_stages * p->stage_bytes;
  return true;
}

std::once_flag g_attr_once[4][64];

template <int NT, int KSW>
cudaError_t ensure_smem_attr() {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  constexpr int variant = (NT - 1) * 2 + (KSW == 4 ? 1 : 0);
  cudaError_t result = cudaSuccess;
  std::call_once(g_attr_once[variant][dev & 63], [&] {
    result = cudaFuncSetAttribute(mma_pipeline_kernel<NT, KSW>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
  });
  return result;
}

}  // namespace

int sm_count() {
  static int counts[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (counts[dev & 63] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
      v = 148;
    counts[dev & 63] = v;
  }
  return counts[dev & 63];
}

bool mma_pipeline_supported(const GemvArgs& a, const char** why) {
  Plan p;
  return make_plan(a, &p, why);
}

cudaError_t launch_mma_pipeline(const GemvArgs& a, cudaStream_t stream) {
  Plan p;
  if (!make_plan(a, &p, nullptr)) return cudaErrorInvalidValue;
  return with_variant(a.m, a.group, [&]<int NT, int KSW>() {
    cudaError_t err = ensure_smem_attr<NT, KSW>();
    if (err != cudaSuccess) return err;
    mma_pipeline_kernel<NT, KSW><<<p.ctas, kThreads, p.smem_bytes, stream>>>(a, p);
    return cudaGetLastError();
  });
}

cudaError_t mma_pipeline_attrs(int m, KernelAttrs* out) {
  return with_variant(m, 128, [&]<int NT, int KSW>() {
    cudaFuncAttributes fa;
    cudaError_t err = cudaFuncGetAttributes(&fa, mma_pipeline_kernel<NT, KSW>);
    if (err != cudaSuccess) return err;
    out->registers = fa.numRegs;
    out->local_bytes = static_cast<int>(fa.localSizeBytes);
    out->max_threads_per_block = fa.maxThreadsPerBlock;
    out->blocks_per_sm = 1;
    out->threads_per_block = kThreads;
    return cudaSuccess;
  });
}

int* device_status_word() {
  static int* words[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  if (!words[dev & 63]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status) != cudaSuccess) return nullptr;
    words[dev & 63] = static_cast<int*>(p);
  }
  return words[dev & 63];
}

cudaError_t read_and_clear_status(int* status) {
  cudaError_t err = cudaDeviceSynchronize();
  if (err != cudaSuccess) return err;
  int v = 0;
  err = cudaMemcpyFromSymbol(&v, g_status, sizeof(int));
  if (err != cudaSuccess) return err;
  const int zero = 0;
  err = cudaMemcpyToSymbol(g_status, &zero, sizeof(int));
  *status = v;
  return err;
}

}  // namespace i4
