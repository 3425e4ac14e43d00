// Device helpers shared by the sm_100a kernels: nibble unpacking, warp reductions, and the
// mbarrier / bulk-copy primitives of the TMA pipeline (inline PTX), with bounded waits.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace i4 {

constexpr int kWarp = 32;

// Status codes a kernel writes to the device status word when a bounded wait gives up.
constexpr int kStatusFullBarrierTimeout = 1;
constexpr int kStatusEmptyBarrierTimeout = 2;
constexpr int kStatusPeerTimeout = 3;  // a peer rank's flag did not arrive within the limit

// About one second at B200 clocks. A correct pipeline never waits more than microseconds.
constexpr long long kWaitLimitCycles = 2000000000LL;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- Nibble unpacking -------------------------------------------------------------------------
//
// A packed word holds q0..q7 (q_j in bits 4j..4j+3). OR-ing a nibble into the mantissa of the
// fp16 constant 1024 (0x6400, mantissa step 1) gives 1024 + q exactly; a nibble in mantissa bits
// 4..7 gives 1024 + 16 q. One LOP3 per half2, one shift per word:
//   h[0] = (1024 + q0,      1024 + q4)
//   h[1] = (1024 + 16 q1,   1024 + 16 q5)
//   h[2] = (1024 + q2,      1024 + q6)
//   h[3] = (1024 + 16 q3,   1024 + 16 q7)
__device__ __forceinline__ void unpack_x16(uint32_t w, uint32_t (&h)[4]) {
  const uint32_t hi = w >> 8;
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(h[0]) : "r"(w), "r"(0x000F000Fu), "r"(0x64006400u));
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(h[1]) : "r"(w), "r"(0x00F000F0u), "r"(0x64006400u));
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(h[2]) : "r"(hi), "r"(0x000F000Fu), "r"(0x64006400u));
  asm("lop3.b32 %0, %1, %2, %3, 0xea;" : "=r"(h[3]) : "r"(hi), "r"(0x00F000F0u), "r"(0x64006400u));
}

// One register of unpack_x16: the nibbles in bits 0..3 and 16..19 of w (high = false) as
// (1024 + q, 1024 + q), or those in bits 4..7 and 20..23 (high = true) as (1024 + 16 q, ...).
__device__ __forceinline__ uint32_t magic_f16(uint32_t w, bool high) {
  uint32_t h;
  asm("lop3.b32 %0, %1, %2, %3, 0xea;"
      : "=r"(h)
      : "r"(w), "r"(high ? 0x00F000F0u : 0x000F000Fu), "r"(0x64006400u));
  return h;
}

// Same trick without the factor 16: h[j] = (1024 + q_j, 1024 + q_{j+4}) for j = 0..3.
__device__ __forceinline__ void unpack_pairs(uint32_t w, uint32_t (&h)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    asm("lop3.b32 %0, %1, %2, %3, 0xea;"
        : "=r"(h[j])
        : "r"(w >> (4 * j)), "r"(0x000F000Fu), "r"(0x64006400u));
  }
}

// Word i (0..3) of a 16-byte vector.
__device__ __forceinline__ uint32_t word_of4(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// x0..x7 (one 8-weight block of x, fp16) -> the B halves that match unpack_x16's A halves:
// (x0, x4), (x1/16, x5/16), (x2, x6), (x3/16, x7/16). Adds the block's B values to bsum and the x
// they stand for (16 times each x/16 half) to xsum, both in fp32.
__device__ __forceinline__ uint4 permute_x_block(const uint4& v, float& bsum, float& xsum) {
  uint32_t lo02, hi02, lo13, hi13;
  asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(lo02) : "r"(v.x), "r"(v.z));  // (x0, x4)
  asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(hi02) : "r"(v.x), "r"(v.z));  // (x1, x5)
  asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(lo13) : "r"(v.y), "r"(v.w));  // (x2, x6)
  asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(hi13) : "r"(v.y), "r"(v.w));  // (x3, x7)
  const __half2 sixteenth = __float2half2_rn(0.0625f);
  __half2 a, b;
  memcpy(&a, &hi02, 4);
  memcpy(&b, &hi13, 4);
  a = __hmul2(a, sixteenth);
  b = __hmul2(b, sixteenth);
  uint4 o;
  o.x = lo02;
  memcpy(&o.y, &a, 4);
  o.z = lo13;
  memcpy(&o.w, &b, 4);
  __half2 l0, l1;
  memcpy(&l0, &lo02, 4);
  memcpy(&l1, &lo13, 4);
  const float2 f0 = __half22float2(l0), f1 = __half22float2(l1);
  const float2 f2 = __half22float2(a), f3 = __half22float2(b);
  const float ones = (f0.x + f0.y) + (f1.x + f1.y);
  const float sixteenths = (f2.x + f2.y) + (f3.x + f3.y);
  bsum += ones + sixteenths;
  xsum += ones + 16.0f * sixteenths;
  return o;
}

// permute_x_block without the sums.
__device__ __forceinline__ uint4 permute_x8(const uint4& v) {
  uint4 o;
  uint32_t hi02, hi13;
  asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(o.x) : "r"(v.x), "r"(v.z));  // (x0, x4)
  asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(hi02) : "r"(v.x), "r"(v.z));  // (x1, x5)
  asm("prmt.b32 %0, %1, %2, 0x5410;" : "=r"(o.z) : "r"(v.y), "r"(v.w));  // (x2, x6)
  asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(hi13) : "r"(v.y), "r"(v.w));  // (x3, x7)
  const uint32_t sixteenth = 0x2C002C00u;                                // (1/16, 1/16)
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o.y) : "r"(hi02), "r"(sixteenth));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o.w) : "r"(hi13), "r"(sixteenth));
  return o;
}

__device__ __forceinline__ float2 half2_bits_to_float2(uint32_t bits) {
  __half2 h;
  memcpy(&h, &bits, sizeof(h));
  return __half22float2(h);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = kWarp / 2; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

__device__ __forceinline__ uint32_t warp_xor(uint32_t v) {
#pragma unroll
  for (int off = kWarp / 2; off > 0; off >>= 1) v ^= __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// ---- Loads ------------------------------------------------------------------------------------

// 16-byte streaming load: read once, keep it out of L1.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// ---- mbarrier and bulk copies (sm_90+ PTX, used here on sm_100a) ------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for the phase with the given parity to complete, for at most kWaitLimitCycles. Returns
// false on timeout (the caller records a status and stops).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - start > kWaitLimitCycles) return false;
  }
  return true;
}

// mbar_wait_bounded with a suspend-time hint: a thread whose phase has not completed is suspended
// in hardware (up to kSuspendHintNs per try, woken when the phase completes) instead of spinning,
// so waiting warps do not take issue slots from the warps doing the work. Same bound, same result.
constexpr uint32_t kSuspendHintNs = 100000;
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded_suspend(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait_suspend(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait_suspend(bar, parity)) {
    if (clock64() - start > kWaitLimitCycles) return false;
  }
  return true;
}

// Releasing a ring stage right after loading it. mbarrier.arrive does not wait for the warp's
// shared-memory loads that are still in flight (measured on B200: with the weights in L2, a refill
// landed before such loads had read the stage). So before the release every lane folds the
// registers it loaded from the stage into one word (XOR) and stores it to a scratch word: that
// store cannot issue before the loads have returned, and the arrive, issued after it in program
// order, then hands back a stage that has been read. Call it from every lane, then __syncwarp(),
// then one lane arrives. `scratch` is 32 words of otherwise unused shared memory.
__device__ __forceinline__ uint32_t fold4(const uint4& v) { return v.x ^ v.y ^ v.z ^ v.w; }

__device__ __forceinline__ void stage_reads_done(uint32_t folded, uint32_t* scratch, int lane) {
  reinterpret_cast<volatile uint32_t*>(scratch)[lane] = folded;
}

// The consumers' side of a stage ring whose full barriers expect one arrival plus the bytes: slot
// and phase kept incrementally (no division). next() waits (bounded) for the next stage and
// returns its slot; after a timeout it records `status` once and stops waiting (ok = false).
struct StageRingSx {
  uint64_t* full;
  int stages;
  int* status;
  bool ok;
  int slot;
  uint32_t phase;
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

// ---- words between ranks (peer memory over NVLink) -----------------------------------------------
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Tagged words between ranks: 32 bits of data and a 32-bit tag (the call number) in one naturally
// aligned 64-bit store, which is single-copy atomic, so a reader that sees the tag sees the data
// that came with it: no fence and no separate flag.
__device__ __forceinline__ void st_tagged(unsigned long long* p, unsigned data, unsigned tag) {
  const unsigned long long v = (static_cast<unsigned long long>(tag) << 32) | data;
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Waits until the word at p carries `tag`, at most `limit_ns` nanoseconds; its data in *data.
__device__ __forceinline__ bool wait_tagged(const unsigned long long* p, unsigned tag,
                                            unsigned* data, unsigned long long limit_ns) {
  unsigned long long v = ld_tagged(p);
  if (static_cast<unsigned>(v >> 32) != tag) {
    const unsigned long long start = global_ns();
    do {
      if (global_ns() - start > limit_ns) return false;
      __nanosleep(64);
      v = ld_tagged(p);
    } while (static_cast<unsigned>(v >> 32) != tag);
  }
  *data = static_cast<unsigned>(v);
  return true;
}

// L2 policy for data read exactly once (the packed weights): evict it first.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// L2 policy for data many CTAs read (x): keep it.
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// 1-D bulk copy global -> shared, completion counted in bytes on `bar`. dst, src and bytes must
// be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// 4-byte asynchronous copy global -> shared (Ampere-style cp.async).
__device__ __forceinline__ void cp_async_4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}

// Arrive on `bar` once every cp.async this thread issued so far has landed. The arrival is one
// of the barrier's expected arrivals (.noinc).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// Named barrier over `threads` threads (a multiple of 32), id 1..15.
__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---- Tensor core (warp-level) -------------------------------------------------------------------

// D = A * B + C, m16n8k16, A row-major f16, B column-major f16, C / D f32. Not volatile: the
// compiler may interleave independent MMAs (a dependent one waits ~21 cycles on B200).
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D = A * B (C = 0): starts an accumulator without zeroing its registers first.
__device__ __forceinline__ void mma_16816_first(float (&d)[4], const uint32_t (&a)[4],
                                                uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%10, %10, %10, %10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.0f));
}

}  // namespace i4
