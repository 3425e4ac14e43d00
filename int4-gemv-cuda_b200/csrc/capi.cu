// The C ABI (include/int4gemv_b200.h): argument checks with the reference's messages, dispatch to
// the launchers, and error reporting through int4gemv_last_error(). No torch; the only device
// allocation is int4gemv_peer_alloc's, which the caller asks for.
#include <algorithm>
#include <atomic>
#include <climits>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "int4gemv_b200.h"
#include "kernels.h"

namespace i4 {
void sequential_cpu(uint16_t* y, const uint16_t* x, const uint32_t* q, const uint16_t* s,
                    const uint16_t* z, int64_t m, int64_t n, int64_t k, int64_t group,
                    int64_t threads);
}  // namespace i4

namespace {

thread_local std::string g_last_error;

// int4gemv_set_strict_weights: when set, the pipelined kernels read the weights only after the
// previous kernel in the stream has completed (see the header).
std::atomic<int> g_strict_weights{0};
bool strict_weights() { return g_strict_weights.load(std::memory_order_relaxed) != 0; }

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int ok() {
  g_last_error.clear();
  return INT4GEMV_OK;
}

int cuda_fail(const char* name, cudaError_t err) {
  return fail(INT4GEMV_ERR_CUDA, "%s: CUDA error %d: %s", name, static_cast<int>(err),
              cudaGetErrorString(err));
}

// The size and group checks of csrc/checks.cpp:9-44 (reference), on raw sizes. The dtype, rank,
// shape-consistency, contiguity and device checks are made by the torch binding, which sees
// tensors; here the caller's sizes define the shapes.
int check_sizes(const char* name, int64_t m, int64_t n, int64_t k, int64_t group) {
  if (m < 0 || n < 0 || k < 0) {
    return fail(INT4GEMV_ERR_INVALID, "%s: M = %lld, N = %lld, K = %lld must not be negative", name,
                static_cast<long long>(m), static_cast<long long>(n), static_cast<long long>(k));
  }
  if (m > INT_MAX || n > INT_MAX || k > INT_MAX) {
    return fail(INT4GEMV_ERR_INVALID, "%s: M = %lld, N = %lld, K = %lld must each fit in int", name,
                static_cast<long long>(m), static_cast<long long>(n), static_cast<long long>(k));
  }
  if (!(group > 0 && group % 8 == 0 && k % group == 0)) {
    return fail(INT4GEMV_ERR_INVALID,
                "%s: group_size %lld must be a positive multiple of 8 dividing K = %lld", name,
                static_cast<long long>(group), static_cast<long long>(k));
  }
  return INT4GEMV_OK;
}

int check_pointers(const char* name, int64_t m, int64_t n, int64_t k, const void* y,
                   const void* x, const void* q, const void* s, const void* z) {
  const bool need_y = m > 0 && n > 0;
  const bool need_in = need_y && k > 0;
  if ((need_y && !y) || (need_in && (!x || !q || !s || !z))) {
    return fail(INT4GEMV_ERR_INVALID, "%s: null pointer for a non-empty tensor", name);
  }
  return INT4GEMV_OK;
}

// csrc/common.cuh:84-89 (reference).
int check_threads(const char* name, int64_t threads) {
  if (!(threads >= 32 && threads <= 1024 && threads % 32 == 0)) {
    return fail(INT4GEMV_ERR_INVALID,
                "%s: threads_per_block must be a multiple of 32 in [32, 1024], got %lld", name,
                static_cast<long long>(threads));
  }
  return INT4GEMV_OK;
}

// csrc/common.cuh:94-101 (reference).
int check_16_byte_loads(const char* name, const void* x, const void* q, int64_t group) {
  if (group % 32 != 0) {
    return fail(INT4GEMV_ERR_INVALID, "%s: group_size must be a multiple of 32, got %lld", name,
                static_cast<long long>(group));
  }
  if (reinterpret_cast<uintptr_t>(x) % 16 != 0 || reinterpret_cast<uintptr_t>(q) % 16 != 0) {
    return fail(INT4GEMV_ERR_INVALID, "%s: x and qweight must be 16-byte aligned", name);
  }
  return INT4GEMV_OK;
}

// csrc/common.cuh:67-82 (reference); the reference's message carries no operator name.
int check_rows_per_warp(int64_t rpw) {
  if (rpw != 1 && rpw != 2 && rpw != 4) {
    return fail(INT4GEMV_ERR_INVALID, "rows_per_warp must be 1, 2 or 4, got %lld",
                static_cast<long long>(rpw));
  }
  return INT4GEMV_OK;
}

// csrc/common.cuh:105-112 (reference): say clearly when registers limit the block size.
int check_launchable(const char* name, int m, int threads, int rpw) {
  int max_threads = 0;
  const cudaError_t err = i4::vectorized_max_threads(m, rpw, &max_threads);
  if (err != cudaSuccess) return cuda_fail(name, err);
  if (threads > max_threads) {
    i4::KernelAttrs at{};
    i4::simt_attrs("vectorized", m, 32, rpw, &at);
    return fail(INT4GEMV_ERR_INVALID,
                "%s: this configuration uses %d registers per thread, so blocks of at most %d "
                "threads fit, not %d",
                name, at.registers, max_threads, threads);
  }
  return INT4GEMV_OK;
}

i4::GemvArgs make_args(void* y, const void* x, const void* q, const void* s, const void* z,
                       int64_t m, int64_t n, int64_t k, int64_t group) {
  return i4::GemvArgs{static_cast<half*>(y),
                      static_cast<const half*>(x),
                      static_cast<const uint32_t*>(q),
                      static_cast<const half*>(s),
                      static_cast<const half*>(z),
                      static_cast<int>(m),
                      static_cast<int>(n),
                      static_cast<int>(k),
                      static_cast<int>(group)};
}

// M or N = 0: nothing to do. K = 0: y is all zeros (an empty sum).
int empty_cases(const char* name, void* y, int64_t m, int64_t n, int64_t k, cudaStream_t stream,
                bool* done) {
  *done = true;
  if (m == 0 || n == 0) return ok();
  if (k == 0) {
    const cudaError_t err = cudaMemsetAsync(y, 0, static_cast<size_t>(m * n * 2), stream);
    return err == cudaSuccess ? ok() : cuda_fail(name, err);
  }
  *done = false;
  return INT4GEMV_OK;
}

int launched(const char* name, cudaError_t err) { return err == cudaSuccess ? ok() : cuda_fail(name, err); }

enum class Pick {
  kStripeMma, kTcDequant, kStreamMma, kTcgen05, kMmaPipeline, kVectorized, kCoalesced
};

// From this many rows of x the tcgen05 kernel (one MMA instruction per 2048 weights, whatever the
// row count up to 64) is faster than the warp-MMA stream, whose MMA count grows with M (measured on
// B200 at 8192 x 8192, 4096 x 14336 and 14336 x 4096: stream_mma ahead at M = 8, tc_dequant from
// M = 10 on).
constexpr int kTcDequantMinM = 9;

Pick pick_kernel(const i4::GemvArgs& a) {
  if (i4::stripe_mma_supported(a, nullptr)) return Pick::kStripeMma;
  if (a.m >= kTcDequantMinM && i4::tc_dequant_supported(a, nullptr)) return Pick::kTcDequant;
  if (i4::stream_mma_supported(a, nullptr)) return Pick::kStreamMma;
  if (i4::mma_pipeline_supported(a, nullptr)) return Pick::kMmaPipeline;
  if (a.group % 32 == 0 && reinterpret_cast<uintptr_t>(a.x) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(a.q) % 16 == 0) {
    return Pick::kVectorized;
  }
  return Pick::kCoalesced;
}

// Launches the kernel pick_kernel chooses for `a` (the dispatch of int4gemv_w4a16).
int run_picked(const char* name, const i4::GemvArgs& a, cudaStream_t st) {
  switch (pick_kernel(a)) {
    case Pick::kStripeMma:
      return launched(name, i4::launch_stripe_mma(a, st, strict_weights()));
    case Pick::kTcDequant:
      return launched(name, i4::launch_tc_dequant(a, st, strict_weights()));
    case Pick::kStreamMma:
      return launched(name, i4::launch_stream_mma(a, st, strict_weights()));
    case Pick::kTcgen05:
      return launched(name, i4::launch_tc_gemv(a, st, strict_weights()));
    case Pick::kMmaPipeline:
      return launched(name, i4::launch_mma_pipeline(a, st));
    case Pick::kVectorized:
      return launched(name, i4::launch_vectorized(a, 128, 2, st));
    default:
      return launched(name, i4::launch_coalesced(a, st));
  }
}

}  // namespace

// ---- Scratch of int4gemv_w4a16_exchange_static: static device memory, no allocation ---------
// A single rank's exchange buffer (two halves of 8-byte tagged words) and its call counters
// (INT4GEMV_PEER_COUNTER_BYTES), in module memory of every device the library is loaded on.
constexpr int64_t kStaticExchangeBytes = 4 << 20;
static __device__ __align__(256) unsigned char g_static_exchange[kStaticExchangeBytes];
static __device__ __align__(256) unsigned char g_static_counters[INT4GEMV_PEER_COUNTER_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
void* g_static_out[kMaxDevices];
void* g_static_counter_ptr[kMaxDevices];

// The current device's static scratch. The first call on a device looks the symbols up and
// clears both arrays (synchronously: it must not happen inside a stream capture).
int static_scratch(const char* name, void** out, void** counters) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return cuda_fail(name, err);
  if (dev < 0 || dev >= kMaxDevices) {
    return fail(INT4GEMV_ERR_INVALID, "%s: device %d out of range", name, dev);
  }
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_out[dev]) {
    void* o = nullptr;
    void* f = nullptr;
    err = cudaGetSymbolAddress(&o, g_static_exchange);
    if (err == cudaSuccess) err = cudaGetSymbolAddress(&f, g_static_counters);
    if (err == cudaSuccess) err = cudaMemset(o, 0, kStaticExchangeBytes);
    if (err == cudaSuccess) err = cudaMemset(f, 0, INT4GEMV_PEER_COUNTER_BYTES);
    if (err == cudaSuccess) err = cudaDeviceSynchronize();
    if (err != cudaSuccess) return cuda_fail(name, err);
    g_static_counter_ptr[dev] = f;
    g_static_out[dev] = o;
  }
  *out = g_static_out[dev];
  *counters = g_static_counter_ptr[dev];
  return INT4GEMV_OK;
}
}  // namespace

extern "C" {

const char* int4gemv_last_error(void) { return g_last_error.c_str(); }

int int4gemv_version(void) { return 100; }

int int4gemv_naive(void* y, const void* x, const void* qweight, const void* scales,
                   const void* zeros, int64_t m, int64_t n, int64_t k, int64_t group_size,
                   void* stream) {
  const char* name = "naive";
  if (int e = check_sizes(name, m, n, k, group_size)) return e;
  if (int e = check_pointers(name, m, n, k, y, x, qweight, scales, zeros)) return e;
  bool done;
  const auto st = static_cast<cudaStream_t>(stream);
  int e = empty_cases(name, y, m, n, k, st, &done);
  if (done) return e;
  return launched(name, i4::launch_naive(make_args(y, x, qweight, scales, zeros, m, n, k, group_size), st));
}

int int4gemv_coalesced(void* y, const void* x, const void* qweight, const void* scales,
                       const void* zeros, int64_t m, int64_t n, int64_t k, int64_t group_size,
                       void* stream) {
  const char* name = "coalesced";
  if (int e = check_sizes(name, m, n, k, group_size)) return e;
  if (int e = check_pointers(name, m, n, k, y, x, qweight, scales, zeros)) return e;
  bool done;
  const auto st = static_cast<cudaStream_t>(stream);
  int e = empty_cases(name, y, m, n, k, st, &done);
  if (done) return e;
  return launched(name,
                  i4::launch_coalesced(make_args(y, x, qweight, scales, zeros, m, n, k, group_size), st));
}

int int4gemv_vectorized(void* y, const void* x, const void* qweight, const void* scales,
                        const void* zeros, int64_t m, int64_t n, int64_t k, int64_t group_size,
                        int64_t threads_per_block, int64_t rows_per_warp, void* stream) {
  const char* name = "vectorized";
  if (int e = check_sizes(name, m, n, k, group_size)) return e;
  if (int e = check_threads(name, threads_per_block)) return e;
  if (int e = check_16_byte_loads(name, x, qweight, group_size)) return e;
  if (int e = check_pointers(name, m, n, k, y, x, qweight, scales, zeros)) return e;
  bool done;
  const auto st = static_cast<cudaStream_t>(stream);
  int e = empty_cases(name, y, m, n, k, st, &done);
  if (done) return e;
  if (int e2 = check_rows_per_warp(rows_per_warp)) return e2;
  if (int e2 = check_launchable(name, static_cast<int>(m), static_cast<int>(threads_per_block),
                                static_cast<int>(rows_per_warp)))
    return e2;
  return launched(name, i4::launch_vectorized(
                            make_args(y, x, qweight, scales, zeros, m, n, k, group_size),
                            static_cast<int>(threads_per_block), static_cast<int>(rows_per_warp), st));
}

int int4gemv_load_only(void* out, const void* x, const void* qweight, const void* scales,
                       const void* zeros, int64_t m, int64_t n, int64_t k, int64_t group_size,
                       int64_t threads_per_block, int64_t rows_per_warp, void* stream) {
  const char* name = "load_only";
  if (int e = check_sizes(name, m, n, k, group_size)) return e;
  if (int e = check_threads(name, threads_per_block)) return e;
  if (m != 1) return fail(INT4GEMV_ERR_INVALID, "load_only: needs M = 1, got %lld", static_cast<long long>(m));
  if (int e = check_16_byte_loads(name, x, qweight, group_size)) return e;
  if (int e = check_pointers(name, 1, n, k, out, x, qweight, scales, zeros)) return e;
  const auto st = static_cast<cudaStream_t>(stream);
  if (n == 0) return ok();
  if (k == 0) {
    const cudaError_t err = cudaMemsetAsync(out, 0, static_cast<size_t>(n * 4), st);
    return err == cudaSuccess ? ok() : cuda_fail(name, err);
  }
  if (int e = check_rows_per_warp(rows_per_warp)) return e;
  if (int e = check_launchable(name, 1, static_cast<int>(threads_per_block),
                               static_cast<int>(rows_per_warp)))
    return e;
  return launched(name, i4::launch_load_only(static_cast<uint32_t*>(out),
                                             make_args(nullptr, x, qweight, scales, zeros, 1, n, k,
                                                       group_size),
                                             static_cast<int>(threads_per_block),
                                             static_cast<int>(rows_per_warp), st));
}

int int4gemv_stripe_load_only(void* out, const void* qweight, const void* scales,
                              const void* zeros, int64_t n, int64_t k, int64_t group_size,
                              void* stream) {
  const char* name = "stripe_load_only";
  if (int e = check_sizes(name, 1, n, k, group_size)) return e;
  if (n > 0 && k > 0 && (!out || !qweight || !scales || !zeros)) {
    return fail(INT4GEMV_ERR_INVALID, "%s: null pointer", name);
  }
  const auto st = static_cast<cudaStream_t>(stream);
  if (n == 0) return ok();
  if (k == 0) {
    const cudaError_t err = cudaMemsetAsync(out, 0, static_cast<size_t>(n * 4), st);
    return err == cudaSuccess ? ok() : cuda_fail(name, err);
  }
  const i4::GemvArgs a = make_args(nullptr, nullptr, qweight, scales, zeros, 1, n, k, group_size);
  const char* why = "unsupported shape";
  if (!i4::stripe_mma_supported(a, &why)) return fail(INT4GEMV_ERR_INVALID, "%s: %s", name, why);
  return launched(name, i4::launch_stripe_load_only(static_cast<uint32_t*>(out), a, st));
}

int int4gemv_kernel_info(const char* kernel, int64_t m, int64_t threads_per_block,
                         int64_t rows_per_warp, int64_t* info) {
  if (!kernel || !info) return fail(INT4GEMV_ERR_INVALID, "kernel_info: null argument");
  if (m < 0 || m > INT_MAX) return fail(INT4GEMV_ERR_INVALID, "kernel_info: bad M = %lld", static_cast<long long>(m));
  i4::KernelAttrs at{};
  cudaError_t err;
  if (std::strcmp(kernel, "vectorized") == 0) {
    if (int e = check_threads("vectorized_info", threads_per_block)) return e;
    if (int e = check_rows_per_warp(rows_per_warp)) return e;
    err = i4::simt_attrs("vectorized", static_cast<int>(m), static_cast<int>(threads_per_block),
                         static_cast<int>(rows_per_warp), &at);
  } else if (std::strcmp(kernel, "naive") == 0 || std::strcmp(kernel, "coalesced") == 0) {
    err = i4::simt_attrs(kernel, static_cast<int>(m), 0, 1, &at);
  } else if (std::strcmp(kernel, "w4a16") == 0) {
    err = m <= 8                ? i4::stripe_mma_attrs(static_cast<int>(m), &at)
          : m < kTcDequantMinM  ? i4::stream_mma_attrs(static_cast<int>(m), &at)
          : m <= 64             ? i4::tc_dequant_attrs(static_cast<int>(m), &at)
                                : i4::mma_pipeline_attrs(16, &at);
  } else {
    return fail(INT4GEMV_ERR_INVALID, "kernel_info: unknown kernel '%s'", kernel);
  }
  if (err != cudaSuccess) return cuda_fail("kernel_info", err);
  info[0] = at.registers;
  info[1] = at.local_bytes;
  info[2] = at.threads_per_block;
  info[3] = at.max_threads_per_block;
  info[4] = at.blocks_per_sm;
  info[5] = static_cast<int64_t>(at.blocks_per_sm) * at.threads_per_block / 32;
  return ok();
}

int int4gemv_sequential(void* y, const void* x, const void* qweight, const void* scales,
                        const void* zeros, int64_t m, int64_t n, int64_t k, int64_t group_size,
                        int64_t threads) {
  const char* name = "sequential";
  if (int e = check_sizes(name, m, n, k, group_size)) return e;
  if (int e = check_pointers(name, m, n, k, y, x, qweight, scales, zeros)) return e;
  if (m == 0 || n == 0) return ok();
  if (k == 0) {
    std::memset(y, 0, static_cast<size_t>(m * n * 2));
    return ok();
  }
  i4::sequential_cpu(static_cast<uint16_t*>(y), static_cast<const uint16_t*>(x),
                     static_cast<const uint32_t*>(qweight), static_cast<const uint16_t*>(scales),
                     static_cast<const uint16_t*>(zeros), m, n, k, group_size, threads);
  return ok();
}

int64_t int4gemv_w4a16_workspace_size(int64_t m, int64_t n, int64_t k, int64_t group_size) {
  if (m <= 0 || n <= 0 || k <= 0 || m > INT_MAX || n > INT_MAX || k > INT_MAX ||
      group_size <= 0 || group_size % 8 || k % group_size) {
    return 0;
  }
  // The size depends on the shape only; aligned stand-in pointers pass the alignment checks.
  const void* aligned = reinterpret_cast<const void*>(static_cast<uintptr_t>(256));
  const i4::GemvArgs a = make_args(nullptr, aligned, aligned, aligned, aligned, m, n, k, group_size);
  return pick_kernel(a) == Pick::kStreamMma ? i4::stream_mma_workspace_bytes(a) : 0;
}

int int4gemv_w4a16(void* y, const void* x, const void* qweight, const void* scales,
                   const void* zeros, int64_t m, int64_t n, int64_t k, int64_t group_size,
                   void* workspace, int64_t workspace_bytes, void* stream) {
  const char* name = "w4a16";
  if (int e = check_sizes(name, m, n, k, group_size)) return e;
  if (int e = check_pointers(name, m, n, k, y, x, qweight, scales, zeros)) return e;
  bool done;
  const auto st = static_cast<cudaStream_t>(stream);
  int e = empty_cases(name, y, m, n, k, st, &done);
  if (done) return e;
  const i4::GemvArgs a = make_args(y, x, qweight, scales, zeros, m, n, k, group_size);
  if (workspace && workspace_bytes > 0 && pick_kernel(a) == Pick::kStreamMma) {
    return launched(name, i4::launch_stream_mma(a, st, strict_weights(), nullptr, nullptr,
                                                workspace, workspace_bytes));
  }
  return run_picked(name, a, st);
}

int int4gemv_w4a16_grouped(int count, void* const* ys, const int64_t* ns, const void* x,
                           const void* qweight, const void* scales, const void* zeros, int64_t m,
                           int64_t k, int64_t group_size, void* stream) {
  const char* name = "w4a16_grouped";
  if (count < 1 || count > INT4GEMV_MAX_GROUP || !ys || !ns) {
    return fail(INT4GEMV_ERR_INVALID, "%s: count %d must be in [1, %d] with ys and ns given", name,
                count, INT4GEMV_MAX_GROUP);
  }
  int64_t total = 0;
  i4::GroupOut go{};
  go.count = count;
  for (int i = 0; i < count; ++i) {
    if (ns[i] < 0) return fail(INT4GEMV_ERR_INVALID, "%s: ns[%d] = %lld < 0", name, i,
                               static_cast<long long>(ns[i]));
    if (ns[i] > 0 && m > 0 && !ys[i]) return fail(INT4GEMV_ERR_INVALID, "%s: null ys[%d]", name, i);
    total += ns[i];
    go.y[i] = static_cast<half*>(ys[i]);
    go.row_end[i] = static_cast<int>(std::min<int64_t>(total, INT_MAX));
  }
  if (int e = check_sizes(name, m, total, k, group_size)) return e;
  if (int e = check_pointers(name, m, total, k, ys[0] ? ys[0] : x, x, qweight, scales, zeros)) {
    return e;
  }
  const auto st = static_cast<cudaStream_t>(stream);
  if (m == 0 || total == 0) return ok();
  i4::GemvArgs a = make_args(ys[0], x, qweight, scales, zeros, m, total, k, group_size);
  if (k > 0 && i4::stream_mma_supported(a, nullptr)) {
    a.epilogue = i4::kGroupedY;
    return launched(name, i4::launch_stream_mma(a, st, strict_weights(), nullptr, &go));
  }
  // Other shapes: one launch per matrix on its rows of the stacked weights.
  int64_t row0 = 0;
  for (int i = 0; i < count; ++i) {
    const int64_t groups = k / group_size;
    const auto* q = static_cast<const uint32_t*>(qweight) + row0 * (k / 8);
    const auto* sc = static_cast<const half*>(scales) + row0 * groups;
    const auto* zc = static_cast<const half*>(zeros) + row0 * groups;
    bool done;
    int e = empty_cases(name, ys[i], m, ns[i], k, st, &done);
    if (!done) e = run_picked(name, make_args(ys[i], x, q, sc, zc, m, ns[i], k, group_size), st);
    if (e != INT4GEMV_OK) return e;
    row0 += ns[i];
  }
  return ok();
}

int int4gemv_w4a16_bias_residual(void* y, const void* x, const void* qweight, const void* scales,
                                 const void* zeros, const void* bias, const void* residual,
                                 int64_t m, int64_t n, int64_t k, int64_t group_size,
                                 void* stream) {
  const char* name = "w4a16_bias_residual";
  if (int e = check_sizes(name, m, n, k, group_size)) return e;
  if (int e = check_pointers(name, m, n, k, y, x, qweight, scales, zeros)) return e;
  const auto st = static_cast<cudaStream_t>(stream);
  if (m == 0 || n == 0) return ok();
  i4::GemvArgs a = make_args(y, x, qweight, scales, zeros, m, n, k, group_size);
  a.bias = static_cast<const half*>(bias);
  a.residual = static_cast<const half*>(residual);
  if (k == 0) return launched(name, i4::launch_bias_residual(a, st));  // y = bias + residual
  return run_picked(name, a, st);
}

const char* int4gemv_w4a16_kernel_name(const void* x, const void* qweight, const void* scales,
                                       const void* zeros, int64_t m, int64_t n, int64_t k,
                                       int64_t group_size) {
  if (m <= 0 || n <= 0 || k <= 0 || m > INT_MAX || n > INT_MAX || k > INT_MAX ||
      group_size <= 0 || group_size % 8 || k % group_size) {
    return "none";
  }
  const i4::GemvArgs a = make_args(nullptr, x, qweight, scales, zeros, m, n, k, group_size);
  switch (pick_kernel(a)) {
    case Pick::kStripeMma:
      return "stripe_mma";
    case Pick::kTcDequant:
      return "tc_dequant";
    case Pick::kStreamMma:
      return "stream_mma";
    case Pick::kTcgen05:
      return "tcgen05";
    case Pick::kMmaPipeline:
      return "mma_pipeline";
    case Pick::kVectorized:
      return "vectorized";
    default:
      return "coalesced";
  }
}

int int4gemv_w4a16_kernel(const char* kernel, void* y, const void* x, const void* qweight,
                          const void* scales, const void* zeros, int64_t m, int64_t n, int64_t k,
                          int64_t group_size, void* stream) {
  const char* name = "w4a16";
  if (!kernel) return fail(INT4GEMV_ERR_INVALID, "w4a16: null kernel name");
  if (int e = check_sizes(name, m, n, k, group_size)) return e;
  if (int e = check_pointers(name, m, n, k, y, x, qweight, scales, zeros)) return e;
  bool done;
  const auto st = static_cast<cudaStream_t>(stream);
  int e = empty_cases(name, y, m, n, k, st, &done);
  if (done) return e;
  const i4::GemvArgs a = make_args(y, x, qweight, scales, zeros, m, n, k, group_size);
  const char* why = "unsupported shape";
  if (std::strcmp(kernel, "stream_mma") == 0) {
    if (!i4::stream_mma_supported(a, &why)) return fail(INT4GEMV_ERR_INVALID, "stream_mma: %s", why);
    return launched(name, i4::launch_stream_mma(a, st, strict_weights()));
  }
  if (std::strcmp(kernel, "stripe_mma") == 0) {
    if (!i4::stripe_mma_supported(a, &why)) return fail(INT4GEMV_ERR_INVALID, "stripe_mma: %s", why);
    return launched(name, i4::launch_stripe_mma(a, st, strict_weights()));
  }
  if (std::strcmp(kernel, "tc_dequant") == 0) {
    if (!i4::tc_dequant_supported(a, &why)) return fail(INT4GEMV_ERR_INVALID, "tc_dequant: %s", why);
    return launched(name, i4::launch_tc_dequant(a, st, strict_weights()));
  }
  if (std::strcmp(kernel, "tc_wide") == 0) {
    if (!i4::tc_wide_supported(a, &why)) return fail(INT4GEMV_ERR_INVALID, "tc_wide: %s", why);
    return launched(name, i4::launch_tc_wide(a, st, strict_weights()));
  }
  if (std::strcmp(kernel, "tcgen05") == 0) {
    if (!i4::tc_gemv_supported(a, &why)) return fail(INT4GEMV_ERR_INVALID, "tcgen05: %s", why);
    return launched(name, i4::launch_tc_gemv(a, st, strict_weights()));
  }
  if (std::strcmp(kernel, "mma_pipeline") == 0) {
    if (!i4::mma_pipeline_supported(a, &why)) return fail(INT4GEMV_ERR_INVALID, "mma_pipeline: %s", why);
    return launched(name, i4::launch_mma_pipeline(a, st));
  }
  if (std::strcmp(kernel, "vectorized") == 0) {
    if (int e2 = check_16_byte_loads("vectorized", x, qweight, group_size)) return e2;
    return launched(name, i4::launch_vectorized(a, 128, 2, st));
  }
  if (std::strcmp(kernel, "coalesced") == 0) return launched(name, i4::launch_coalesced(a, st));
  if (std::strcmp(kernel, "naive") == 0) return launched(name, i4::launch_naive(a, st));
  return fail(INT4GEMV_ERR_INVALID, "w4a16: unknown kernel '%s'", kernel);
}

int int4gemv_w4a16_silu_mul(void* y, const void* x, const void* qweight, const void* scales,
                            const void* zeros, int64_t m, int64_t n, int64_t k, int64_t group_size,
                            void* stream) {
  const char* name = "w4a16_silu_mul";
  if (int e = check_sizes(name, m, n, k, group_size)) return e;
  if (n % 2 != 0) {
    return fail(INT4GEMV_ERR_INVALID, "%s: N = %lld must be even (gate and up rows interleaved)",
                name, static_cast<long long>(n));
  }
  if (int e = check_pointers(name, m, n, k, y, x, qweight, scales, zeros)) return e;
  const auto st = static_cast<cudaStream_t>(stream);
  if (m == 0 || n == 0) return ok();
  if (k == 0) {  // silu(0) * 0
    const cudaError_t err = cudaMemsetAsync(y, 0, static_cast<size_t>(m * (n / 2) * 2), st);
    return err == cudaSuccess ? ok() : cuda_fail(name, err);
  }
  i4::GemvArgs a = make_args(y, x, qweight, scales, zeros, m, n, k, group_size);
  a.epilogue = i4::kSiluMul;
  const char* why = "unsupported shape";
  if (!i4::stream_mma_supported(a, &why)) return fail(INT4GEMV_ERR_INVALID, "%s: %s", name, why);
  return launched(name, i4::launch_stream_mma(a, st, strict_weights()));
}

int int4gemv_w4a16_f32(void* y, const void* x, const void* qweight, const void* scales,
                       const void* zeros, int64_t m, int64_t n, int64_t k, int64_t group_size,
                       void* stream) {
  const char* name = "w4a16_f32";
  if (int e = check_sizes(name, m, n, k, group_size)) return e;
  if (int e = check_pointers(name, m, n, k, y, x, qweight, scales, zeros)) return e;
  const auto st = static_cast<cudaStream_t>(stream);
  if (m == 0 || n == 0) return ok();
  if (k == 0) {
    const cudaError_t err = cudaMemsetAsync(y, 0, static_cast<size_t>(m * n * 4), st);
    return err == cudaSuccess ? ok() : cuda_fail(name, err);
  }
  i4::GemvArgs a = make_args(y, x, qweight, scales, zeros, m, n, k, group_size);
  a.epilogue = i4::kStoreF32;
  if (a.m >= kTcDequantMinM && i4::tc_dequant_supported(a, nullptr)) {
    return launched(name, i4::launch_tc_dequant(a, st, strict_weights()));
  }
  if (i4::stream_mma_supported(a, nullptr)) {
    return launched(name, i4::launch_stream_mma(a, st, strict_weights()));
  }
  // any other shape (e.g. a K shard that is not a multiple of 1024): the SIMT kernels
  if (a.group % 32 == 0 && reinterpret_cast<uintptr_t>(a.x) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(a.q) % 16 == 0) {
    return launched(name, i4::launch_vectorized(a, 128, 2, st));
  }
  return launched(name, i4::launch_coalesced(a, st));
}

int int4gemv_unpack(void* q, const void* qweight, int64_t n, int64_t k, void* stream) {
  const char* name = "unpack";
  if (n < 0 || k < 0 || k % 8 != 0) {
    return fail(INT4GEMV_ERR_INVALID, "unpack: N = %lld, K = %lld: K must be a non-negative multiple of 8",
                static_cast<long long>(n), static_cast<long long>(k));
  }
  if (n == 0 || k == 0) return ok();
  if (!q || !qweight) return fail(INT4GEMV_ERR_INVALID, "unpack: null pointer");
  if (reinterpret_cast<uintptr_t>(q) % 16 != 0) {
    return fail(INT4GEMV_ERR_INVALID, "unpack: output must be 16-byte aligned");
  }
  return launched(name, i4::launch_unpack(static_cast<int32_t*>(q), static_cast<const uint32_t*>(qweight),
                                          n, k, static_cast<cudaStream_t>(stream)));
}

int int4gemv_dequantize(void* w, const void* qweight, const void* scales, const void* zeros,
                        int64_t n, int64_t k, int64_t group_size, void* stream) {
  const char* name = "dequantize";
  if (int e = check_sizes(name, 0, n, k, group_size)) return e;
  if (n == 0 || k == 0) return ok();
  if (!w || !qweight || !scales || !zeros) return fail(INT4GEMV_ERR_INVALID, "dequantize: null pointer");
  if (reinterpret_cast<uintptr_t>(w) % 16 != 0) {
    return fail(INT4GEMV_ERR_INVALID, "dequantize: output must be 16-byte aligned");
  }
  return launched(name, i4::launch_dequantize(static_cast<float*>(w), static_cast<const uint32_t*>(qweight),
                                              static_cast<const half*>(scales), static_cast<const half*>(zeros),
                                              n, k, group_size, static_cast<cudaStream_t>(stream)));
}

int int4gemv_quantize(void* qweight, void* scales, void* zeros, const void* w, int dtype,
                      int64_t n, int64_t k, int64_t group_size, void* stream) {
  const char* name = "quantize";
  if (dtype != INT4GEMV_DTYPE_F32 && dtype != INT4GEMV_DTYPE_F16 && dtype != INT4GEMV_DTYPE_BF16) {
    return fail(INT4GEMV_ERR_INVALID, "quantize: unknown weight dtype %d", dtype);
  }
  if (int e = check_sizes(name, 0, n, k, group_size)) return e;
  if (n == 0 || k == 0) return ok();
  if (!qweight || !scales || !zeros || !w) return fail(INT4GEMV_ERR_INVALID, "quantize: null pointer");
  if (reinterpret_cast<uintptr_t>(w) % 16 != 0) {
    return fail(INT4GEMV_ERR_INVALID, "quantize: w must be 16-byte aligned");
  }
  return launched(name, i4::launch_quantize(static_cast<uint32_t*>(qweight), static_cast<half*>(scales),
                                            static_cast<half*>(zeros), w, dtype, n, k, group_size,
                                            static_cast<cudaStream_t>(stream)));
}

int int4gemv_pack(void* qweight, const void* q, int64_t n, int64_t k, void* stream) {
  const char* name = "pack";
  if (n < 0 || k < 0 || k % 8 != 0) {
    return fail(INT4GEMV_ERR_INVALID, "pack: N = %lld, K = %lld: K must be a non-negative multiple of 8",
                static_cast<long long>(n), static_cast<long long>(k));
  }
  if (n == 0 || k == 0) return ok();
  if (!q || !qweight) return fail(INT4GEMV_ERR_INVALID, "pack: null pointer");
  if (reinterpret_cast<uintptr_t>(q) % 16 != 0) {
    return fail(INT4GEMV_ERR_INVALID, "pack: q must be 16-byte aligned");
  }
  return launched(name, i4::launch_pack(static_cast<uint32_t*>(qweight), static_cast<const int32_t*>(q), n,
                                        k, static_cast<cudaStream_t>(stream)));
}

namespace {
int repack(const char* name, bool awq, void* qweight, void* scales, void* zeros,
           const void* ck_qweight, const void* ck_qzeros, const void* ck_scales, int zero_offset,
           int64_t n, int64_t k, int64_t group_size, void* stream) {
  if (int e = check_sizes(name, 0, n, k, group_size)) return e;
  if (n % 8 != 0) {
    return fail(INT4GEMV_ERR_INVALID, "%s: N = %lld must be a multiple of 8 (packed zero points)",
                name, static_cast<long long>(n));
  }
  if (zero_offset < 0 || zero_offset > 1) {
    return fail(INT4GEMV_ERR_INVALID, "%s: zero_offset %d must be 0 or 1", name, zero_offset);
  }
  if (n == 0 || k == 0) return ok();
  if (!qweight || !scales || !zeros || !ck_qweight || !ck_qzeros || !ck_scales) {
    return fail(INT4GEMV_ERR_INVALID, "%s: null pointer", name);
  }
  return launched(name, i4::launch_repack(awq, static_cast<uint32_t*>(qweight), static_cast<half*>(scales),
                                          static_cast<half*>(zeros), static_cast<const uint32_t*>(ck_qweight),
                                          static_cast<const uint32_t*>(ck_qzeros),
                                          static_cast<const half*>(ck_scales), n, k, group_size,
                                          zero_offset, static_cast<cudaStream_t>(stream)));
}
}  // namespace

int int4gemv_repack_awq(void* qweight, void* scales, void* zeros, const void* awq_qweight,
                        const void* awq_qzeros, const void* awq_scales, int64_t n, int64_t k,
                        int64_t group_size, void* stream) {
  return repack("repack_awq", true, qweight, scales, zeros, awq_qweight, awq_qzeros, awq_scales, 0,
                n, k, group_size, stream);
}

int int4gemv_repack_gptq(void* qweight, void* scales, void* zeros, const void* gptq_qweight,
                         const void* gptq_qzeros, const void* gptq_scales, int zero_offset,
                         int64_t n, int64_t k, int64_t group_size, void* stream) {
  return repack("repack_gptq", false, qweight, scales, zeros, gptq_qweight, gptq_qzeros,
                gptq_scales, zero_offset, n, k, group_size, stream);
}

static_assert(INT4GEMV_MAX_PEERS == i4::kMaxPeers, "peer count");
static_assert(INT4GEMV_MAX_GROUP == i4::kMaxGroup, "group count");
static_assert(INT4GEMV_PEER_COUNTER_BYTES == 4 * i4::kPeerCounters, "counter words");

size_t int4gemv_peers_struct_bytes(void) { return sizeof(int4gemv_peers_t); }

int int4gemv_peer_alloc(int64_t bytes, void** ptr, void* ipc_handle) {
  if (bytes <= 0 || !ptr || !ipc_handle) return fail(INT4GEMV_ERR_INVALID, "peer_alloc: bad argument");
  void* p = nullptr;
  cudaError_t err = cudaMalloc(&p, static_cast<size_t>(bytes));
  if (err != cudaSuccess) return cuda_fail("peer_alloc", err);
  err = cudaMemset(p, 0, static_cast<size_t>(bytes));
  cudaIpcMemHandle_t h;
  if (err == cudaSuccess) err = cudaIpcGetMemHandle(&h, p);
  if (err != cudaSuccess) {
    cudaFree(p);
    return cuda_fail("peer_alloc", err);
  }
  static_assert(sizeof(h) == INT4GEMV_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return ok();
}

int int4gemv_peer_open(const void* ipc_handle, void** ptr) {
  if (!ipc_handle || !ptr) return fail(INT4GEMV_ERR_INVALID, "peer_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  const cudaError_t err = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return err == cudaSuccess ? ok() : cuda_fail("peer_open", err);
}

int int4gemv_peer_close(void* ptr) {
  const cudaError_t err = cudaIpcCloseMemHandle(ptr);
  return err == cudaSuccess ? ok() : cuda_fail("peer_close", err);
}

int int4gemv_peer_free(void* ptr) {
  const cudaError_t err = cudaFree(ptr);
  return err == cudaSuccess ? ok() : cuda_fail("peer_free", err);
}

int int4gemv_w4a16_exchange(void* y, const void* x, const void* qweight, const void* scales,
                            const void* zeros, int64_t m, int64_t n, int64_t k, int64_t group_size,
                            const int4gemv_peers_t* peers, void* stream) {
  const char* name = "w4a16_exchange";
  if (!peers) return fail(INT4GEMV_ERR_INVALID, "%s: null peers", name);
  const int mode = peers->mode;
  if (mode != INT4GEMV_SHARD_ROWS && mode != INT4GEMV_SHARD_K) {
    return fail(INT4GEMV_ERR_INVALID, "%s: unknown mode %d", name, mode);
  }
  if (peers->world < 1 || peers->world > INT4GEMV_MAX_PEERS || peers->rank < 0 ||
      peers->rank >= peers->world) {
    return fail(INT4GEMV_ERR_INVALID, "%s: rank %d of world %d (at most %d ranks)", name,
                peers->rank, peers->world, INT4GEMV_MAX_PEERS);
  }
  for (int r = 0; r < peers->world; ++r) {
    if (!peers->out[r]) return fail(INT4GEMV_ERR_INVALID, "%s: null buffer of rank %d", name, r);
  }
  if (!peers->counters) return fail(INT4GEMV_ERR_INVALID, "%s: null counters", name);
  if (int e = check_sizes(name, m, n, k, group_size)) return e;
  if (m == 0 || n == 0 || k == 0) {
    return fail(INT4GEMV_ERR_INVALID, "%s: M, N and K must be positive", name);
  }
  if (int e = check_pointers(name, m, n, k, y, x, qweight, scales, zeros)) return e;
  const int64_t n_out = mode == INT4GEMV_SHARD_ROWS ? peers->n_total : n;
  if (mode == INT4GEMV_SHARD_ROWS &&
      (peers->n_total != n * peers->world || peers->col0 != n * peers->rank)) {
    return fail(INT4GEMV_ERR_INVALID,
                "%s: rows split needs equal shards: n_total = %lld must be %lld x %d and col0 = "
                "%lld must be %lld x %d",
                name, static_cast<long long>(peers->n_total), static_cast<long long>(n),
                peers->world, static_cast<long long>(peers->col0), static_cast<long long>(n),
                peers->rank);
  }
  const int64_t need = 8 * (mode == INT4GEMV_SHARD_ROWS ? m * n_out : peers->world * m * n);
  if (peers->out_bytes < 2 * need) {
    return fail(INT4GEMV_ERR_INVALID, "%s: out buffers of %lld bytes, %lld needed (two halves)",
                name, static_cast<long long>(peers->out_bytes), static_cast<long long>(2 * need));
  }
  if (n_out > INT_MAX) return fail(INT4GEMV_ERR_INVALID, "%s: y too wide", name);
  i4::GemvArgs a = make_args(y, x, qweight, scales, zeros, m, n, k, group_size);
  a.epilogue = mode == INT4GEMV_SHARD_ROWS ? i4::kGatherPeers : i4::kReducePeers;
  const char* why = "unsupported shape";
  // the M <= 8 stripe kernel where it takes the shape, else the stream kernel
  const bool stripe = i4::stripe_mma_supported(a, nullptr);
  if (!stripe && !i4::stream_mma_supported(a, &why)) {
    return fail(INT4GEMV_ERR_INVALID, "%s: %s", name, why);
  }
  i4::PeerSet ps{};
  for (int r = 0; r < peers->world; ++r) ps.out[r] = peers->out[r];
  ps.counters = static_cast<unsigned*>(peers->counters);
  ps.out_half = (peers->out_bytes / 2) / 16 * 16;
  ps.world = peers->world;
  ps.rank = peers->rank;
  ps.n_total = static_cast<int>(n_out);
  ps.col0 = static_cast<int>(mode == INT4GEMV_SHARD_ROWS ? peers->col0 : 0);
  const auto st = static_cast<cudaStream_t>(stream);
  return launched(name, stripe ? i4::launch_stripe_mma(a, st, strict_weights(), &ps)
                               : i4::launch_stream_mma(a, st, strict_weights(), &ps));
}

int int4gemv_w4a16_exchange_static(void* y, const void* x, const void* qweight,
                                   const void* scales, const void* zeros, int64_t m, int64_t n,
                                   int64_t k, int64_t group_size, int mode, void* stream) {
  const char* name = "w4a16_exchange_static";
  if (mode != INT4GEMV_SHARD_ROWS && mode != INT4GEMV_SHARD_K) {
    return fail(INT4GEMV_ERR_INVALID, "%s: unknown mode %d", name, mode);
  }
  // Every check that can reject the call runs before the first-call setup below, so an invalid
  // call never triggers the synchronous setup.
  if (int e = check_sizes(name, m, n, k, group_size)) return e;
  if (m == 0 || n == 0 || k == 0) {
    return fail(INT4GEMV_ERR_INVALID, "%s: M, N and K must be positive", name);
  }
  if (int e = check_pointers(name, m, n, k, y, x, qweight, scales, zeros)) return e;
  // One 8-byte tagged word per output in each of two halves, either mode: M x N <= bytes / 16.
  // Compared by division, so no product of the (int-sized) M and N can overflow.
  constexpr int64_t kMaxOutputs = kStaticExchangeBytes / 16;
  if (n > kMaxOutputs / m) {
    return fail(INT4GEMV_ERR_INVALID,
                "%s: M = %lld, N = %lld needs more exchange buffer than there is; the static "
                "buffer holds %lld bytes (M x N <= %lld)",
                name, static_cast<long long>(m), static_cast<long long>(n),
                static_cast<long long>(kStaticExchangeBytes), static_cast<long long>(kMaxOutputs));
  }
  {
    i4::GemvArgs a = make_args(y, x, qweight, scales, zeros, m, n, k, group_size);
    a.epilogue = mode == INT4GEMV_SHARD_ROWS ? i4::kGatherPeers : i4::kReducePeers;
    const char* why = "unsupported shape";
    if (!i4::stripe_mma_supported(a, nullptr) && !i4::stream_mma_supported(a, &why)) {
      return fail(INT4GEMV_ERR_INVALID, "%s: %s", name, why);
    }
  }
  void* out = nullptr;
  void* counters = nullptr;
  if (int e = static_scratch(name, &out, &counters)) return e;
  int4gemv_peers_t peers{};
  peers.world = 1;
  peers.rank = 0;
  peers.mode = mode;
  peers.n_total = n;
  peers.col0 = 0;
  peers.out_bytes = kStaticExchangeBytes;
  peers.out[0] = out;
  peers.counters = counters;
  return int4gemv_w4a16_exchange(y, x, qweight, scales, zeros, m, n, k, group_size, &peers,
                                 stream);
}

int int4gemv_set_strict_weights(int strict) {
  if (strict != 0 && strict != 1) {
    return fail(INT4GEMV_ERR_INVALID, "set_strict_weights: strict must be 0 or 1, got %d", strict);
  }
  g_strict_weights.store(strict, std::memory_order_relaxed);
  return ok();
}

int int4gemv_device_status(int* status) {
  if (!status) return fail(INT4GEMV_ERR_INVALID, "device_status: null argument");
  const cudaError_t err = i4::read_and_clear_status(status);
  return err == cudaSuccess ? ok() : cuda_fail("device_status", err);
}

}  // extern "C"
