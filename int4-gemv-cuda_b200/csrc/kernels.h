// Internal interface between the C ABI (capi.cu) and the kernel launchers. Host-only types, no
// torch. Every launcher assumes its arguments were validated by the C ABI layer and M, N > 0.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace i4 {

// What the GEMV writes. kStoreY: y [m, n]. kSiluMul: the rows of W are gate and up rows
// interleaved (row 2i = gate i, row 2i + 1 = up i) and y [m, n / 2] = silu(gate) * up.
// kGatherPeers / kReducePeers (stripe_mma and stream_mma): the fused exchange of a layer sharded
// over the ranks of one node (PeerSet below): rows split (every rank's y gets this rank's columns) or K split (every rank
// gets this rank's fp32 partial sums, then each adds all ranks' partials in rank order).
// kGroupedY: the rows of W are several matrices stacked (GroupOut below) and each matrix's
// outputs go to its own y.
// kStoreF32: y [m, n] fp32, the row sums themselves (the partial sums of a K-split layer, added
// across ranks before the one rounding to fp16).
enum Epilogue : int {
  kStoreY = 0, kSiluMul = 1, kGatherPeers = 2, kReducePeers = 3, kGroupedY = 4, kStoreF32 = 5
};

constexpr int kMaxPeers = 8;
constexpr int kPeerCounters = 1024;  // counter words per rank (two used: call number, CTAs done)
constexpr unsigned long long kPeerWaitNs = 2000000000ull;  // limit of one wait on a peer's word

// Peer buffers of a sharded layer. out[r] is rank r's exchange buffer mapped into this process
// (out[rank] is this rank's own): two halves of out_half bytes used by alternate calls (a rank
// can run at most one call ahead of another), each an array of 64-bit tagged words (32 bits of
// data, 32 bits of call number). kGatherPeers: a half is [m, n_total] words (fp16 bits of y);
// this rank writes columns [col0, col0 + n) of every rank's half, then each CTA copies the rows
// it needs into this rank's y as their tags show this call. kReducePeers: a half is
// [world, m, n] words (fp32 partial sums); this rank writes slot `rank` of every rank's half.
// counters: this rank's kPeerCounters words: [0] the number of the last completed call, [1] the
// CTAs of the running call that have finished. A call's number is [0] + 1, read on the device,
// so a captured graph replays correctly.
struct PeerSet {
  void* out[kMaxPeers];
  unsigned* counters;
  long long out_half;
  int world, rank;
  int n_total, col0;
};

// Outputs of a grouped launch: matrix i is rows [row_end[i - 1], row_end[i]) of the stacked
// weights (row_end[-1] = 0) and writes y[i] [m, row_end[i] - row_end[i - 1]].
constexpr int kMaxGroup = 8;
struct GroupOut {
  half* y[kMaxGroup];
  int row_end[kMaxGroup];
  int count;
};

// Epilogue inputs beyond GemvArgs, one kernel parameter.
struct EpilogueExtra {
  PeerSet peers;
  GroupOut groups;
};

struct GemvArgs {
  half* y;             // [m, n] (kSiluMul: [m, n / 2])
  const half* x;       // [m, k]
  const uint32_t* q;   // [n, k / 8]
  const half* s;       // [n, k / group]
  const half* z;       // [n, k / group]
  int m, n, k, group;
  int epilogue = kStoreY;  // kSiluMul etc.: stream_mma; kStoreF32: stream_mma, tc_dequant, SIMT
  // kStoreY only, each optional: y[m, r] = sum + bias[r] + residual[m, r], rounded to fp16 once.
  // residual may be y itself (each output is read and written by the same thread).
  const half* bias = nullptr;      // [n]
  const half* residual = nullptr;  // [m, n]
};

#if defined(__CUDACC__)
// The fp16 value a GEMV kernel stores for output (m, r) of row sum `sum` (kStoreY).
__device__ __forceinline__ half store_value(const GemvArgs& a, int m, int r, float sum) {
  if (a.bias) sum += __half2float(a.bias[r]);
  if (a.residual) sum += __half2float(a.residual[static_cast<int64_t>(m) * a.n + r]);
  return __float2half_rn(sum);
}
#endif

// Attributes of one compiled kernel, for the *_info entry points.
struct KernelAttrs {
  int registers;
  int local_bytes;
  int max_threads_per_block;
  int blocks_per_sm;  // occupancy at the given block size and dynamic shared memory
  int threads_per_block;
};

// SIMT kernels (simt.cu): the reference operators' mappings, rewritten for sm_100a.
cudaError_t launch_naive(const GemvArgs& a, cudaStream_t stream);
cudaError_t launch_coalesced(const GemvArgs& a, cudaStream_t stream);
cudaError_t launch_vectorized(const GemvArgs& a, int threads_per_block, int rows_per_warp,
                              cudaStream_t stream);
cudaError_t launch_load_only(uint32_t* out, const GemvArgs& a, int threads_per_block,
                             int rows_per_warp, cudaStream_t stream);
// Registers etc. of the kernel instance the launcher would pick for (m, threads, rows_per_warp).
cudaError_t simt_attrs(const char* kernel, int m, int threads_per_block, int rows_per_warp,
                       KernelAttrs* out);
// Largest block the vectorized instance for (m, rows_per_warp) can launch with (registers).
cudaError_t vectorized_max_threads(int m, int rows_per_warp, int* max_threads);

// tcgen05 GEMV for M <= 8 (tc_gemv.cu). Launched with programmatic stream
// serialization; strict = read the weights only after the previous kernel in the stream is done.
bool tc_gemv_supported(const GemvArgs& a, const char** why);
cudaError_t launch_tc_gemv(const GemvArgs& a, cudaStream_t stream, bool strict);
cudaError_t tc_gemv_attrs(int m, KernelAttrs* out);

// TMA-tile-fed mma.sync GEMV for M <= 32, group 128, K % 1024 == 0 (stream_mma.cu): the M <= 8
// shapes stripe_mma does not take, and the fused epilogues. Launched with programmatic stream
// serialization like launch_tc_gemv.
bool stream_mma_supported(const GemvArgs& a, const char** why);
// With a workspace of at least stream_mma_workspace_bytes(a) bytes (> 0 for the wide path, M >= 5,
// plain stores), a small pre-kernel permutes x once and the GEMV's CTAs copy it instead of each
// permuting all of x; without one, each CTA permutes x itself.
cudaError_t launch_stream_mma(const GemvArgs& a, cudaStream_t stream, bool strict,
                              const PeerSet* peers = nullptr, const GroupOut* groups = nullptr,
                              void* workspace = nullptr, int64_t workspace_bytes = 0);
int64_t stream_mma_workspace_bytes(const GemvArgs& a);
cudaError_t stream_mma_attrs(int m, KernelAttrs* out);

// Stripe-fed mma.sync GEMV for M <= 8, group 128, K % 2048 == 0 (stripe_mma.cu): 2-D TMA tiles of
// 32 rows x 2048 weights, the whole ring issued before the dependency wait unless strict.
bool stripe_mma_supported(const GemvArgs& a, const char** why);
// With peers (kGatherPeers / kReducePeers) it runs the fused exchange like launch_stream_mma.
cudaError_t launch_stripe_mma(const GemvArgs& a, cudaStream_t stream, bool strict,
                              const PeerSet* peers = nullptr);
cudaError_t stripe_mma_attrs(int m, KernelAttrs* out);
// The loads-only ceiling of the stripe stream (M = 1 plan, no x, no MMA): out[row] = XOR of the
// row's packed words and of (scale bits | zero bits << 16) of each of its groups. a.y, a.x and
// a.m are ignored.
cudaError_t launch_stripe_load_only(uint32_t* out, const GemvArgs& a, cudaStream_t stream);

// tcgen05 GEMV for M <= 64, group 128, K % 1024 == 0 (tc_dequant.cu): weights dequantized into
// TMEM, one accumulator per 128-row tile, stream-K split over the SMs with a fixed-order reduction
// of shared tiles through static device memory (calls in different streams are ordered by an
// event). Plain stores only (kStoreY with bias / residual, or kStoreF32).
bool tc_dequant_supported(const GemvArgs& a, const char** why);
cudaError_t launch_tc_dequant(const GemvArgs& a, cudaStream_t stream, bool strict);
cudaError_t tc_dequant_attrs(int m, KernelAttrs* out);

// tcgen05 GEMV for M <= 64 with the weights as the MMA's N operand (tc_wide.cu): 256-row tiles,
// x and the dequantised weights both in shared memory, stream-K like tc_dequant with its own
// static partial sums and counters.
bool tc_wide_supported(const GemvArgs& a, const char** why);
cudaError_t launch_tc_wide(const GemvArgs& a, cudaStream_t stream, bool strict);
cudaError_t tc_wide_attrs(int m, KernelAttrs* out);

// TMA-bulk-fed mma.sync pipeline (mma_pipeline.cu). `why` gets a reason when unsupported.
bool mma_pipeline_supported(const GemvArgs& a, const char** why);
cudaError_t launch_mma_pipeline(const GemvArgs& a, cudaStream_t stream);
cudaError_t mma_pipeline_attrs(int m, KernelAttrs* out);
// Device address of the status word of the current device (cached per device), or null.
int* device_status_word();
// Reads and clears the device status word of the current device (synchronous).
cudaError_t read_and_clear_status(int* status);

// Packed-format helpers (packed.cu).
cudaError_t launch_unpack(int32_t* q, const uint32_t* qweight, int64_t n, int64_t k,
                          cudaStream_t stream);
cudaError_t launch_dequantize(float* w, const uint32_t* qweight, const half* s, const half* z,
                              int64_t n, int64_t k, int64_t group, cudaStream_t stream);
// y = bias + residual (the K = 0 case of a GEMV with a bias / residual epilogue).
cudaError_t launch_bias_residual(const GemvArgs& a, cudaStream_t stream);

// Group quantisation and packing (quantize.cu). The weight element types quantize reads.
enum WeightType : int { kWeightF32 = 0, kWeightF16 = 1, kWeightBF16 = 2 };
cudaError_t launch_quantize(uint32_t* qweight, half* scales, half* zeros, const void* w,
                            int dtype, int64_t n, int64_t k, int64_t group, cudaStream_t stream);
cudaError_t launch_pack(uint32_t* qweight, const int32_t* q, int64_t n, int64_t k,
                        cudaStream_t stream);

// AWQ / GPTQ checkpoint tensors -> this layout (repack.cu). awq selects the AWQ layout, else
// GPTQ's; zero_offset is added to every stored zero point (1 for GPTQ's "gptq" format).
cudaError_t launch_repack(bool awq, uint32_t* qweight, half* scales, half* zeros,
                          const uint32_t* ck_qweight, const uint32_t* ck_qzeros,
                          const half* ck_scales, int64_t n, int64_t k, int64_t group,
                          int zero_offset, cudaStream_t stream);

// SM count of the current device (cached per device).
int sm_count();

}  // namespace i4
