/*
 * int4gemv_b200: C ABI of the B200-native (sm_100a) W4A16 GEMV library.
 *
 * The operator is y = x @ dequant(W)^T with w = (q - z) * s, every group_size weights along K
 * sharing one fp16 scale s and one fp16 zero z. Layouts follow the reference operator contract
 * (Yu-TingLee/int4-GEMV-cuda, csrc/w4a16.h:10-16), all contiguous row-major:
 *   x        [M, K]          fp16
 *   qweight  [N, K / 8]      int32, eight 4-bit q per word, weight k in bits 4*(k%8).. of word k/8
 *   scales   [N, K / group]  fp16
 *   zeros    [N, K / group]  fp16
 *   y        [M, N]          fp16 (written)
 * Unless stated otherwise pointers are DEVICE pointers on the current CUDA device, `stream` is a
 * cudaStream_t (NULL = the legacy default stream), and calls are asynchronous: they enqueue work on
 * `stream` and return. Only int4gemv_device_status, int4gemv_peer_alloc / _open / _close / _free
 * and the first call of int4gemv_w4a16_exchange_static on a device synchronise.
 *
 * Every entry point returns INT4GEMV_OK (0) or an error code; int4gemv_last_error() then gives a
 * message for the calling thread. Argument errors use the reference's check messages
 * (csrc/checks.cpp:9-44, csrc/common.cuh:84-112), prefixed by the operator name.
 * M or N equal to 0 is valid and launches nothing (y is empty); K = 0 gives y = 0 (plus bias and
 * residual where the entry point takes them).
 */
#ifndef INT4GEMV_B200_H_
#define INT4GEMV_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define INT4GEMV_OK 0
#define INT4GEMV_ERR_INVALID 1     /* an argument fails a check; nothing was launched */
#define INT4GEMV_ERR_CUDA 2        /* a CUDA runtime call failed */
#define INT4GEMV_ERR_WORKSPACE 3   /* workspace missing or smaller than *_workspace_size */

/* Message for the last failing call on this thread ("" if none). Valid until the next call. */
const char* int4gemv_last_error(void);

/* Library version as MAJOR * 10000 + MINOR * 100 + PATCH. */
int int4gemv_version(void);

/* ---- The reference's operators (csrc/w4a16.h), re-implemented for sm_100a -------------------- */

/* Replaces int4gemv::naive (csrc/w4a16.h:27-28): one thread per output row. */
int int4gemv_naive(void* y, const void* x, const void* qweight, const void* scales,
                   const void* zeros, int64_t m, int64_t n, int64_t k, int64_t group_size,
                   void* stream);

/* Replaces int4gemv::coalesced (csrc/w4a16.h:32-33): one warp per output row. */
int int4gemv_coalesced(void* y, const void* x, const void* qweight, const void* scales,
                       const void* zeros, int64_t m, int64_t n, int64_t k, int64_t group_size,
                       void* stream);

/* Replaces int4gemv::vectorized (csrc/w4a16.h:38-40): rows_per_warp (1, 2 or 4) rows per warp,
 * threads_per_block a multiple of 32 in [32, 1024], 16-byte loads. Needs group_size % 32 == 0 and
 * 16-byte aligned x and qweight (csrc/common.cuh:94-101). */
int int4gemv_vectorized(void* y, const void* x, const void* qweight, const void* scales,
                        const void* zeros, int64_t m, int64_t n, int64_t k, int64_t group_size,
                        int64_t threads_per_block, int64_t rows_per_warp, void* stream);

/* Replaces int4gemv::load_only (csrc/w4a16.h:45-47): the vectorized loads without the GEMV math,
 * M = 1 only. out is uint32 [N]; out[r] is the XOR of every 32-bit word of qweight row r, of the
 * zero-extended 16-bit patterns of scales/zeros row r, and of the words of x read with each chunk. */
int int4gemv_load_only(void* out, const void* x, const void* qweight, const void* scales,
                       const void* zeros, int64_t m, int64_t n, int64_t k, int64_t group_size,
                       int64_t threads_per_block, int64_t rows_per_warp, void* stream);

/* Replaces naive_info / coalesced_info / vectorized_info (csrc/w4a16.h:29,34,41;
 * csrc/common.cuh:115-128). kernel is "naive", "coalesced", "vectorized" or "w4a16".
 * threads_per_block / rows_per_warp are used by "vectorized" only. Writes six values to info:
 * registers, local_bytes, threads_per_block, max_threads_per_block, blocks_per_sm, warps_per_sm. */
int int4gemv_kernel_info(const char* kernel, int64_t m, int64_t threads_per_block,
                         int64_t rows_per_warp, int64_t* info);

/* Replaces int4gemv::sequential (csrc/w4a16.h:23-24): the CPU path. HOST pointers. Same order of
 * fp32 operations as the reference, so the result is bit-identical; rows are spread over
 * `threads` host threads (0 = one per hardware thread), which does not change the result. */
int int4gemv_sequential(void* y, const void* x, const void* qweight, const void* scales,
                        const void* zeros, int64_t m, int64_t n, int64_t k, int64_t group_size,
                        int64_t threads);

/* ---- The B200 fast path (new; no counterpart in the reference) ------------------------------- */

/* Bytes of device workspace int4gemv_w4a16 can use for this shape (0 if none): for the shapes with
 * 5 <= M <= 8 that go to stream_mma (those stripe_mma does not take), room for x permuted once per
 * call by a pre-kernel instead of in every CTA. */
int64_t int4gemv_w4a16_workspace_size(int64_t m, int64_t n, int64_t k, int64_t group_size);

/* y = x @ dequant(W)^T through the fastest kernel for the shape: a persistent, TMA-bulk-fed,
 * tensor-core dequant GEMV when the shape allows it, else the SIMT kernels. Same inputs and result
 * contract as the operators above (csrc/w4a16.h:10-16), parity with int4gemv/reference.py within
 * rtol = 1e-2, atol = 1e-2. workspace is optional: NULL (or smaller than
 * int4gemv_w4a16_workspace_size) gives the same result through the slower path. It is used only
 * within the call, in stream order. */
int int4gemv_w4a16(void* y, const void* x, const void* qweight, const void* scales,
                   const void* zeros, int64_t m, int64_t n, int64_t k, int64_t group_size,
                   void* workspace, int64_t workspace_bytes, void* stream);

/* Name of the kernel int4gemv_w4a16 picks for this shape and these pointers ("stripe_mma" for
 * M <= 8 when K is a multiple of 2048 and its x panels and partials fit in shared memory,
 * "tc_dequant" for 9 <= M <= 64, "stream_mma" otherwise up to M = 32 when group_size is 128 and K
 * a multiple of 1024; "mma_pipeline", "vectorized", "coalesced" for the other shapes); for
 * tests and the benchmark. Static storage.
 *
 * tc_dequant keeps split-K partial sums and per-tile counters in static device memory, so two of
 * its calls must not run at the same time on one device: calls in one stream are ordered, and
 * before a call in a different stream than the previous one that stream waits for an event
 * recorded after the previous call (host-side, nothing to do for the caller). Calls captured into
 * CUDA graphs are ordered only by the graphs' own streams: replays of such graphs must not
 * overlap on one device. */
const char* int4gemv_w4a16_kernel_name(const void* x, const void* qweight, const void* scales,
                                       const void* zeros, int64_t m, int64_t n, int64_t k,
                                       int64_t group_size);

/* The loads-only ceiling of the M <= 4 fast path (new; the reference's load_only above is the
 * same idea for its SIMT kernel, csrc/w4a16.h:45-47): the stripe_mma weight stream (2-D TMA tiles,
 * the same ring, grid and launch) with the arithmetic replaced by a fold, no x. out is uint32 [N];
 * out[r] is the XOR of every 32-bit word of qweight row r and, for each group of the row, of
 * (scale bits | zero bits << 16). Needs group_size 128, K a multiple of 2048, 16-byte aligned
 * qweight, scales and zeros; INT4GEMV_ERR_INVALID with the reason otherwise. For measuring how
 * close the GEMV comes to the stream it rides on. */
int int4gemv_stripe_load_only(void* out, const void* qweight, const void* scales,
                              const void* zeros, int64_t n, int64_t k, int64_t group_size,
                              void* stream);

/* Runs one named kernel instead of the automatic choice: "stripe_mma", "tc_dequant",
 * "stream_mma", "tcgen05", "tc_wide", "mma_pipeline", "vectorized" (128 threads, 2 rows per warp),
 * "coalesced" or "naive". For tests and benchmarks. "tcgen05" and "tc_wide" are tcgen05 designs
 * that the automatic choice does not use (slower than the kernels it picks, at every shape
 * measured); "tc_wide" (1 <= M <= 64, K % 1024 == 0) keeps its own static split-K scratch and
 * orders its calls across streams like tc_dequant.
 * Fails with
 * INT4GEMV_ERR_INVALID if that kernel does not support the shape or the pointers' alignment. */
int int4gemv_w4a16_kernel(const char* kernel, void* y, const void* x, const void* qweight,
                          const void* scales, const void* zeros, int64_t m, int64_t n, int64_t k,
                          int64_t group_size, void* stream);

/* Fused gate / up projection (new; no counterpart in the reference): qweight, scales and zeros hold
 * 2 * n_out rows with the gate and up rows interleaved (row 2i = gate i, row 2i + 1 = up i, see
 * int4gemv/quant.py interleave_rows), n = 2 * n_out, and y [m, n_out] fp16 =
 * silu(x @ gate^T) * (x @ up^T), computed from the fp32 sums and rounded once. One weight stream
 * and one read of x for both projections. Needs the fast path's shapes (group_size 128, K a
 * multiple of 1024, M <= 32, 16-byte aligned x, qweight, scales, zeros); INT4GEMV_ERR_INVALID
 * with the reason otherwise. */
int int4gemv_w4a16_silu_mul(void* y, const void* x, const void* qweight, const void* scales,
                            const void* zeros, int64_t m, int64_t n, int64_t k, int64_t group_size,
                            void* stream);

/* y [M, N] = x @ W^T + bias + residual with both additions fused into the GEMV's store: the fp32
 * row sum plus bias[n] plus residual[m, n], rounded to fp16 once. bias ([N] fp16) and residual
 * ([M, N] fp16) may each be NULL; residual may be y itself (in-place residual add). Same kernel
 * choice and checks as int4gemv_w4a16; with K = 0, y = bias + residual. New: the reference has no
 * fused epilogue (a caller adds bias and residual with separate elementwise kernels). */
int int4gemv_w4a16_bias_residual(void* y, const void* x, const void* qweight, const void* scales,
                                 const void* zeros, const void* bias, const void* residual,
                                 int64_t m, int64_t n, int64_t k, int64_t group_size,
                                 void* stream);

/* One launch for several matrices that share x (q / k / v, or gate / up kept apart): their
 * packed weights stacked by rows into one qweight [sum ns, K/8], scales and zeros
 * [sum ns, K/group_size] (stack them once at load time), and each matrix i's output written to
 * its own ys[i] [m, ns[i]] fp16. count <= INT4GEMV_MAX_GROUP. On the fast path's shapes this is a
 * single stream_mma launch over all the rows (one x load, one tail); otherwise one launch per
 * matrix. New: the reference launches one GEMV per matrix. */
#define INT4GEMV_MAX_GROUP 8
int int4gemv_w4a16_grouped(int count, void* const* ys, const int64_t* ns, const void* x,
                           const void* qweight, const void* scales, const void* zeros, int64_t m,
                           int64_t k, int64_t group_size, void* stream);

/* y [M, N] fp32 = x @ W^T, the fp32 row sums themselves with no rounding to fp16: the local partial
 * sums of a layer split along K over several GPUs, which are added across ranks and rounded to
 * fp16 once (int4gemv/sharded.py). Same inputs and checks as int4gemv_w4a16, any shape they
 * accept: on the fast path's shapes (group_size 128, K a multiple of 1024, M <= 64) stream_mma or
 * tc_dequant, otherwise the SIMT kernels (vectorized when group_size % 32 == 0 and x, qweight are
 * 16-byte aligned, else coalesced). New: the reference returns fp16 only. */
int int4gemv_w4a16_f32(void* y, const void* x, const void* qweight, const void* scales,
                       const void* zeros, int64_t m, int64_t n, int64_t k, int64_t group_size,
                       void* stream);

/* ---- Packed-format helpers on the device (int4gemv/quant.py:40-53), bit-exact ---------------- */

/* q [N, K] int32 = the 4-bit values of qweight [N, K/8]   (quant.py:40-44). */
int int4gemv_unpack(void* q, const void* qweight, int64_t n, int64_t k, void* stream);

/* w [N, K] fp32 = (q - z) * s with one fp32 subtraction and one fp32 multiplication per weight
 * (quant.py:47-53), bit-identical to the reference. */
int int4gemv_dequantize(void* w, const void* qweight, const void* scales, const void* zeros,
                        int64_t n, int64_t k, int64_t group_size, void* stream);

/* Group quantisation of w [N, K] on the device, bit-exact with quant.py:14-29 (quantize) for
 * finite weights: per group of group_size weights along K, lo = min(w, 0), hi = max(w, 0),
 * s = fp16((hi - lo) / 15 clamped to >= 1e-6), z = clamp(round(-lo / s), 0, 15),
 * q = clamp(round(w / s + z), 0, 15) with round half to even, then packed as by int4gemv_pack.
 * w holds fp32, fp16 or bf16 (dtype, INT4GEMV_DTYPE_*) and must be 16-byte aligned; the reference
 * widens w to fp32 first, which is exact for fp16 and bf16. Writes qweight [N, K/8] int32,
 * scales and zeros [N, K/group_size] fp16. New: the reference quantises with torch on the host. */
#define INT4GEMV_DTYPE_F32 0
#define INT4GEMV_DTYPE_F16 1
#define INT4GEMV_DTYPE_BF16 2
int int4gemv_quantize(void* qweight, void* scales, void* zeros, const void* w, int dtype,
                      int64_t n, int64_t k, int64_t group_size, void* stream);

/* qweight [N, K/8] int32 from q [N, K] int32 (16-byte aligned): word = sum over j of
 * q[8w + j] << 4j, modulo 2^32, as quant.py:32-37 (pack) computes it in int64 and casts to int32
 * (values outside 0..15 carry into the neighbouring nibbles the same way). */
int int4gemv_pack(void* qweight, const void* q, int64_t n, int64_t k, void* stream);

/* ---- Checkpoint repacking (new: the reference reads only unquantised fp16 / bf16 weights) ---- */

/* AWQ checkpoint tensors -> qweight [N, K/8] int32, scales and zeros [N, K/group_size] fp16.
 * awq_qweight [K, N/8] int32 and awq_qzeros [K/group_size, N/8] int32 hold column 8c + j of word
 * c in nibble (j % 2) * 4 + j / 2 (AutoAWQ's order 0 2 4 6 1 3 5 7); awq_scales [K/group_size, N]
 * fp16. Exact bit movement; N must be a multiple of 8. All pointers are device addresses. */
int int4gemv_repack_awq(void* qweight, void* scales, void* zeros, const void* awq_qweight,
                        const void* awq_qzeros, const void* awq_scales, int64_t n, int64_t k,
                        int64_t group_size, void* stream);

/* GPTQ checkpoint tensors -> the same outputs. gptq_qweight [K/8, N] int32 holds weight 8r + i of
 * column n in nibble i of word (r, n); gptq_qzeros [K/group_size, N/8] int32 holds column 8c + i in
 * nibble i, stored as z - zero_offset (1 for the original "gptq" format, 0 for "gptq_v2");
 * gptq_scales [K/group_size, N] fp16. Groups must be contiguous (no act-order g_idx). */
int int4gemv_repack_gptq(void* qweight, void* scales, void* zeros, const void* gptq_qweight,
                         const void* gptq_qzeros, const void* gptq_scales, int zero_offset,
                         int64_t n, int64_t k, int64_t group_size, void* stream);

/* ---- Sharded layers with the exchange fused into the GEMV (new: the reference is single-GPU) -- */

/* One process per GPU of a node. Each rank allocates its exchange buffers with
 * int4gemv_peer_alloc (zeroed device memory plus a CUDA IPC handle of INT4GEMV_IPC_HANDLE_BYTES),
 * sends the handle to the other ranks (any host channel) and maps theirs with int4gemv_peer_open.
 * Release with int4gemv_peer_close (mapped peers' buffers) and int4gemv_peer_free (own). */
#define INT4GEMV_IPC_HANDLE_BYTES 64
int int4gemv_peer_alloc(int64_t bytes, void** ptr, void* ipc_handle);
int int4gemv_peer_open(const void* ipc_handle, void** ptr);
int int4gemv_peer_close(void* ptr);
int int4gemv_peer_free(void* ptr);

#define INT4GEMV_MAX_PEERS 8
#define INT4GEMV_SHARD_ROWS 0  /* N split: every rank gets y [m, n_total] (all-gather) */
#define INT4GEMV_SHARD_K 1     /* K split: every rank gets y [m, n] = sum of partials */
#define INT4GEMV_PEER_COUNTER_BYTES 4096  /* a rank's call counter words */

typedef struct {
  int32_t world, rank, mode, reserved;
  int64_t n_total;    /* ROWS: columns of the gathered y; must be n x world (equal shards) */
  int64_t col0;       /* ROWS: first column of this rank's shard in y; must be n x rank */
  int64_t out_bytes;  /* size of every rank's out buffer, the same on every rank */
  /* out[r]: rank r's exchange buffer, mapped here (out[rank] is this rank's own), two halves used
   * by alternate calls, each an array of 8-byte words (data and call number in one store).
   * ROWS: a half holds m x n_total words (out_bytes >= 16 m n_total). K: a half holds
   * world x m x n words (out_bytes >= 16 world m n). */
  void* out[INT4GEMV_MAX_PEERS];
  /* this rank's call counters, INT4GEMV_PEER_COUNTER_BYTES, zeroed once at allocation
   * (int4gemv_peer_alloc does) and then owned by the kernel: they hold the number of the last
   * completed call, so calls need no host-side state and replay from a captured CUDA graph.
   * Use one out buffer set and one counter buffer per sharded matrix. */
  void* counters;
} int4gemv_peers_t;

/* sizeof(int4gemv_peers_t), for bindings that build the struct themselves. */
size_t int4gemv_peers_struct_bytes(void);

/* The GEMV of this rank's shard with the exchange fused into its epilogue, on the fast path's
 * shapes (group_size 128, K % 1024 == 0, M <= 32), y [m, n_total] (ROWS) or [m, n] (K) fp16.
 * The shard's GEMV runs on stripe_mma where it takes the shape (M <= 8, K % 2048 == 0, 16-byte
 * aligned pointers), else on stream_mma; ranks whose K shares differ may run different kernels,
 * the exchange words are the same.
 * ROWS: the shard's rows are columns [col0, col0 + n) of y; each CTA writes its outputs, each
 * tagged with the call number in the same 8-byte store, into every rank's exchange buffer over
 * NVLink (peer stores), then copies the rows its counterpart CTAs wrote into y as their tags show
 * this call, so when the kernel completes y is whole. K: each CTA writes its fp32 partial sums,
 * tagged, into every rank's exchange buffer and writes y = the ranks' partials added in rank order
 * (bit-identical on every rank).
 * Every rank must make the same sequence of calls on a set of buffers with the same m and n (the
 * call number advances once per call on every rank), and a rank's calls on one set of buffers
 * must be ordered on one stream (each after the previous one has completed or, with programmatic
 * dependent launch, past its dependency). A wait on a peer's word is bounded (2 s); when it runs out the kernel records
 * status 3 (int4gemv_device_status) and finishes with an undefined y. */
int int4gemv_w4a16_exchange(void* y, const void* x, const void* qweight, const void* scales,
                            const void* zeros, int64_t m, int64_t n, int64_t k, int64_t group_size,
                            const int4gemv_peers_t* peers, void* stream);

/* int4gemv_w4a16_exchange for a single rank (world 1, rank 0) with no allocation at all: its
 * exchange buffer and call-counter words are static device arrays in the library
 * (4 MiB + 4 KiB per device), so no int4gemv_peer_alloc and no caller buffers. mode
 * INT4GEMV_SHARD_ROWS or INT4GEMV_SHARD_K; y [m, n] fp16 as int4gemv_w4a16 computes it, through
 * the exchange epilogue. Sizes needing more than the static buffer (m x n > 256 Ki in either
 * mode) are rejected with INT4GEMV_ERR_INVALID and a message giving the limit; so are the shapes
 * the fast path does not take (same checks as int4gemv_w4a16_exchange). Every such check runs
 * before the setup below, so a rejected call does no setup.
 * The first valid call on a device does the setup (looks up the arrays with cudaGetSymbolAddress
 * and clears the exchange buffer and the counters, synchronously), so it must come before any
 * stream capture. The looked-up addresses are kept for the life of the process: after
 * cudaDeviceReset on a device this entry point must not be used on that device again. All calls
 * on a device share the one buffer, whatever their shapes: calls that overlap in time (different
 * streams, or other host threads) race. No counterpart in the reference. */
int int4gemv_w4a16_exchange_static(void* y, const void* x, const void* qweight,
                                   const void* scales, const void* zeros, int64_t m, int64_t n,
                                   int64_t k, int64_t group_size, int mode, void* stream);

/* ---- Stream ordering of the weights ---------------------------------------------------------- */

/* The pipelined kernels (stripe_mma, tc_dequant, stream_mma, tcgen05, and the fused epilogues and
 * exchange on them) are launched with programmatic dependent launch: a call may start while the
 * previous kernel in the stream is still running, and by default it already streams its qweight,
 * scales and zeros then; x is read, and y written, only after that kernel has completed. This is
 * what lets back-to-back GEMVs keep HBM busy, and it is safe whenever the weights were not written
 * by the kernel right before the call in the same stream (weights loaded or repacked earlier, or
 * written by work that was followed by another kernel, an event or a copy, are fine). A caller
 * that does write the weights in the immediately preceding kernel (e.g. re-quantising in place and
 * then multiplying) calls int4gemv_set_strict_weights(1): every pipelined kernel then reads its
 * weights only after the previous kernel has completed, at some cost in overlap. Process-wide; 0
 * restores the default. INT4GEMV_ERR_INVALID for other values. No counterpart in the reference
 * (its kernels use plain stream order).
 */
int int4gemv_set_strict_weights(int strict);

/* ---- Device-side status --------------------------------------------------------------------- */

/* Reads and clears the current device's kernel status word: 0 if every pipelined kernel since the
 * last call finished normally, else a nonzero code recorded by a kernel whose bounded wait on a
 * shared-memory barrier timed out (the kernel then skipped its work and returned). Synchronises
 * the current device. */
int int4gemv_device_status(int* status);

#ifdef __cplusplus
}
#endif

#endif /* INT4GEMV_B200_H_ */
