// The weight stream shared by the fast kernels: a producer warp moves the packed weights, scales
// and zeros of a CTA's rows into a ring of shared-memory stages with 2-D TMA tile copies.
//
// A stage is one block of up to 32 rows x 8 items (an item = 128 weights = one quantisation group):
//   [0, 16384)          4 column chunks of 128 bytes x 32 rows (128-byte swizzle): packed words
//   [16384, 16896)      scales, 32 rows x 8 fp16
//   [16896, 17408)      zeros,  32 rows x 8 fp16
// Boxes are the binary decomposition of the block's row count (rounded up to 4) into 32 / 16 / 8 / 4
// rows, largest first, so a CTA never fetches a row it does not own and every box lands 1024-byte
// aligned. On B200 these 4 KB tiles stream at the same rate as large contiguous copies, while
// per-row 512-byte 1-D bulk copies reach less than half of it.
//
// Requirements (checked by weight_stream_supported): group_size == 128, K % 1024 == 0, qweight,
// scales and zeros 16-byte aligned.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"

namespace i4 {

constexpr int kItemK = 128;                                   // weights per item = group size
constexpr int kItemBytes = kItemK / 2;                        // packed bytes per item and row
constexpr int kItemsPerStage = 8;
constexpr int kStageRowBytes = kItemsPerStage * kItemBytes;   // 512: 4 chunks of 128 bytes
constexpr int kBlockRows = 32;
constexpr int kChunkBytes = kBlockRows * 128;
constexpr int kSzRowBytes = kItemsPerStage * 2;
constexpr int kStageQBytes = 4 * kChunkBytes;
constexpr int kStageBytes = kStageQBytes + 2 * kBlockRows * kSzRowBytes;  // 17408
constexpr int kStageTx = kStageRowBytes + 2 * kSzRowBytes;   // bytes landing per row per stage

// Box heights 32 >> h for tensor maps h = 0..3.
__host__ __device__ constexpr int box_height(int h) { return kBlockRows >> h; }

// qweight viewed as [N rows][K / 2 bytes] (128-byte boxes, 128-byte swizzle); scales and zeros as
// [N rows][K / 128] fp16 (8-group boxes); each with boxes of 32, 16, 8 and 4 rows.
struct WeightMaps {
  CUtensorMap q[4];
  CUtensorMap s[4];
  CUtensorMap z[4];
};

bool weight_stream_supported(const GemvArgs& a, const char** why);
// Encoded maps for this call's tensors (cached per device and pointer set).
cudaError_t weight_maps_for(const GemvArgs& a, WeightMaps* out);

// The tile this lane copies for a block of up to 32 rows: lane l copies weight column chunk l % 4
// of box l / 4 (lanes 0..15), or the scales (lanes 16..19) or zeros (lanes 20..23) of box l % 4.
// Boxes are the binary decomposition of the block's row count (rounded up to 4), largest first.
// Returns false if the lane has no box in this block.
struct LaneBox {
  const CUtensorMap* map;
  int dst_off;  // byte offset inside a stage
  int y;        // first row
  int kind;     // 0 weights, 1 scales, 2 zeros
  int chunk;
};

__device__ __forceinline__ bool lane_box(const WeightMaps& maps, int lane, int rows4, int block_row0,
                                         LaneBox* b) {
  const int box_idx = lane < 16 ? lane / 4 : lane % 4;
  int box_map = -1, box_off = 0;
  int n = 0, off = 0;
  for (int hi = 0; hi < 4; ++hi) {
    if (rows4 & box_height(hi)) {
      if (n == box_idx) {
        box_map = hi;
        box_off = off;
      }
      ++n;
      off += box_height(hi);
    }
  }
  if (lane >= 24 || box_map < 0) return false;
  b->kind = lane < 16 ? 0 : lane < 20 ? 1 : 2;
  b->chunk = lane % 4;
  b->y = block_row0 + box_off;
  b->map = b->kind == 0 ? &maps.q[box_map] : b->kind == 1 ? &maps.s[box_map] : &maps.z[box_map];
  b->dst_off = b->kind == 0   ? b->chunk * kChunkBytes + box_off * 128
               : b->kind == 1 ? kStageQBytes + box_off * kSzRowBytes
                              : kStageQBytes + (kBlockRows + box_off) * kSzRowBytes;
  return true;
}

__device__ __forceinline__ int box_x(const LaneBox& b, int j) {
  return b.kind == 0 ? j * kStageRowBytes + b.chunk * 128 : j * kItemsPerStage;
}

// One stage of one block: lane 0 arms full_bar with the stage's bytes, then every lane with a box
// copies its tile into `stage`.
__device__ __forceinline__ void issue_stage(const LaneBox& b, bool has_box, int j, int rows4,
                                            unsigned char* stage, uint64_t* full_bar,
                                            uint64_t policy, int lane) {
  if (lane == 0) mbar_arrive_expect_tx(full_bar, static_cast<uint32_t>(rows4 * kStageTx));
  __syncwarp();
  if (has_box) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(stage + b.dst_off)),
        "l"(b.map), "r"(box_x(b, j)), "r"(b.y), "r"(smem_addr(full_bar)), "l"(policy)
        : "memory");
  }
}

// The producer warp's loop. Streams the CTA's `rows` rows (from row_begin) in k-panels of
// `panel_steps` stages (panel_steps >= steps gives one panel): for each panel, for each block of
// 32 rows, the panel's stages in k order, through `n_stages` ring buffers. full[s] expects one
// arrival (lane 0's expect_tx) plus the bytes; empty[s] is released by the consumers. Returns
// after its last copies have landed. (Requesting the stages beyond the ring into L2 ahead of time
// was measured slower on B200: it delays other CTAs' tiles more than it hides latency.)
__device__ __forceinline__ void produce_weight_stages(const WeightMaps& maps, int row_begin,
                                                      int rows, int steps, int panel_steps,
                                                      unsigned char* stages, int n_stages,
                                                      uint64_t* full, uint64_t* empty,
                                                      int* status) {
  const int lane = threadIdx.x % kWarp;
  const uint64_t policy = l2_evict_first_policy();
  const int blocks = (rows + kBlockRows - 1) / kBlockRows;
  bool ok = true;
  int it = 0;
  int slot = 0, use = 0;
  for (int p0 = 0; p0 < steps; p0 += panel_steps) {
    const int p1 = min(steps, p0 + panel_steps);
    for (int blk = 0; blk < blocks; ++blk) {
      const int rows4 = (min(kBlockRows, rows - blk * kBlockRows) + 3) & ~3;
      LaneBox b;
      const bool has_box = lane_box(maps, lane, rows4, row_begin + blk * kBlockRows, &b);
      for (int j = p0; j < p1; ++j, ++it) {
        if (ok && use > 0 && !mbar_wait_bounded(&empty[slot], (use - 1) & 1)) {
          ok = false;
          if (lane == 0) atomicExch(status, kStatusEmptyBarrierTimeout);
        }
        if (ok) {
          issue_stage(b, has_box, j, rows4, stages + slot * kStageBytes, &full[slot], policy, lane);
        }
        if (++slot == n_stages) {
          slot = 0;
          ++use;
        }
      }
    }
  }
  // Do not leave while copies into this CTA's shared memory may be in flight.
  if (ok) {
    for (int back = 1; back <= min(it, n_stages); ++back) {
      const int j = it - back;
      if (!mbar_wait_bounded(&full[j % n_stages], (j / n_stages) & 1)) break;
    }
  }
}

// Words 4 c .. 4 c + 3 of item `item_s` (0..7) of block row `row` in a landed stage.
__device__ __forceinline__ uint4 stage_words(const unsigned char* stage, int row, int item_s,
                                             int c) {
  const int granule = ((item_s & 1) * 4 + c) ^ (row & 7);
  return *reinterpret_cast<const uint4*>(stage + (item_s >> 1) * kChunkBytes + row * 128 +
                                         granule * 16);
}

// Scale bits | zero bits << 16 of item `item_s` of block row `row` in a landed stage.
__device__ __forceinline__ uint32_t stage_sz(const unsigned char* stage, int row, int item_s) {
  const uint16_t* s = reinterpret_cast<const uint16_t*>(stage + kStageQBytes);
  const uint16_t* z = s + kBlockRows * kItemsPerStage;
  return static_cast<uint32_t>(s[row * kItemsPerStage + item_s]) |
         (static_cast<uint32_t>(z[row * kItemsPerStage + item_s]) << 16);
}

__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace i4
