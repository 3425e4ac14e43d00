// Host side of the TMA weight stream: support checks and the tensor maps (encoded once per
// device and tensor set, then cached, so a decode loop over the same weights encodes nothing).
#include "weight_stream.cuh"

#include <mutex>
#include <vector>

namespace i4 {
namespace {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

struct MapEntry {
  int dev;
  const void* q;
  const void* s;
  const void* z;
  int n, k;
  WeightMaps maps;
};
std::mutex g_map_mu;
std::vector<MapEntry> g_maps;  // most recently used first
constexpr size_t kMapCache = 64;

}  // namespace

bool weight_stream_supported(const GemvArgs& a, const char** why) {
  auto fail = [&](const char* reason) {
    if (why) *why = reason;
    return false;
  };
  if (a.group != kItemK) return fail("group_size must be 128");
  if (a.k % (kItemK * kItemsPerStage) != 0) return fail("K must be a multiple of 1024");
  if (reinterpret_cast<uintptr_t>(a.q) % 16 || reinterpret_cast<uintptr_t>(a.s) % 16 ||
      reinterpret_cast<uintptr_t>(a.z) % 16)
    return fail("qweight, scales and zeros must be 16-byte aligned");
  return true;
}

cudaError_t weight_maps_for(const GemvArgs& a, WeightMaps* out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  std::lock_guard<std::mutex> lock(g_map_mu);
  for (size_t i = 0; i < g_maps.size(); ++i) {
    const MapEntry& e = g_maps[i];
    if (e.dev == dev && e.q == a.q && e.s == a.s && e.z == a.z && e.n == a.n && e.k == a.k) {
      *out = e.maps;
      if (i != 0) std::swap(g_maps[i], g_maps[0]);
      return cudaSuccess;
    }
  }
  auto encode = encode_fn();
  if (!encode) return cudaErrorNotSupported;
  MapEntry e{dev, a.q, a.s, a.z, a.n, a.k, {}};
  const cuuint32_t estr[2] = {1, 1};
  for (int hi = 0; hi < 4; ++hi) {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(a.k / 2), static_cast<cuuint64_t>(a.n)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.k / 2)};
    const cuuint32_t box[2] = {128, static_cast<cuuint32_t>(box_height(hi))};
    const CUresult r = encode(&e.maps.q[hi], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                              const_cast<uint32_t*>(a.q), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
    const int groups = a.k / a.group;
    const cuuint64_t sdims[2] = {static_cast<cuuint64_t>(groups), static_cast<cuuint64_t>(a.n)};
    const cuuint64_t sstrides[1] = {static_cast<cuuint64_t>(groups) * 2};
    const cuuint32_t sbox[2] = {static_cast<cuuint32_t>(kItemsPerStage),
                                static_cast<cuuint32_t>(box_height(hi))};
    for (int which = 0; which < 2; ++which) {
      const CUresult rs = encode(which == 0 ? &e.maps.s[hi] : &e.maps.z[hi],
                                 CU_TENSOR_MAP_DATA_TYPE_UINT16, 2,
                                 const_cast<half*>(which == 0 ? a.s : a.z), sdims, sstrides, sbox,
                                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                 CU_TENSOR_MAP_L2_PROMOTION_NONE,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (rs != CUDA_SUCCESS) return cudaErrorInvalidValue;
    }
  }
  g_maps.insert(g_maps.begin(), e);
  if (g_maps.size() > kMapCache) g_maps.pop_back();
  *out = e.maps;
  return cudaSuccess;
}

}  // namespace i4
