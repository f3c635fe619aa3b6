// Tensor-map construction and cache (see lm_tmap.cuh).
#include <mutex>
#include <string>
#include <vector>

#include "lm_common.cuh"
#include "lm_tmap.cuh"

namespace lm {
namespace {

constexpr int BK = 64;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

struct MapKey {
  const void* ptr;
  uint64_t d[2];
  int rank;
  int box_rows;
  int box_depth;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && d[0] == o.d[0] && d[1] == o.d[1] && rank == o.rank &&
           box_rows == o.box_rows && box_depth == o.box_depth;
  }
};

struct MapCache {
  std::mutex mu;
  std::vector<std::pair<MapKey, CUtensorMap>> entries;
};

MapCache& map_cache() {
  static MapCache c;
  return c;
}

}  // namespace

int make_map(CUtensorMap* out, const void* ptr, int rank, uint64_t d0, uint64_t d1,
             int box_rows, int box_depth) {
  const MapKey key{ptr, {d0, d1}, rank, box_rows, box_depth};
  MapCache& cache = map_cache();
  {
    std::lock_guard<std::mutex> lk(cache.mu);
    for (auto& e : cache.entries)
      if (e.first == key) {
        *out = e.second;
        return LM_OK;
      }
  }
  auto fn = encode_fn();
  if (fn == nullptr) return fail(LM_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3];
  cuuint64_t strides[2];
  if (rank == 2) {
    dims[0] = d0;
    dims[1] = d1;
    strides[0] = d0 * 2;
  } else {
    dims[0] = BK;
    dims[1] = 128;
    dims[2] = d0;  // number of 128 x 64 tiles
    strides[0] = BK * 2;
    strides[1] = BK * 128 * 2;
  }
  cuuint32_t box[3] = {static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(box_rows),
                       static_cast<cuuint32_t>(box_depth)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMap m;
  const CUresult r = fn(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, static_cast<cuuint32_t>(rank),
                        const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(LM_ERR_CUDA, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(r));
  {
    std::lock_guard<std::mutex> lk(cache.mu);
    if (cache.entries.size() >= 256) cache.entries.erase(cache.entries.begin());
    cache.entries.emplace_back(key, m);
  }
  *out = m;
  return LM_OK;
}


}  // namespace lm
