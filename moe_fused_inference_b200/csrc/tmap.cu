// tmap.cu — TMA tensor maps through the driver entry point exposed by the
// runtime (no link-time dependency on libcuda).
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>
#include <tuple>
#include <map>

#include "tmap.cuh"

namespace mfi {

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

static bool encode(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows,
                   uint32_t box_bytes, uint32_t box_rows, bool swizzle) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {row_bytes, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_bytes, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE,
            swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_tmap(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows,
               uint32_t box_rows) {
  return encode(m, base, row_bytes, rows, 128, box_rows, true);
}

static bool cached(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows,
                   uint32_t box_bytes, uint32_t box_rows, bool swizzle) {
  using Key = std::tuple<const void*, uint64_t, uint64_t, uint32_t, uint32_t, bool>;
  static std::mutex mu;
  static std::map<Key, CUtensorMap> cache;
  const Key key{base, row_bytes, rows, box_bytes, box_rows, swizzle};
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *m = it->second;
      return true;
    }
  }
  if (!encode(m, base, row_bytes, rows, box_bytes, box_rows, swizzle)) return false;
  std::lock_guard<std::mutex> g(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *m);
  return true;
}

bool get_tmap(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows,
              uint32_t box_rows) {
  return cached(m, base, row_bytes, rows, 128, box_rows, true);
}

bool get_tmap_plain(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows,
                    uint32_t box_bytes, uint32_t box_rows) {
  return cached(m, base, row_bytes, rows, box_bytes, box_rows, false);
}

cudaError_t ensure_dynamic_smem(const void* fn, size_t bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, size_t> granted;
  std::lock_guard<std::mutex> g(mu);
  size_t& have = granted[{dev, fn}];
  if (have >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
  if (e == cudaSuccess) have = bytes;
  return e;
}

}  // namespace mfi
