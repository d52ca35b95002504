// Host encoding of TMA tensor maps (driver entry point reached through the
// runtime, so the library needs no direct libcuda link).
#include "tensor_map.hpp"

#include <map>
#include <mutex>
#include <tuple>

namespace lfm3 {
namespace {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t,
                                 void*, const cuuint64_t*, const cuuint64_t*,
                                 const cuuint32_t*, const cuuint32_t*,
                                 CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion,
                                 CUtensorMapFloatOOBfill);

EncodeTiled Encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult status;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p,
                                cudaEnableDefault, &status) == cudaSuccess &&
        status == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

}  // namespace

cudaError_t encode_q8_rows(CUtensorMap* map, const void* base, size_t row_bytes,
                           int rows, int box_bytes, int box_rows) {
  const EncodeTiled encode = Encoder();
  if (!encode)
    return cudaErrorNotSupported;
  if (row_bytes % 16 || box_bytes % 16 || box_bytes < 16 ||
      box_bytes / 8 > 256 || box_rows < 1 || box_rows > 256 || rows < 1 ||
      reinterpret_cast<uintptr_t>(base) % 16)
    return cudaErrorInvalidValue;
  const cuuint64_t dims[2] = {row_bytes / 8, cuuint64_t(rows)};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {cuuint32_t(box_bytes / 8), cuuint32_t(box_rows)};
  const cuuint32_t element_strides[2] = {1, 1};
  const CUresult r = encode(
      map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims,
      strides, box, element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
      CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t encode_activation_map(CUtensorMap* map, const void* base, int rows,
                                  int cols, int box_rows, int box_cols) {
  const EncodeTiled encode = Encoder();
  if (!encode)
    return cudaErrorNotSupported;
  if (rows < 1 || cols % 8 || box_cols * 2 != 64 || box_rows < 1 ||
      box_rows > 256 || reinterpret_cast<uintptr_t>(base) % 16)
    return cudaErrorInvalidValue;
  const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(cols) * 2};
  const cuuint32_t box[2] = {cuuint32_t(box_cols), cuuint32_t(box_rows)};
  const cuuint32_t element_strides[2] = {1, 1};
  const CUresult r = encode(
      map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
      strides, box, element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
      CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

namespace {
// kind, base, size, rows, box width, box rows
using MapKey = std::tuple<int, const void*, size_t, int, int, int>;
std::mutex g_map_mutex;
std::map<MapKey, CUtensorMap> g_maps;

template <typename Encode>
cudaError_t Cached(const MapKey& key, CUtensorMap* map, Encode encode) {
  {
    std::lock_guard<std::mutex> lock(g_map_mutex);
    const auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *map = it->second;
      return cudaSuccess;
    }
  }
  const cudaError_t e = encode();
  if (e != cudaSuccess)
    return e;
  std::lock_guard<std::mutex> lock(g_map_mutex);
  if (g_maps.size() >= 4096)
    g_maps.clear();
  g_maps.emplace(key, *map);
  return cudaSuccess;
}
}  // namespace

cudaError_t cached_q8_rows(CUtensorMap* map, const void* base, size_t row_bytes,
                           int rows, int box_bytes, int box_rows) {
  return Cached(MapKey{0, base, row_bytes, rows, box_bytes, box_rows}, map,
                [&] {
                  return encode_q8_rows(map, base, row_bytes, rows, box_bytes,
                                        box_rows);
                });
}

cudaError_t cached_activation_map(CUtensorMap* map, const void* base, int rows,
                                  int cols, int box_rows, int box_cols) {
  return Cached(MapKey{1, base, size_t(cols), rows, box_cols, box_rows}, map,
                [&] {
                  return encode_activation_map(map, base, rows, cols, box_rows,
                                               box_cols);
                });
}

}  // namespace lfm3
