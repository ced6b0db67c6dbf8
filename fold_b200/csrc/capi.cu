// Status reporting, device queries and the TMA descriptor cache of the C-ABI.
#include <cudaTypedefs.h>

#include <mutex>
#include <string>
#include <unordered_map>

#include "host_common.h"

namespace fold {

namespace {
thread_local std::string g_last_error;

struct MapKey {
  uintptr_t ptr;
  int pages, hkv, hd, box_rows, device;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && pages == o.pages && hkv == o.hkv && hd == o.hd && box_rows == o.box_rows &&
           device == o.device;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<uintptr_t>()(k.ptr);
    h ^= (static_cast<size_t>(k.pages) * 0x9E3779B97F4A7C15ull) + (h << 6) + (h >> 2);
    h ^= static_cast<size_t>(k.hkv) << 1 ^ static_cast<size_t>(k.hd) << 9 ^ static_cast<size_t>(k.box_rows) << 19 ^
         static_cast<size_t>(k.device) << 29;
    return h;
  }
};
std::mutex g_map_mutex;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int load_encode() {
  if (g_encode) return FOLD_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
    return fail(FOLD_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled is not available from the driver");
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return FOLD_OK;
}
}  // namespace

int fail(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return FOLD_OK;
  return fail(FOLD_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int check_launch(const char* what) { return check_cuda(cudaGetLastError(), what); }

int device_sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return n;
}

int side_tensor_map(const void* side, int pages, int hkv, int hd, int box_rows, CUtensorMap* out) {
  int dev = 0;
  if (int s = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return s;
  MapKey key{reinterpret_cast<uintptr_t>(side), pages, hkv, hd, box_rows, dev};
  std::lock_guard<std::mutex> lock(g_map_mutex);
  auto it = g_maps.find(key);
  if (it != g_maps.end()) {
    *out = it->second;
    return FOLD_OK;
  }
  if (int s = load_encode()) return s;
  if (!aligned16(side)) return fail(FOLD_ERR_ALIGNMENT, "side cache pointer is not 16-byte aligned");
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(2 * hd), 256u,
                              static_cast<cuuint64_t>(pages) * static_cast<cuuint64_t>(hkv)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(2 * hd) * 2u, static_cast<cuuint64_t>(256 * 2 * hd) * 2u};
  const cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(box_rows), 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  CUtensorMap m;
  CUresult r = g_encode(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(side), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FOLD_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(r));
  if (g_maps.size() > 4096) g_maps.clear();
  g_maps.emplace(key, m);
  *out = m;
  return FOLD_OK;
}

int fp8_side_tensor_map(const void* side8, int pages, int hkv, CUtensorMap* out) {
  int dev = 0;
  if (int s = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return s;
  // hd -1 marks the fp8 layout in the cache key
  MapKey key{reinterpret_cast<uintptr_t>(side8), pages, hkv, -1, 128, dev};
  std::lock_guard<std::mutex> lock(g_map_mutex);
  auto it = g_maps.find(key);
  if (it != g_maps.end()) {
    *out = it->second;
    return FOLD_OK;
  }
  if (int s = load_encode()) return s;
  if (!aligned16(side8)) return fail(FOLD_ERR_ALIGNMENT, "fp8 side cache pointer is not 16-byte aligned");
  // [pages][hkv][2 planes][2 halves][128 rows] rows of 128 bytes; one box = one 16 KB block
  const cuuint64_t dims[2] = {128u, static_cast<cuuint64_t>(pages) * static_cast<cuuint64_t>(hkv) * 512u};
  const cuuint64_t strides[1] = {128u};
  const cuuint32_t box[2] = {128u, 128u};
  const cuuint32_t estr[2] = {1u, 1u};
  CUtensorMap m;
  CUresult r = g_encode(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(side8), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(FOLD_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled (fp8 side cache) failed with CUresult " +
                                         std::to_string(r));
  if (g_maps.size() > 4096) g_maps.clear();
  g_maps.emplace(key, m);
  *out = m;
  return FOLD_OK;
}

int side_tensor_map_uncached(const void* side, int pages, int hkv, int hd, int box_rows, CUtensorMap* out) {
  {
    std::lock_guard<std::mutex> lock(g_map_mutex);
    if (int s = load_encode()) return s;
  }
  if (!aligned16(side)) return fail(FOLD_ERR_ALIGNMENT, "side cache pointer is not 16-byte aligned");
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(2 * hd), 256u,
                              static_cast<cuuint64_t>(pages) * static_cast<cuuint64_t>(hkv)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(2 * hd) * 2u, static_cast<cuuint64_t>(256 * 2 * hd) * 2u};
  const cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(box_rows), 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = g_encode(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(side), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FOLD_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled failed");
  return FOLD_OK;
}

}  // namespace fold

extern "C" {

const char* fold_status_string(int status) {
  switch (status) {
    case FOLD_OK: return "ok";
    case FOLD_ERR_INVALID_ARGUMENT: return "invalid argument";
    case FOLD_ERR_UNSUPPORTED: return "unsupported configuration";
    case FOLD_ERR_ALIGNMENT: return "misaligned pointer or stride";
    case FOLD_ERR_CUDA: return "CUDA error";
    case FOLD_ERR_TENSOR_MAP: return "TMA descriptor error";
    default: return "unknown status";
  }
}

const char* fold_last_error(void) { return fold::g_last_error.c_str(); }

int fold_version(void) { return 1; }

int fold_num_sms(void) { return fold::device_sm_count(); }

}  // extern "C"
