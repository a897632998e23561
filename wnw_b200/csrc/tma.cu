// Host side of the tensor-map cache (cuTensorMapEncodeTiled through the
// runtime's driver entry point; no libcuda link needed).
#include <cudaTypedefs.h>

#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "tma.cuh"

namespace wnw {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

using Key = std::tuple<uintptr_t, int64_t, int, int, int>;
std::mutex g_mu;
std::map<Key, CUtensorMap> g_maps;

}  // namespace

bool kv_tensor_map(CUtensorMap* out, const void* base, int64_t rows, int head_dim, int dtype, int box_rows) {
  const Key key{reinterpret_cast<uintptr_t>(base), rows, head_dim, dtype, box_rows};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *out = it->second;
      return true;
    }
  }
  auto fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return false;
  }
  if (dtype == WNW_F32) {
    set_error("tensor maps are built for 16-bit stores only");
    return false;
  }
  CUtensorMap m;
  std::memset(&m, 0, sizeof(m));
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(head_dim) * 2};
  const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = dtype == WNW_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = fn(&m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (%d) for %lld rows x %d", static_cast<int>(r),
              static_cast<long long>(rows), head_dim);
    return false;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_maps.size() > 4096) g_maps.clear();  // stores are long-lived; bound the cache anyway
  g_maps[key] = m;
  *out = m;
  return true;
}

}  // namespace wnw
