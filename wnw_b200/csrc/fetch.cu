// Zero-copy fetch of offloaded KV rows from pinned host memory (sm_100a).
//
// The reference gathers the planned CPU ranges into a pinned staging buffer
// with host memcpy and then issues one H2D copy (cache.py:868-889,
// planner.cpp:113-122).  At decode-time churn that host memcpy is the
// bottleneck, so here the GPU reads the rows itself: pinned host memory is
// mapped into the device address space, and a kernel on the copy stream
// streams every planned range over PCIe / C2C straight into the device
// landing buffer, one launch (and one event) per layer so layer l's rows
// arrive while earlier layers compute.
#include <algorithm>

#include "common.cuh"

namespace wnw {

constexpr int kFetchThreads = 256;
constexpr int kFetchUnroll = 8;

// ranges: [n][2] source rows [s, e); dst_row[i] = destination row of range i
__global__ void __launch_bounds__(kFetchThreads)
    fetch_rows_kernel(const uint4* __restrict__ src_k, const uint4* __restrict__ src_v, const int32_t* ranges,
                      const int64_t* dst_row, int n, uint4* dst_k, uint4* dst_v, int chunks_per_row) {
  for (int r = blockIdx.x; r < n; r += gridDim.x) {
    const int64_t s = ranges[2 * r];
    const int64_t e = ranges[2 * r + 1];
    const int64_t nchunk = (e - s) * chunks_per_row;
    const uint4* sk = src_k + s * chunks_per_row;
    const uint4* sv = src_v + s * chunks_per_row;
    uint4* dk = dst_k + dst_row[r] * chunks_per_row;
    uint4* dv = dst_v + dst_row[r] * chunks_per_row;
    for (int64_t base = 0; base < nchunk; base += int64_t(kFetchThreads) * kFetchUnroll) {
      uint4 bk[kFetchUnroll], bv[kFetchUnroll];
#pragma unroll
      for (int u = 0; u < kFetchUnroll; ++u) {
        const int64_t i = base + int64_t(u) * kFetchThreads + threadIdx.x;
        if (i < nchunk) {
          bk[u] = sk[i];
          bv[u] = sv[i];
        }
      }
#pragma unroll
      for (int u = 0; u < kFetchUnroll; ++u) {
        const int64_t i = base + int64_t(u) * kFetchThreads + threadIdx.x;
        if (i < nchunk) {
          dk[i] = bk[u];
          dv[i] = bv[u];
        }
      }
    }
  }
}

// Plain copy of n 16-byte words (the source may be mapped host memory).
__global__ void __launch_bounds__(kFetchThreads) copy_words_kernel(const uint4* __restrict__ src,
                                                                    uint4* __restrict__ dst, int64_t n) {
  for (int64_t i = int64_t(blockIdx.x) * kFetchThreads + threadIdx.x; i < n; i += int64_t(gridDim.x) * kFetchThreads)
    dst[i] = src[i];
}

}  // namespace wnw

extern "C" wnw_status wnw_copy_mapped(void* dst, const void* src, int64_t bytes, int max_ctas, void* stream) {
  using namespace wnw;
  if (bytes <= 0) return WNW_OK;
  WNW_CHECK_ARG(dst && src, "null pointer argument");
  WNW_CHECK_ARG(bytes % 16 == 0 && aligned16(dst) && aligned16(src), "16-byte aligned sizes and addresses only");
  const int64_t n = bytes / 16;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(max_ctas > 0 ? max_ctas : 32,
                                                                           (n + kFetchThreads - 1) / kFetchThreads)));
  copy_words_kernel<<<grid, kFetchThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), static_cast<uint4*>(dst), n);
  WNW_CUDA_TRY(cudaGetLastError());
  return WNW_OK;
}

extern "C" wnw_status wnw_host_device_pointer(const void* host_ptr, void** dev_ptr) {
  using namespace wnw;
  WNW_CHECK_ARG(host_ptr && dev_ptr, "null pointer argument");
  void* d = nullptr;
  WNW_CUDA_TRY(cudaHostGetDevicePointer(&d, const_cast<void*>(host_ptr), 0));
  *dev_ptr = d;
  return WNW_OK;
}

extern "C" wnw_status wnw_fetch_rows(const void* src_k, const void* src_v, int64_t row_bytes,
                                     const int32_t* ranges, const int64_t* dst_row, int n_ranges, void* dst_k,
                                     void* dst_v, int max_ctas, void* stream) {
  using namespace wnw;
  if (n_ranges <= 0) return WNW_OK;
  WNW_CHECK_ARG(src_k && src_v && ranges && dst_row && dst_k && dst_v, "null pointer argument");
  WNW_CHECK_ARG(row_bytes > 0 && row_bytes % 16 == 0, "row size must be a positive multiple of 16 bytes");
  WNW_CHECK_ARG(aligned16(src_k) && aligned16(src_v) && aligned16(dst_k) && aligned16(dst_v),
                "buffers must be 16-byte aligned");
  const int grid = std::max(1, std::min(n_ranges, max_ctas > 0 ? max_ctas : 1024));
  fetch_rows_kernel<<<grid, kFetchThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src_k), static_cast<const uint4*>(src_v), ranges, dst_row, n_ranges,
      static_cast<uint4*>(dst_k), static_cast<uint4*>(dst_v), static_cast<int>(row_bytes / 16));
  WNW_CUDA_TRY(cudaGetLastError());
  return WNW_OK;
}

extern "C" wnw_status wnw_fetch_layers(const void* src_k, const void* src_v, int64_t row_bytes,
                                       const int32_t* ranges, const int64_t* dst_row, const int32_t* layer_ranges,
                                       int num_layers, void* dst_k, void* dst_v, int max_ctas, void* stream,
                                       void* const* events) {
  using namespace wnw;
  WNW_CHECK_ARG(layer_ranges && num_layers >= 0, "null layer offsets");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int l = 0; l < num_layers; ++l) {
    const int r0 = layer_ranges[l], r1 = layer_ranges[l + 1];
    WNW_CHECK_ARG(r1 >= r0 && r0 >= 0, "layer range offsets must be non-decreasing");
    if (r1 > r0) {
      const wnw_status st = wnw_fetch_rows(src_k, src_v, row_bytes, ranges + 2 * int64_t(r0), dst_row + r0,
                                           r1 - r0, dst_k, dst_v, max_ctas, stream);
      if (st != WNW_OK) return st;
    }
    if (events && events[l]) WNW_CUDA_TRY(cudaEventRecord(static_cast<cudaEvent_t>(events[l]), s));
  }
  return WNW_OK;
}
