// C-ABI plumbing: status strings, thread-local error messages, host gather of
// offloaded rows into pinned staging, and the per-layer async H2D copy.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/wnw_b200.h"

namespace wnw {

namespace {
thread_local char g_err[512] = {0};
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

wnw_status cuda_status(cudaError_t e, const char* what) {
  set_error("%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
  return WNW_ERR_CUDA;
}

}  // namespace wnw

extern "C" {

int wnw_abi_version(void) { return WNW_ABI_VERSION; }

const char* wnw_status_string(wnw_status s) {
  switch (s) {
    case WNW_OK: return "ok";
    case WNW_ERR_INVALID: return "invalid argument";
    case WNW_ERR_CUDA: return "CUDA error";
    case WNW_ERR_CAPACITY: return "capacity exceeded";
    case WNW_ERR_STATE: return "invalid state";
    case WNW_ERR_TIMEOUT: return "timed out";
    case WNW_ERR_UNSUPPORTED: return "unsupported";
  }
  return "unknown status";
}

const char* wnw_last_error(void) { return wnw::g_err; }

// planner.cpp:104-122: rows of every planned range, in plan order, packed
// back to back.  Ranges are split over threads by destination row so each
// thread copies a contiguous slice of the staging buffer.
wnw_status wnw_gather_rows(const void* src_k, const void* src_v, int64_t row_bytes, const int32_t* ranges,
                           int n_pairs, void* dst_k, void* dst_v, int n_threads) {
  if (n_pairs <= 0) return WNW_OK;
  if (!src_k || !src_v || !ranges || !dst_k || !dst_v || row_bytes <= 0) {
    wnw::set_error("null argument or bad row size");
    return WNW_ERR_INVALID;
  }
  std::vector<int64_t> dst_row(n_pairs + 1, 0);
  for (int i = 0; i < n_pairs; ++i) {
    const int64_t n = int64_t(ranges[2 * i + 1]) - ranges[2 * i];
    if (n < 0 || ranges[2 * i] < 0) {
      wnw::set_error("bad range %d: [%d, %d)", i, ranges[2 * i], ranges[2 * i + 1]);
      return WNW_ERR_INVALID;
    }
    dst_row[i + 1] = dst_row[i] + n;
  }
  const char* sk = static_cast<const char*>(src_k);
  const char* sv = static_cast<const char*>(src_v);
  char* dk = static_cast<char*>(dst_k);
  char* dv = static_cast<char*>(dst_v);
  auto work = [&](int lo, int hi) {
    for (int i = lo; i < hi; ++i) {
      const int64_t n = dst_row[i + 1] - dst_row[i];
      std::memcpy(dk + dst_row[i] * row_bytes, sk + int64_t(ranges[2 * i]) * row_bytes, n * row_bytes);
      std::memcpy(dv + dst_row[i] * row_bytes, sv + int64_t(ranges[2 * i]) * row_bytes, n * row_bytes);
    }
  };
  const int64_t total_bytes = dst_row[n_pairs] * row_bytes * 2;
  int nt = std::max(1, std::min(n_threads, n_pairs));
  if (total_bytes < (4 << 20)) nt = 1;  // thread start-up costs more than small copies
  if (nt == 1) {
    work(0, n_pairs);
    return WNW_OK;
  }
  std::vector<std::thread> th;
  th.reserve(nt);
  const int64_t per = (dst_row[n_pairs] + nt - 1) / nt;
  int lo = 0;
  for (int t = 0; t < nt && lo < n_pairs; ++t) {
    const int64_t target = std::min<int64_t>(dst_row[n_pairs], per * (t + 1));
    int hi = lo;
    while (hi < n_pairs && dst_row[hi + 1] <= target) ++hi;
    if (t == nt - 1) hi = n_pairs;
    if (hi == lo && lo < n_pairs) hi = lo + 1;
    th.emplace_back(work, lo, hi);
    lo = hi;
  }
  for (auto& t : th) t.join();
  return WNW_OK;
}

wnw_status wnw_copy_async(void* dst, const void* src, int64_t bytes, void* stream) {
  if (bytes <= 0) return WNW_OK;
  if (!dst || !src) {
    wnw::set_error("null argument");
    return WNW_ERR_INVALID;
  }
  const cudaError_t e = cudaMemcpyAsync(dst, src, size_t(bytes), cudaMemcpyDefault, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return wnw::cuda_status(e, "cudaMemcpyAsync");
  return WNW_OK;
}

wnw_status wnw_stream_wait_event(void* stream, void* event) {
  if (!event) {
    wnw::set_error("null event");
    return WNW_ERR_INVALID;
  }
  const cudaError_t e = cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), static_cast<cudaEvent_t>(event), 0);
  if (e != cudaSuccess) return wnw::cuda_status(e, "cudaStreamWaitEvent");
  return WNW_OK;
}

wnw_status wnw_h2d_async(void* dst_k, void* dst_v, const void* src_k, const void* src_v, int64_t bytes,
                         void* stream, void* event) {
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bytes > 0) {
    if (!dst_k || !dst_v || !src_k || !src_v) {
      wnw::set_error("null argument");
      return WNW_ERR_INVALID;
    }
    cudaError_t e = cudaMemcpyAsync(dst_k, src_k, size_t(bytes), cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return wnw::cuda_status(e, "cudaMemcpyAsync(K)");
    e = cudaMemcpyAsync(dst_v, src_v, size_t(bytes), cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return wnw::cuda_status(e, "cudaMemcpyAsync(V)");
  }
  if (event) {
    cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(event), s);
    if (e != cudaSuccess) return wnw::cuda_status(e, "cudaEventRecord");
  }
  return WNW_OK;
}

}  // extern "C"
