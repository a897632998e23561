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
#include <cstring>
#include <map>
#include <memory>
#include <mutex>

#include "common.cuh"
#include "fetch_graph.h"

namespace wnw {

constexpr int kFetchThreads = 256;
constexpr int kFetchUnroll = 8;

// Copy range r (source rows [s, e) -> destination row dst_row[r]) with the
// block's threads, eight 16-byte words per thread in flight per tensor.
__device__ __forceinline__ void fetch_range(const uint4* __restrict__ src_k, const uint4* __restrict__ src_v,
                                            const int32_t* ranges, const int64_t* dst_row, int r, uint4* dst_k,
                                            uint4* dst_v, int chunks_per_row) {
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

// ranges: [n][2] source rows [s, e); dst_row[i] = destination row of range i
__global__ void __launch_bounds__(kFetchThreads)
    fetch_rows_kernel(const uint4* __restrict__ src_k, const uint4* __restrict__ src_v, const int32_t* ranges,
                      const int64_t* dst_row, int n, uint4* dst_k, uint4* dst_v, int chunks_per_row) {
  for (int r = blockIdx.x; r < n; r += gridDim.x)
    fetch_range(src_k, src_v, ranges, dst_row, r, dst_k, dst_v, chunks_per_row);
}

// The ranges of one layer, [layer_ranges[layer], layer_ranges[layer + 1]),
// read from device memory so the launch itself is the same every step.
__global__ void __launch_bounds__(kFetchThreads)
    fetch_layer_kernel(const uint4* __restrict__ src_k, const uint4* __restrict__ src_v, const int32_t* ranges,
                       const int64_t* dst_row, const int32_t* layer_ranges, int layer, uint4* dst_k, uint4* dst_v,
                       int chunks_per_row) {
  const int r0 = layer_ranges[layer], r1 = layer_ranges[layer + 1];
  for (int r = r0 + static_cast<int>(blockIdx.x); r < r1; r += gridDim.x)
    fetch_range(src_k, src_v, ranges, dst_row, r, dst_k, dst_v, chunks_per_row);
}

// ------------------------------------------------------------ step graph
// The per-step fetch as one CUDA graph, built once per set of buffers: the
// plan / range / offset tables go up (memcpy nodes, sizes updated per step),
// then per layer one fetch_layer_kernel followed by an external record of the
// layer's event.  One graph launch replaces 3 copies, L launches and L event
// records on the host.
struct FetchGraph {
  FetchGraphKey key;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  cudaGraphNode_t cp_plan = nullptr, cp_rng = nullptr, cp_dst = nullptr, cp_lr = nullptr;
  int32_t* lr_host = nullptr;
  int32_t* lr_dev = nullptr;
  ~FetchGraph() {
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    if (lr_host) cudaFreeHost(lr_host);
    if (lr_dev) cudaFree(lr_dev);
  }
};

static std::mutex g_graph_mu;
static std::map<const void*, std::unique_ptr<FetchGraph>> g_graphs;

static wnw_status build_graph(FetchGraph* fg, const FetchGraphKey& k, void* const* events) {
  fg->key = k;
  const bool planned = k.layer_ranges_dev != nullptr;
  WNW_CUDA_TRY(cudaGraphCreate(&fg->graph, 0));
  cudaGraph_t g = fg->graph;
  cudaGraphNode_t prev[4] = {};
  int nprev = 0;
  if (!planned) {
    WNW_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void**>(&fg->lr_host), sizeof(int32_t) * (k.L + 1),
                               cudaHostAllocDefault));
    WNW_CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(&fg->lr_dev), sizeof(int32_t) * (k.L + 1)));
    // placeholder sizes (16 bytes); the real ones are set before every launch
    WNW_CUDA_TRY(cudaGraphAddMemcpyNode1D(&fg->cp_plan, g, nullptr, 0, k.plan_dev, k.plan_host, 16,
                                          cudaMemcpyHostToDevice));
    WNW_CUDA_TRY(cudaGraphAddMemcpyNode1D(&fg->cp_rng, g, nullptr, 0, k.ranges_dev, k.ranges_host, 16,
                                          cudaMemcpyHostToDevice));
    WNW_CUDA_TRY(cudaGraphAddMemcpyNode1D(&fg->cp_dst, g, nullptr, 0, k.dst_dev, k.dst_host, 16,
                                          cudaMemcpyHostToDevice));
    WNW_CUDA_TRY(cudaGraphAddMemcpyNode1D(&fg->cp_lr, g, nullptr, 0, fg->lr_dev, fg->lr_host,
                                          sizeof(int32_t) * (k.L + 1), cudaMemcpyHostToDevice));
    prev[0] = fg->cp_plan;
    prev[1] = fg->cp_rng;
    prev[2] = fg->cp_dst;
    prev[3] = fg->cp_lr;
    nprev = 4;
  }
  const int cpr = static_cast<int>(k.row_bytes / 16);
  for (int l = 0; l < k.L; ++l) {
    const uint4* sk = static_cast<const uint4*>(k.src_k);
    const uint4* sv = static_cast<const uint4*>(k.src_v);
    const int32_t* rng = static_cast<const int32_t*>(k.ranges_dev);
    const int64_t* dst = static_cast<const int64_t*>(k.dst_dev);
    const int32_t* lr = planned ? k.layer_ranges_dev : fg->lr_dev;
    int layer = l;
    uint4* dk = static_cast<uint4*>(k.land_k);
    uint4* dv = static_cast<uint4*>(k.land_v);
    int c = cpr;
    void* args[] = {&sk, &sv, &rng, &dst, &lr, &layer, &dk, &dv, &c};
    cudaKernelNodeParams kp = {};
    kp.func = reinterpret_cast<void*>(fetch_layer_kernel);
    kp.gridDim = dim3(std::max(1, k.max_ctas), 1, 1);
    kp.blockDim = dim3(kFetchThreads, 1, 1);
    kp.sharedMemBytes = 0;
    kp.kernelParams = args;
    cudaGraphNode_t kn, en;
    WNW_CUDA_TRY(cudaGraphAddKernelNode(&kn, g, prev, nprev, &kp));
    if (events && events[l]) {
      WNW_CUDA_TRY(cudaGraphAddEventRecordNode(&en, g, &kn, 1, static_cast<cudaEvent_t>(events[l])));
    }
    prev[0] = kn;
    nprev = 1;
  }
  WNW_CUDA_TRY(cudaGraphInstantiate(&fg->exec, g, 0));
  return WNW_OK;
}

wnw_status fetch_graph_issue(const void* owner, const FetchGraphKey& k, int64_t plan_ints, int64_t n_ranges,
                             const int32_t* layer_ranges, void* stream, void* const* events) {
  std::lock_guard<std::mutex> lock(g_graph_mu);
  auto& slot = g_graphs[owner];
  if (!slot || !(slot->key == k)) {
    slot.reset(new FetchGraph());
    const wnw_status st = build_graph(slot.get(), k, events);
    if (st != WNW_OK) {
      slot.reset();
      return st;
    }
  }
  FetchGraph* fg = slot.get();
  std::memcpy(fg->lr_host, layer_ranges, sizeof(int32_t) * (k.L + 1));
  const size_t nr = static_cast<size_t>(std::max<int64_t>(n_ranges, 1));
  WNW_CUDA_TRY(cudaGraphExecMemcpyNodeSetParams1D(fg->exec, fg->cp_plan, k.plan_dev, k.plan_host,
                                                   sizeof(int32_t) * std::max<int64_t>(plan_ints, 4),
                                                   cudaMemcpyHostToDevice));
  WNW_CUDA_TRY(cudaGraphExecMemcpyNodeSetParams1D(fg->exec, fg->cp_rng, k.ranges_dev, k.ranges_host,
                                                   sizeof(int32_t) * 2 * nr, cudaMemcpyHostToDevice));
  WNW_CUDA_TRY(cudaGraphExecMemcpyNodeSetParams1D(fg->exec, fg->cp_dst, k.dst_dev, k.dst_host, sizeof(int64_t) * nr,
                                                   cudaMemcpyHostToDevice));
  WNW_CUDA_TRY(cudaGraphLaunch(fg->exec, static_cast<cudaStream_t>(stream)));
  return WNW_OK;
}

wnw_status fetch_graph_issue_planned(const void* owner, const FetchGraphKey& k, void* stream) {
  if (!k.layer_ranges_dev) {
    set_error("fetch_graph_issue_planned: no device layer offsets");
    return WNW_ERR_INVALID;
  }
  std::lock_guard<std::mutex> lock(g_graph_mu);
  auto& slot = g_graphs[owner];
  if (!slot || !(slot->key == k)) {
    slot.reset(new FetchGraph());
    const wnw_status st = build_graph(slot.get(), k, k.events);
    if (st != WNW_OK) {
      slot.reset();
      return st;
    }
  }
  WNW_CUDA_TRY(cudaGraphLaunch(slot->exec, static_cast<cudaStream_t>(stream)));
  return WNW_OK;
}

void fetch_graph_release(const void* owner) {
  std::lock_guard<std::mutex> lock(g_graph_mu);
  g_graphs.erase(owner);
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
