// Decode attention for callers that cannot allocate device memory.
//
// wnw_decode_attn needs two pieces of scratch besides its inputs and outputs:
// the per-cluster partial softmax states and the per-segment arrival
// counters.  Some hosts of this path own every byte of device memory
// themselves -- a serving engine that partitions a fixed memory budget up
// front, or a plugin host that hands an extension only the buffers it
// created -- and a cudaMalloc from inside the decode step would either fail
// there or bypass the host's accounting (and it also synchronises the
// device).  For them this entry point keeps the scratch in a file-scope
// device array of fixed size, so the call allocates nothing.
//
// The array is one per device per process, shared by every call: calls that
// overlap on the GPU (different streams, or concurrent host threads) race on
// it.  Each call clears the counters it uses before the launch.  The device
// address of the array is looked up on the first call made in a CUDA context
// (with that context current) and again whenever the current context of the
// device changes (after a cudaDeviceReset, say); make the first call of a
// context before any stream capture.
#include <cuda.h>

#include <mutex>

#include "decode_attn.cuh"

namespace wnw {
namespace {

constexpr int64_t kPartialBytes = int64_t(WNW_NOALLOC_MAX_PARTIAL_FLOATS) * 4;
constexpr int64_t kCounterBytes = int64_t(WNW_NOALLOC_MAX_SEGS) * 4;
constexpr int64_t kScratchBytes = kPartialBytes + kCounterBytes;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

std::mutex g_mu;
void* g_addr[kMaxDevices] = {};
CUcontext g_ctx[kMaxDevices] = {};

// the driver's cuCtxGetCurrent (this library links only the CUDA runtime)
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  }
  return fn;
}

// device address of g_noalloc_scratch in the current context of the current
// device; an address taken in a context that has since been destroyed is
// never reused
wnw_status scratch_address(void** out) {
  int dev = 0;
  WNW_CUDA_TRY(cudaGetDevice(&dev));
  WNW_CHECK_ARG(dev >= 0 && dev < kMaxDevices, "device index %d out of range", dev);
  const CtxGetCurrentFn get = ctx_get_current();
  if (get == nullptr) {
    set_error("cuCtxGetCurrent is not available from the driver");
    return WNW_ERR_CUDA;
  }
  CUcontext ctx = nullptr;
  if (get(&ctx) == CUDA_SUCCESS && ctx == nullptr) {
    WNW_CUDA_TRY(cudaSetDevice(dev));  // makes the device's primary context current
    get(&ctx);
  }
  if (ctx == nullptr) {
    set_error("no current CUDA context on device %d", dev);
    return WNW_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_addr[dev] == nullptr || g_ctx[dev] != ctx) {
    void* p = nullptr;
    WNW_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_addr[dev] = p;
    g_ctx[dev] = ctx;
  }
  *out = g_addr[dev];
  return WNW_OK;
}

}  // namespace
}  // namespace wnw

extern "C" wnw_status wnw_decode_attn_noalloc(const wnw_decode_attn_args* a, void* stream) {
  using namespace wnw;
  WNW_CHECK_ARG(a != nullptr, "null args");
  WNW_CHECK_ARG(a->err != nullptr, "err (a device word the caller owns) is required");
  WNW_CHECK_ARG(a->n_clusters >= 0 && a->plan_parts >= 0 && a->group >= 1 && a->head_dim > 0 && a->num_segs >= 0,
                "bad sizes");
  // partial slots: the plan's cluster partials (tensor-core path) or one per cluster
  const bool plan = a->plan != nullptr;
  const int slots = plan ? a->plan_parts : a->n_clusters;
  const int64_t need = int64_t(slots) * a->group * (a->head_dim + 2);
  if (need > WNW_NOALLOC_MAX_PARTIAL_FLOATS) {
    set_error("%lld partial floats needed (%d %s x group %d x (head_dim %d + 2)); the static scratch holds %d",
              static_cast<long long>(need), slots, plan ? "plan partials" : "clusters", a->group, a->head_dim,
              WNW_NOALLOC_MAX_PARTIAL_FLOATS);
    return WNW_ERR_CAPACITY;
  }
  if (a->num_segs > WNW_NOALLOC_MAX_SEGS) {
    set_error("%d segments; the static scratch holds counters for %d", a->num_segs, WNW_NOALLOC_MAX_SEGS);
    return WNW_ERR_CAPACITY;
  }
  void* base = nullptr;
  const wnw_status st = scratch_address(&base);
  if (st != WNW_OK) return st;
  wnw_decode_attn_args b = *a;
  b.partials = static_cast<float*>(base);
  b.counters = reinterpret_cast<int32_t*>(static_cast<unsigned char*>(base) + kPartialBytes);
  if ((!plan || a->plan_combine > 0) && b.num_segs > 0)  // arrival counters start at zero
    WNW_CUDA_TRY(cudaMemsetAsync(b.counters, 0, size_t(b.num_segs) * 4, static_cast<cudaStream_t>(stream)));
  return wnw_decode_attn(&b, stream);
}
