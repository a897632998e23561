// Tensor-parallel o_proj exchange in one kernel (sm_100a, NVLink peer memory).
//
// Under tensor parallelism by kv head, rank r holds the attention output of
// its query heads x_r [B, K] and the matching column slice of o_proj,
// W_r [N, K]; the layer output is y = sum_r x_r . W_r^T [B, N].  Each CTA
// owns a chunk of the N outputs: it computes this rank's partial sums for the
// chunk (a GEMV streaming W_r from HBM), stores them straight into every
// rank's receive buffer over NVLink, raises that rank's flag for the chunk
// (release at system scope), waits for every rank's flag in its own memory
// (acquire, bounded by a deadline) and adds the ranks' partials in rank order
// -- the same fp32 additions on every rank, so y is bit-identical everywhere.
//
// Receive buffers are double-buffered by the parity of the call's epoch: a
// rank cannot start call e+2 before every rank has finished reading call e,
// since call e+1 waits for every rank's call e+1 partials, which a rank
// sends only after its call e.
#include <algorithm>
#include <cstring>

#include "common.cuh"

namespace wnw {

constexpr int kTpThreads = 256;
constexpr int kTpWarps = kTpThreads / 32;
constexpr int kTpMaxBatch = 8;

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

struct TpParams {
  const void* x;
  const void* w;
  void* y;
  float* recv[WNW_TP_MAX_RANKS];
  uint32_t* flags[WNW_TP_MAX_RANKS];
  int batch, recv_batch, n_out, k_in, rank, world, chunk;
  uint32_t epoch;
  uint64_t timeout_ns;
  int32_t* err;
};

// recv layout on every rank: [2 parities][world][recv_batch][n_out] fp32
// flags layout on every rank: [world][n_chunks] u32 (last epoch received)
template <typename T>
__global__ void __launch_bounds__(kTpThreads) oproj_allreduce_kernel(const TpParams p) {
  __shared__ float part[kTpMaxBatch][64];
  const int c = blockIdx.x;
  const int c0 = c * p.chunk;
  const int c1 = min(p.n_out, c0 + p.chunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kv = p.k_in / 8;  // 16-byte vectors per weight row
  const T* x = static_cast<const T*>(p.x);
  const uint4* w = static_cast<const uint4*>(p.w);

  // ---- this rank's partial sums of the chunk: warp per output row, four
  // 16-byte weight loads in flight per lane
  for (int n = c0 + warp; n < c1; n += kTpWarps) {
    float acc[kTpMaxBatch];
#pragma unroll
    for (int b = 0; b < kTpMaxBatch; ++b) acc[b] = 0.f;
    const uint4* wr = w + int64_t(n) * kv;
#pragma unroll 4
    for (int i = lane; i < kv; i += 32) {
      float wf[8];
      unpack16<T>(__ldg(wr + i), wf);
#pragma unroll
      for (int b = 0; b < kTpMaxBatch; ++b) {
        if (b < p.batch) {
          float xf[8];
          unpack16<T>(__ldg(reinterpret_cast<const uint4*>(x + int64_t(b) * p.k_in) + i), xf);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[b] += wf[e] * xf[e];
        }
      }
    }
#pragma unroll
    for (int b = 0; b < kTpMaxBatch; ++b) {
      float v = acc[b];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0 && b < p.batch) part[b][n - c0] = v;
    }
  }
  __syncthreads();
  const int m = c1 - c0;
  if (p.world == 1) {  // no peers: the partial is the output
    T* y = static_cast<T*>(p.y);
    for (int idx = threadIdx.x; idx < p.batch * m; idx += kTpThreads)
      y[int64_t(idx / m) * p.n_out + c0 + idx % m] = DT<T>::from_f(part[idx / m][idx % m]);
    return;
  }

  // ---- push the partials into every rank's receive buffer (NVLink stores)
  const int par = p.epoch & 1;
  for (int idx = threadIdx.x; idx < p.world * p.batch * m; idx += kTpThreads) {
    const int dst = idx / (p.batch * m);
    const int rem = idx % (p.batch * m);
    const int b = rem / m, j = rem % m;
    float* r = p.recv[dst] + ((int64_t(par) * p.world + p.rank) * p.recv_batch + b) * p.n_out + c0 + j;
    *r = part[b][j];
  }
  __syncthreads();
  if (threadIdx.x < p.world) {
    fence_acq_rel_sys();  // this CTA's partial stores before the flag (cumulative via the barrier)
    st_release_sys(p.flags[threadIdx.x] + int64_t(p.rank) * gridDim.x + c, p.epoch);
  }

  // ---- wait for every rank's partials of this chunk, bounded by a deadline
  __shared__ int s_timeout;
  if (threadIdx.x == 0) s_timeout = 0;
  __syncthreads();
  if (threadIdx.x < p.world) {
    const uint32_t* f = p.flags[p.rank] + int64_t(threadIdx.x) * gridDim.x + c;
    const uint64_t t0 = global_ns();
    while (static_cast<int32_t>(ld_acquire_sys(f) - p.epoch) < 0) {
      if (global_ns() - t0 > p.timeout_ns) {
        atomicOr(p.err, WNW_DEVERR_PEER_TIMEOUT);
        s_timeout = 1;
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();

  // ---- rank-order sum of the chunk -> y
  T* y = static_cast<T*>(p.y);
  const float* own = p.recv[p.rank] + int64_t(par) * p.world * p.recv_batch * p.n_out;
  for (int idx = threadIdx.x; idx < p.batch * m; idx += kTpThreads) {
    const int b = idx / m, j = idx % m;
    float s = 0.f;
    for (int r = 0; r < p.world; ++r) s += __ldcg(own + (int64_t(r) * p.recv_batch + b) * p.n_out + c0 + j);
    y[int64_t(b) * p.n_out + c0 + j] = DT<T>::from_f(s_timeout ? 0.f : s);
  }
}

}  // namespace wnw

extern "C" int wnw_oproj_allreduce_chunks(int n_out) {
  // one output row per warp (8 per CTA), up to 8 CTAs per SM of a B200
  // (1184); beyond that up to 64 rows per CTA
  if (n_out <= 0) return 0;
  const int chunk = std::min(64, std::max(8, (n_out + 1183) / 1184));
  return (n_out + chunk - 1) / chunk;
}

extern "C" wnw_status wnw_oproj_allreduce(const wnw_oproj_allreduce_args* a, void* stream) {
  using namespace wnw;
  WNW_CHECK_ARG(a != nullptr, "null args");
  WNW_CHECK_ARG(a->world >= 1 && a->world <= WNW_TP_MAX_RANKS && a->rank >= 0 && a->rank < a->world,
                "rank %d / world %d out of range (world <= %d)", a->rank, a->world, WNW_TP_MAX_RANKS);
  WNW_CHECK_ARG(a->batch >= 1 && a->batch <= kTpMaxBatch, "batch %d not in 1..%d", a->batch, kTpMaxBatch);
  WNW_CHECK_ARG(a->n_out > 0 && a->k_in > 0 && a->k_in % 8 == 0, "n_out > 0 and k_in a multiple of 8 required");
  WNW_CHECK_ARG(a->recv_batch >= 1 && a->recv_batch <= kTpMaxBatch, "recv_batch %d not in 1..%d", a->recv_batch,
                kTpMaxBatch);
  if (a->batch > a->recv_batch) {
    wnw::set_error("wnw_oproj_allreduce: batch %d exceeds the receive buffers' %d rows", a->batch, a->recv_batch);
    return WNW_ERR_CAPACITY;
  }
  WNW_CHECK_ARG(a->x && a->w && a->y && a->err, "null pointer argument");
  WNW_CHECK_ARG(aligned16(a->x) && aligned16(a->w), "x and w must be 16-byte aligned");
  WNW_CHECK_ARG(a->dtype == WNW_BF16 || a->dtype == WNW_F16, "dtype must be bf16 or f16");
  for (int r = 0; r < a->world; ++r)
    WNW_CHECK_ARG(a->recv[r] && a->flags[r], "receive buffer / flags of rank %d missing", r);
  const int nchunks = wnw_oproj_allreduce_chunks(a->n_out);
  TpParams p;
  p.x = a->x;
  p.w = a->w;
  p.y = a->y;
  for (int r = 0; r < WNW_TP_MAX_RANKS; ++r) {
    p.recv[r] = r < a->world ? a->recv[r] : nullptr;
    p.flags[r] = r < a->world ? a->flags[r] : nullptr;
  }
  p.batch = a->batch;
  p.recv_batch = a->recv_batch;
  p.n_out = a->n_out;
  p.k_in = a->k_in;
  p.rank = a->rank;
  p.world = a->world;
  p.chunk = (a->n_out + nchunks - 1) / nchunks;
  p.epoch = a->epoch;
  p.timeout_ns = a->timeout_ns ? a->timeout_ns : uint64_t(2000000000);
  p.err = a->err;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a->dtype == WNW_BF16)
    oproj_allreduce_kernel<__nv_bfloat16><<<nchunks, kTpThreads, 0, s>>>(p);
  else
    oproj_allreduce_kernel<__half><<<nchunks, kTpThreads, 0, s>>>(p);
  WNW_CUDA_TRY(cudaGetLastError());
  return WNW_OK;
}

extern "C" wnw_status wnw_ipc_alloc(int64_t bytes, void** ptr, void* handle) {
  using namespace wnw;
  WNW_CHECK_ARG(bytes > 0 && ptr && handle, "bad arguments");
  void* d = nullptr;
  WNW_CUDA_TRY(cudaMalloc(&d, size_t(bytes)));
  cudaError_t e = cudaMemset(d, 0, size_t(bytes));
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), d);
  if (e != cudaSuccess) {
    cudaFree(d);
    return cuda_status(e, "wnw_ipc_alloc");
  }
  *ptr = d;
  return WNW_OK;
}

extern "C" wnw_status wnw_ipc_open(const void* handle, void** ptr) {
  using namespace wnw;
  WNW_CHECK_ARG(handle && ptr, "null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  WNW_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return WNW_OK;
}

extern "C" wnw_status wnw_ipc_close(void* ptr, int owned) {
  using namespace wnw;
  WNW_CHECK_ARG(ptr, "null pointer");
  if (owned)
    WNW_CUDA_TRY(cudaFree(ptr));
  else
    WNW_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return WNW_OK;
}
