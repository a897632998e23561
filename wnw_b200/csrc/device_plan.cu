// Device-planned fetch: the step's loads planned on the GPU from the device
// top-k, so the copy stream starts fetching without a host round trip.
//
// One thread block restates, for the fetch only, what the host planner
// (planner.cpp) does with the same top-k:
//  * needed  = union of the segments of the top-k chunks, per sample; a
//    sample with no top-k entry is left untouched;
//  * to_load = needed and not loaded; a loaded segment that is not needed
//    bumps its counter and is evicted once the counter reaches the lag; a
//    needed one resets its counter (the loaded maps and counters live on the
//    device and advance with every step);
//  * the loads become host ranges in the planner's order -- layer, then
//    sample, then class-B kv head in configuration order, then segment
//    ascending -- skipping (layer, head, segment)s with no host rows, and
//    each range lands at the running row count, so the landing layout is the
//    one the host planner's rebuild plan expects.
// The host planner still runs (it plans the rebuild) and wnw_dplan_verify
// compares its landing rows, loaded maps and counters with the device's.
#include <algorithm>
#include <cstring>
#include <new>
#include <vector>

#include "common.cuh"
#include "fetch_graph.h"
#include "planner_tables.h"

namespace wnw {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kPlanWarps = kPlanThreads / 32;
constexpr int kRowBits = 40;  // scan key: (ranges << 40) | rows
constexpr size_t kPlanSmemMax = 200 * 1024;

struct DPlanArgs {
  const int32_t* topk;
  int topk_stride, B, L, H, total_segs, evict_lag;
  const int32_t* chunk_base;
  const int32_t* c2s_off;
  const int32_t* c2s_flat;
  const int32_t* seg_base;
  const int32_t* seg_sample;
  uint8_t* loaded;
  int32_t* counters;
  const int64_t* meta_base;
  const int32_t* cpu_s;
  const int32_t* cpu_e;
  int64_t n_meta;
  const int32_t* classb_off;
  const int32_t* classb;
  int32_t* ranges;
  int64_t* dst;
  int64_t ranges_cap, land_rows;
  int32_t* layer_ranges;  // [L+1] device, read by the fetch kernels
  int32_t* layer_rows;    // [L+1] device
  int32_t* rb_layer_rows;  // mapped host read-back of the step's results
  uint8_t* rb_loaded;
  int32_t* rb_counters;
  int32_t* err;
};

// Exclusive prefix of v over the block (all kPlanThreads threads call it);
// `total` receives the block's sum.
__device__ int64_t block_excl_scan(int64_t v, int64_t* ws, int64_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int64_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) ws[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int64_t w = ws[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    ws[lane] = w;
  }
  __syncthreads();
  const int64_t excl = x - v + (warp > 0 ? ws[warp - 1] : 0);
  total = ws[kPlanWarps - 1];
  __syncthreads();
  return excl;
}

// first index in a[0, n) with a[i] >= key (a non-decreasing)
__device__ __forceinline__ int lower_bound_i(const int32_t* a, int n, int key) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (a[mid] < key) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

__global__ void __launch_bounds__(kPlanThreads) fetch_plan_kernel(const DPlanArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  int64_t* ws = reinterpret_cast<int64_t*>(smem);
  int32_t* list = reinterpret_cast<int32_t*>(ws + kPlanWarps);  // to-load segments, sample-local ids
  int32_t* lo = list + a.total_segs;                             // [B+1] list offset per sample
  int32_t* active = lo + a.B + 1;                                // [B]
  int32_t* eoff = active + a.B;                                  // [L+1] entry offset per layer
  uint8_t* flag = reinterpret_cast<uint8_t*>(eoff + a.L + 1);   // [total_segs]
  __shared__ int bad;
  const int tid = threadIdx.x;
  const int L = a.L, B = a.B, S = a.B * a.H;
  if (tid == 0) bad = 0;
  for (int i = tid; i < a.total_segs; i += kPlanThreads) flag[i] = 0;
  for (int b = tid; b < B; b += kPlanThreads) active[b] = 0;
  __syncthreads();

  // 1. needed segments
  const int nk = B * a.topk_stride;
  for (int j = tid; j < nk; j += kPlanThreads) {
    const int b = j / a.topk_stride;
    const int c = a.topk[j];
    if (c < 0) continue;
    active[b] = 1;
    const int cb = a.chunk_base[b];
    if (c >= a.chunk_base[b + 1] - cb - 1) {
      bad = 1;
      continue;
    }
    const int sb = a.seg_base[b], nsb = a.seg_base[b + 1] - sb;
    for (int q = a.c2s_off[cb + c]; q < a.c2s_off[cb + c + 1]; ++q) {
      const int s = a.c2s_flat[q];
      if (s < 0 || s >= nsb) {
        bad = 1;
        continue;
      }
      flag[sb + s] = 1;
    }
  }
  __syncthreads();
  if (bad) {  // nothing is fetched and the state does not advance
    for (int l = tid; l <= L; l += kPlanThreads) a.layer_ranges[l] = a.layer_rows[l] = 0;
    if (tid == 0) atomicOr(a.err, WNW_DEVERR_BAD_INDEX);
    return;
  }

  // 2. selection diff with eviction lag; flag becomes "load"
  for (int i = tid; i < a.total_segs; i += kPlanThreads) {
    int ld = a.loaded[i], cnt = a.counters[i], load = 0;
    if (active[a.seg_sample[i]]) {
      const int nd = flag[i];
      int ev = 0;
      if (ld) {
        if (!nd) {
          cnt += 1;
          ev = cnt >= a.evict_lag;
          if (ev) cnt = 0;
        } else {
          cnt = 0;
        }
      }
      load = nd && !ld;
      ld = load ? 1 : (ev ? 0 : ld);
      a.loaded[i] = static_cast<uint8_t>(ld);
      a.counters[i] = cnt;
    }
    flag[i] = static_cast<uint8_t>(load);
    a.rb_loaded[i] = static_cast<uint8_t>(ld);
    a.rb_counters[i] = cnt;
  }
  __syncthreads();

  // 3. to-load lists, ascending, and each sample's offset into them
  int64_t carry = 0, tot = 0;
  for (int base = 0; base < a.total_segs; base += kPlanThreads) {
    const int i = base + tid;
    const int v = i < a.total_segs ? flag[i] : 0;
    const int p = static_cast<int>(block_excl_scan(v, ws, tot) + carry);
    if (i < a.total_segs) {
      const int b = a.seg_sample[i];
      if (v) list[p] = i - a.seg_base[b];
      if (i == a.seg_base[b])  // first segment of b (and of any empty samples before it)
        for (int bb = lower_bound_i(a.seg_base, B + 1, i); bb <= B && a.seg_base[bb] == i; ++bb) lo[bb] = p;
    }
    carry += tot;
  }
  if (tid == 0) {
    for (int bb = lower_bound_i(a.seg_base, B + 1, a.total_segs); bb <= B; ++bb) lo[bb] = static_cast<int>(carry);
    const int nl = static_cast<int>(carry);
    int e = 0;
    for (int l = 0; l < L; ++l) {
      eoff[l] = e;
      e += (a.classb_off[l + 1] - a.classb_off[l]) * nl;
    }
    eoff[L] = e;
  }
  __syncthreads();

  // 4. ranges and landing rows in the planner's order
  const int E = eoff[L];
  const int64_t row_mask = (int64_t(1) << kRowBits) - 1;
  carry = 0;
  for (int base = 0; base < E; base += kPlanThreads) {
    const int e = base + tid;
    int cs = -1, ce = -1;
    int64_t v = 0;
    if (e < E) {
      const int l = lower_bound_i(eoff, L + 1, e + 1) - 1;  // eoff[l] <= e < eoff[l+1]
      const int h0 = a.classb_off[l], nh = a.classb_off[l + 1] - h0;
      const int w = e - eoff[l];
      const int b = lower_bound_i(lo, B + 1, w / nh + 1) - 1;  // lo[b] <= w / nh < lo[b+1]
      const int nlb = lo[b + 1] - lo[b];
      const int wp = w - nh * lo[b];
      const int h = a.classb[h0 + wp / nlb];
      const int s = list[lo[b] + wp % nlb];
      const int64_t m = a.meta_base[int64_t(l) * S + b * a.H + h] + s;
      if (m >= 0 && m < a.n_meta) {
        cs = a.cpu_s[m];
        ce = a.cpu_e[m];
      } else {
        bad = 1;
      }
      if (cs >= 0) v = (int64_t(1) << kRowBits) | int64_t(ce - cs);
    }
    const int64_t p = block_excl_scan(v, ws, tot) + carry;
    const int64_t ri = p >> kRowBits, row = p & row_mask;
    if (cs >= 0 && ri < a.ranges_cap) {
      a.ranges[2 * ri] = cs;
      a.ranges[2 * ri + 1] = ce;
      a.dst[ri] = row;
    }
    if (e < E)
      for (int l = lower_bound_i(eoff, L + 1, e); l <= L && eoff[l] == e; ++l) {
        a.layer_ranges[l] = static_cast<int32_t>(ri);
        a.layer_rows[l] = static_cast<int32_t>(row);
      }
    carry += tot;
  }
  if (tid == 0)
    for (int l = lower_bound_i(eoff, L + 1, E); l <= L; ++l) {
      a.layer_ranges[l] = static_cast<int32_t>(carry >> kRowBits);
      a.layer_rows[l] = static_cast<int32_t>(carry & row_mask);
    }
  __syncthreads();
  const bool over = (carry >> kRowBits) > a.ranges_cap || (carry & row_mask) > a.land_rows;
  if (bad || over) {  // fetch nothing; the host raises on the error word
    __syncthreads();
    for (int l = tid; l <= L; l += kPlanThreads) a.layer_ranges[l] = 0;
    if (tid == 0) atomicOr(a.err, bad ? WNW_DEVERR_BAD_INDEX : WNW_DEVERR_CAPACITY);
  }
  for (int l = tid; l <= L; l += kPlanThreads) a.rb_layer_rows[l] = a.layer_rows[l];
  __threadfence_system();
}

template <typename T>
wnw_status upload(T** dev, const std::vector<T>& host) {
  const size_t n = std::max<size_t>(host.size(), 1);
  WNW_CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(dev), sizeof(T) * n));
  if (!host.empty()) WNW_CUDA_TRY(cudaMemcpy(*dev, host.data(), sizeof(T) * host.size(), cudaMemcpyHostToDevice));
  return WNW_OK;
}

template <typename T>
wnw_status mapped(T** host, T** dev, size_t n) {
  WNW_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void**>(host), sizeof(T) * std::max<size_t>(n, 1),
                             cudaHostAllocMapped));
  std::memset(*host, 0, sizeof(T) * std::max<size_t>(n, 1));
  WNW_CUDA_TRY(cudaHostGetDevicePointer(reinterpret_cast<void**>(dev), *host, 0));
  return WNW_OK;
}

}  // namespace
}  // namespace wnw

struct wnw_dplan {
  int L = 0, H = 0, B = 0, total_segs = 0, evict_lag = 1;
  int64_t n_meta = 0, ranges_cap = 0;
  size_t smem = 0;
  int32_t *chunk_base = nullptr, *c2s_off = nullptr, *c2s_flat = nullptr, *seg_base = nullptr,
          *seg_sample = nullptr, *counters = nullptr, *cpu_s = nullptr, *cpu_e = nullptr, *classb_off = nullptr,
          *classb = nullptr, *ranges = nullptr, *layer_ranges = nullptr, *layer_rows = nullptr;
  uint8_t* loaded = nullptr;
  int64_t *meta_base = nullptr, *dst = nullptr;
  int32_t *rb_rows_h = nullptr, *rb_rows_d = nullptr, *rb_cnt_h = nullptr, *rb_cnt_d = nullptr;
  uint8_t *rb_ld_h = nullptr, *rb_ld_d = nullptr;
  cudaEvent_t planned = nullptr;

  ~wnw_dplan() {
    wnw::fetch_graph_release(this);
    for (void* p : {static_cast<void*>(chunk_base), static_cast<void*>(c2s_off), static_cast<void*>(c2s_flat),
                    static_cast<void*>(seg_base), static_cast<void*>(seg_sample), static_cast<void*>(counters),
                    static_cast<void*>(cpu_s), static_cast<void*>(cpu_e), static_cast<void*>(classb_off),
                    static_cast<void*>(classb), static_cast<void*>(ranges), static_cast<void*>(layer_ranges),
                    static_cast<void*>(layer_rows), static_cast<void*>(loaded), static_cast<void*>(meta_base),
                    static_cast<void*>(dst)})
      if (p) cudaFree(p);
    for (void* p : {static_cast<void*>(rb_rows_h), static_cast<void*>(rb_cnt_h), static_cast<void*>(rb_ld_h)})
      if (p) cudaFreeHost(p);
    if (planned) cudaEventDestroy(planned);
  }
};

extern "C" {

wnw_status wnw_dplan_create(const wnw_planner* p, wnw_dplan** out) {
  using namespace wnw;
  WNW_CHECK_ARG(p && out, "null argument");
  *out = nullptr;
  PlannerTables t;
  wnw_status st = planner_tables(p, &t);
  if (st != WNW_OK) return st;
  const int total = t.seg_base.back();
  const size_t smem = sizeof(int64_t) * kPlanWarps +
                      sizeof(int32_t) * (size_t(total) + (t.B + 1) + t.B + (t.L + 1)) + size_t(total);
  if (smem > kPlanSmemMax) {
    set_error("device fetch plan: %d segments need %zu bytes of shared memory", total, smem);
    return WNW_ERR_UNSUPPORTED;
  }
  wnw_dplan* d = new (std::nothrow) wnw_dplan();
  if (!d) {
    set_error("out of host memory");
    return WNW_ERR_INVALID;
  }
  d->L = t.L;
  d->H = t.H;
  d->B = t.B;
  d->total_segs = total;
  d->evict_lag = t.evict_lag;
  d->n_meta = static_cast<int64_t>(t.cpu_s.size());
  d->smem = (smem + 15) / 16 * 16;
  int64_t cap = 0;
  for (int l = 0; l < t.L; ++l) cap += int64_t(t.classb_off[l + 1] - t.classb_off[l]) * total;
  d->ranges_cap = std::max<int64_t>(cap, 1);
  st = WNW_OK;
#define WNW_DP_TRY(expr)            \
  if ((st = (expr)) != WNW_OK) {    \
    delete d;                       \
    return st;                      \
  }
  WNW_DP_TRY(upload(&d->chunk_base, t.chunk_base));
  WNW_DP_TRY(upload(&d->c2s_off, t.c2s_off));
  WNW_DP_TRY(upload(&d->c2s_flat, t.c2s_flat));
  WNW_DP_TRY(upload(&d->seg_base, t.seg_base));
  WNW_DP_TRY(upload(&d->seg_sample, t.seg_sample));
  WNW_DP_TRY(upload(&d->loaded, t.loaded));
  WNW_DP_TRY(upload(&d->counters, t.counters));
  WNW_DP_TRY(upload(&d->meta_base, t.meta_base));
  WNW_DP_TRY(upload(&d->cpu_s, t.cpu_s));
  WNW_DP_TRY(upload(&d->cpu_e, t.cpu_e));
  WNW_DP_TRY(upload(&d->classb_off, t.classb_off));
  WNW_DP_TRY(upload(&d->classb, t.classb));
  WNW_DP_TRY(upload(&d->ranges, std::vector<int32_t>(size_t(2 * d->ranges_cap), 0)));
  WNW_DP_TRY(upload(&d->dst, std::vector<int64_t>(size_t(d->ranges_cap), 0)));
  WNW_DP_TRY(upload(&d->layer_ranges, std::vector<int32_t>(size_t(t.L + 1), 0)));
  WNW_DP_TRY(upload(&d->layer_rows, std::vector<int32_t>(size_t(t.L + 1), 0)));
  WNW_DP_TRY(mapped(&d->rb_rows_h, &d->rb_rows_d, size_t(t.L + 1)));
  WNW_DP_TRY(mapped(&d->rb_ld_h, &d->rb_ld_d, size_t(total)));
  WNW_DP_TRY(mapped(&d->rb_cnt_h, &d->rb_cnt_d, size_t(total)));
#undef WNW_DP_TRY
  cudaError_t e = cudaEventCreateWithFlags(&d->planned, cudaEventDisableTiming);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(fetch_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(d->smem));
  if (e != cudaSuccess) {
    delete d;
    return cuda_status(e, "wnw_dplan_create");
  }
  *out = d;
  return WNW_OK;
}

void wnw_dplan_destroy(wnw_dplan* dp) { delete dp; }

wnw_status wnw_dplan_step(wnw_dplan* dp, const int32_t* topk_dev, int topk_stride, int32_t* err, const void* src_k,
                          const void* src_v, int64_t row_bytes, void* land_k, void* land_v, int64_t land_rows,
                          int max_ctas, void* compute_stream, void* copy_stream, void* const* events) {
  using namespace wnw;
  WNW_CHECK_ARG(dp && topk_dev && err && src_k && src_v && land_k && land_v && events, "null argument");
  WNW_CHECK_ARG(topk_stride > 0 && land_rows >= 0, "bad top-k stride or landing rows");
  WNW_CHECK_ARG(row_bytes > 0 && row_bytes % 16 == 0, "row bytes must be a positive multiple of 16");
  DPlanArgs a;
  a.topk = topk_dev;
  a.topk_stride = topk_stride;
  a.B = dp->B;
  a.L = dp->L;
  a.H = dp->H;
  a.total_segs = dp->total_segs;
  a.evict_lag = dp->evict_lag;
  a.chunk_base = dp->chunk_base;
  a.c2s_off = dp->c2s_off;
  a.c2s_flat = dp->c2s_flat;
  a.seg_base = dp->seg_base;
  a.seg_sample = dp->seg_sample;
  a.loaded = dp->loaded;
  a.counters = dp->counters;
  a.meta_base = dp->meta_base;
  a.cpu_s = dp->cpu_s;
  a.cpu_e = dp->cpu_e;
  a.n_meta = dp->n_meta;
  a.classb_off = dp->classb_off;
  a.classb = dp->classb;
  a.ranges = dp->ranges;
  a.dst = dp->dst;
  a.ranges_cap = dp->ranges_cap;
  a.land_rows = land_rows;
  a.layer_ranges = dp->layer_ranges;
  a.layer_rows = dp->layer_rows;
  a.rb_layer_rows = dp->rb_rows_d;
  a.rb_loaded = dp->rb_ld_d;
  a.rb_counters = dp->rb_cnt_d;
  a.err = err;
  cudaStream_t cs = static_cast<cudaStream_t>(compute_stream);
  fetch_plan_kernel<<<1, kPlanThreads, dp->smem, cs>>>(a);
  WNW_CUDA_TRY(cudaGetLastError());
  WNW_CUDA_TRY(cudaEventRecord(dp->planned, cs));
  WNW_CUDA_TRY(cudaStreamWaitEvent(static_cast<cudaStream_t>(copy_stream), dp->planned, 0));
  FetchGraphKey k;
  k.src_k = src_k;
  k.src_v = src_v;
  k.row_bytes = row_bytes;
  k.ranges_dev = dp->ranges;
  k.dst_dev = dp->dst;
  k.land_k = land_k;
  k.land_v = land_v;
  k.max_ctas = max_ctas > 0 ? max_ctas : 12;
  k.L = dp->L;
  k.events = events;
  k.layer_ranges_dev = dp->layer_ranges;
  return fetch_graph_issue_planned(dp, k, copy_stream);
}

wnw_status wnw_dplan_verify(const wnw_dplan* dp, const wnw_planner* p) {
  WNW_CHECK_ARG(dp && p, "null argument");
  return wnw::planner_check_mirror(p, dp->rb_rows_h, dp->rb_ld_h, dp->rb_cnt_h);
}

}  // extern "C"
