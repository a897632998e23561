// In-place layout maintenance for the slot layout of the flat varlen cache.
//
// Every (sample, kv head) segment owns a fixed slot [seg_base, seg_base+cap)
// of its layer's K / V store.  A chunk update of the reference rewrites the
// whole flat buffer (rebuild_append_kv, src/algorithms/wnw/code/kernels.py:
// 375-473); here only the changed segments move rows inside their own slot:
// evicted ranges are squeezed out (later kept rows shift down) and the rows
// fetched from host memory are spliced after the kept rows.  Moving rows down
// inside one buffer in parallel would let a write clobber a source another
// thread has not read yet, so the moving rows go through a scratch buffer in
// two grid-wide launches (gather, then scatter).  The step's new token is
// appended afterwards by the decode-attention kernel.
#include <algorithm>
#include <vector>

#include "common.cuh"

namespace wnw {

constexpr int kRbThreads = 256;
constexpr int kRbMaxBlocks = 148 * 4;

// One layer record of the device plan (see wnw_planner_device_plan).
struct RbRec {
  int n, moved_total, out_total;
  const int32_t *seg, *old_len, *new_len, *lsrc, *llen, *mov_off, *out_off, *ev_off, *ev_s, *ev_e;
  __device__ explicit RbRec(const int32_t* blob, int layer) {
    const int32_t* h = blob + blob[layer];
    n = h[0];
    moved_total = h[1];
    out_total = h[2];
    seg = h + 3;
    old_len = seg + n;
    new_len = old_len + n;
    lsrc = new_len + n;
    llen = lsrc + n;
    mov_off = llen + n;
    out_off = mov_off + n + 1;
    ev_off = out_off + n + 1;
    ev_s = ev_off + n + 1;
    ev_e = ev_s + ev_off[n];
  }
  // record index i with off[i] <= x < off[i+1] (off non-decreasing, off[0] = 0)
  __device__ int find(const int32_t* off, int x) const {
    int lo = 0, hi = n;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (off[mid] <= x) lo = mid; else hi = mid;
    }
    return lo;
  }
};

// Whether layer `layer`'s record lies inside the blob and its offset arrays
// are well formed (start at 0, non-decreasing, end at the totals), with at
// most num_segs records -- checked before anything else reads the record.
__device__ inline bool record_well_formed(const int32_t* blob, int64_t blob_ints, int layer, int num_segs) {
  if (layer < 0 || int64_t(layer) >= blob_ints) return false;
  const int64_t o = blob[layer];
  if (o < 0 || o + 3 > blob_ints) return false;
  const int64_t n = blob[o];
  if (n < 0 || n > num_segs) return false;
  const int64_t fixed = 3 + 5 * n + 3 * (n + 1);
  if (o + fixed > blob_ints) return false;
  const int32_t* h = blob + o;
  const int32_t* mov_off = h + 3 + 5 * n;
  const int32_t* out_off = mov_off + n + 1;
  const int32_t* ev_off = out_off + n + 1;
  if (h[1] < 0 || h[2] < 0 || mov_off[0] != 0 || out_off[0] != 0 || ev_off[0] != 0) return false;
  for (int64_t i = 0; i < n; ++i)
    if (mov_off[i + 1] < mov_off[i] || out_off[i + 1] < out_off[i] || ev_off[i + 1] < ev_off[i]) return false;
  if (mov_off[n] != h[1] || out_off[n] != h[2]) return false;
  return o + fixed + 2 * int64_t(ev_off[n]) <= blob_ints;
}

// Every CTA checks the layer record once; on a malformed record the block 0
// thread 0 raises the error bit and every CTA returns before reading it.
__device__ inline bool cta_record_ok(const int32_t* blob, int64_t blob_ints, int layer, int num_segs, int32_t* err,
                                     bool first_cta) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    s_ok = record_well_formed(blob, blob_ints, layer, num_segs) ? 1 : 0;
    if (!s_ok && first_cta) atomicOr(err, WNW_DEVERR_LEN_MISMATCH);
  }
  __syncthreads();
  return s_ok != 0;
}

// Kept-row index k (0-based among the kept rows after the first evicted
// range) -> slot-relative source row.
__device__ inline int kept_source_row(const RbRec& r, int i, int k) {
  const int e0 = r.ev_off[i], e1 = r.ev_off[i + 1];
  int run_lo = r.ev_e[e0];
  for (int e = e0; e < e1; ++e) {
    const int run_hi = (e + 1 < e1) ? r.ev_s[e + 1] : r.old_len[i];
    const int n = run_hi - run_lo;
    if (k < n) return run_lo + k;
    k -= n;
    if (e + 1 < e1) run_lo = r.ev_e[e + 1];
  }
  return -1;
}

// Phase 1 of one layer, by CTA `cta` of `ncta`: validate every record,
// gather the moving kept rows into scratch.
__device__ void gather_layer(const uint4* k_store, const uint4* v_store, const int64_t* seg_base,
                             const int32_t* seg_len, const int32_t* seg_cap, const int32_t* blob, int64_t blob_ints,
                             int layer, int num_segs, int64_t land_rows, uint4* k_move, uint4* v_move,
                             int64_t move_rows, int32_t* status, int32_t* err, int cpr, int cta, int ncta) {
  if (!cta_record_ok(blob, blob_ints, layer, num_segs, err, cta == 0)) return;
  const RbRec r(blob, layer);
  const int64_t gtid = int64_t(cta) * blockDim.x + threadIdx.x;
  const int64_t nthreads = int64_t(ncta) * blockDim.x;
  for (int i = static_cast<int>(gtid); i < r.n; i += static_cast<int>(nthreads)) {
    const int seg = r.seg[i];
    const int e0 = r.ev_off[i], e1 = r.ev_off[i + 1];
    if (seg < 0 || seg >= num_segs) {  // nothing of this record is read or written
      atomicOr(err, WNW_DEVERR_LEN_MISMATCH);
      status[i] = 0;
      continue;
    }
    int ok = seg_len[seg] == r.old_len[i] ? 1 : 0;
    int prev = 0, evicted = 0;
    for (int e = e0; e < e1 && ok; ++e) {
      if (r.ev_s[e] < prev || r.ev_e[e] < r.ev_s[e] || r.ev_e[e] > r.old_len[i]) ok = 0;
      prev = r.ev_e[e];
      evicted += r.ev_e[e] - r.ev_s[e];
    }
    const int moved = r.mov_off[i + 1] - r.mov_off[i];
    if (ok && (r.old_len[i] - evicted + r.llen[i] != r.new_len[i] || r.llen[i] < 0 || r.lsrc[i] < 0 ||
               moved != (e1 > e0 ? r.old_len[i] - evicted - r.ev_s[e0] : 0) ||
               r.out_off[i + 1] - r.out_off[i] != moved + r.llen[i] ||
               int64_t(r.lsrc[i]) + r.llen[i] > (r.llen[i] > 0 ? land_rows : int64_t(INT32_MAX))))
      ok = 0;
    if (!ok) atomicOr(err, WNW_DEVERR_LEN_MISMATCH);
    if (ok && r.new_len[i] + 1 > seg_cap[seg]) {
      ok = 0;
      atomicOr(err, WNW_DEVERR_CAPACITY);
    }
    status[i] = ok;
  }
  if (r.moved_total > move_rows) {
    if (gtid == 0) atomicOr(err, WNW_DEVERR_CAPACITY);
    return;
  }
  const int64_t total = int64_t(r.moved_total) * cpr;
  for (int64_t x = gtid; x < total; x += nthreads) {
    const int row = static_cast<int>(x / cpr);
    const int c = static_cast<int>(x % cpr);
    const int i = r.find(r.mov_off, row);
    const int seg = r.seg[i];
    if (seg < 0 || seg >= num_segs) continue;  // malformed record: refused by status[i]
    const int src = kept_source_row(r, i, row - r.mov_off[i]);
    if (src < 0 || src >= seg_cap[seg]) continue;
    const int64_t s = (seg_base[seg] + src) * cpr + c;
    k_move[int64_t(row) * cpr + c] = k_store[s];
    v_move[int64_t(row) * cpr + c] = v_store[s];
  }
}

__global__ void __launch_bounds__(kRbThreads)
    rebuild_gather_kernel(const uint4* k_store, const uint4* v_store, const int64_t* seg_base, const int32_t* seg_len,
                          const int32_t* seg_cap, const int32_t* blob, int64_t blob_ints, int layer, int num_segs,
                          int64_t land_rows, uint4* k_move, uint4* v_move, int64_t move_rows, int32_t* status,
                          int32_t* err, int cpr) {
  pdl_launch_dependents();  // the scatter may start validating its record now
  gather_layer(k_store, v_store, seg_base, seg_len, seg_cap, blob, blob_ints, layer, num_segs, land_rows, k_move,
               v_move, move_rows, status, err, cpr, blockIdx.x, gridDim.x);
}

// Phase 2 of one layer, by CTA `cta` of `ncta` of a launch dependent on the
// gather's (it checks the layer's record, then waits for the gather): write
// moved and fetched rows to their final slot rows; set seg_len.
__device__ void scatter_layer(uint4* k_store, uint4* v_store, const int64_t* seg_base, int32_t* seg_len,
                              const uint4* k_land, const uint4* v_land, const int32_t* blob, int64_t blob_ints,
                              int layer, int num_segs, int64_t move_rows, const uint4* k_move, const uint4* v_move,
                              const int32_t* status, int32_t* err, int cpr, int cta, int ncta) {
  if (!cta_record_ok(blob, blob_ints, layer, num_segs, err, cta == 0)) return;  // reads the plan blob only
  pdl_wait();  // the gather's status words and moved rows are complete
  const RbRec r(blob, layer);
  if (r.moved_total > move_rows) return;  // refused by the gather (error bit set there)
  const int64_t gtid = int64_t(cta) * blockDim.x + threadIdx.x;
  const int64_t nthreads = int64_t(ncta) * blockDim.x;
  const int64_t total = int64_t(r.out_total) * cpr;
  for (int64_t x = gtid; x < total; x += nthreads) {
    const int row = static_cast<int>(x / cpr);
    const int c = static_cast<int>(x % cpr);
    const int i = r.find(r.out_off, row);
    if (!status[i]) continue;
    const int seg = r.seg[i];
    const int k = row - r.out_off[i];
    const int moved = r.mov_off[i + 1] - r.mov_off[i];
    const int64_t dst = (seg_base[seg] + (k < moved ? r.ev_s[r.ev_off[i]] + k
                                                    : r.new_len[i] - r.llen[i] + (k - moved))) * cpr + c;
    if (k < moved) {
      const int64_t s = int64_t(r.mov_off[i] + k) * cpr + c;
      k_store[dst] = k_move[s];
      v_store[dst] = v_move[s];
    } else {
      const int64_t s = int64_t(r.lsrc[i] + (k - moved)) * cpr + c;
      k_store[dst] = k_land[s];
      v_store[dst] = v_land[s];
    }
  }
  for (int i = static_cast<int>(gtid); i < r.n; i += static_cast<int>(nthreads))
    if (status[i]) seg_len[r.seg[i]] = r.new_len[i];
}

__global__ void __launch_bounds__(kRbThreads)
    rebuild_scatter_kernel(uint4* k_store, uint4* v_store, const int64_t* seg_base, int32_t* seg_len,
                           const int32_t* seg_cap, const uint4* k_land, const uint4* v_land, const int32_t* blob,
                           int64_t blob_ints, int layer, int num_segs, int64_t move_rows, const uint4* k_move,
                           const uint4* v_move, const int32_t* status, int32_t* err, int cpr) {
  // the layer's decode attention (launched with programmatic dependent launch)
  // may start its layout-only prologue now; it waits for this grid to finish
  // before it reads anything written here
  pdl_launch_dependents();
  scatter_layer(k_store, v_store, seg_base, seg_len, k_land, v_land, blob, blob_ints, layer, num_segs, move_rows,
                k_move, v_move, status, err, cpr, blockIdx.x, gridDim.x);
}

// ------------------------------------------------ every changed layer at once
// One gather and one scatter launch for all the changed layers of a step:
// blockIdx.y picks the layer, blockIdx.x / gridDim.x the CTA within it; each
// layer does exactly what its own wnw_rebuild_segments pair would, with its
// moved rows in a region of the move buffers of their own and its status
// words at status_base.
constexpr int kRbMultiMax = 48;  // layers per launch pair (by-value kernel argument, < 4 KB)
struct RbLayer {
  uint4* k_store;
  uint4* v_store;
  const int64_t* seg_base;
  int32_t* seg_len;
  const int32_t* seg_cap;
  int layer, num_segs, status_base;
};
struct RbMulti {
  RbLayer l[kRbMultiMax];
  int n;
};

// First row of the i-th layer's moved rows in the move buffers: the moved-row
// totals of the launch's earlier layers, read from their records (a record
// outside the blob counts 0; its own layer refuses it).  Every thread of the
// CTA returns the same value.
__device__ int64_t move_base_of(const RbMulti& m, int i, const int32_t* blob, int64_t blob_ints) {
  __shared__ unsigned long long s_base;
  if (threadIdx.x == 0) s_base = 0;
  __syncthreads();
  for (int j = threadIdx.x; j < i; j += blockDim.x) {
    const int l = m.l[j].layer;
    if (l >= 0 && int64_t(l) < blob_ints) {
      const int64_t o = blob[l];
      if (o >= 0 && o + 3 <= blob_ints && blob[o + 1] > 0) atomicAdd(&s_base, static_cast<unsigned long long>(blob[o + 1]));
    }
  }
  __syncthreads();
  return static_cast<int64_t>(s_base);
}

__global__ void __launch_bounds__(kRbThreads)
    rebuild_gather_multi_kernel(const RbMulti m, const int32_t* blob, int64_t blob_ints, int64_t land_rows,
                                uint4* k_move, uint4* v_move, int64_t move_rows, int32_t* status, int32_t* err,
                                int cpr) {
  pdl_launch_dependents();  // the scatter may start validating its records now
  const int i = blockIdx.y;
  const RbLayer& L = m.l[i];
  const int64_t mb = move_base_of(m, i, blob, blob_ints);
  const int64_t room = mb <= move_rows ? move_rows - mb : -1;  // a negative room refuses every moved row
  gather_layer(L.k_store, L.v_store, L.seg_base, L.seg_len, L.seg_cap, blob, blob_ints, L.layer, L.num_segs,
               land_rows, k_move + (room >= 0 ? mb : 0) * cpr, v_move + (room >= 0 ? mb : 0) * cpr, room,
               status + L.status_base, err, cpr, blockIdx.x, gridDim.x);
}

__global__ void __launch_bounds__(kRbThreads)
    rebuild_scatter_multi_kernel(const RbMulti m, const uint4* k_land, const uint4* v_land, const int32_t* blob,
                                 int64_t blob_ints, int64_t move_rows, const uint4* k_move, const uint4* v_move,
                                 const int32_t* status, int32_t* err, int cpr) {
  pdl_launch_dependents();
  const int i = blockIdx.y;
  const RbLayer& L = m.l[i];
  const int64_t mb = move_base_of(m, i, blob, blob_ints);
  const int64_t room = mb <= move_rows ? move_rows - mb : -1;
  scatter_layer(L.k_store, L.v_store, L.seg_base, L.seg_len, k_land, v_land, blob, blob_ints, L.layer, L.num_segs,
                room, k_move + (room >= 0 ? mb : 0) * cpr, v_move + (room >= 0 ? mb : 0) * cpr,
                status + L.status_base, err, cpr, blockIdx.x, gridDim.x);
}

// ------------------------------------------------------------ segment copy
__global__ void copy_segments_kernel(const uint4* src_k, const uint4* src_v, const int64_t* src_base,
                                     uint4* dst_k, uint4* dst_v, const int64_t* dst_base,
                                     const int32_t* len, int chunks_per_row) {
  const int seg = blockIdx.y;
  const int64_t n = int64_t(len[seg]) * chunks_per_row;
  const int64_t s0 = src_base[seg] * chunks_per_row;
  const int64_t d0 = dst_base[seg] * chunks_per_row;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  // four rows' chunks of K and V in flight per thread: the loads of a
  // round are issued before its stores
  for (; i + 3 * stride < n; i += 4 * stride) {
    uint4 k[4], v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      k[j] = src_k[s0 + i + j * stride];
      v[j] = src_v[s0 + i + j * stride];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      dst_k[d0 + i + j * stride] = k[j];
      dst_v[d0 + i + j * stride] = v[j];
    }
  }
  for (; i < n; i += stride) {
    dst_k[d0 + i] = src_k[s0 + i];
    dst_v[d0 + i] = src_v[s0 + i];
  }
}

// reference-layout append: out row of segment s
__global__ void interleave_append_kernel(const uint4* old, const uint4* nt, const int32_t* cu_old,
                                         uint4* out, int chunks_per_row) {
  const int seg = blockIdx.y;
  const int64_t a = cu_old[seg], b = cu_old[seg + 1];
  const int64_t n = (b - a + 1) * chunks_per_row;
  const int64_t o0 = (a + seg) * chunks_per_row;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t row = i / chunks_per_row;
    const int64_t c = i % chunks_per_row;
    out[o0 + i] = (row < b - a) ? old[(a + row) * chunks_per_row + c] : nt[int64_t(seg) * chunks_per_row + c];
  }
}

__global__ void advance_kernel(int32_t* len, int64_t n) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    len[i] += 1;
}

inline int row_bytes_of(int dtype, int head_dim) { return head_dim * (dtype == WNW_F32 ? 4 : 2); }

}  // namespace wnw

extern "C" wnw_status wnw_rebuild_segments(int dtype, int head_dim, void* k_store, void* v_store,
                                           const int64_t* seg_base, int32_t* seg_len, const int32_t* seg_cap,
                                           int num_segs, const void* k_landing, const void* v_landing,
                                           int64_t land_rows, const int32_t* plan_blob, int64_t blob_ints,
                                           int layer, void* k_move, void* v_move, int64_t move_rows,
                                           int32_t* status, int32_t* err, void* stream) {
  using namespace wnw;
  WNW_CHECK_ARG(k_store && v_store && seg_base && seg_len && seg_cap && plan_blob && status && err,
                "null pointer argument");
  WNW_CHECK_ARG(layer >= 0 && num_segs >= 0 && land_rows >= 0 && blob_ints > layer,
                "negative layer / sizes, or a blob too small for the layer table");
  WNW_CHECK_ARG(aligned16(k_store) && aligned16(v_store), "stores must be 16-byte aligned");
  WNW_CHECK_ARG(k_landing == nullptr || (aligned16(k_landing) && aligned16(v_landing)),
                "landing buffers must be 16-byte aligned");
  WNW_CHECK_ARG(move_rows == 0 || (k_move && v_move && aligned16(k_move) && aligned16(v_move)),
                "move buffers must be given and 16-byte aligned when move_rows > 0");
  const int rb = row_bytes_of(dtype, head_dim);
  WNW_CHECK_ARG(rb > 0 && rb % 16 == 0, "row size must be a positive multiple of 16 bytes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  rebuild_gather_kernel<<<kRbMaxBlocks, kRbThreads, 0, s>>>(
      static_cast<const uint4*>(k_store), static_cast<const uint4*>(v_store), seg_base, seg_len, seg_cap, plan_blob,
      blob_ints, layer, num_segs, k_landing ? land_rows : 0, static_cast<uint4*>(k_move),
      static_cast<uint4*>(v_move), move_rows, status, err, rb / 16);
  WNW_CUDA_TRY(cudaGetLastError());
  // programmatic dependent launch: the scatter's CTAs validate their record
  // while the gather finishes, then wait for it (griddepcontrol.wait)
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kRbMaxBlocks, 1, 1);
  cfg.blockDim = dim3(kRbThreads, 1, 1);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  WNW_CUDA_TRY(cudaLaunchKernelEx(&cfg, rebuild_scatter_kernel, static_cast<uint4*>(k_store),
                                  static_cast<uint4*>(v_store), seg_base, seg_len, seg_cap,
                                  static_cast<const uint4*>(k_landing), static_cast<const uint4*>(v_landing),
                                  plan_blob, blob_ints, layer, num_segs, move_rows,
                                  static_cast<const uint4*>(k_move), static_cast<const uint4*>(v_move),
                                  static_cast<const int32_t*>(status), err, rb / 16));
  return WNW_OK;
}

extern "C" wnw_status wnw_rebuild_layers(int dtype, int head_dim, int num_layers, const int32_t* layer_changed,
                                         void* const* k_store, void* const* v_store,
                                         const int64_t* const* seg_base, int32_t* const* seg_len,
                                         const int32_t* const* seg_cap, const int32_t* num_segs,
                                         const void* k_landing, const void* v_landing, int64_t land_rows,
                                         const int32_t* plan_blob, int64_t blob_ints, void* k_move, void* v_move,
                                         int64_t move_rows, int32_t* status, int32_t* err,
                                         void* const* wait_events, void* const* record_events, void* stream) {
  using namespace wnw;
  WNW_CHECK_ARG(num_layers >= 0, "num_layers < 0");
  WNW_CHECK_ARG(num_layers == 0 || (layer_changed && k_store && v_store && seg_base && seg_len && seg_cap &&
                                    num_segs),
                "null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int l = 0; l < num_layers; ++l) {
    if (!layer_changed[l]) continue;
    if (wait_events && wait_events[l]) WNW_CUDA_TRY(cudaStreamWaitEvent(s, static_cast<cudaEvent_t>(wait_events[l]), 0));
    const wnw_status st = wnw_rebuild_segments(dtype, head_dim, k_store[l], v_store[l], seg_base[l], seg_len[l],
                                               seg_cap[l], num_segs[l], k_landing, v_landing, land_rows, plan_blob,
                                               blob_ints, l, k_move, v_move, move_rows, status, err, stream);
    if (st != WNW_OK) return st;
    if (record_events && record_events[l])
      WNW_CUDA_TRY(cudaEventRecord(static_cast<cudaEvent_t>(record_events[l]), s));
  }
  return WNW_OK;
}

extern "C" wnw_status wnw_rebuild_layers_fused(int dtype, int head_dim, int num_layers, const int32_t* layer_changed,
                                               void* const* k_store, void* const* v_store,
                                               const int64_t* const* seg_base, int32_t* const* seg_len,
                                               const int32_t* const* seg_cap, const int32_t* num_segs,
                                               const void* k_landing, const void* v_landing, int64_t land_rows,
                                               const int32_t* plan_blob, int64_t blob_ints, void* k_move,
                                               void* v_move, int64_t move_rows, int32_t* status,
                                               int64_t status_len, int32_t* err, void* const* wait_events,
                                               void* const* record_events, void* stream) {
  using namespace wnw;
  WNW_CHECK_ARG(num_layers >= 0, "num_layers < 0");
  if (num_layers == 0) return WNW_OK;
  WNW_CHECK_ARG(layer_changed && k_store && v_store && seg_base && seg_len && seg_cap && num_segs && plan_blob &&
                    status && err,
                "null pointer argument");
  WNW_CHECK_ARG(land_rows >= 0 && move_rows >= 0 && status_len >= 0 && blob_ints > num_layers,
                "negative sizes, or a blob too small for the layer table");
  WNW_CHECK_ARG(k_landing == nullptr || (aligned16(k_landing) && aligned16(v_landing)),
                "landing buffers must be 16-byte aligned");
  WNW_CHECK_ARG(move_rows == 0 || (k_move && v_move && aligned16(k_move) && aligned16(v_move)),
                "move buffers must be given and 16-byte aligned when move_rows > 0");
  const int rb = row_bytes_of(dtype, head_dim);
  WNW_CHECK_ARG(rb > 0 && rb % 16 == 0, "row size must be a positive multiple of 16 bytes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the changed layers, checked and cut into launch pairs of kRbMultiMax
  std::vector<int> chg;
  int64_t st_need = 0;
  for (int l = 0; l < num_layers; ++l) {
    if (!layer_changed[l]) continue;
    WNW_CHECK_ARG(k_store[l] && v_store[l] && seg_base[l] && seg_len[l] && seg_cap[l] && num_segs[l] >= 0,
                  "layer %d: null store or table, or negative num_segs", l);
    WNW_CHECK_ARG(aligned16(k_store[l]) && aligned16(v_store[l]), "layer %d: stores must be 16-byte aligned", l);
    chg.push_back(l);
    st_need += num_segs[l];
  }
  WNW_CHECK_ARG(st_need <= status_len, "status needs %lld entries (the changed layers' num_segs), has %lld",
                static_cast<long long>(st_need), static_cast<long long>(status_len));
  if (chg.empty()) return WNW_OK;
  // every launch reads rows any earlier fetch may land: wait for all of them
  if (wait_events)
    for (int l : chg)
      if (wait_events[l]) WNW_CUDA_TRY(cudaStreamWaitEvent(s, static_cast<cudaEvent_t>(wait_events[l]), 0));
  int64_t status_base = 0;
  for (size_t c0 = 0; c0 < chg.size(); c0 += kRbMultiMax) {
    const int n = static_cast<int>(std::min<size_t>(kRbMultiMax, chg.size() - c0));
    RbMulti m = {};
    m.n = n;
    for (int i = 0; i < n; ++i) {
      const int l = chg[c0 + i];
      m.l[i] = RbLayer{static_cast<uint4*>(k_store[l]), static_cast<uint4*>(v_store[l]), seg_base[l], seg_len[l],
                       seg_cap[l], l, num_segs[l], static_cast<int>(status_base)};
      status_base += num_segs[l];
    }
    // about eight CTAs per SM over the launch's layers, at least 8 per layer
    const dim3 grid(std::max(8, (2 * kRbMaxBlocks + n - 1) / n), n);
    rebuild_gather_multi_kernel<<<grid, kRbThreads, 0, s>>>(m, plan_blob, blob_ints, k_landing ? land_rows : 0,
                                                             static_cast<uint4*>(k_move),
                                                             static_cast<uint4*>(v_move), move_rows, status, err,
                                                             rb / 16);
    WNW_CUDA_TRY(cudaGetLastError());
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kRbThreads, 1, 1);
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    WNW_CUDA_TRY(cudaLaunchKernelEx(&cfg, rebuild_scatter_multi_kernel, m, static_cast<const uint4*>(k_landing),
                                    static_cast<const uint4*>(v_landing), plan_blob, blob_ints, move_rows,
                                    static_cast<const uint4*>(k_move), static_cast<const uint4*>(v_move),
                                    static_cast<const int32_t*>(status), err, rb / 16));
  }
  if (record_events)
    for (int l : chg)
      if (record_events[l]) WNW_CUDA_TRY(cudaEventRecord(static_cast<cudaEvent_t>(record_events[l]), s));
  return WNW_OK;
}

extern "C" wnw_status wnw_copy_segments(int dtype, int head_dim, const void* src_k, const void* src_v,
                                        const int64_t* src_base, void* dst_k, void* dst_v,
                                        const int64_t* dst_base, const int32_t* len, int num_segs,
                                        void* stream) {
  using namespace wnw;
  WNW_CHECK_ARG(src_k && src_v && src_base && dst_k && dst_v && dst_base && len, "null pointer argument");
  WNW_CHECK_ARG(aligned16(src_k) && aligned16(src_v) && aligned16(dst_k) && aligned16(dst_v),
                "buffers must be 16-byte aligned");
  const int rb = row_bytes_of(dtype, head_dim);
  WNW_CHECK_ARG(rb > 0 && rb % 16 == 0, "row size must be a positive multiple of 16 bytes");
  if (num_segs <= 0) return WNW_OK;
  WNW_CHECK_ARG(num_segs <= 65535, "at most 65535 segments per call");
  // about four CTAs per SM over all segments (148 SMs), at least one per segment
  dim3 grid(std::min(64, std::max(1, (4 * 148 + num_segs - 1) / num_segs)), num_segs);
  copy_segments_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src_k), static_cast<const uint4*>(src_v), src_base, static_cast<uint4*>(dst_k),
      static_cast<uint4*>(dst_v), dst_base, len, rb / 16);
  WNW_CUDA_TRY(cudaGetLastError());
  return WNW_OK;
}

extern "C" wnw_status wnw_interleave_append(int dtype, int head_dim, const void* old, const void* new_tokens,
                                            const int32_t* cu_old, int num_segs, void* out, void* stream) {
  using namespace wnw;
  WNW_CHECK_ARG(new_tokens && cu_old && out, "null pointer argument");
  WNW_CHECK_ARG((old == nullptr || aligned16(old)) && aligned16(new_tokens) && aligned16(out),
                "buffers must be 16-byte aligned");
  const int rb = row_bytes_of(dtype, head_dim);
  WNW_CHECK_ARG(rb > 0 && rb % 16 == 0, "row size must be a positive multiple of 16 bytes");
  if (num_segs <= 0) return WNW_OK;
  WNW_CHECK_ARG(num_segs <= 65535, "at most 65535 segments per call");
  dim3 grid(4, num_segs);
  interleave_append_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(old), static_cast<const uint4*>(new_tokens), cu_old, static_cast<uint4*>(out),
      rb / 16);
  WNW_CUDA_TRY(cudaGetLastError());
  return WNW_OK;
}

extern "C" wnw_status wnw_advance_lengths(int32_t* seg_len, int64_t n, void* stream) {
  using namespace wnw;
  WNW_CHECK_ARG(seg_len != nullptr || n == 0, "null pointer argument");
  if (n <= 0) return WNW_OK;
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 1024));
  advance_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(seg_len, n);
  WNW_CUDA_TRY(cudaGetLastError());
  return WNW_OK;
}
