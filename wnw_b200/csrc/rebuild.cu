// In-place layout maintenance for the slot layout of the flat varlen cache.
//
// Every (sample, kv head) segment owns a fixed slot [seg_base, seg_base+cap)
// of its layer's K / V store.  A chunk update of the reference rewrites the
// whole flat buffer (rebuild_append_kv, src/algorithms/wnw/code/kernels.py:
// 375-473); here only the changed segments move rows inside their own slot:
// evicted ranges are squeezed out (later rows shift down) and the rows fetched
// from host memory are spliced after the kept rows.  The step's new token is
// appended afterwards by the decode-attention kernel.
#include <algorithm>

#include "common.cuh"

namespace wnw {

constexpr int kRbThreads = 128;
constexpr int kRbStages = 8;
constexpr int kRbStageBytes = 8 * 1024;  // per tensor per stage

// One tile of a row move: `n` rows from src (slot-relative row or landing
// row) to dst (slot-relative row).
struct RbTile {
  int src;
  int dst;
  int n;
  int landing;
};

// Walks the moves of one segment in ascending source order: the kept runs
// after the first evicted range (each shifted down by the rows evicted before
// it), then the spliced landing rows.
struct RbWalker {
  const int32_t* ev_s;
  const int32_t* ev_e;
  int n_ev;
  int old_len;
  int kept_len;
  int load_src;
  int load_len;
  int tile_rows;
  // state
  int k;      // current run (0..n_ev-1), n_ev = splice phase, n_ev+1 = done
  int off;    // rows of the current piece already emitted
  int shift;  // rows evicted up to and including run k's range

  __device__ void init() {
    k = 0;
    off = 0;
    shift = n_ev > 0 ? (ev_e[0] - ev_s[0]) : 0;
    if (n_ev == 0) k = 0;  // no runs: go straight to the splice phase
  }
  __device__ bool next(RbTile& t) {
    while (k < n_ev) {
      const int run_lo = ev_e[k];
      const int run_hi = (k + 1 < n_ev) ? ev_s[k + 1] : old_len;
      const int left = run_hi - run_lo - off;
      if (left > 0) {
        const int n = min(left, tile_rows);
        t.src = run_lo + off;
        t.dst = run_lo + off - shift;
        t.n = n;
        t.landing = 0;
        off += n;
        return true;
      }
      ++k;
      off = 0;
      if (k < n_ev) shift += ev_e[k] - ev_s[k];
    }
    if (k == n_ev) {
      const int left = load_len - off;
      if (left > 0) {
        const int n = min(left, tile_rows);
        t.src = load_src + off;
        t.dst = kept_len + off;
        t.n = n;
        t.landing = 1;
        off += n;
        return true;
      }
      k = n_ev + 1;
    }
    return false;
  }
};

template <int ROW_BYTES>
__global__ void __launch_bounds__(kRbThreads)
    rebuild_kernel(uint8_t* k_store, uint8_t* v_store, const int64_t* seg_base, int32_t* seg_len,
                   const int32_t* seg_cap, const uint8_t* k_land, const uint8_t* v_land,
                   const int32_t* blob, int layer, int32_t* err) {
  constexpr int TR = kRbStageBytes / ROW_BYTES;  // rows per tile
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[kRbStages];
  __shared__ RbTile tiles[kRbStages];

  const int32_t* rec = blob + blob[layer];
  const int n = rec[0];
  const int i = blockIdx.x;
  if (i >= n) return;
  const int seg = rec[1 + i];
  const int old_len = rec[1 + n + i];
  const int new_len = rec[1 + 2 * n + i];
  const int load_src = rec[1 + 3 * n + i];
  const int load_len = rec[1 + 4 * n + i];
  const int32_t* ev_off = rec + 1 + 5 * n;
  const int n_ev_total = ev_off[n];
  const int32_t* ev_s = ev_off + n + 1 + ev_off[i];
  const int32_t* ev_e = ev_off + n + 1 + n_ev_total + ev_off[i];
  const int n_ev = ev_off[i + 1] - ev_off[i];

  if (threadIdx.x != 0) return;  // a single thread drives the bulk-copy pipeline
  if (seg_len[seg] != old_len) {
    atomicOr(err, WNW_DEVERR_LEN_MISMATCH);
    return;
  }
  // ranges must be sorted, disjoint and inside the segment: a malformed plan
  // is refused rather than allowed to move rows outside the slot
  int evicted = 0, prev_end = 0;
  for (int e = 0; e < n_ev; ++e) {
    if (ev_s[e] < prev_end || ev_e[e] < ev_s[e] || ev_e[e] > old_len) {
      atomicOr(err, WNW_DEVERR_LEN_MISMATCH);
      return;
    }
    prev_end = ev_e[e];
    evicted += ev_e[e] - ev_s[e];
  }
  if (load_len < 0 || load_src < 0) {
    atomicOr(err, WNW_DEVERR_LEN_MISMATCH);
    return;
  }
  const int kept_len = old_len - evicted;
  if (kept_len + load_len != new_len) {
    atomicOr(err, WNW_DEVERR_LEN_MISMATCH);
    return;
  }
  if (seg_cap != nullptr && new_len + 1 > seg_cap[seg]) {
    atomicOr(err, WNW_DEVERR_CAPACITY);
    return;
  }
  for (int s = 0; s < kRbStages; ++s) mbar_init(&bars[s], 1);
  fence_mbar_init();
  fence_proxy_async();

  uint8_t* kbase = k_store + seg_base[seg] * ROW_BYTES;
  uint8_t* vbase = v_store + seg_base[seg] * ROW_BYTES;
  RbWalker walk{ev_s, ev_e, n_ev, old_len, kept_len, load_src, load_len, TR, 0, 0, 0};
  walk.init();

  // Loads run up to kRbStages tiles ahead of the stores.  Sources of later
  // tiles lie at or above the end of every earlier tile's source, and a tile's
  // destination never extends past its own source's end, so no store can
  // clobber a source that is still to be read; stores are issued in tile
  // order after the tile's own load (and hence all earlier loads) completed.
  int issued = 0, done = 0;
  bool more = true;
  for (;;) {
    while (more && issued - done < kRbStages) {
      RbTile t;
      if (!walk.next(t)) {
        more = false;
        break;
      }
      const int s = issued % kRbStages;
      if (issued >= kRbStages) bulk_wait_read<0>();  // the stage's previous store has read smem
      tiles[s] = t;
      const uint32_t bytes = uint32_t(t.n) * ROW_BYTES;
      uint8_t* ks = smem + s * 2 * kRbStageBytes;
      uint8_t* vs = ks + kRbStageBytes;
      mbar_arrive_expect_tx(&bars[s], 2 * bytes);
      const uint8_t* ksrc = t.landing ? (k_land + int64_t(t.src) * ROW_BYTES) : (kbase + int64_t(t.src) * ROW_BYTES);
      const uint8_t* vsrc = t.landing ? (v_land + int64_t(t.src) * ROW_BYTES) : (vbase + int64_t(t.src) * ROW_BYTES);
      bulk_g2s(ks, ksrc, bytes, &bars[s]);
      bulk_g2s(vs, vsrc, bytes, &bars[s]);
      ++issued;
    }
    if (done == issued) break;
    const int s = done % kRbStages;
    if (!mbar_wait(&bars[s], (done / kRbStages) & 1, err)) break;
    const RbTile t = tiles[s];
    uint8_t* ks = smem + s * 2 * kRbStageBytes;
    uint8_t* vs = ks + kRbStageBytes;
    bulk_s2g(kbase + int64_t(t.dst) * ROW_BYTES, ks, uint32_t(t.n) * ROW_BYTES);
    bulk_s2g(vbase + int64_t(t.dst) * ROW_BYTES, vs, uint32_t(t.n) * ROW_BYTES);
    bulk_commit();
    ++done;
  }
  bulk_wait_all();
  seg_len[seg] = new_len;
}

template <int ROW_BYTES>
wnw_status launch_rebuild(void* k_store, void* v_store, const int64_t* seg_base, int32_t* seg_len,
                          const int32_t* seg_cap, const void* kl, const void* vl, const int32_t* plan,
                          int layer, int max_changed, int32_t* err, cudaStream_t s) {
  auto kern = rebuild_kernel<ROW_BYTES>;
  constexpr int smem = kRbStages * 2 * kRbStageBytes;
  static bool configured = false;
  if (!configured) {
    WNW_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured = true;
  }
  kern<<<max_changed, kRbThreads, smem, s>>>(static_cast<uint8_t*>(k_store), static_cast<uint8_t*>(v_store),
                                             seg_base, seg_len, seg_cap, static_cast<const uint8_t*>(kl),
                                             static_cast<const uint8_t*>(vl), plan, layer, err);
  WNW_CUDA_TRY(cudaGetLastError());
  return WNW_OK;
}

// ------------------------------------------------------------ segment copy
__global__ void copy_segments_kernel(const uint4* src_k, const uint4* src_v, const int64_t* src_base,
                                     uint4* dst_k, uint4* dst_v, const int64_t* dst_base,
                                     const int32_t* len, int chunks_per_row) {
  const int seg = blockIdx.y;
  const int64_t n = int64_t(len[seg]) * chunks_per_row;
  const int64_t s0 = src_base[seg] * chunks_per_row;
  const int64_t d0 = dst_base[seg] * chunks_per_row;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
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
                                           const void* k_landing, const void* v_landing, const int32_t* plan_blob,
                                           int layer, int max_changed, int32_t* err, void* stream) {
  using namespace wnw;
  WNW_CHECK_ARG(k_store && v_store && seg_base && seg_len && plan_blob && err, "null pointer argument");
  WNW_CHECK_ARG(layer >= 0, "negative layer");
  WNW_CHECK_ARG(aligned16(k_store) && aligned16(v_store), "stores must be 16-byte aligned");
  WNW_CHECK_ARG(k_landing == nullptr || (aligned16(k_landing) && aligned16(v_landing)),
                "landing buffers must be 16-byte aligned");
  if (max_changed <= 0) return WNW_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (row_bytes_of(dtype, head_dim)) {
    case 32: return launch_rebuild<32>(k_store, v_store, seg_base, seg_len, seg_cap, k_landing, v_landing, plan_blob, layer, max_changed, err, s);
    case 64: return launch_rebuild<64>(k_store, v_store, seg_base, seg_len, seg_cap, k_landing, v_landing, plan_blob, layer, max_changed, err, s);
    case 128: return launch_rebuild<128>(k_store, v_store, seg_base, seg_len, seg_cap, k_landing, v_landing, plan_blob, layer, max_changed, err, s);
    case 256: return launch_rebuild<256>(k_store, v_store, seg_base, seg_len, seg_cap, k_landing, v_landing, plan_blob, layer, max_changed, err, s);
    case 512: return launch_rebuild<512>(k_store, v_store, seg_base, seg_len, seg_cap, k_landing, v_landing, plan_blob, layer, max_changed, err, s);
    default: set_error("row size %d bytes not compiled", row_bytes_of(dtype, head_dim)); return WNW_ERR_UNSUPPORTED;
  }
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
  dim3 grid(8, num_segs);
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
