// C ABI of the decode-attention kernel: argument checks, dtype dispatch and
// the host-side work-table builder.
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "decode_attn.cuh"

namespace wnw {

int split_rows_for(int dtype, int head_dim) {
  const int esz = dtype == WNW_F32 ? 4 : 2;
  if (head_dim <= 0) return 0;
  if (esz == 2 && (head_dim == 64 || head_dim == 128)) return 128;  // tensor-core kernel tile
  return kAttnTileBytes / (2 * head_dim * esz);
}

}  // namespace wnw

extern "C" int wnw_split_rows(int dtype, int head_dim) { return wnw::split_rows_for(dtype, head_dim); }

namespace wnw {

// Resident CTAs (clusters x size) of the tensor-core kernel, cached per
// device, head_dim, cluster size and stage count.
static wnw_status mma_slots(int head_dim, int cs, int nstages, int* slots) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int>, int> cache;
  int dev = 0;
  WNW_CUDA_TRY(cudaGetDevice(&dev));
  const auto key = std::make_tuple(dev, head_dim, cs, nstages);
  {
    std::lock_guard<std::mutex> g(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *slots = it->second;
      return WNW_OK;
    }
  }
  int n = 0;
  const wnw_status st = attn_mma_active_clusters_any(head_dim, cs, nstages, &n);
  if (st != WNW_OK) return st;
  std::lock_guard<std::mutex> g(mu);
  cache[key] = n * cs;
  *slots = n * cs;
  return WNW_OK;
}

}  // namespace wnw

extern "C" wnw_status wnw_attn_launch_shape(int dtype, int head_dim, const int32_t* seg_cap, int num_segs,
                                            int* split_rows, int* cluster_size) {
  using namespace wnw;
  WNW_CHECK_ARG(seg_cap && split_rows && cluster_size, "null pointer argument");
  WNW_CHECK_ARG(num_segs >= 0, "num_segs < 0");
  const int base = split_rows_for(dtype, head_dim);
  WNW_CHECK_ARG(base > 0, "unsupported head_dim %d", head_dim);
  std::vector<int64_t> units(num_segs);
  int64_t maxu = 1;
  for (int s = 0; s < num_segs; ++s) {
    WNW_CHECK_ARG(seg_cap[s] >= 0, "negative capacity at segment %d", s);
    units[s] = (int64_t(seg_cap[s]) + 1 + base - 1) / base;
    maxu = std::max(maxu, units[s]);
  }
  const bool mma = dtype != WNW_F32 && (head_dim == 64 || head_dim == 128);
  if (!mma) {
    // CUDA-core kernel: one tile per CTA, clusters of up to 8, smaller when
    // even the longest segment needs fewer splits
    int cs = 1;
    while (cs < maxu && cs < 8) cs *= 2;
    *split_rows = base;
    *cluster_size = cs;
    return WNW_OK;
  }
  int dev = 0, nsm = 0;
  WNW_CUDA_TRY(cudaGetDevice(&dev));
  WNW_CUDA_TRY(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
  // Tiles per CTA T and cluster size cs.  Cost, in tile-stream times of one
  // SM: every wave of resident CTAs pays a fixed latency (first copy issued
  // only after the segment length is read, merge chain at the end: about
  // kWaveFixed tiles) plus T tiles for each CTA sharing an SM.  Then the
  // fewest cross-cluster partials, then the smaller T.
  constexpr int64_t kWaveFixed = 3;
  int64_t best_cost = INT64_MAX, best_ncl = INT64_MAX;
  int best_t = 1, best_cs = 1;
  for (int64_t t = 1;; t = (t < 4) ? t + 1 : (t % 3 == 0 ? t / 3 * 4 : t / 2 * 3)) {
    const int64_t max_ctas = (maxu + t - 1) / t;  // CTAs of the longest segment
    for (int cs = 8; cs >= 1; cs /= 2) {
      if (cs > 1 && cs / 2 >= max_ctas) continue;  // the longest segment would leave half a cluster idle
      int64_t ctas = 0, ncl_max = 0;
      for (int s = 0; s < num_segs; ++s) {
        const int64_t ncl = std::max<int64_t>(1, ((units[s] + t - 1) / t + cs - 1) / cs);
        ctas += ncl * cs;
        ncl_max = std::max(ncl_max, ncl);
      }
      int slots = 0;
      const wnw_status st = mma_slots(head_dim, cs, mma_stages(t), &slots);
      if (st != WNW_OK) return st;
      if (slots <= 0 || ctas == 0) continue;
      const int64_t waves = (ctas + slots - 1) / slots;
      const int64_t per_sm = (std::min<int64_t>(ctas, slots) + nsm - 1) / nsm;
      const int64_t cost = waves * (kWaveFixed + t * per_sm);
      if (cost < best_cost || (cost == best_cost && ncl_max < best_ncl)) {
        best_cost = cost;
        best_ncl = ncl_max;
        best_t = static_cast<int>(t);
        best_cs = cs;
      }
    }
    if (t >= maxu || t * base >= (int64_t(1) << 30)) break;
  }
  *split_rows = best_t * base;
  *cluster_size = best_cs;
  return WNW_OK;
}

extern "C" wnw_status wnw_decode_attn(const wnw_decode_attn_args* a, void* stream) {
  using namespace wnw;
  WNW_CHECK_ARG(a != nullptr, "null args");
  WNW_CHECK_ARG(a->q && a->k_store && a->v_store && a->seg_base && a->seg_len && a->work && a->out &&
                    a->partials && a->counters && a->err,
                "null pointer argument");
  WNW_CHECK_ARG((a->new_k == nullptr) == (a->new_v == nullptr), "new_k and new_v must both be given or both null");
  WNW_CHECK_ARG(a->num_segs > 0 && a->num_kv_heads > 0, "bad segment counts");
  WNW_CHECK_ARG(a->cluster_size == 1 || a->cluster_size == 2 || a->cluster_size == 4 || a->cluster_size == 8 ||
                    a->cluster_size == 16,
                "cluster_size must be 1, 2, 4, 8 or 16");
  WNW_CHECK_ARG(a->n_clusters >= 0, "n_clusters < 0");
  WNW_CHECK_ARG(aligned16(a->q) && aligned16(a->k_store) && aligned16(a->v_store) && aligned16(a->out) &&
                    aligned16(a->partials) &&
                    (a->new_k == nullptr || (aligned16(a->new_k) && aligned16(a->new_v))),
                "q, stores, out, partials and new rows must be 16-byte aligned");
  if (a->score_slot != nullptr)
    WNW_CHECK_ARG(a->audio_start && a->audio_end && a->logits && a->logits_off,
                  "scoring needs audio ranges, logits and offsets");
  if (a->n_clusters == 0) return WNW_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (a->dtype) {
    case WNW_F32: return dispatch_dtype<float>(a, s);
    case WNW_F16: return dispatch_dtype<__half>(a, s);
    case WNW_BF16: return dispatch_dtype<__nv_bfloat16>(a, s);
    default: set_error("unknown dtype %d", a->dtype); return WNW_ERR_UNSUPPORTED;
  }
}

extern "C" wnw_status wnw_decode_attn_step(const wnw_decode_attn_args* a, const void* q, const void* new_k,
                                           const void* new_v, void* out, void* stream) {
  using namespace wnw;
  WNW_CHECK_ARG(a != nullptr, "null args");
  wnw_decode_attn_args b = *a;
  b.q = q;
  b.new_k = new_k;
  b.new_v = new_v;
  b.out = out;
  return wnw_decode_attn(&b, stream);
}

extern "C" wnw_status wnw_build_work_table(const int32_t* seg_cap, int num_segs, int split_rows,
                                           int cluster_size, int32_t* work, int max_clusters,
                                           int* n_clusters) {
  using namespace wnw;
  WNW_CHECK_ARG(seg_cap && n_clusters && (work || max_clusters == 0), "null pointer argument");
  WNW_CHECK_ARG(split_rows > 0 && cluster_size > 0, "split_rows and cluster_size must be positive");
  WNW_CHECK_ARG(num_segs >= 0, "num_segs < 0");
  std::vector<int64_t> ncl(num_segs);
  int64_t n = 0;
  for (int s = 0; s < num_segs; ++s) {
    WNW_CHECK_ARG(seg_cap[s] >= 0, "negative capacity at segment %d", s);
    const int64_t nsplit = (int64_t(seg_cap[s]) + 1 + split_rows - 1) / split_rows;
    ncl[s] = std::max<int64_t>(1, (nsplit + cluster_size - 1) / cluster_size);
    n += ncl[s];
  }
  WNW_CHECK_ARG(n <= INT32_MAX, "work table too large");
  *n_clusters = static_cast<int>(n);
  if (work == nullptr) return WNW_OK;
  if (n > max_clusters) {
    set_error("work table needs %lld clusters, capacity %d", static_cast<long long>(n), max_clusters);
    return WNW_ERR_CAPACITY;
  }
  // segments split over several clusters first: they are launched (and get
  // their rows) first, so their longer cross-cluster merge overlaps the loads
  // of the single-cluster segments; a segment's clusters stay consecutive
  std::vector<int> order(num_segs);
  for (int s = 0; s < num_segs; ++s) order[s] = s;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return ncl[a] > ncl[b]; });
  int k = 0;
  for (int s : order) {
    for (int64_t j = 0; j < ncl[s]; ++j, ++k) {
      work[2 * k] = s;
      work[2 * k + 1] = static_cast<int32_t>(j);
    }
  }
  return WNW_OK;
}
