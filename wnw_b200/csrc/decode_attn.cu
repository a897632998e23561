// C ABI of the decode-attention kernel: argument checks, dtype dispatch and
// the host-side work-table builder.
#include <algorithm>
#include <cstdint>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "decode_attn.cuh"

namespace wnw {

int split_rows_for(int dtype, int head_dim) {
  const int esz = dtype == WNW_F32 ? 4 : 2;
  if (head_dim <= 0) return 0;
  if (esz == 2 && (head_dim == 64 || head_dim == 128)) return 0;  // tensor-core kernel: takes a plan
  return kAttnTileBytes / (2 * head_dim * esz);
}

bool uses_plan(int dtype, int head_dim) { return dtype != WNW_F32 && (head_dim == 64 || head_dim == 128); }

}  // namespace wnw

extern "C" int wnw_split_rows(int dtype, int head_dim) { return wnw::split_rows_for(dtype, head_dim); }

namespace wnw {

}  // namespace wnw

extern "C" wnw_status wnw_attn_launch_shape(int dtype, int head_dim, const int32_t* seg_cap, int num_segs,
                                            int* split_rows, int* cluster_size) {
  using namespace wnw;
  WNW_CHECK_ARG(seg_cap && split_rows && cluster_size, "null pointer argument");
  WNW_CHECK_ARG(num_segs >= 0, "num_segs < 0");
  WNW_CHECK_ARG(!uses_plan(dtype, head_dim),
                "16-bit K/V with head_dim %d take the tensor-core kernel, launched from a plan (wnw_attn_plan)",
                head_dim);
  const int base = split_rows_for(dtype, head_dim);
  WNW_CHECK_ARG(base > 0, "unsupported head_dim %d", head_dim);
  std::vector<int64_t> units(num_segs);
  int64_t maxu = 1;
  for (int s = 0; s < num_segs; ++s) {
    WNW_CHECK_ARG(seg_cap[s] >= 0, "negative capacity at segment %d", s);
    units[s] = (int64_t(seg_cap[s]) + 1 + base - 1) / base;
    maxu = std::max(maxu, units[s]);
  }
  // CUDA-core kernel: one tile per CTA, clusters of up to 8, smaller when
  // even the longest segment needs fewer splits
  int cs = 1;
  while (cs < maxu && cs < 8) cs *= 2;
  *split_rows = base;
  *cluster_size = cs;
  return WNW_OK;
}

extern "C" wnw_status wnw_decode_attn(const wnw_decode_attn_args* a, void* stream) {
  using namespace wnw;
  WNW_CHECK_ARG(a != nullptr, "null args");
  WNW_CHECK_ARG(a->q && a->k_store && a->v_store && a->seg_base && a->seg_len && a->out && a->partials && a->err,
                "null pointer argument");
  WNW_CHECK_ARG((a->new_k == nullptr) == (a->new_v == nullptr), "new_k and new_v must both be given or both null");
  WNW_CHECK_ARG(a->num_segs > 0 && a->num_kv_heads > 0, "bad segment counts");
  WNW_CHECK_ARG(aligned16(a->q) && aligned16(a->k_store) && aligned16(a->v_store) && aligned16(a->out) &&
                    aligned16(a->partials) &&
                    (a->new_k == nullptr || (aligned16(a->new_k) && aligned16(a->new_v))),
                "q, stores, out, partials and new rows must be 16-byte aligned");
  WNW_CHECK_ARG((a->flags & ~WNW_ATTN_ROWS_READY) == 0, "unknown flags 0x%x", a->flags);
  if (a->score_slot != nullptr)
    WNW_CHECK_ARG(a->audio_start && a->audio_end && a->logits && a->logits_off,
                  "scoring needs audio ranges, logits and offsets");
  if (!uses_plan(a->dtype, a->head_dim)) {
    WNW_CHECK_ARG(a->work && a->counters, "the CUDA-core path needs a work table and counters");
    WNW_CHECK_ARG(a->cluster_size == 1 || a->cluster_size == 2 || a->cluster_size == 4 || a->cluster_size == 8 ||
                      a->cluster_size == 16,
                  "cluster_size must be 1, 2, 4, 8 or 16");
    WNW_CHECK_ARG(a->n_clusters >= 0, "n_clusters < 0");
    if (a->n_clusters == 0) return WNW_OK;
  }
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

extern "C" wnw_status wnw_attn_resident_clusters(int head_dim, int cluster, int* n) {
  using namespace wnw;
  WNW_CHECK_ARG(n, "null pointer argument");
  WNW_CHECK_ARG(cluster >= 1 && cluster <= 16, "cluster must be in 1..16");
  return attn_mma_active_clusters_any(head_dim, cluster, n);
}

extern "C" wnw_status wnw_attn_plan(const int32_t* seg_cap, int num_segs, int sm_count, int max_cluster,
                                    int32_t* plan, int64_t max_ints, wnw_attn_plan_info* info) {
  using namespace wnw;
  constexpr int64_t kUnit = 32;           // rows: one TMA box pair of two warps
  constexpr int64_t kMaxShareUnits = 48;  // 1,536 rows: most a CTA takes to keep a segment in one cluster
  constexpr int64_t kWaveOverheadUnits = 16;  // a CTA's fixed cost (prologue, merge) ~ streaming 512 rows
  WNW_CHECK_ARG(seg_cap && info && (plan || max_ints == 0), "null pointer argument");
  WNW_CHECK_ARG(num_segs > 0, "num_segs must be positive");
  WNW_CHECK_ARG(max_cluster <= 16, "max_cluster must be in 1..16 (or <= 0 for the device's)");
  // CTA slots the device holds at once in clusters of c (the SM count when
  // the caller gives one)
  const bool query = sm_count <= 0;
  int dev = 0;
  if (query) {
    WNW_CUDA_TRY(cudaGetDevice(&dev));
    WNW_CUDA_TRY(cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev));
  }
  // residency queries take a while and never change for a device: kept per
  // (device, cluster size) for the life of the process
  static std::mutex slot_mu;
  static std::map<std::pair<int, int>, int64_t> slot_cache;
  auto slots_for = [&](int c) -> int64_t {
    if (!query) return sm_count;
    std::lock_guard<std::mutex> lock(slot_mu);
    auto it = slot_cache.find({dev, c});
    if (it != slot_cache.end()) return it->second;
    int n = 0;
    const int64_t v = attn_mma_active_clusters_any(128, c, &n) != WNW_OK || n <= 0
                          ? sm_count
                          : std::min<int64_t>(sm_count, int64_t(n) * c);
    slot_cache[{dev, c}] = v;
    return v;
  };
  if (max_cluster <= 0) max_cluster = slots_for(16) >= 16 ? 16 : 8;  // the largest cluster the device holds
  std::vector<int64_t> units(num_segs);
  int64_t total = 0, umax = 1;
  for (int s = 0; s < num_segs; ++s) {
    WNW_CHECK_ARG(seg_cap[s] >= 0 && seg_cap[s] < (1 << 30), "capacity of segment %d out of range", s);
    units[s] = (int64_t(seg_cap[s]) + 1 + kUnit - 1) / kUnit;  // capacity + the step's token
    total += units[s];
    umax = std::max(umax, units[s]);
  }
  // Units per CTA: an equal share of the device's CTA slots, raised so the
  // longest segment fits one cluster as long as that keeps shares <=
  // kMaxShareUnits; every segment then merges in distributed shared memory.
  // When a segment does not fit one cluster anyway, or the equal share itself
  // exceeds kMaxShareUnits (a large layer), segments may span several
  // clusters (merged by the last of them to finish): then clusters of at most 4 --
  // large clusters tie a segment's CTAs to a few GPCs and stream long
  // segments slower -- and a share sized to whole waves of resident CTAs.
  int cl = max_cluster;
  int c = 1;  // the cluster size of the plan at share sh (set by ctas_at)
  auto ctas_at = [&](int64_t sh) {  // the CTAs the packing below makes at share sh
    int64_t km = 1;
    for (int s = 0; s < num_segs; ++s) km = std::max(km, (units[s] + sh - 1) / sh);
    c = 1;
    while (c < std::min<int64_t>(km, cl)) c *= 2;
    int64_t n = 0, clusters = 0;
    std::vector<int64_t> need(c + 1, 0), free(c + 1, 0);  // segments by CTAs; clusters by free ranks
    for (int s = 0; s < num_segs; ++s) {
      const int64_t k = std::max<int64_t>(1, (units[s] + sh - 1) / sh);
      if (k > c)
        n += (k + c - 1) / c * c;
      else
        ++need[k];
    }
    for (int k = c; k >= 1; --k) {
      for (; need[k] > 0; --need[k]) {
        int f = k;
        while (f < c && free[f] == 0) ++f;
        if (f == c) ++clusters;
        else --free[f];
        if (f - k > 0) ++free[f - k];
      }
    }
    return n + clusters * c;
  };
  int64_t share = std::max<int64_t>((total + slots_for(cl) - 1) / slots_for(cl),
                                    std::min<int64_t>(kMaxShareUnits, (umax + cl - 1) / cl));
  int64_t limit = 0;  // > 0: plan for at most this many SMs (see below)
  auto slots_of = [&](int x) {  // CTA slots a plan may fill per wave
    return limit > 0 ? std::max<int64_t>(1, std::min<int64_t>(slots_for(x), limit)) : slots_for(x);
  };
  // Segments spanning clusters: clusters of at most 4; for w = 1..4 waves,
  // the smallest share whose CTAs fit w waves of the resident slots (or
  // every segment down to one CTA); then the w whose waves x (share + a
  // CTA's fixed cost) -- the busiest SM's time -- is least.  One wave avoids
  // a short tail wave; a few waves balance layers of many short segments
  // beside a few long ones.  Sets cl; returns the share.
  auto spread_share = [&]() {
    cl = std::min(cl, 4);
    int64_t best = INT64_MAX, best_sh = 1;
    for (int64_t w = 1; w <= 4; ++w) {
      const int64_t slots1 = slots_of(cl);
      int64_t sh = std::max<int64_t>(1, (total + w * slots1 - 1) / (w * slots1));
      for (int it = 0; it < 256 && ctas_at(sh) > w * slots_of(c) && sh < umax; ++it)
        sh = std::min(umax, sh + std::max<int64_t>(1, sh / 16));
      const int64_t slots = slots_of(c);
      const int64_t cost = (ctas_at(sh) + slots - 1) / slots * (sh + kWaveOverheadUnits);
      if (cost < best) {
        best = cost;
        best_sh = sh;
      }
    }
    return best_sh;
  };
  if ((umax + share - 1) / share <= cl && share <= kMaxShareUnits) {
    // one cluster per segment: keep the launch to one wave of the clusters
    // the device holds at once (a larger share means fewer CTAs per segment
    // and smaller clusters)
    for (int it = 0; it < 256 && ctas_at(share) > slots_for(c) && share < umax; ++it)
      share = std::min(umax, share + std::max<int64_t>(1, share / 16));
    // Clusters above 4 CTAs tie each long segment to one GPC, which streams
    // it at about 1 TB/s.  When that makes a CTA's streaming outweigh its
    // fixed cost (shares above kWaveOverheadUnits), the layer is planned
    // again with segments spanning clusters of 4 on half, then two thirds of
    // the SMs, and the first of those plans whose share is smaller is taken.
    // Back to back, the next layer's CTAs then find free SMs (one CTA per
    // SM) and load their first stages while this layer's CTAs stream and
    // merge.  Measured on a B200, layers of 2-5 segments of 15.1k rows beside
    // 2.3k-row ones, back to back: one class-A segment 9.80 -> 9.17 us (half),
    // two 10.07 -> 9.38 (half), three 10.41 -> 9.91 and four 11.37 -> 10.76
    // (two thirds); all the SMs (clusters of 4) gave 9.75-11.27 us.
    if (c > 4 && share > kWaveOverheadUnits) {
      const int keep_cl = cl;
      for (const int64_t part : {int64_t(sm_count) / 2, int64_t(sm_count) * 2 / 3}) {
        if (part < 1 || (total + part - 1) / part > kMaxShareUnits) continue;
        limit = part;
        const int64_t sh = spread_share();
        if (sh < share) {
          share = sh;
          break;
        }
        limit = 0;
        cl = keep_cl;
      }
    }
  } else {
    share = spread_share();
  }
  std::vector<int64_t> k(num_segs);
  int64_t kmax = 1;
  for (int s = 0; s < num_segs; ++s) {
    k[s] = std::max<int64_t>(1, (units[s] + share - 1) / share);
    kmax = std::max(kmax, k[s]);
  }
  int C = 1;
  while (C < std::min<int64_t>(kmax, cl)) C *= 2;

  struct Slot {
    int32_t seg, r0, r1, meta;
  };
  std::vector<Slot> slots;       // clusters x C
  std::vector<int32_t> part_r0;  // first row of each cluster partial
  std::vector<int32_t> comb;     // seg, first part, parts, 0
  auto new_cluster = [&]() {
    const size_t at = slots.size();
    slots.resize(at + C, Slot{-1, 0, 0, 0});
    return at;
  };
  // ranks [r, r + n) of the cluster at `at` attend units [u0, u1) of segment
  // s, split evenly (the first ranks take the extra units)
  auto place = [&](size_t at, int r, int n, int s, int64_t u0, int64_t u1, bool to_part, int64_t part) {
    const int64_t nu = u1 - u0;
    int64_t u = u0;
    for (int i = 0; i < n; ++i) {
      const int64_t take = nu / n + (i < nu % n ? 1 : 0);
      const uint32_t meta = static_cast<uint32_t>(r) | (static_cast<uint32_t>(n) << 5) |
                            ((to_part ? 1u : 0u) << 10) | (static_cast<uint32_t>(part) << 11);
      slots[at + r + i] = Slot{s, static_cast<int32_t>(u * kUnit), static_cast<int32_t>((u + take) * kUnit),
                               static_cast<int32_t>(meta)};
      u += take;
    }
  };
  // segments needing more CTAs than a cluster holds: whole clusters, each
  // an even share of the segment's units; the last cluster to finish merges them
  for (int s = 0; s < num_segs; ++s) {
    if (k[s] <= C) continue;
    const int64_t ncl = (k[s] + C - 1) / C;
    comb.insert(comb.end(), {s, static_cast<int32_t>(part_r0.size()), static_cast<int32_t>(ncl), 0});
    for (int64_t j = 0; j < ncl; ++j) {
      const int64_t u0 = units[s] * j / ncl, u1 = units[s] * (j + 1) / ncl;
      WNW_CHECK_ARG(part_r0.size() < (size_t(1) << 21), "too many cluster partials");
      const size_t at = new_cluster();
      place(at, 0, C, s, u0, u1, true, static_cast<int64_t>(part_r0.size()));
      part_r0.push_back(static_cast<int32_t>(u0 * kUnit));
    }
  }
  // the others: packed into clusters, largest first, each into the cluster
  // with the fewest free ranks that still hold it
  std::vector<int> order;
  for (int s = 0; s < num_segs; ++s)
    if (k[s] <= C) order.push_back(s);
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return k[a] > k[b]; });
  std::vector<std::vector<size_t>> by_free(C + 1);  // clusters by free ranks
  std::vector<int> used;                            // ranks taken per cluster (index: at / C)
  for (int s : order) {
    const int need = static_cast<int>(k[s]);
    size_t at = SIZE_MAX;
    for (int f = need; f < C && at == SIZE_MAX; ++f) {
      if (!by_free[f].empty()) {
        at = by_free[f].back();
        by_free[f].pop_back();
      }
    }
    if (at == SIZE_MAX) {
      at = new_cluster();
      used.resize(slots.size() / C, 0);
    }
    int& r = used[at / C];
    place(at, r, need, s, 0, units[s], false, 0);
    r += need;
    if (r < C) by_free[C - r].push_back(at);
  }
  const int64_t ctas = static_cast<int64_t>(slots.size());
  const int64_t parts = static_cast<int64_t>(part_r0.size());
  const int64_t ints = 8 + 4 * ctas + (parts + 3) / 4 * 4 + static_cast<int64_t>(comb.size());
  WNW_CHECK_ARG(ctas < INT32_MAX && ints < INT32_MAX, "plan too large");
  info->ctas = static_cast<int>(ctas);
  info->cluster = C;
  info->parts = static_cast<int>(parts);
  info->combine = static_cast<int>(comb.size() / 4);
  info->ints = ints;
  if (plan == nullptr) return WNW_OK;
  if (max_ints < ints) {
    set_error("the plan needs %lld ints, capacity %lld", static_cast<long long>(ints),
              static_cast<long long>(max_ints));
    return WNW_ERR_CAPACITY;
  }
  std::fill(plan, plan + ints, 0);
  plan[0] = info->ctas;
  plan[1] = C;
  plan[2] = info->parts;
  plan[3] = info->combine;
  for (int64_t c = 0; c < ctas; ++c) {
    plan[8 + 4 * c] = slots[c].seg;
    plan[8 + 4 * c + 1] = slots[c].r0;
    plan[8 + 4 * c + 2] = slots[c].r1;
    plan[8 + 4 * c + 3] = slots[c].meta;
  }
  std::copy(part_r0.begin(), part_r0.end(), plan + 8 + 4 * ctas);
  std::copy(comb.begin(), comb.end(), plan + 8 + 4 * ctas + (parts + 3) / 4 * 4);
  return WNW_OK;
}
