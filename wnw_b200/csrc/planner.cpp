// Host planner of the WnW decode path: selection diff with eviction lag and
// per-layer evict / load / length planning.
//
// Same integer semantics as the reference Planner
// (src/algorithms/wnw_cpp/code/planner.cpp:19-306) and the Python path it
// mirrors (src/algorithms/wnw/code/cache.py:609-630, 756-866):
//  * needed  = union of the segments of the top-k chunks;
//  * to_load = needed - loaded;
//  * a loaded segment that is not needed bumps its counter and is evicted once
//    the counter reaches eviction_lag; a needed one resets its counter;
//  * per layer and per changed sample, each class-B head drops its evicted
//    ranges (sorted, segment-relative), shifts the remaining loaded ranges
//    down, and appends the loads in ascending segment order at
//    len - evicted; new_len = len - evicted + loaded + 1.
//
// State is kept in flat arrays (restore metadata indexed by a per-(layer,
// segment) base offset, loaded sets as byte maps) rather than nested vectors
// and std::set; iteration is always in ascending segment order, which is the
// order both reference implementations observe.
#include <algorithm>
#include <cstring>
#include <new>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/wnw_b200.h"
#include "fetch_graph.h"
#include "planner_tables.h"

namespace wnw {
void set_error(const char* fmt, ...);
wnw_status cuda_status(cudaError_t e, const char* what);
}

struct wnw_planner {
  int L = 0, H = 0, B = 0, S = 0;
  int top_k = 0, evict_lag = 1;
  bool prev_changed = false;
  bool have_seg_count = false, have_meta = false, have_lens = false;
  std::vector<int> seg_count;                    // [B]
  std::vector<std::vector<int>> c2s_flat, c2s_off;  // per sample CSR
  std::vector<std::vector<int>> class_b;          // per layer, kv heads
  std::vector<int64_t> meta_base;                 // [L*S] -> offset into meta arrays
  std::vector<int> cpu_s, cpu_e, gpu_s, gpu_e;    // flat restore metadata
  std::vector<std::vector<uint8_t>> loaded;       // [B][seg_count]
  std::vector<std::vector<int>> counters;         // [B][seg_count]
  std::vector<int> seq_lens;                      // [L*S]

  // results of the last compute_and_prepare
  std::vector<int32_t> ev_starts, ev_ends, cpu_ranges;
  std::vector<int32_t> layer_rows;                // [L+1] transfer-row offsets
  std::vector<int32_t> layer_ranges;              // [L+1] cpu-range offsets
  std::vector<std::vector<int>> to_load, to_evict;  // [B] sorted
  std::vector<int> changed;                       // changed samples
  // per layer: changed segments and their records (for the device plan)
  struct Chg {
    int seg, old_len, new_len, load_src, load_len, ev_lo, ev_hi;
  };
  std::vector<std::vector<Chg>> chg;              // [L]
  bool last_change = false;

  int64_t midx(int l, int fi) const { return meta_base[size_t(l) * S + fi]; }
};

namespace {

wnw_status bad(const char* msg) {
  wnw::set_error("%s", msg);
  return WNW_ERR_INVALID;
}

}  // namespace

extern "C" {

wnw_status wnw_planner_create(int num_layers, int num_kv_heads, int batch_size, int num_kv_groups,
                              wnw_planner** out) {
  (void)num_kv_groups;  // accepted for interface parity (planner.cpp:21); unused
  if (!out) return bad("null output pointer");
  if (num_layers <= 0 || num_kv_heads <= 0 || batch_size <= 0) return bad("dimensions must be positive");
  wnw_planner* p = new (std::nothrow) wnw_planner();
  if (!p) {
    wnw::set_error("out of host memory");
    return WNW_ERR_INVALID;
  }
  p->L = num_layers;
  p->H = num_kv_heads;
  p->B = batch_size;
  p->S = batch_size * num_kv_heads;
  p->c2s_flat.resize(p->B);
  p->c2s_off.resize(p->B);
  p->class_b.resize(p->L);
  p->loaded.resize(p->B);
  p->counters.resize(p->B);
  p->to_load.resize(p->B);
  p->to_evict.resize(p->B);
  p->chg.resize(p->L);
  p->layer_rows.assign(p->L + 1, 0);
  p->layer_ranges.assign(p->L + 1, 0);
  *out = p;
  return WNW_OK;
}

void wnw_planner_destroy(wnw_planner* p) {
  if (p) wnw::fetch_graph_release(p);
  delete p;
}

wnw_status wnw_planner_set_config(wnw_planner* p, int top_k_chunks, int eviction_lag) {
  if (!p) return bad("null planner");
  p->top_k = top_k_chunks;
  p->evict_lag = eviction_lag;
  return WNW_OK;
}

wnw_status wnw_planner_set_seg_count(wnw_planner* p, const int32_t* seg_count, int n) {
  if (!p || (!seg_count && n > 0)) return bad("null argument");
  if (n != p->B) return bad("seg_count must have batch_size entries");
  p->seg_count.assign(seg_count, seg_count + n);
  for (int b = 0; b < p->B; ++b) {
    if (p->seg_count[b] < 0) return bad("negative segment count");
    p->loaded[b].assign(p->seg_count[b], 0);
    p->counters[b].assign(p->seg_count[b], 0);
  }
  p->meta_base.assign(size_t(p->L) * p->S, 0);
  int64_t acc = 0;
  for (int l = 0; l < p->L; ++l)
    for (int fi = 0; fi < p->S; ++fi) {
      p->meta_base[size_t(l) * p->S + fi] = acc;
      acc += p->seg_count[fi / p->H];
    }
  p->have_seg_count = true;
  return WNW_OK;
}

wnw_status wnw_planner_set_chunk_to_segs(wnw_planner* p, int b, const int32_t* flat_segs, int n_flat,
                                         const int32_t* offsets, int n_offsets) {
  if (!p || !offsets || (!flat_segs && n_flat > 0)) return bad("null argument");
  if (b < 0 || b >= p->B) return bad("sample index out of range");
  if (!p->have_seg_count) return bad("set_seg_count must come first");
  if (n_offsets < 1 || offsets[0] != 0 || offsets[n_offsets - 1] != n_flat) return bad("bad chunk offsets");
  for (int i = 0; i + 1 < n_offsets; ++i)
    if (offsets[i + 1] < offsets[i]) return bad("chunk offsets must be non-decreasing");
  for (int i = 0; i < n_flat; ++i)
    if (flat_segs[i] < 0 || flat_segs[i] >= p->seg_count[b]) return bad("chunk references a missing segment");
  p->c2s_flat[b].assign(flat_segs, flat_segs + n_flat);
  p->c2s_off[b].assign(offsets, offsets + n_offsets);
  return WNW_OK;
}

wnw_status wnw_planner_set_class_b(wnw_planner* p, int layer, const int32_t* kv_heads, int n) {
  if (!p || (!kv_heads && n > 0)) return bad("null argument");
  if (layer < 0 || layer >= p->L) return bad("layer out of range");
  for (int i = 0; i < n; ++i)
    if (kv_heads[i] < 0 || kv_heads[i] >= p->H) return bad("kv head out of range");
  p->class_b[layer].assign(kv_heads, kv_heads + n);
  return WNW_OK;
}

wnw_status wnw_planner_set_restore_meta(wnw_planner* p, const int32_t* cpu_s, const int32_t* cpu_e,
                                        const int32_t* gpu_s, const int32_t* gpu_e, int64_t n) {
  if (!p || !cpu_s || !cpu_e || !gpu_s || !gpu_e) return bad("null argument");
  if (!p->have_seg_count) return bad("set_seg_count must come first");
  int64_t need = 0;
  for (int fi = 0; fi < p->S; ++fi) need += p->seg_count[fi / p->H];
  need *= p->L;
  if (n != need) return bad("restore metadata size does not match L * sum(seg_count)");
  p->cpu_s.assign(cpu_s, cpu_s + n);
  p->cpu_e.assign(cpu_e, cpu_e + n);
  p->gpu_s.assign(gpu_s, gpu_s + n);
  p->gpu_e.assign(gpu_e, gpu_e + n);
  p->have_meta = true;
  return WNW_OK;
}

wnw_status wnw_planner_set_loaded(wnw_planner* p, int b, const int32_t* segs, int n) {
  if (!p || (!segs && n > 0)) return bad("null argument");
  if (b < 0 || b >= p->B) return bad("sample index out of range");
  if (!p->have_seg_count) return bad("set_seg_count must come first");
  std::fill(p->loaded[b].begin(), p->loaded[b].end(), 0);
  for (int i = 0; i < n; ++i) {
    if (segs[i] < 0 || segs[i] >= p->seg_count[b]) return bad("loaded segment out of range");
    p->loaded[b][segs[i]] = 1;
  }
  return WNW_OK;
}

wnw_status wnw_planner_set_seq_lens(wnw_planner* p, const int32_t* seq_lens, int64_t n) {
  if (!p || !seq_lens) return bad("null argument");
  if (!p->have_seg_count) return bad("set_seg_count must come first");
  if (n != int64_t(p->L) * p->S) return bad("seq_lens must have num_layers * num_segs entries");
  p->seq_lens.assign(seq_lens, seq_lens + n);
  for (int b = 0; b < p->B; ++b) std::fill(p->counters[b].begin(), p->counters[b].end(), 0);
  p->prev_changed = false;
  p->have_lens = true;
  return WNW_OK;
}

wnw_status wnw_planner_get_loaded_segments(const wnw_planner* p, int b, int32_t* out, int cap, int* n_out) {
  if (!p || !n_out) return bad("null argument");
  if (b < 0 || b >= p->B) return bad("sample index out of range");
  int n = 0;
  for (int s = 0; s < int(p->loaded[b].size()); ++s)
    if (p->loaded[b][s]) {
      if (out && n < cap) out[n] = s;
      ++n;
    }
  *n_out = n;
  if (n > cap && out) {
    wnw::set_error("output capacity %d < %d loaded segments", cap, n);
    return WNW_ERR_CAPACITY;
  }
  return WNW_OK;
}

wnw_status wnw_planner_compute_and_prepare(wnw_planner* p, const int32_t* topk_idx, const int32_t* topk_off,
                                           int32_t* load_starts_2d, int32_t* load_lens_2d, int32_t* cu_new_2d,
                                           int32_t* new_lens_2d, int32_t* evict_offsets_2d, int32_t* evict_max,
                                           int32_t* evict_layer_ptr, int* any_change, int* total_tokens) {
  if (!p || !topk_off || !any_change || !total_tokens) return bad("null argument");
  if (!p->have_seg_count || !p->have_meta || !p->have_lens) return bad("planner state incomplete");
  const int L = p->L, S = p->S, H = p->H, B = p->B;
  if (!p->prev_changed)
    for (auto& x : p->seq_lens) x += 1;  // the previous step appended one row everywhere

  // ---- selection diff per sample (cache.py:609-630)
  bool change = false;
  std::vector<uint8_t> needed;
  for (int b = 0; b < B; ++b) {
    p->to_load[b].clear();
    p->to_evict[b].clear();
    const int lo = topk_off[b], hi = topk_off[b + 1];
    if (hi < lo) return bad("topk offsets must be non-decreasing");
    if (hi == lo) continue;
    const int nsb = p->seg_count[b];
    const int nchunks = int(p->c2s_off[b].size()) - 1;
    needed.assign(nsb, 0);
    for (int j = lo; j < hi; ++j) {
      const int c = topk_idx[j];
      if (c < 0 || c >= nchunks) return bad("top-k chunk index out of range");
      for (int k = p->c2s_off[b][c]; k < p->c2s_off[b][c + 1]; ++k) needed[p->c2s_flat[b][k]] = 1;
    }
    auto& ld = p->loaded[b];
    auto& cnt = p->counters[b];
    for (int s = 0; s < nsb; ++s) {
      if (needed[s] && !ld[s]) p->to_load[b].push_back(s);
      if (ld[s]) {
        if (!needed[s]) {
          cnt[s] += 1;
          if (cnt[s] >= p->evict_lag) p->to_evict[b].push_back(s);
        } else {
          cnt[s] = 0;
        }
      }
    }
    for (int s : p->to_load[b]) ld[s] = 1;
    for (int s : p->to_evict[b]) {
      ld[s] = 0;
      cnt[s] = 0;
    }
    if (!p->to_load[b].empty() || !p->to_evict[b].empty()) change = true;
  }

  p->ev_starts.clear();
  p->ev_ends.clear();
  p->cpu_ranges.clear();
  p->changed.clear();
  for (auto& v : p->chg) v.clear();
  std::fill(p->layer_rows.begin(), p->layer_rows.end(), 0);
  std::fill(p->layer_ranges.begin(), p->layer_ranges.end(), 0);
  p->last_change = change;
  if (!change) {
    p->prev_changed = false;
    *any_change = 0;
    *total_tokens = 0;
    return WNW_OK;
  }
  if (!load_starts_2d || !load_lens_2d || !cu_new_2d || !new_lens_2d || !evict_offsets_2d || !evict_max ||
      !evict_layer_ptr)
    return bad("null output array");
  for (int b = 0; b < B; ++b)
    if (!p->to_load[b].empty() || !p->to_evict[b].empty()) p->changed.push_back(b);

  // ---- per-layer planning (cache.py:771-823)
  std::vector<int> new_lens(size_t(L) * S);
  std::vector<std::pair<int, int>> ev;
  int gts = 0;
  for (int l = 0; l < L; ++l) {
    p->layer_rows[l] = gts;
    p->layer_ranges[l] = static_cast<int32_t>(p->cpu_ranges.size() / 2);
    int32_t* ls = load_starts_2d + size_t(l) * S;
    int32_t* ll = load_lens_2d + size_t(l) * S;
    int32_t* cun = cu_new_2d + size_t(l) * (S + 1);
    int32_t* nl = new_lens_2d + size_t(l) * S;
    for (int fi = 0; fi < S; ++fi) {
      new_lens[size_t(l) * S + fi] = p->seq_lens[size_t(l) * S + fi] + 1;
      ls[fi] = -1;
      ll[fi] = 0;
    }
    for (int b : p->changed) {
      for (int h : p->class_b[l]) {
        const int fi = b * H + h;
        const int seg_len = p->seq_lens[size_t(l) * S + fi];
        const int64_t m0 = p->midx(l, fi);
        int* gs = p->gpu_s.data() + m0;
        int* ge = p->gpu_e.data() + m0;
        const int* cs = p->cpu_s.data() + m0;
        const int* ce = p->cpu_e.data() + m0;
        const int nsb = p->seg_count[b];
        int evicted = 0;
        ev.clear();
        if (!p->to_evict[b].empty()) {
          for (int s : p->to_evict[b]) {
            if (cs[s] >= 0 && gs[s] >= 0) {
              ev.emplace_back(gs[s], ge[s]);
              gs[s] = ge[s] = -1;
            }
          }
          std::sort(ev.begin(), ev.end());
          for (auto& r : ev) evicted += r.second - r.first;
          if (!ev.empty()) {
            // shift the still-resident loaded ranges down (cache.py:792-799)
            std::vector<uint8_t> evicting(nsb, 0);
            for (int s : p->to_evict[b]) evicting[s] = 1;
            for (int s = 0; s < nsb; ++s) {
              if (cs[s] < 0 || gs[s] < 0 || evicting[s]) continue;
              int shift = 0;
              for (auto& r : ev)
                if (r.second <= gs[s]) shift += r.second - r.first;
              gs[s] -= shift;
              ge[s] -= shift;
            }
          }
        }
        const int ev_lo = static_cast<int>(p->ev_starts.size());
        for (auto& r : ev) {
          p->ev_starts.push_back(r.first);
          p->ev_ends.push_back(r.second);
        }
        const int ev_hi = static_cast<int>(p->ev_starts.size());
        int rel = seg_len - evicted;
        int loaded_n = 0;
        const int load_src = gts;
        for (int s : p->to_load[b]) {
          if (cs[s] < 0) continue;
          const int n = ce[s] - cs[s];
          p->cpu_ranges.push_back(cs[s]);
          p->cpu_ranges.push_back(ce[s]);
          if (ls[fi] < 0) ls[fi] = gts;
          ll[fi] += n;
          gs[s] = rel;
          ge[s] = rel + n;
          rel += n;
          loaded_n += n;
          gts += n;
        }
        new_lens[size_t(l) * S + fi] = seg_len - evicted + loaded_n + 1;
        p->chg[l].push_back({fi, seg_len, seg_len - evicted + loaded_n, load_src, loaded_n, ev_lo, ev_hi});
      }
    }
    cun[0] = 0;
    for (int fi = 0; fi < S; ++fi) {
      nl[fi] = new_lens[size_t(l) * S + fi];
      cun[fi + 1] = cun[fi] + nl[fi];
    }
  }
  // The planning loop visits (sample, class-B head) in configuration order;
  // the reference lays each layer's evict ranges out by segment index
  // (planner.cpp:281-292, cache.py:840-850), so re-pack them that way.
  {
    std::vector<int32_t> es, ee;
    es.reserve(p->ev_starts.size());
    ee.reserve(p->ev_ends.size());
    evict_layer_ptr[0] = 0;
    for (int l = 0; l < L; ++l) {
      std::vector<std::pair<int, size_t>> order;
      for (size_t i = 0; i < p->chg[l].size(); ++i) order.emplace_back(p->chg[l][i].seg, i);
      std::sort(order.begin(), order.end());
      int32_t* eo = evict_offsets_2d + size_t(l) * (S + 1);
      const int layer_base = static_cast<int>(es.size());
      size_t oi = 0;
      int emax = 0;
      eo[0] = 0;
      for (int fi = 0; fi < S; ++fi) {
        while (oi < order.size() && order[oi].first == fi) {
          auto& c = p->chg[l][order[oi].second];
          const int lo = static_cast<int>(es.size());
          for (int e = c.ev_lo; e < c.ev_hi; ++e) {
            es.push_back(p->ev_starts[e]);
            ee.push_back(p->ev_ends[e]);
          }
          c.ev_lo = lo;
          c.ev_hi = static_cast<int>(es.size());
          emax = std::max(emax, c.ev_hi - c.ev_lo);
          ++oi;
        }
        eo[fi + 1] = static_cast<int32_t>(es.size()) - layer_base;
      }
      evict_max[l] = emax;
      evict_layer_ptr[l + 1] = static_cast<int32_t>(es.size());
    }
    p->ev_starts.swap(es);
    p->ev_ends.swap(ee);
  }
  p->layer_rows[L] = gts;
  p->layer_ranges[L] = static_cast<int32_t>(p->cpu_ranges.size() / 2);
  p->seq_lens.swap(new_lens);
  p->prev_changed = true;
  *any_change = 1;
  *total_tokens = gts;
  return WNW_OK;
}

wnw_status wnw_planner_get_evictions(const wnw_planner* p, int32_t* starts, int32_t* ends, int cap, int* n) {
  if (!p || !n) return bad("null argument");
  const int m = static_cast<int>(p->ev_starts.size());
  *n = m;
  if (m > cap) {
    if (starts || ends) {
      wnw::set_error("capacity %d < %d eviction ranges", cap, m);
      return WNW_ERR_CAPACITY;
    }
    return WNW_OK;
  }
  if (starts) std::memcpy(starts, p->ev_starts.data(), sizeof(int32_t) * m);
  if (ends) std::memcpy(ends, p->ev_ends.data(), sizeof(int32_t) * m);
  return WNW_OK;
}

wnw_status wnw_planner_get_cpu_ranges(const wnw_planner* p, int32_t* ranges, int cap_pairs, int* n_pairs) {
  if (!p || !n_pairs) return bad("null argument");
  const int m = static_cast<int>(p->cpu_ranges.size() / 2);
  *n_pairs = m;
  if (m > cap_pairs) {
    if (ranges) {
      wnw::set_error("capacity %d < %d cpu ranges", cap_pairs, m);
      return WNW_ERR_CAPACITY;
    }
    return WNW_OK;
  }
  if (ranges) std::memcpy(ranges, p->cpu_ranges.data(), sizeof(int32_t) * 2 * m);
  return WNW_OK;
}

wnw_status wnw_planner_get_layer_transfer(const wnw_planner* p, int32_t* layer_rows, int32_t* layer_ranges) {
  if (!p || !layer_rows) return bad("null argument");
  std::memcpy(layer_rows, p->layer_rows.data(), sizeof(int32_t) * (p->L + 1));
  if (layer_ranges) std::memcpy(layer_ranges, p->layer_ranges.data(), sizeof(int32_t) * (p->L + 1));
  return WNW_OK;
}

wnw_status wnw_planner_get_changes(const wnw_planner* p, int b, int32_t* to_load, int cap_load, int* n_load,
                                   int32_t* to_evict, int cap_evict, int* n_evict) {
  if (!p || !n_load || !n_evict) return bad("null argument");
  if (b < 0 || b >= p->B) return bad("sample index out of range");
  const auto& a = p->to_load[b];
  const auto& e = p->to_evict[b];
  *n_load = static_cast<int>(a.size());
  *n_evict = static_cast<int>(e.size());
  if ((to_load && int(a.size()) > cap_load) || (to_evict && int(e.size()) > cap_evict)) {
    wnw::set_error("output capacity too small");
    return WNW_ERR_CAPACITY;
  }
  if (to_load) std::copy(a.begin(), a.end(), to_load);
  if (to_evict) std::copy(e.begin(), e.end(), to_evict);
  return WNW_OK;
}

}  // extern "C"

namespace {

// Sizes of the last plan (blob ints, landed rows, ranges, most rows a layer
// moves) and which layers it changes.
wnw_status fill_fetch_info(const wnw_planner* p, wnw_fetch_info* info) {
  const int L = p->L;
  int64_t used = 0;
  wnw_status st = wnw_planner_device_plan(p, nullptr, 0, &used);
  if (st != WNW_OK) return st;
  int64_t moved = 0;
  for (int l = 0; l < L; ++l) {
    int64_t m = 0;
    for (const auto& c : p->chg[l]) {
      const int n_ev = c.ev_hi - c.ev_lo;
      if (n_ev > 0) m += (c.new_len - c.load_len) - p->ev_starts[c.ev_lo];
    }
    moved = std::max(moved, m);
    if (info->layer_changed) info->layer_changed[l] = p->chg[l].empty() ? 0 : 1;
  }
  info->plan_ints = used;
  info->total_rows = p->layer_rows.empty() ? 0 : p->layer_rows[L];
  info->fetch_launches = 0;
  for (int l = 0; l < L; ++l) info->fetch_launches += p->layer_ranges[l + 1] > p->layer_ranges[l] ? 1 : 0;
  info->n_ranges = static_cast<int64_t>(p->cpu_ranges.size() / 2);
  info->max_moved_rows = moved;
  return WNW_OK;
}

}  // namespace

namespace wnw {

wnw_status planner_tables(const wnw_planner* p, PlannerTables* t) {
  if (!p || !t) return bad("null argument");
  if (!p->have_seg_count || !p->have_meta) return bad("planner state incomplete");
  t->L = p->L;
  t->H = p->H;
  t->B = p->B;
  t->evict_lag = p->evict_lag;
  t->chunk_base.assign(1, 0);
  t->c2s_off.clear();
  t->c2s_flat.clear();
  t->seg_base.assign(1, 0);
  t->seg_sample.clear();
  t->loaded.clear();
  t->counters.clear();
  for (int b = 0; b < p->B; ++b) {
    const int fb = static_cast<int>(t->c2s_flat.size());
    if (p->c2s_off[b].empty()) {
      t->c2s_off.push_back(fb);  // no chunks
    } else {
      for (int o : p->c2s_off[b]) t->c2s_off.push_back(fb + o);
      t->c2s_flat.insert(t->c2s_flat.end(), p->c2s_flat[b].begin(), p->c2s_flat[b].end());
    }
    t->chunk_base.push_back(static_cast<int32_t>(t->c2s_off.size()));
    const int nsb = p->seg_count[b];
    t->seg_base.push_back(t->seg_base.back() + nsb);
    for (int s = 0; s < nsb; ++s) {
      t->seg_sample.push_back(b);
      t->loaded.push_back(p->loaded[b][s]);
      t->counters.push_back(p->counters[b][s]);
    }
  }
  t->meta_base = p->meta_base;
  t->cpu_s = p->cpu_s;
  t->cpu_e = p->cpu_e;
  t->classb_off.assign(1, 0);
  t->classb.clear();
  for (int l = 0; l < p->L; ++l) {
    t->classb.insert(t->classb.end(), p->class_b[l].begin(), p->class_b[l].end());
    t->classb_off.push_back(static_cast<int32_t>(t->classb.size()));
  }
  return WNW_OK;
}

wnw_status planner_check_mirror(const wnw_planner* p, const int32_t* layer_rows, const uint8_t* loaded,
                                const int32_t* counters) {
  if (!p || !layer_rows || !loaded || !counters) return bad("null argument");
  for (int l = 0; l <= p->L; ++l) {
    const int32_t want = p->layer_rows.empty() ? 0 : p->layer_rows[l];
    if (layer_rows[l] != want) {
      wnw::set_error("device fetch plan: layer %d lands at row %d, the planner's plan at %d", l, layer_rows[l],
                     want);
      return WNW_ERR_STATE;
    }
  }
  int64_t i = 0;
  for (int b = 0; b < p->B; ++b)
    for (int s = 0; s < p->seg_count[b]; ++s, ++i)
      if (loaded[i] != p->loaded[b][s] || counters[i] != p->counters[b][s]) {
        wnw::set_error("device fetch plan: sample %d segment %d loaded/counter %d/%d, planner %d/%d", b, s,
                       int(loaded[i]), counters[i], int(p->loaded[b][s]), p->counters[b][s]);
        return WNW_ERR_STATE;
      }
  return WNW_OK;
}

}  // namespace wnw

extern "C" {

wnw_status wnw_planner_device_plan(const wnw_planner* p, int32_t* blob, int64_t cap, int64_t* used) {
  if (!p || !used) return bad("null argument");
  const int L = p->L;
  int64_t need = L + 1;
  for (int l = 0; l < L; ++l) {
    const int64_t n = static_cast<int64_t>(p->chg[l].size());
    int64_t ne = 0;
    for (auto& c : p->chg[l]) ne += c.ev_hi - c.ev_lo;
    need += 3 + 5 * n + 3 * (n + 1) + 2 * ne;
  }
  *used = need;
  if (!blob) return WNW_OK;
  if (need > cap) {
    wnw::set_error("device plan needs %lld ints, capacity %lld", (long long)need, (long long)cap);
    return WNW_ERR_CAPACITY;
  }
  int64_t o = L + 1;
  for (int l = 0; l < L; ++l) {
    blob[l] = static_cast<int32_t>(o);
    const auto& cl = p->chg[l];
    const int n = static_cast<int>(cl.size());
    int32_t* h = blob + o;  // n, moved rows, output rows
    int32_t* seg = h + 3;
    int32_t* old_len = seg + n;
    int32_t* new_len = old_len + n;
    int32_t* lsrc = new_len + n;
    int32_t* llen = lsrc + n;
    int32_t* mov_off = llen + n;
    int32_t* out_off = mov_off + n + 1;
    int32_t* ev_off = out_off + n + 1;
    int32_t* es = ev_off + n + 1;
    mov_off[0] = out_off[0] = ev_off[0] = 0;
    for (int i = 0; i < n; ++i) {
      const auto& c = cl[i];
      seg[i] = c.seg;
      old_len[i] = c.old_len;
      new_len[i] = c.new_len;
      lsrc[i] = c.load_src;
      llen[i] = c.load_len;
      const int n_ev = c.ev_hi - c.ev_lo;
      // rows that move: the kept rows after the first evicted range
      const int moved = n_ev > 0 ? (c.new_len - c.load_len) - p->ev_starts[c.ev_lo] : 0;
      mov_off[i + 1] = mov_off[i] + moved;
      out_off[i + 1] = out_off[i] + moved + c.load_len;
      ev_off[i + 1] = ev_off[i] + n_ev;
    }
    const int ne = ev_off[n];
    int32_t* ee = es + ne;
    int k = 0;
    for (int i = 0; i < n; ++i)
      for (int e = cl[i].ev_lo; e < cl[i].ev_hi; ++e, ++k) {
        es[k] = p->ev_starts[e];
        ee[k] = p->ev_ends[e];
      }
    h[0] = n;
    h[1] = mov_off[n];
    h[2] = out_off[n];
    o += 3 + 5 * n + 3 * (n + 1) + 2 * ne;
  }
  blob[L] = static_cast<int32_t>(o);
  return WNW_OK;
}

wnw_status wnw_planner_upload_plan(const wnw_planner* p, int32_t* plan_host, int32_t* plan_dev, int64_t plan_cap,
                                   void* stream, wnw_fetch_info* info) {
  if (!p || !info) return bad("null argument");
  wnw_status st = fill_fetch_info(p, info);
  if (st != WNW_OK) return st;
  if (info->plan_ints > plan_cap) {
    wnw::set_error("upload_plan needs %lld ints, capacity %lld", (long long)info->plan_ints, (long long)plan_cap);
    return WNW_ERR_CAPACITY;
  }
  if (!plan_host || !plan_dev) return bad("null buffer");
  int64_t used = 0;
  st = wnw_planner_device_plan(p, plan_host, plan_cap, &used);
  if (st != WNW_OK) return st;
  info->fetch_launches = 0;
  const cudaError_t e = cudaMemcpyAsync(plan_dev, plan_host, sizeof(int32_t) * used, cudaMemcpyHostToDevice,
                                        static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? WNW_OK : wnw::cuda_status(e, "cudaMemcpyAsync(plan)");
}

wnw_status wnw_planner_issue_fetch(const wnw_planner* p, int32_t* plan_host, int32_t* plan_dev, int64_t plan_cap,
                                   int32_t* ranges_host, int32_t* ranges_dev, int64_t* dst_host, int64_t* dst_dev,
                                   int64_t ranges_cap, const void* src_k, const void* src_v, int64_t row_bytes,
                                   void* land_k, void* land_v, int64_t land_rows, int max_ctas, void* stream,
                                   void* const* events, wnw_fetch_info* info) {
  if (!p || !info) return bad("null argument");
  const int L = p->L;
  // sizes first: nothing is issued unless every buffer is large enough
  wnw_status st = fill_fetch_info(p, info);
  if (st != WNW_OK) return st;
  int64_t used = info->plan_ints;
  const int64_t nr = info->n_ranges, rows = info->total_rows;
  if (used > plan_cap || nr > ranges_cap || rows > land_rows) {
    wnw::set_error("issue_fetch needs plan %lld / ranges %lld / rows %lld; capacity %lld / %lld / %lld",
                   (long long)used, (long long)nr, (long long)rows, (long long)plan_cap, (long long)ranges_cap,
                   (long long)land_rows);
    return WNW_ERR_CAPACITY;
  }
  if (!plan_host || !plan_dev || (nr > 0 && (!ranges_host || !ranges_dev || !dst_host || !dst_dev || !src_k ||
                                             !src_v || !land_k || !land_v)))
    return bad("null buffer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = wnw_planner_device_plan(p, plan_host, plan_cap, &used);
  if (st != WNW_OK) return st;
  if (ranges_cap > 0 && ranges_host && ranges_dev && dst_host && dst_dev && land_k && land_v && src_k && src_v) {
    // one graph launch: tables up, then per layer its fetch and its event
    int64_t acc = 0;
    for (int64_t i = 0; i < nr; ++i) {
      ranges_host[2 * i] = p->cpu_ranges[2 * i];
      ranges_host[2 * i + 1] = p->cpu_ranges[2 * i + 1];
      dst_host[i] = acc;
      acc += p->cpu_ranges[2 * i + 1] - p->cpu_ranges[2 * i];
    }
    wnw::FetchGraphKey k;
    k.src_k = src_k;
    k.src_v = src_v;
    k.row_bytes = row_bytes;
    k.plan_host = plan_host;
    k.plan_dev = plan_dev;
    k.ranges_host = ranges_host;
    k.ranges_dev = ranges_dev;
    k.dst_host = dst_host;
    k.dst_dev = dst_dev;
    k.land_k = land_k;
    k.land_v = land_v;
    k.max_ctas = max_ctas > 0 ? max_ctas : 32;
    k.L = L;
    k.events = events;
    info->fetch_launches = L;  // the graph runs every layer's fetch kernel
    return wnw::fetch_graph_issue(p, k, used, nr, p->layer_ranges.data(), stream, events);
  }
  cudaError_t e = cudaMemcpyAsync(plan_dev, plan_host, sizeof(int32_t) * used, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return wnw::cuda_status(e, "cudaMemcpyAsync(plan)");
  if (nr > 0) {
    std::memcpy(ranges_host, p->cpu_ranges.data(), sizeof(int32_t) * 2 * nr);
    int64_t acc = 0;
    for (int64_t i = 0; i < nr; ++i) {
      dst_host[i] = acc;
      acc += p->cpu_ranges[2 * i + 1] - p->cpu_ranges[2 * i];
    }
    e = cudaMemcpyAsync(ranges_dev, ranges_host, sizeof(int32_t) * 2 * nr, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(dst_dev, dst_host, sizeof(int64_t) * nr, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return wnw::cuda_status(e, "cudaMemcpyAsync(ranges)");
  }
  return wnw_fetch_layers(src_k, src_v, row_bytes, ranges_dev, dst_dev, p->layer_ranges.data(), L, land_k, land_v,
                          max_ctas, stream, events);
}

}  // extern "C"
