// The per-step fetch graph shared by fetch.cu (which builds and launches it)
// and planner.cpp (which fills its tables): host-only declarations.
#pragma once

#include <stdint.h>

#include "../../include/wnw_b200.h"

namespace wnw {

// Everything a built graph bakes in; a different key rebuilds the graph.
struct FetchGraphKey {
  const void* src_k = nullptr;
  const void* src_v = nullptr;
  int64_t row_bytes = 0;
  int32_t* plan_host = nullptr;
  int32_t* plan_dev = nullptr;
  int32_t* ranges_host = nullptr;
  int32_t* ranges_dev = nullptr;
  int64_t* dst_host = nullptr;
  int64_t* dst_dev = nullptr;
  void* land_k = nullptr;
  void* land_v = nullptr;
  int max_ctas = 0;
  int L = 0;
  void* const* events = nullptr;
  // device-planned step: the range tables and layer offsets are already in
  // device memory (layer offsets here); the graph uploads nothing
  const int32_t* layer_ranges_dev = nullptr;
  bool operator==(const FetchGraphKey& o) const {
    return src_k == o.src_k && src_v == o.src_v && row_bytes == o.row_bytes && plan_host == o.plan_host &&
           plan_dev == o.plan_dev && ranges_host == o.ranges_host && ranges_dev == o.ranges_dev &&
           dst_host == o.dst_host && dst_dev == o.dst_dev && land_k == o.land_k && land_v == o.land_v &&
           max_ctas == o.max_ctas && L == o.L && events == o.events && layer_ranges_dev == o.layer_ranges_dev;
  }
};

// Upload the step's tables (plan_ints ints of plan, n_ranges ranges, the
// L + 1 layer offsets) and run the step's fetch as one graph launch.
wnw_status fetch_graph_issue(const void* owner, const FetchGraphKey& k, int64_t plan_ints, int64_t n_ranges,
                             const int32_t* layer_ranges, void* stream, void* const* events);
// Device-planned step (k.layer_ranges_dev set): the per-layer fetch and event
// records only, as one graph launch.
wnw_status fetch_graph_issue_planned(const void* owner, const FetchGraphKey& k, void* stream);
// Drop the graph built for `owner` (the planner is being destroyed).
void fetch_graph_release(const void* owner);

}  // namespace wnw
