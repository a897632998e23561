// The planner state the device fetch plan (device_plan.cu) mirrors, exported
// by planner.cpp as flat arrays: host-only declarations.
#pragma once

#include <stdint.h>

#include <vector>

#include "../../include/wnw_b200.h"

namespace wnw {

struct PlannerTables {
  int L = 0, H = 0, B = 0, evict_lag = 1;
  std::vector<int32_t> chunk_base;  // [B+1] sample b's chunk offsets start at c2s_off[chunk_base[b]]
  std::vector<int32_t> c2s_off;     // per sample nchunks+1 offsets into c2s_flat (absolute)
  std::vector<int32_t> c2s_flat;    // segment ids (sample-local)
  std::vector<int32_t> seg_base;    // [B+1] sample b's segments are state rows [seg_base[b], seg_base[b+1])
  std::vector<int32_t> seg_sample;  // [total segments] owning sample
  std::vector<uint8_t> loaded;      // [total segments]
  std::vector<int32_t> counters;    // [total segments]
  std::vector<int64_t> meta_base;   // [L*S] offset of (layer, slot) into cpu_s / cpu_e
  std::vector<int32_t> cpu_s, cpu_e;
  std::vector<int32_t> classb_off;  // [L+1] offsets into classb
  std::vector<int32_t> classb;      // class-B kv heads, per layer in configuration order
};

wnw_status planner_tables(const wnw_planner* p, PlannerTables* t);

// WNW_OK when the device's results of the last step (per-layer landing-row
// offsets [L+1], loaded maps and counters in seg_base order) equal the
// planner's; WNW_ERR_STATE with a message naming the first difference.
wnw_status planner_check_mirror(const wnw_planner* p, const int32_t* layer_rows, const uint8_t* loaded,
                                const int32_t* counters);

}  // namespace wnw
