// Tensor maps (TMA descriptors) for the K / V stores, built once per store
// and cached: 2-D [rows, head_dim] maps with 128-byte swizzle, box =
// 64 bf16/f16 columns x `box_rows` rows.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace wnw {

// Returns false (with the error set) when the driver entry point or the
// encode call fails.  Thread-safe; maps are cached by (base, rows, dtype, D).
bool kv_tensor_map(CUtensorMap* out, const void* base, int64_t rows, int head_dim, int dtype, int box_rows);

__device__ inline void tma_load_2d(void* dst_smem, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst_smem)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace wnw
