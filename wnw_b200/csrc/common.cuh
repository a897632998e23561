// Shared device helpers for the sm_100a WnW kernels: status plumbing, dtype
// traits, mbarrier / bulk-copy (TMA) PTX wrappers with bounded waits.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/wnw_b200.h"

namespace wnw {

// ---------------------------------------------------------------- host side
void set_error(const char* fmt, ...);
wnw_status cuda_status(cudaError_t e, const char* what);

#define WNW_CHECK_ARG(cond, ...)          \
  do {                                    \
    if (!(cond)) {                        \
      ::wnw::set_error(__VA_ARGS__);      \
      return WNW_ERR_INVALID;             \
    }                                     \
  } while (0)

#define WNW_CUDA_TRY(expr)                                     \
  do {                                                         \
    cudaError_t _e = (expr);                                   \
    if (_e != cudaSuccess) return ::wnw::cuda_status(_e, #expr); \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ------------------------------------------------------------- dtype traits
template <typename T> struct DT;
template <> struct DT<float> {
  static constexpr int code = WNW_F32;
  __device__ static inline float to_f(float x) { return x; }
  __device__ static inline float from_f(float x) { return x; }
};
template <> struct DT<__half> {
  static constexpr int code = WNW_F16;
  __device__ static inline float to_f(__half x) { return __half2float(x); }
  __device__ static inline __half from_f(float x) { return __float2half_rn(x); }
};
template <> struct DT<__nv_bfloat16> {
  static constexpr int code = WNW_BF16;
  __device__ static inline float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ static inline __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

// Unpack a 16-byte chunk into fp32 values (EPC = 16 / sizeof(T) elements).
template <typename T>
__device__ inline void unpack16(const uint4& u, float* f);

template <>
__device__ inline void unpack16<float>(const uint4& u, float* f) {
  f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
  f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
}
template <>
__device__ inline void unpack16<__nv_bfloat16>(const uint4& u, float* f) {
  // bf16 -> fp32 is exact: the bf16 bits are the high half of the fp32 bits.
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <>
__device__ inline void unpack16<__half>(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    float2 x = __half22float2(h);
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
}

// Hardware base-2 exponential (MUFU.EX2); ex2(-inf) = +0.
__device__ inline float ex2(float x) {
  float y;
  asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ------------------------------------------------------- mbarrier + TMA bulk
__device__ inline uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ inline void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make mbarrier initialisation visible to the async (TMA) proxy.
__device__ inline void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// acquire-release fence at gpu scope (cheaper than the sequentially
// consistent __threadfence)
__device__ inline void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
// atomic add with acquire-release semantics at gpu scope: releases what this
// thread has observed (cumulative) and acquires what earlier releasers of the
// same location published, in one memory round trip instead of fence + atomic
// + fence; returns the old value
__device__ inline int atom_add_acq_rel_gpu(int* addr, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
  return old;
}
// split cluster barrier: arrive (release) now, wait (acquire) later; every
// thread of every CTA of the cluster executes both, in this order
__device__ inline void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ inline void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// Programmatic dependent launch: wait until the preceding kernel in the
// stream has completed and its writes are visible / let the next kernel in
// the stream start its prologue.
// Bulk prefetch of [ptr, ptr + bytes) into L2 (16-byte aligned, bytes a
// multiple of 16); a hint with no completion to wait for.
__device__ inline void prefetch_l2(const void* ptr, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(ptr), "r"(bytes) : "memory");
}
__device__ inline void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ inline void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ inline void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ inline void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Plain arrive (no transaction bytes): completes a phase of a barrier whose
// expected arrival count is 1 without any copy.
__device__ inline void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 1-D bulk async copy global -> shared (this CTA), completion on `bar`.
__device__ inline void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 1-D bulk async copy shared -> global, tracked by the bulk-group mechanism.
__device__ inline void bulk_s2g(void* dst_gmem, const void* src_smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst_gmem),
               "r"(smem_u32(src_smem)), "r"(bytes)
               : "memory");
}
__device__ inline void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ inline void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ inline void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ inline bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and sets *err) when the phase never completes.
// try_wait already suspends in hardware for a while per poll, so the bound is
// a few seconds at most.
constexpr uint32_t kMaxPolls = 1u << 22;
__device__ inline bool mbar_wait(uint64_t* bar, uint32_t parity, int32_t* err) {
  for (uint32_t i = 0; i < kMaxPolls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i > 64) __nanosleep(64);
  }
  if (err) atomicOr(err, WNW_DEVERR_MBAR_TIMEOUT);
  return false;
}

}  // namespace wnw
