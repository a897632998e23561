// Instantiations of the decode-attention kernel for one dtype (split per
// dtype so the three translation units compile in parallel).
#include <algorithm>

#include "decode_attn_mma.cuh"

namespace wnw {

template <typename T, int D>
static wnw_status dispatch_g(const wnw_decode_attn_args* a, cudaStream_t s) {
  switch (a->group) {
    case 1: return launch_attn<T, D, 1>(a, s);
    case 2: return launch_attn<T, D, 2>(a, s);
    case 3: return launch_attn<T, D, 3>(a, s);
    case 4: return launch_attn<T, D, 4>(a, s);
    case 5: return launch_attn<T, D, 5>(a, s);
    case 6: return launch_attn<T, D, 6>(a, s);
    case 7: return launch_attn<T, D, 7>(a, s);
    case 8: return launch_attn<T, D, 8>(a, s);
    default: set_error("group %d not compiled (1..8)", a->group); return WNW_ERR_UNSUPPORTED;
  }
}

template <typename T, int D>
static wnw_status dispatch_mma(const wnw_decode_attn_args* a, cudaStream_t s) {
  switch (a->group) {
    case 1: return launch_attn_mma<T, D, 1>(a, s);
    case 2: return launch_attn_mma<T, D, 2>(a, s);
    case 3: return launch_attn_mma<T, D, 3>(a, s);
    case 4: return launch_attn_mma<T, D, 4>(a, s);
    case 5: return launch_attn_mma<T, D, 5>(a, s);
    case 6: return launch_attn_mma<T, D, 6>(a, s);
    case 7: return launch_attn_mma<T, D, 7>(a, s);
    case 8: return launch_attn_mma<T, D, 8>(a, s);
    default: set_error("group %d not compiled (1..8)", a->group); return WNW_ERR_UNSUPPORTED;
  }
}

template <>
wnw_status dispatch_dtype<__nv_bfloat16>(const wnw_decode_attn_args* a, cudaStream_t s) {
  switch (a->head_dim) {
    case 16: return dispatch_g<__nv_bfloat16, 16>(a, s);
    case 32: return dispatch_g<__nv_bfloat16, 32>(a, s);
    case 64: return dispatch_mma<__nv_bfloat16, 64>(a, s);
    case 128: return dispatch_mma<__nv_bfloat16, 128>(a, s);
    default: set_error("head_dim %d not compiled (16, 32, 64, 128)", a->head_dim); return WNW_ERR_UNSUPPORTED;
  }
}

}  // namespace wnw

namespace wnw {

// Residency of the tensor-core kernel for the plan builder.  The f16 and
// bf16 instantiations (and every group size) use the same resources per CTA,
// so the bf16, group-4 one stands for all of them.
wnw_status attn_mma_active_clusters_any(int head_dim, int cs, int* n) {
  switch (head_dim) {
    case 64: return attn_mma_active_clusters<__nv_bfloat16, 64, 4>(cs, n);
    case 128: return attn_mma_active_clusters<__nv_bfloat16, 128, 4>(cs, n);
    default: set_error("head_dim %d has no tensor-core kernel", head_dim); return WNW_ERR_UNSUPPORTED;
  }
}

}  // namespace wnw

#ifdef WNW_ATTN_TRACE
// Trace build only (not part of the product ABI): clear and read the bf16
// tensor-core kernel's phase records.
extern "C" wnw_status wnw_attn_trace_reset(void) {
  using namespace wnw;
  const int zero = 0;
  WNW_CUDA_TRY(cudaMemcpyToSymbol(g_attn_trace_n, &zero, sizeof(int)));
  return WNW_OK;
}
extern "C" wnw_status wnw_attn_trace_read(unsigned long long* out, int max_records, int* n) {
  using namespace wnw;
  WNW_CHECK_ARG(out && n && max_records >= 0, "null pointer argument");
  int cnt = 0;
  WNW_CUDA_TRY(cudaMemcpyFromSymbol(&cnt, g_attn_trace_n, sizeof(int)));
  cnt = std::min(std::min(cnt, kTraceCap), max_records);
  if (cnt > 0) WNW_CUDA_TRY(cudaMemcpyFromSymbol(out, g_attn_trace, size_t(cnt) * 8 * sizeof(unsigned long long)));
  *n = cnt;
  return WNW_OK;
}
#endif
