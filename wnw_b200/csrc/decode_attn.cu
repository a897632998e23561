// C ABI of the decode-attention kernel: argument checks, dtype dispatch and
// the host-side work-table builder.
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
                    (a->new_k == nullptr || (aligned16(a->new_k) && aligned16(a->new_v))),
                "q, stores, out and new rows must be 16-byte aligned");
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

extern "C" wnw_status wnw_build_work_table(const int32_t* seg_cap, int num_segs, int split_rows,
                                           int cluster_size, int32_t* work, int max_clusters,
                                           int* n_clusters) {
  using namespace wnw;
  WNW_CHECK_ARG(seg_cap && n_clusters && (work || max_clusters == 0), "null pointer argument");
  WNW_CHECK_ARG(split_rows > 0 && cluster_size > 0, "split_rows and cluster_size must be positive");
  int n = 0;
  for (int s = 0; s < num_segs; ++s) {
    WNW_CHECK_ARG(seg_cap[s] >= 0, "negative capacity at segment %d", s);
    const int64_t nsplit = (int64_t(seg_cap[s]) + 1 + split_rows - 1) / split_rows;
    const int64_t ncl = std::max<int64_t>(1, (nsplit + cluster_size - 1) / cluster_size);
    for (int64_t j = 0; j < ncl; ++j) {
      if (work != nullptr && n < max_clusters) {
        work[2 * n] = s;
        work[2 * n + 1] = static_cast<int32_t>(j);
      }
      ++n;
    }
  }
  *n_clusters = n;
  if (work != nullptr && n > max_clusters) {
    set_error("work table needs %d clusters, capacity %d", n, max_clusters);
    return WNW_ERR_CAPACITY;
  }
  return WNW_OK;
}
