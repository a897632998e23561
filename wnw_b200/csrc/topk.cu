// Class-A score finalisation and fused chunk scoring + top-k (sm_100a).
//
// The decode-attention kernel leaves, per class-A (layer, segment), the base-2
// logits of the audio rows and the merged softmax statistics.  Here:
//  * wnw_score_finalize forms acc[t] = sum over the step's class-A terms of
//    sum_g 2^(x - m_g) / l_g -- the probabilities the reference accumulates
//    in fused_attn.py:107-121 and kernels.py:302-370 -- no atomics, a fixed
//    summation order (8 interleaved partial sums over the layer-major /
//    ascending-kv term list, combined in order);
//  * wnw_chunk_topk computes the chunk means of cache.py:632-640 and the top-k
//    of cache.py:648 (ties -> lower index) in one CTA per sample, the top-k
//    by ranking every chunk against all others in one pass.  The prefix
//    sums are taken at segment boundaries only, accumulated in fp64 and rounded
//    to fp32, which is what torch's CPU cumsum produces for an fp32 input.
#include <algorithm>

#include "common.cuh"

namespace wnw {

// One CTA per (32 audio tokens, sample): the 8 warps split the sample's
// class-A terms (warp w takes terms w, w+8, ...; lane = token) and the warp
// sums are added in warp order -- a fixed order, so results repeat bit for bit.
constexpr int kFinWarps = 8;
__global__ void __launch_bounds__(kFinWarps * 32)
    score_finalize_kernel(const float* logits, const float* stats, const int64_t* logit_off, const int64_t* stat_off,
                          const uint32_t* qmask, const int32_t* term_off, int group, const int32_t* score_off,
                          float* acc) {
  __shared__ float part[kFinWarps][32];
  const int b = blockIdx.y;
  const int n = score_off[b + 1] - score_off[b];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 32 + lane;
  const int i0 = term_off[b], i1 = term_off[b + 1];
  float sum = 0.f;
  if (t < n) {
    // terms w, w + 8, w + 16, ... added in that order; four terms' loads in
    // flight at a time
    constexpr int U = 4;
    for (int i = i0 + warp; i < i1; i += U * kFinWarps) {
      float p[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int ii = i + u * kFinWarps;
        p[u] = 0.f;
        if (ii < i1) {
          const float* st = stats + __ldg(stat_off + ii);
          const float* lg = logits + __ldg(logit_off + ii) + int64_t(t) * group;
          const uint32_t mask = __ldg(qmask + ii);
          for (int g = 0; g < group; ++g)
            if (mask & (1u << g)) p[u] += ex2(__ldcs(lg + g) - __ldg(st + g)) / __ldg(st + group + g);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) sum += p[u];
    }
  }
  part[warp][lane] = sum;
  __syncthreads();
  if (warp == 0 && t < n) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kFinWarps; ++w) s += part[w][lane];
    acc[score_off[b] + t] = s;
  }
}

constexpr int kTopkThreads = 512;

// (value, index) ordering: larger value first, then lower index.
__device__ inline bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

__global__ void __launch_bounds__(kTopkThreads)
    chunk_topk_kernel(const float* acc, const int32_t* score_off, int max_audio, int stride, int spc,
                      int top_k, int32_t* topk, float* chunk_scores, const int32_t* chunk_off) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int b = blockIdx.x;
  const int n = score_off[b + 1] - score_off[b];
  if (n > max_audio || n < 0) {  // shared memory was sized for max_audio tokens
    for (int j = threadIdx.x; j < top_k; j += blockDim.x) topk[b * top_k + j] = -1;
    return;
  }
  const int nseg = (n + stride - 1) / stride;
  double* segsum = reinterpret_cast<double*>(smem);        // [nseg + 1], becomes the prefix
  float* cs = reinterpret_cast<float*>(segsum + nseg + 1);  // [nseg] chunk scores
  __shared__ double carry;
  const float* a = acc + score_off[b];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = kTopkThreads / 32;

  // 1. per-segment sums in fp64 (fixed per-lane order, fixed shuffle tree)
  for (int s = warp; s < nseg; s += nwarps) {
    const int lo = s * stride, hi = min(n, lo + stride);
    double x = 0.0;
    int t = lo + lane;
    for (; t + 96 < hi; t += 128) {  // four loads in flight, added in the same order
      const float v0 = a[t], v1 = a[t + 32], v2 = a[t + 64], v3 = a[t + 96];
      x += double(v0);
      x += double(v1);
      x += double(v2);
      x += double(v3);
    }
    for (; t < hi; t += 32) x += double(a[t]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
    if (lane == 0) segsum[s] = x;
  }
  __syncthreads();
  // 2. exclusive prefix over segments (warp 0, 32 at a time) -> P at boundaries
  if (warp == 0) {
    if (lane == 0) carry = 0.0;
    __syncwarp();
    for (int s0 = 0; s0 <= nseg; s0 += 32) {
      const int s = s0 + lane;
      const double v = (s < nseg) ? segsum[s] : 0.0;
      double inc = v;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, inc, off);
        if (lane >= off) inc += y;
      }
      const double c = carry;
      __syncwarp();
      if (s <= nseg) segsum[s] = c + inc - v;  // exclusive prefix
      const double tot = __shfl_sync(0xffffffffu, inc, 31);
      if (lane == 0) carry = c + tot;
      __syncwarp();
    }
  }
  __syncthreads();
  // 3. chunk means in fp32: (P[end] - P[start]) / max(1, end - start)
  for (int c = tid; c < nseg; c += kTopkThreads) {
    const int e = min(c + spc, nseg);
    const int start = c * stride;
    const int end = (e == nseg) ? n : e * stride;
    const float pe = float(segsum[e]);
    const float ps = float(segsum[c]);
    const float len = float(max(1, end - start));
    const float v = __fdiv_rn(__fsub_rn(pe, ps), len);
    cs[c] = v;
    if (chunk_scores != nullptr) chunk_scores[chunk_off[b] + c] = v;
  }
  __syncthreads();
  // 4. top-k in one pass: a chunk's rank is the number of chunks that beat
  // it (larger score, then lower index: a strict total order, so ranks are
  // distinct); NaN ranks as -inf.  Chunks ranked below k write themselves.
  const int k = min(top_k, nseg);
  for (int j = k + tid; j < top_k; j += kTopkThreads) topk[b * top_k + j] = -1;
  for (int c = tid; c < nseg; c += kTopkThreads) {
    float v = cs[c];
    if (isnan(v)) v = -INFINITY;
    int rank = 0;
    for (int o = 0; o < nseg && rank < k; ++o) {
      float w = cs[o];
      if (isnan(w)) w = -INFINITY;
      rank += better(w, o, v, c) ? 1 : 0;
    }
    if (rank < k) topk[b * top_k + rank] = c;
  }
}

}  // namespace wnw

extern "C" wnw_status wnw_score_finalize(const float* logits, const float* stats, const int64_t* logit_off,
                                         const int64_t* stat_off, const uint32_t* qmask, const int32_t* term_off,
                                         int group, int batch, const int32_t* score_off, int max_audio,
                                         float* acc, void* stream) {
  using namespace wnw;
  WNW_CHECK_ARG(logits && stats && logit_off && stat_off && qmask && term_off && score_off && acc,
                "null pointer argument");
  WNW_CHECK_ARG(group >= 1 && group <= 32, "group must be in 1..32");
  WNW_CHECK_ARG(batch >= 0 && batch <= 65535, "batch must be in 0..65535");
  if (batch == 0 || max_audio <= 0) return WNW_OK;
  dim3 grid((max_audio + 31) / 32, batch);
  score_finalize_kernel<<<grid, kFinWarps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      logits, stats, logit_off, stat_off, qmask, term_off, group, score_off, acc);
  WNW_CUDA_TRY(cudaGetLastError());
  return WNW_OK;
}

namespace wnw {
// shared memory needed for a sample with `max_audio` tokens
inline size_t topk_smem(int max_audio, int stride) {
  const int nseg = (max_audio + stride - 1) / stride;
  return size_t(nseg + 1) * sizeof(double) + size_t(nseg) * sizeof(float) + 16;
}
}  // namespace wnw

extern "C" wnw_status wnw_chunk_topk(const float* acc, const int32_t* score_off, int batch, int max_audio,
                                     int stride, int segs_per_chunk, int top_k, int32_t* topk,
                                     float* chunk_scores, const int32_t* chunk_off, void* stream) {
  using namespace wnw;
  WNW_CHECK_ARG(acc && score_off && topk, "null pointer argument");
  WNW_CHECK_ARG(stride > 0 && segs_per_chunk > 0 && top_k >= 0 && max_audio >= 0, "bad chunk geometry");
  WNW_CHECK_ARG(chunk_scores == nullptr || chunk_off != nullptr, "chunk_scores needs chunk_off");
  if (batch <= 0 || top_k == 0) return WNW_OK;
  const size_t smem = topk_smem(max_audio, stride);
  WNW_CHECK_ARG(smem <= 200 * 1024, "too many segments per sample for one CTA (%d tokens / stride %d)",
                max_audio, stride);
  static size_t configured = 48 * 1024;
  if (smem > configured) {
    WNW_CUDA_TRY(cudaFuncSetAttribute(chunk_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem)));
    configured = smem;
  }
  chunk_topk_kernel<<<batch, kTopkThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      acc, score_off, max_audio, stride, segs_per_chunk, top_k, topk, chunk_scores, chunk_off);
  WNW_CUDA_TRY(cudaGetLastError());
  return WNW_OK;
}
