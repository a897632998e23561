// GQA split-K flash-decoding over per-head KV segments (sm_100a).
//
// Replaces the reference's q1_decode_attn / q1_decode_attn_score Triton
// kernels (src/common/kv/fused_attn.py:9-156) and the varlen_attn call of
// src/algorithms/wnw/code/session.py:90-106, and fuses the per-step append of
// src/common/kv/kernels.py:7-73.
//
// Design (HBM-bound, q_len = 1):
//  * every CTA owns `SPLIT` consecutive rows of one segment; its K and V rows
//    are staged into shared memory by 1-D bulk async copies (TMA engine), one
//    copy per warp chunk per tensor, each completing on its own mbarrier, so
//    the whole 64 KB tile is in flight before any math starts;
//  * each warp scores 4 (or 2) rows at a time with 8 (or 16) lanes per row;
//    lanes hold fixed 16-byte chunks of q (fp32, pre-scaled into the base-2
//    domain) and reduce dot products with xor shuffles; online softmax uses
//    the MUFU ex2 unit;
//  * CTAs of a segment are grouped into thread-block clusters; partial
//    (max, sum, o) states are merged through distributed shared memory, and
//    clusters of long segments merge through a global partial buffer with
//    the last-arriving cluster doing the final merge (a counter, no waiting);
//  * the step's new K/V row is attended from the caller's buffer and written
//    into the segment's slot (fused append);
//  * for class-A scoring segments the base-2 logits of the audio rows and the
//    merged softmax statistics are stored, and a later kernel forms the
//    per-token probabilities without re-reading K.
#pragma once
#include <cooperative_groups.h>

#include <algorithm>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace wnw {

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = 4;
constexpr int kAttnTileBytes = 64 * 1024;  // K + V rows staged per CTA
constexpr int kMaxCluster = 16;             // CTAs per cluster (16 needs the non-portable opt-in)
constexpr float kLog2e = 1.4426950408889634f;

template <typename T, int D, int G>
struct AttnCfg {
  static constexpr int ESZ = sizeof(T);
  static constexpr int ROW_BYTES = D * ESZ;
  static constexpr int CPR = ROW_BYTES / 16;                 // 16-byte chunks per row
  static constexpr int LPR_WANT = (G <= 4) ? 8 : 16;
  static constexpr int LPR = (LPR_WANT > CPR) ? CPR : LPR_WANT;  // lanes per row
  static constexpr int CPL = CPR / LPR;                      // chunks per lane
  static constexpr int EPC = 16 / ESZ;                       // elements per chunk
  static constexpr int EPL = CPL * EPC;                      // elements per lane
  static constexpr int RPW = 32 / LPR;                       // rows per warp pass
  static constexpr int U = 2;                                // rows per lane group per pass
  static constexpr int SPLIT = kAttnTileBytes / (2 * ROW_BYTES);
  static constexpr int WROWS = SPLIT / kAttnWarps;
  static_assert(CPR % LPR == 0, "lanes must tile a row");
  static_assert(WROWS % (RPW * U) == 0, "warp chunk must tile into passes");
  // merge scratch (reuses the tile region): wm, wl [warps][G], wo [warps][G][D],
  // then the CTA partial Po [G][D], Pm, Pl [G]
  static constexpr int MERGE_FLOATS = 2 * kAttnWarps * G + kAttnWarps * G * D + 2 * G + G * D;
  static_assert(MERGE_FLOATS * 4 <= kAttnTileBytes, "merge scratch fits the tile");
};

struct AttnParams {
  const void* q;
  const void* new_k;
  const void* new_v;
  void* k_store;
  void* v_store;
  const int64_t* seg_base;
  const int32_t* seg_len;
  const int32_t* seg_cap;
  const int32_t* work;
  void* out;
  float scale_log2;
  int num_kv_heads;
  int num_segs;
  const int32_t* score_slot;
  const int32_t* audio_start;
  const int32_t* audio_end;
  float* logits;
  const int64_t* logits_off;
  float* stats;
  float* partials;
  int32_t* counters;
  int32_t* err;
};

// A global partial is {o[G*D], max[G], sum[G]} (stride G * (D + 2) floats);
// its o row is read / written as float4 when that stride keeps 16-byte
// alignment (G even), else element-wise.
template <int D, int G>
struct PartIO {
  static constexpr int kStride = G * (D + 2);
  static constexpr bool kVec = (kStride % 4) == 0;
  __device__ static float4 ld(const float* p) {
    if constexpr (kVec) {
      return __ldcg(reinterpret_cast<const float4*>(p));
    } else {
      return make_float4(__ldcg(p), __ldcg(p + 1), __ldcg(p + 2), __ldcg(p + 3));
    }
  }
  __device__ static void st(float* p, float4 v) {
    if constexpr (kVec) {
      *reinterpret_cast<float4*>(p) = v;
    } else {
      p[0] = v.x;
      p[1] = v.y;
      p[2] = v.z;
      p[3] = v.w;
    }
  }
};

// Output (and class-A stats) of the 4 merged elements [i, i + 4) of one head.
template <typename T, int D, int G>
__device__ __forceinline__ void attn_store4(const AttnParams& p, int seg, int i, float mx, float ls, float4 acc) {
  T* outp = reinterpret_cast<T*>(p.out) + int64_t(seg) * G * D + i;
  const bool nz = ls > 0.f;
  outp[0] = DT<T>::from_f(nz ? acc.x / ls : 0.f);
  outp[1] = DT<T>::from_f(nz ? acc.y / ls : 0.f);
  outp[2] = DT<T>::from_f(nz ? acc.z / ls : 0.f);
  outp[3] = DT<T>::from_f(nz ? acc.w / ls : 0.f);
  if (i % D == 0 && p.stats != nullptr) {
    const int g = i / D;
    p.stats[int64_t(seg) * 2 * G + g] = mx;
    p.stats[int64_t(seg) * 2 * G + G + g] = ls;
  }
}

__device__ __forceinline__ void fma4(float4& acc, float4 v, float f) {
  acc.x += v.x * f;
  acc.y += v.y * f;
  acc.z += v.z * f;
  acc.w += v.w * f;
}
__device__ __forceinline__ void scale4(float4& acc, float f) {
  acc.x *= f;
  acc.y *= f;
  acc.z *= f;
  acc.w *= f;
}

// Merge the 4 warp partials (wm, wl, wo at the start of `smem`) of elements
// [i, i + 4) (one head g) into (max, sum, o).
template <int D, int G>
__device__ __forceinline__ void merge_warps4(const float* smem, int i, float& mx, float& ls, float4& acc) {
  const float* wm = smem;
  const float* wl = wm + kAttnWarps * G;
  const float* wo = wl + kAttnWarps * G;
  const int g = i / D, d = i % D;
  mx = -INFINITY;
#pragma unroll
  for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, wm[w * G + g]);
  const float bse = (mx == -INFINITY) ? 0.f : mx;
  ls = 0.f;
  acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int w = 0; w < kAttnWarps; ++w) {
    const float f = ex2(wm[w * G + g] - bse);
    fma4(acc, *reinterpret_cast<const float4*>(wo + (w * G + g) * D + d), f);
    ls += wl[w * G + g] * f;
  }
}

// Final merge of a segment's `ncl` global partials (part0 = the first),
// written as the output; this CTA's threads take 4 elements at a time.
template <typename T, int D, int G>
__device__ __forceinline__ void attn_merge_partials(const AttnParams& p, const float* part0, int seg, int ncl) {
  using IO = PartIO<D, G>;
  constexpr int kBatch = 16;  // partials loaded per round trip
  for (int i = 4 * static_cast<int>(threadIdx.x); i < G * D; i += 4 * kAttnThreads) {
    const int g = i / D;
    float mx = -INFINITY, ls = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c0 = 0; c0 < ncl; c0 += kBatch) {
      float bm[kBatch], bl[kBatch];
      float4 bo[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int c = c0 + u;
        if (c < ncl) {
          const float* pc = part0 + int64_t(c) * IO::kStride;
          bm[u] = __ldcg(pc + G * D + g);
          bl[u] = __ldcg(pc + G * D + G + g);
          bo[u] = IO::ld(pc + i);
        } else {
          bm[u] = -INFINITY;
          bl[u] = 0.f;
          bo[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      float mn = mx;
#pragma unroll
      for (int u = 0; u < kBatch; ++u) mn = fmaxf(mn, bm[u]);
      const float bse = (mn == -INFINITY) ? 0.f : mn;
      const float a = ex2(mx - bse);
      scale4(acc, a);
      ls *= a;
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const float f = ex2(bm[u] - bse);
        fma4(acc, bo[u], f);
        ls += bl[u] * f;
      }
      mx = mn;
    }
    attn_store4<T, D, G>(p, seg, i, mx, ls, acc);
  }
}

// Write this CTA's (or cluster's) merged partial to global memory, arrive at
// the segment's counter and, if last, merge all of the segment's partials.
// The caller has stored its elements of `part` from this CTA's threads.
template <typename T, int D, int G>
__device__ __forceinline__ void attn_arrive_and_merge(const AttnParams& p, int seg, int j, int cid, int ncl) {
  __shared__ int s_last;
  __syncthreads();  // the CTA's partial is written (CTA scope) ...
  if (threadIdx.x == 0) {
    fence_acq_rel_gpu();  // ... and released at gpu scope (cumulative) before the arrival
    const int old = atomicAdd(p.counters + seg, 1);
    const int last = (old == ncl - 1) ? 1 : 0;
    if (last) {
      p.counters[seg] = 0;  // every partial of this launch has arrived
      fence_acq_rel_gpu();  // acquire the other partials
    }
    s_last = last;
  }
  __syncthreads();
  if (s_last) attn_merge_partials<T, D, G>(p, p.partials + int64_t(cid - j) * PartIO<D, G>::kStride, seg, ncl);
}

// Merge the 4 warp partials (wm, wl, wo at the start of `smem`) into the
// output, or -- segments split over several clusters -- into a global
// partial merged by the last-arriving cluster.  Clusters of several CTAs
// first combine their CTAs through distributed shared memory: every CTA
// parks its merged partial in its own shared memory, rank 0 gathers them
// and carries on alone while the other ranks leave.
template <typename T, int D, int G>
__device__ __forceinline__ void attn_finish(const AttnParams& p, uint8_t* smem, int seg, int j, int cid, int ncl) {
  using IO = PartIO<D, G>;
  cg::cluster_group cluster = cg::this_cluster();
  const int cs = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int tid = threadIdx.x;
  const float* ws = reinterpret_cast<const float*>(smem);
  float* part = p.partials + int64_t(cid) * IO::kStride;
  if (cs == 1) {
    for (int i = 4 * tid; i < G * D; i += 4 * kAttnThreads) {
      float mx, ls;
      float4 acc;
      merge_warps4<D, G>(ws, i, mx, ls, acc);
      if (ncl == 1) {
        attn_store4<T, D, G>(p, seg, i, mx, ls, acc);
      } else {
        IO::st(part + i, acc);
        if (i % D == 0) {
          part[G * D + i / D] = mx;
          part[G * D + G + i / D] = ls;
        }
      }
    }
    if (ncl > 1) attn_arrive_and_merge<T, D, G>(p, seg, j, cid, ncl);
    return;
  }
  // CTA partial behind the warp partials: Po [G*D] (16-byte aligned), Pm, Pl [G]
  float* Po = reinterpret_cast<float*>(smem) + 2 * kAttnWarps * G + kAttnWarps * G * D;
  float* Pm = Po + G * D;
  float* Pl = Pm + G;
  for (int i = 4 * tid; i < G * D; i += 4 * kAttnThreads) {
    float mx, ls;
    float4 acc;
    merge_warps4<D, G>(ws, i, mx, ls, acc);
    *reinterpret_cast<float4*>(Po + i) = acc;
    if (i % D == 0) {
      Pm[i / D] = mx;
      Pl[i / D] = ls;
    }
  }
  cluster_arrive();  // CTA partials visible to the cluster
  cluster_wait();
  if (rank != 0) {
    cluster_arrive();  // keep this CTA's shared memory until rank 0 has read it
    cluster_wait();
    return;
  }
  for (int i = 4 * tid; i < G * D; i += 4 * kAttnThreads) {
    const int g = i / D;
    // pull every rank's (max, sum, o) first so the remote loads overlap
    float pm[kMaxCluster], pl[kMaxCluster];
    float4 po[kMaxCluster];
#pragma unroll
    for (int r = 0; r < kMaxCluster; ++r) {
      if (r < cs) {
        pm[r] = *cluster.map_shared_rank(Pm + g, r);
        pl[r] = *cluster.map_shared_rank(Pl + g, r);
        po[r] = *reinterpret_cast<const float4*>(cluster.map_shared_rank(Po + i, r));
      } else {
        pm[r] = -INFINITY;
        pl[r] = 0.f;
        po[r] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    float mx = -INFINITY;
#pragma unroll
    for (int r = 0; r < kMaxCluster; ++r) mx = fmaxf(mx, pm[r]);
    const float bse = (mx == -INFINITY) ? 0.f : mx;
    float ls = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kMaxCluster; ++r) {
      const float f = ex2(pm[r] - bse);
      fma4(acc, po[r], f);
      ls += pl[r] * f;
    }
    if (ncl == 1) {
      attn_store4<T, D, G>(p, seg, i, mx, ls, acc);
    } else {
      IO::st(part + i, acc);
      if (i % D == 0) {
        part[G * D + g] = mx;
        part[G * D + G + g] = ls;
      }
    }
  }
  cluster_arrive();  // done with the other ranks' shared memory
  if (ncl > 1) attn_arrive_and_merge<T, D, G>(p, seg, j, cid, ncl);
  cluster_wait();
}

template <typename T, int D, int G>
__global__ void __launch_bounds__(kAttnThreads)
    decode_attn_kernel(const AttnParams p) {
  using C = AttnCfg<T, D, G>;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[kAttnWarps];

  cg::cluster_group cluster = cg::this_cluster();
  const int cs = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int cid = blockIdx.x / cs;
  const int seg = p.work[2 * cid];
  const int j = p.work[2 * cid + 1];
  const int len = p.seg_len[seg];
  const bool append = p.new_k != nullptr;
  const int total = len + (append ? 1 : 0);
  const int nsplit = (total + C::SPLIT - 1) / C::SPLIT;
  const int ncl = max(1, (nsplit + cs - 1) / cs);
  if (j >= ncl) return;  // the whole cluster is idle at this length (uniform)

  const int split = j * cs + rank;
  const int row0 = split * C::SPLIT;
  const int nvalid = max(0, min(C::SPLIT, total - row0));
  const int64_t base = p.seg_base[seg];
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int grp = lane / C::LPR;
  const int pos = lane % C::LPR;

  T* Ks = reinterpret_cast<T*>(smem);
  T* Vs = reinterpret_cast<T*>(smem + C::SPLIT * C::ROW_BYTES);
  const T* kst = reinterpret_cast<const T*>(p.k_store);
  const T* vst = reinterpret_cast<const T*>(p.v_store);

  if (tid == 0) {
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) mbar_init(&bars[w], 1);
    fence_mbar_init();
  }
  __syncthreads();

  // ---- producer: stage this CTA's rows (store rows + the new token row)
  const int new_local = append ? (len - row0) : -1;
  if (tid == 0 && nvalid > 0) {
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const int lo = w * C::WROWS;
      const int hi = min(lo + C::WROWS, nvalid);
      if (hi <= lo) continue;
      const int s_hi = min(hi, len - row0);
      const bool has_new = append && new_local >= lo && new_local < hi;
      uint32_t bytes = 0;
      if (s_hi > lo) bytes += 2u * (s_hi - lo) * C::ROW_BYTES;
      if (has_new) bytes += 2u * C::ROW_BYTES;
      mbar_arrive_expect_tx(&bars[w], bytes);
      if (s_hi > lo) {
        const int64_t g0 = (base + row0 + lo) * D;
        bulk_g2s(Ks + lo * D, kst + g0, (s_hi - lo) * C::ROW_BYTES, &bars[w]);
        bulk_g2s(Vs + lo * D, vst + g0, (s_hi - lo) * C::ROW_BYTES, &bars[w]);
      }
      if (has_new) {
        bulk_g2s(Ks + new_local * D, reinterpret_cast<const T*>(p.new_k) + int64_t(seg) * D,
                 C::ROW_BYTES, &bars[w]);
        bulk_g2s(Vs + new_local * D, reinterpret_cast<const T*>(p.new_v) + int64_t(seg) * D,
                 C::ROW_BYTES, &bars[w]);
      }
    }
  }

  // ---- per-lane q (fp32, base-2 scaled) for this lane's fixed chunks
  float qr[G][C::EPL];
  {
    const T* qs = reinterpret_cast<const T*>(p.q) + int64_t(seg) * G * D;
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
      for (int k = 0; k < C::CPL; ++k) {
        const int c = pos + C::LPR * k;
        const uint4 u = *reinterpret_cast<const uint4*>(qs + g * D + c * C::EPC);
        float f[C::EPC];
        unpack16<T>(u, f);
#pragma unroll
        for (int i = 0; i < C::EPC; ++i) qr[g][k * C::EPC + i] = f[i] * p.scale_log2;
      }
    }
  }

  // scoring geometry
  int slot = -1, a0 = 0, a1 = 0;
  float* lg = nullptr;
  if (p.score_slot != nullptr) {
    slot = p.score_slot[seg];
    if (slot >= 0) {
      const int b = seg / p.num_kv_heads;
      a0 = p.audio_start[b];
      a1 = p.audio_end[b];
      lg = p.logits + p.logits_off[slot];
    }
  }

  float m[G], l[G], o[G][C::EPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.f;
#pragma unroll
    for (int e = 0; e < C::EPL; ++e) o[g][e] = 0.f;
  }

  // ---- consumer: this warp's chunk of rows
  const int lo = warp * C::WROWS;
  const int hi = min(lo + C::WROWS, nvalid);
  if (hi > lo) {
    mbar_wait(&bars[warp], 0, p.err);
    // fused append: copy the new token row from the tile into the slot
    if (append && new_local >= lo && new_local < hi) {
      const bool fits = (p.seg_cap == nullptr) || (len + 1 <= p.seg_cap[seg]);
      if (fits) {
        uint4* dk = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.k_store) + (base + len) * D);
        uint4* dv = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.v_store) + (base + len) * D);
        const uint4* sk = reinterpret_cast<const uint4*>(Ks + new_local * D);
        const uint4* sv = reinterpret_cast<const uint4*>(Vs + new_local * D);
        for (int c = lane; c < C::CPR; c += 32) {
          dk[c] = sk[c];
          dv[c] = sv[c];
        }
      } else if (lane == 0) {
        atomicOr(p.err, WNW_DEVERR_CAPACITY);
      }
    }
    for (int r = lo; r < hi; r += C::RPW * C::U) {
      float s[C::U][G];
      bool valid[C::U];
#pragma unroll
      for (int u = 0; u < C::U; ++u) {
        const int row = r + u * C::RPW + grp;
        valid[u] = row < hi;
#pragma unroll
        for (int g = 0; g < G; ++g) s[u][g] = 0.f;
        if (valid[u]) {
          const T* kr = Ks + row * D;
#pragma unroll
          for (int k = 0; k < C::CPL; ++k) {
            const int c = pos + C::LPR * k;
            const uint4 uu = *reinterpret_cast<const uint4*>(kr + c * C::EPC);
            float f[C::EPC];
            unpack16<T>(uu, f);
#pragma unroll
            for (int g = 0; g < G; ++g) {
#pragma unroll
              for (int i = 0; i < C::EPC; ++i) s[u][g] = fmaf(qr[g][k * C::EPC + i], f[i], s[u][g]);
            }
          }
        }
      }
#pragma unroll
      for (int off = C::LPR / 2; off > 0; off >>= 1) {
#pragma unroll
        for (int u = 0; u < C::U; ++u) {
#pragma unroll
          for (int g = 0; g < G; ++g) s[u][g] += __shfl_xor_sync(0xffffffffu, s[u][g], off);
        }
      }
#pragma unroll
      for (int u = 0; u < C::U; ++u) {
        if (!valid[u]) {
#pragma unroll
          for (int g = 0; g < G; ++g) s[u][g] = -INFINITY;
        } else if (lg != nullptr) {
          const int srow = row0 + r + u * C::RPW + grp;
          if (srow >= a0 && srow < a1 && pos < G) {
            float v = s[u][0];
#pragma unroll
            for (int g = 1; g < G; ++g)
              if (pos == g) v = s[u][g];
            lg[int64_t(srow - a0) * G + pos] = v;
          }
        }
      }
      float pu[C::U][G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float mx = m[g];
#pragma unroll
        for (int u = 0; u < C::U; ++u) mx = fmaxf(mx, s[u][g]);
        const float bse = (mx == -INFINITY) ? 0.f : mx;
        const float alpha = ex2(m[g] - bse);
        float lsum = l[g] * alpha;
#pragma unroll
        for (int u = 0; u < C::U; ++u) {
          pu[u][g] = ex2(s[u][g] - bse);
          lsum += pu[u][g];
        }
        l[g] = lsum;
        m[g] = mx;
#pragma unroll
        for (int e = 0; e < C::EPL; ++e) o[g][e] *= alpha;
      }
#pragma unroll
      for (int u = 0; u < C::U; ++u) {
        if (!valid[u]) continue;
        const T* vr = Vs + (r + u * C::RPW + grp) * D;
#pragma unroll
        for (int k = 0; k < C::CPL; ++k) {
          const int c = pos + C::LPR * k;
          const uint4 uu = *reinterpret_cast<const uint4*>(vr + c * C::EPC);
          float f[C::EPC];
          unpack16<T>(uu, f);
#pragma unroll
          for (int g = 0; g < G; ++g) {
#pragma unroll
            for (int i = 0; i < C::EPC; ++i) o[g][k * C::EPC + i] = fmaf(pu[u][g], f[i], o[g][k * C::EPC + i]);
          }
        }
      }
    }
  }

  // ---- merge the lane groups of this warp (same chunk positions)
#pragma unroll
  for (int off = C::LPR; off < 32; off <<= 1) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float mo = __shfl_xor_sync(0xffffffffu, m[g], off);
      const float lo2 = __shfl_xor_sync(0xffffffffu, l[g], off);
      const float mx = fmaxf(m[g], mo);
      const float bse = (mx == -INFINITY) ? 0.f : mx;
      const float a = ex2(m[g] - bse), b = ex2(mo - bse);
      l[g] = l[g] * a + lo2 * b;
      m[g] = mx;
#pragma unroll
      for (int e = 0; e < C::EPL; ++e) {
        const float oo = __shfl_xor_sync(0xffffffffu, o[g][e], off);
        o[g][e] = o[g][e] * a + oo * b;
      }
    }
  }

  // ---- merge the warps of this CTA (the tile region is reused)
  __syncthreads();
  float* wm = reinterpret_cast<float*>(smem);
  float* wl = wm + kAttnWarps * G;
  float* wo = wl + kAttnWarps * G;
  if (lane < C::LPR) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      if (lane == 0) {
        wm[warp * G + g] = m[g];
        wl[warp * G + g] = l[g];
      }
#pragma unroll
      for (int k = 0; k < C::CPL; ++k) {
#pragma unroll
        for (int i = 0; i < C::EPC; ++i) {
          const int d = (pos + C::LPR * k) * C::EPC + i;
          wo[(warp * G + g) * D + d] = o[g][k * C::EPC + i];
        }
      }
    }
  }
  __syncthreads();
  attn_finish<T, D, G>(p, smem, seg, j, cid, ncl);
}

inline AttnParams make_params(const wnw_decode_attn_args* a) {
  AttnParams p;
  p.q = a->q;
  p.new_k = a->new_k;
  p.new_v = a->new_v;
  p.k_store = a->k_store;
  p.v_store = a->v_store;
  p.seg_base = a->seg_base;
  p.seg_len = a->seg_len;
  p.seg_cap = a->seg_cap;
  p.work = a->work;
  p.out = a->out;
  p.scale_log2 = a->scale * kLog2e;
  p.num_kv_heads = a->num_kv_heads;
  p.num_segs = a->num_segs;
  p.score_slot = a->score_slot;
  p.audio_start = a->audio_start;
  p.audio_end = a->audio_end;
  p.logits = a->logits;
  p.logits_off = a->logits_off;
  p.stats = a->stats;
  p.partials = a->partials;
  p.counters = a->counters;
  p.err = a->err;
  return p;
}

template <typename T, int D, int G>
wnw_status launch_attn(const wnw_decode_attn_args* a, cudaStream_t stream) {
  using C = AttnCfg<T, D, G>;
  static bool configured = false;  // attribute setting is idempotent; a race only repeats it
  auto kern = decode_attn_kernel<T, D, G>;
  if (!configured) {
    WNW_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnTileBytes));
    WNW_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    configured = true;
  }
  WNW_CHECK_ARG(a->split_rows == C::SPLIT, "split_rows %d does not match kernel split %d", a->split_rows,
                C::SPLIT);
  AttnParams p = make_params(a);

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a->n_clusters * a->cluster_size, 1, 1);
  cfg.blockDim = dim3(kAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = kAttnTileBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a->cluster_size;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  WNW_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p));
  return WNW_OK;
}


template <typename T>
wnw_status dispatch_dtype(const wnw_decode_attn_args* a, cudaStream_t s);

// co-resident clusters of `cs` CTAs of the tensor-core kernel (decode_attn_bf16.cu)
wnw_status attn_mma_active_clusters_any(int head_dim, int cs, int* n);

}  // namespace wnw
