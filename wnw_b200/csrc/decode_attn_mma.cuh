// Tensor-core decode attention for 16-bit K/V (bf16 / fp16, head_dim 64 or
// 128), launched from a work plan (wnw_attn_plan).
//
// Work decomposition: every CTA attends one row range of one segment.  A
// segment's CTAs sit in consecutive ranks of one thread-block cluster (up to
// 16 CTAs), so their partial softmax states merge through distributed shared
// memory -- no global-memory round trip; only a segment too long for one
// cluster's CTAs spans several clusters, whose cluster partials the last
// cluster to arrive at the segment's counter merges in order (one atomic,
// then the partials' loads).  The plan gives each CTA about the same rows
// (capped so a long segment fits one cluster) and packs short segments into
// shared clusters.
//
// A CTA streams its rows as 128-row tiles through three shared-memory stages
// (2-D TMA, 128-byte swizzle).  Its eight warps own 16 rows of every tile
// each (two warps per scheduler, so one warp's latency hides behind the
// other's): a warp waits for its rows, runs the two products on the tensor
// cores with fp32 accumulation,
//   S^T[16 x g] = K[16 x D] . q^T[D x g]       (mma m16n8k16, A = K via ldmatrix)
//   O^T[D x g] += V^T[D x 16] . P^T[16 x g]    (A = V^T via ldmatrix.trans,
//                                               B = P^T via movmatrix.trans)
// with the GQA group (<= 8 heads) as the n = 8 dimension, keeps an online
// softmax (base 2, MUFU ex2; the running sum stays per lane until the end)
// and refills its rows of the stage with a later tile as soon as it is done.
//
// Programmatic dependent launch: the prologue overlaps the preceding kernel;
// with WNW_ATTN_ROWS_READY the lengths are read and the first stages' loads
// issued before the dependency wait as well.
#pragma once

#include "decode_attn.cuh"
#include "mma.cuh"
#include "tma.cuh"

namespace wnw {

constexpr int kTcThreads = 256;    // 8 warps
constexpr int kTcWarps = 8;
constexpr int kTcWarpRows = 16;    // one m16 block per warp and tile
constexpr int kTcTileRows = 128;   // 8 warps x 16 rows
constexpr int kTcStages = 3;
constexpr int kTcMaxCluster = 16;

#ifdef WNW_ATTN_TRACE
// Phase timestamps of every CTA (the trace build only: python -m
// wnw_b200.build --trace).  Per record: meta (block | smid << 16 | cluster
// rank << 24 | rows << 32), the plan pointer (which layer), and %globaltimer
// at kernel entry, after the dependency wait, after the last tile, after the
// CTA merge, after the first cluster barrier and at exit.
constexpr int kTraceCap = 16384;
static __device__ unsigned long long g_attn_trace[kTraceCap][8];
static __device__ int g_attn_trace_n;
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#define WNW_TR(i)                   \
  do {                              \
    if (tid == 0) tr_[i] = gtimer(); \
  } while (0)
#else
#define WNW_TR(i) \
  do {            \
  } while (0)
#endif

// byte offset of (row, 16-byte chunk) inside a 128-byte-swizzled tile whose
// base is 1024-byte aligned
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return uint32_t(row) * 128u + (uint32_t(chunk ^ (row & 7)) << 4);
}


// Device view of a wnw_attn_plan blob.
//   cta[c]   = {segment (-1: an idle rank), row_begin, row_end, meta}
//   meta     = leader rank (bits 0-4) | ranks of the segment in this cluster
//              (bits 5-9) | writes a cluster partial (bit 10) | partial slot
//              (bits 11-31)
//   part_r0  = first row of each cluster partial's range
//   comb[e]  = {segment, first partial, partials, 0}
struct AttnPlanView {
  const int4* cta;
  const int32_t* part_r0;
  const int4* comb;
  int parts;
  int combine;  // entries of comb
  int ready;    // WNW_ATTN_ROWS_READY given
};

// rows of a segment attended at this launch: stored rows + the step's token
__device__ __forceinline__ int seg_total(const AttnParams& p, int seg) {
  return p.seg_len[seg] + (p.new_k != nullptr ? 1 : 0);
}

template <typename T, int D, int G>
__global__ void __launch_bounds__(kTcThreads, 1)
    decode_attn_mma_kernel(const AttnParams p, const AttnPlanView pv, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV) {
  static_assert(D == 64 || D == 128, "tensor-core path covers head_dim 64 and 128");
  static_assert(G >= 1 && G <= 8, "GQA group is the mma n=8 dimension");
  constexpr int NH = D / 64;                // 128-byte halves per row
  constexpr int HALF = kTcTileRows * 128;   // bytes of one half tile
  constexpr int STAGE = 2 * NH * HALF;      // K + V of one 128-row tile
  constexpr int NS = D / 16;                // k-steps over D / m-tiles of O^T
  constexpr int NW = kTcWarps;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bars[kTcStages][NW];

  cg::cluster_group cluster = cg::this_cluster();
  const int cs = static_cast<int>(cluster.num_blocks());
  const int crank = static_cast<int>(cluster.block_rank());
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
#ifdef WNW_ATTN_TRACE
  unsigned long long tr_[6] = {0, 0, 0, 0, 0, 0};
#endif
  WNW_TR(0);

  // ---- this CTA's item (plan constants: read before the dependency wait)
  const int4 it = __ldg(pv.cta + blockIdx.x);
  const int leader = it.w & 31;
  const int nranks = (it.w >> 5) & 31;
  const bool to_part = ((it.w >> 10) & 1) != 0;
  const int part = static_cast<int>(static_cast<uint32_t>(it.w) >> 11);
  bool active = it.x >= 0;
  if (active && (it.x >= p.num_segs || it.y < 0 || it.z < it.y || nranks < 1 || leader + nranks > cs ||
                 crank < leader || crank >= leader + nranks || (to_part && part >= pv.parts))) {
    if (tid == 0) atomicOr(p.err, WNW_DEVERR_BAD_INDEX);  // not a wnw_attn_plan: attend nothing
    active = false;
  }
  const int seg = active ? it.x : 0;
  const int64_t base = active ? __ldg(p.seg_base + seg) : 0;
  if (tid == 0) {
#pragma unroll
    for (int st = 0; st < kTcStages; ++st)
#pragma unroll
      for (int w = 0; w < NW; ++w) mbar_init(&bars[st][w], 1);
    fence_mbar_init();
  }
  __syncthreads();

  // class-A scoring geometry: layout constants, read before the dependency wait
  int a0 = 0, a1 = 0;
  float* lg = nullptr;
  if (active && p.score_slot != nullptr) {
    const int slot = __ldg(p.score_slot + seg);
    if (slot >= 0) {
      const int b = seg / p.num_kv_heads;
      a0 = __ldg(p.audio_start + b);
      a1 = __ldg(p.audio_end + b);
      lg = p.logits + __ldg(p.logits_off + slot);
    }
  }
  // q comes from the preceding kernel: bring its lines into L2 now (L2 is the
  // point of coherence, so the loads after the wait see the final values)
  if (active && tid == 32) prefetch_l2(reinterpret_cast<const T*>(p.q) + int64_t(seg) * G * D, G * D * sizeof(T));

  int total = 0, rows = 0, ntiles = 0;
  auto schedule = [&]() {
    if (!active) return;
    total = seg_total(p, seg);
    rows = max(0, min(it.z, total) - it.y);
    ntiles = (rows + kTcTileRows - 1) / kTcTileRows;
  };
  // this warp's 16 rows of tile t -> stage t % kTcStages (lane 0); a warp
  // with no rows in the tile still completes the barrier's phase
  auto issue = [&](int t) {
    const int st = t % kTcStages;
    uint8_t* sK = smem + st * STAGE;
    uint8_t* sV = sK + NH * HALF;
    const int trow = t * kTcTileRows;
    const int lo = warp * kTcWarpRows;
    if (lo >= rows - trow) {
      mbar_arrive(&bars[st][warp]);
      return;
    }
    mbar_arrive_expect_tx(&bars[st][warp], 2u * NH * kTcWarpRows * 128u);
    const int y = static_cast<int>(base + it.y + trow + lo);
#pragma unroll
    for (int h = 0; h < NH; ++h) {
      tma_load_2d(sK + h * HALF + lo * 128, &tmK, h * 64, y, &bars[st][warp]);
      tma_load_2d(sV + h * HALF + lo * 128, &tmV, h * 64, y, &bars[st][warp]);
    }
  };
  // A leader CTA of a segment spanning clusters looks up, in the prologue,
  // the combine entry of its partial (cfirst, cn; cok: the entry checks out)
  // and how many of the segment's partials cover rows at this launch (nact),
  // so that the tail after its arrival is one atomic and the partials' loads.
  // Warp 0 holds the values; everything it reads is a plan constant but the
  // row count.
  const bool spans = active && to_part && crank == leader;
  int cfirst = 0, cn = 0, nact = 1;
  bool cok = false;
  auto find_entry = [&]() {
    if (!spans || warp != 0) return;
    int4 e = make_int4(-1, 0, 0, 0);
    if (lane == 0 && pv.combine > 0) {  // entries are ordered by first partial
      int lo = 0, hi = pv.combine;
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (__ldg(&pv.comb[mid].y) <= part) lo = mid; else hi = mid;
      }
      e = __ldg(pv.comb + lo);
    }
    e.x = __shfl_sync(0xffffffffu, e.x, 0);
    e.y = __shfl_sync(0xffffffffu, e.y, 0);
    e.z = __shfl_sync(0xffffffffu, e.z, 0);
    cok = e.x == seg && e.y <= part && part < e.y + e.z && e.y + e.z <= pv.parts;
    cfirst = e.y;
    cn = e.z;
  };
  auto count_active = [&]() {  // partials whose range starts below the row count (the first always counts)
    if (!cok) return;          // warp-uniform
    int n = 0;
    for (int c = 1 + lane; c < cn; c += 32) n += __ldg(pv.part_r0 + cfirst + c) < total ? 1 : 0;
    nact = 1 + __reduce_add_sync(0xffffffffu, n);
  };
  if (pv.ready) {  // lengths and rows are final: start streaming before the wait
    schedule();
    if (lane == 0)
      for (int t = 0; t < min(ntiles, kTcStages); ++t) issue(t);
    find_entry();
    count_active();
    pdl_wait();  // q, the new rows and the outputs may belong to the preceding kernel
    WNW_TR(1);
  } else {
    find_entry();
    // L2 prefetch of this CTA's first rows by capacity (layout constants
    // only; L2 is the point of coherence, so rows the preceding kernel still
    // writes are read correctly after the wait)
    if (active && tid < 2 * kTcStages) {
      const int r0 = it.y + (tid >> 1) * kTcTileRows;
      const int r1 = min(r0 + kTcTileRows, it.z);
      if (r1 > r0) {
        const T* src = reinterpret_cast<const T*>((tid & 1) ? p.v_store : p.k_store) + (base + r0) * D;
        prefetch_l2(src, uint32_t(r1 - r0) * D * sizeof(T));
      }
    }
    pdl_wait();  // seg_len, K/V rows and q may come from the preceding kernel
    WNW_TR(1);
    schedule();
    if (lane == 0)
      for (int t = 0; t < min(ntiles, kTcStages); ++t) issue(t);
    count_active();
  }
  pdl_launch_dependents();  // the next kernel may start its own prologue now

  const int gid = lane >> 2;
  const int tig = lane & 3;
  const int jm = lane >> 3;  // which 8x8 matrix this lane addresses in ldmatrix
  const bool append = p.new_k != nullptr;
  const int len = total - (append ? 1 : 0);

  // q as the mma B operand: b[k = d][n = g], zero for padded heads
  uint32_t qb[NS][2];
  {
    const T* qs = reinterpret_cast<const T*>(p.q) + int64_t(seg) * G * D;
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      if (active && gid < G) {
        qb[s][0] = *reinterpret_cast<const uint32_t*>(qs + gid * D + 16 * s + 2 * tig);
        qb[s][1] = *reinterpret_cast<const uint32_t*>(qs + gid * D + 16 * s + 8 + 2 * tig);
      } else {
        qb[s][0] = qb[s][1] = 0u;
      }
    }
  }
  // running softmax of this warp: per lane heads g0 = 2*tig, g1 = 2*tig+1;
  // the maxima are warp-uniform, the sums stay per lane until the end
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float o[NS][4];
#pragma unroll
  for (int u = 0; u < NS; ++u) o[u][0] = o[u][1] = o[u][2] = o[u][3] = 0.f;

  for (int t = 0; t < ntiles; ++t) {
    const int st = t % kTcStages;
    uint8_t* sK = smem + st * STAGE;
    uint8_t* sV = sK + NH * HALF;
    const int trow0 = it.y + t * kTcTileRows;  // segment row of the tile's first row
    const int tv = min(kTcTileRows, rows - t * kTcTileRows);
    const int lo = warp * kTcWarpRows;
    const int hi = min(lo + kTcWarpRows, tv);
    if (hi > lo) {
      mbar_wait(&bars[st][warp], (t / kTcStages) & 1, p.err);
      const int new_local = append ? (len - trow0) : -1;
      if (append && new_local >= lo && new_local < hi) {
        // the step's token: into the tile (swizzled) and into its slot row
        const uint4* nk = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.new_k) + int64_t(seg) * D);
        const uint4* nv = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.new_v) + int64_t(seg) * D);
        const bool fits = (p.seg_cap == nullptr) || (len + 1 <= p.seg_cap[seg]);
        if (lane < NH * 8) {
          const uint4 vk = nk[lane], vv = nv[lane];
          const int h = lane >> 3, c = lane & 7;
          *reinterpret_cast<uint4*>(sK + h * HALF + swz(new_local, c)) = vk;
          *reinterpret_cast<uint4*>(sV + h * HALF + swz(new_local, c)) = vv;
          if (fits) {
            reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.k_store) + (base + len) * D)[lane] = vk;
            reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.v_store) + (base + len) * D)[lane] = vv;
          }
        }
        if (!fits && lane == 0) atomicOr(p.err, WNW_DEVERR_CAPACITY);
        __syncwarp();
      }
      if (hi - lo < kTcWarpRows) {
        // rows past the range's end are masked out of the softmax, but their
        // V bytes still enter the mma: zero them so stale or non-finite
        // memory (slack rows, a neighbouring slot) cannot reach the output
        const int n0 = (lo + kTcWarpRows - hi) * NH * 8;
        for (int idx = lane; idx < n0; idx += 32) {
          const int r = hi + idx / (NH * 8);
          const int rem = idx % (NH * 8);
          *reinterpret_cast<uint4*>(sV + (rem >> 3) * HALF + swz(r, rem & 7)) = make_uint4(0u, 0u, 0u, 0u);
        }
        __syncwarp();
      }
      const uint32_t kbase = smem_u32(sK);
      const uint32_t vbase = smem_u32(sV);
      // S^T of the warp's 16 rows, as two independent accumulation chains
      float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
      {
        const int row = lo + (lane & 7) + 8 * (jm & 1);
#pragma unroll
        for (int s = 0; s < NS; ++s) {
          const int h = (16 * s) >> 6;
          const int c = ((16 * s) & 63) / 8 + (jm >> 1);
          uint32_t r0_, r1_, r2_, r3_;
          ldsm_x4(kbase + h * HALF + swz(row, c), r0_, r1_, r2_, r3_);
          if (s & 1)
            mma16816<T>(sb, r0_, r1_, r2_, r3_, qb[s][0], qb[s][1]);
          else
            mma16816<T>(sa, r0_, r1_, r2_, r3_, qb[s][0], qb[s][1]);
        }
      }
      float sc[4];
      // base-2 scaling, masking of rows past the end, class-A logits
#pragma unroll
      for (int hrow = 0; hrow < 2; ++hrow) {
        const int rw = lo + gid + 8 * hrow;
        const bool valid = rw < hi;
        const float x0 = (sa[2 * hrow] + sb[2 * hrow]) * p.scale_log2;
        const float x1 = (sa[2 * hrow + 1] + sb[2 * hrow + 1]) * p.scale_log2;
        sc[2 * hrow] = valid ? x0 : -INFINITY;
        sc[2 * hrow + 1] = valid ? x1 : -INFINITY;
        if (lg != nullptr && valid) {
          const int srow = trow0 + rw;
          if (srow >= a0 && srow < a1) {
            float* dst = lg + int64_t(srow - a0) * G;
            if (2 * tig < G) dst[2 * tig] = x0;
            if (2 * tig + 1 < G) dst[2 * tig + 1] = x1;
          }
        }
      }
      // online softmax: the 8 lanes sharing tig hold the same heads
      float mx0 = fmaxf(sc[0], sc[2]);
      float mx1 = fmaxf(sc[1], sc[3]);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      mx0 = fmaxf(mx0, m0);
      mx1 = fmaxf(mx1, m1);
      const float b0s = (mx0 == -INFINITY) ? 0.f : mx0;
      const float b1s = (mx1 == -INFINITY) ? 0.f : mx1;
      const float al0 = ex2(m0 - b0s), al1 = ex2(m1 - b1s);
      sc[0] = ex2(sc[0] - b0s);
      sc[1] = ex2(sc[1] - b1s);
      sc[2] = ex2(sc[2] - b0s);
      sc[3] = ex2(sc[3] - b1s);
      m0 = mx0;
      m1 = mx1;
      l0 = l0 * al0 + (sc[0] + sc[2]);
      l1 = l1 * al1 + (sc[1] + sc[3]);
#pragma unroll
      for (int u = 0; u < NS; ++u) {
        o[u][0] *= al0;
        o[u][2] *= al0;
        o[u][1] *= al1;
        o[u][3] *= al1;
      }
      // O^T += V^T . P^T
      const uint32_t pb0 = movm_t(pack2<T>(sc[0], sc[1]));  // rows 0-7 of the block
      const uint32_t pb1 = movm_t(pack2<T>(sc[2], sc[3]));  // rows 8-15
      const int row = lo + (lane & 7) + 8 * (jm >> 1);
#pragma unroll
      for (int u = 0; u < NS; ++u) {
        const int h = (16 * u) >> 6;
        const int c = ((16 * u) & 63) / 8 + (jm & 1);
        uint32_t r0_, r1_, r2_, r3_;
        ldsm_x4_t(vbase + h * HALF + swz(row, c), r0_, r1_, r2_, r3_);
        mma16816<T>(o[u], r0_, r1_, r2_, r3_, pb0, pb1);
      }
    }
    __syncwarp();  // the warp is done with its rows of this stage
    if (lane == 0 && t + kTcStages < ntiles) issue(t + kTcStages);
  }
  WNW_TR(2);
  // the lane-held sums over the warp's rows
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }

  // ---- merge the eight warps (the stage region is free: every load issued
  // has been waited for), then the segment's CTAs of this cluster
  __syncthreads();
  float* wm = reinterpret_cast<float*>(smem);
  float* wl = wm + NW * G;
  float* wo = wl + NW * G;
  float* Po = wo + NW * G * D;  // this CTA's partial: Po [G*D], Pm, Pl [G]
  float* Pm = Po + G * D;
  float* Pl = Pm + G;
  const int g0 = 2 * tig, g1 = 2 * tig + 1;
  if (gid == 0) {
    if (g0 < G) {
      wm[warp * G + g0] = m0;
      wl[warp * G + g0] = l0;
    }
    if (g1 < G) {
      wm[warp * G + g1] = m1;
      wl[warp * G + g1] = l1;
    }
  }
#pragma unroll
  for (int u = 0; u < NS; ++u) {
    const int d0 = 16 * u + gid, d1 = d0 + 8;
    if (g0 < G) {
      wo[(warp * G + g0) * D + d0] = o[u][0];
      wo[(warp * G + g0) * D + d1] = o[u][2];
    }
    if (g1 < G) {
      wo[(warp * G + g1) * D + d0] = o[u][1];
      wo[(warp * G + g1) * D + d1] = o[u][3];
    }
  }
  __syncthreads();
  for (int i = 4 * tid; i < G * D; i += 4 * kTcThreads) {
    const int g = i / D, d = i % D;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < NW; ++w) mx = fmaxf(mx, wm[w * G + g]);
    const float bse = (mx == -INFINITY) ? 0.f : mx;
    float ls = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      const float f = ex2(wm[w * G + g] - bse);
      fma4(acc, *reinterpret_cast<const float4*>(wo + (w * G + g) * D + d), f);
      ls += wl[w * G + g] * f;
    }
    *reinterpret_cast<float4*>(Po + i) = acc;
    if (d == 0) {
      Pm[g] = mx;
      Pl[g] = ls;
    }
  }
  WNW_TR(3);
  cluster_arrive();  // CTA partials visible to the cluster
  cluster_wait();
  WNW_TR(4);
  // every rank of the segment merges a slice of the output -- float4 group q
  // of the G*D/4 goes to rank q % nranks -- from all the ranks' partials over
  // DSMEM; a cluster partial whose range starts past the rows is not written
  const int range0 = (active && to_part) ? __ldg(pv.part_r0 + part) : 0;  // part < parts when active
  if (active && !(to_part && range0 >= total && range0 > 0)) {
    float* part_out = to_part ? p.partials + int64_t(part) * PartIO<D, G>::kStride : nullptr;
    for (int q = (crank - leader) + nranks * tid; q < G * D / 4; q += nranks * kTcThreads) {
      const int i = 4 * q;
      const int g = i / D;
      // every rank's (max, sum, o) first, so the remote loads overlap
      float pm[kTcMaxCluster], pl[kTcMaxCluster];
      float4 po[kTcMaxCluster];
#pragma unroll
      for (int r = 0; r < kTcMaxCluster; ++r) {
        if (r < nranks) {
          pm[r] = *cluster.map_shared_rank(Pm + g, leader + r);
          pl[r] = *cluster.map_shared_rank(Pl + g, leader + r);
          po[r] = *reinterpret_cast<const float4*>(cluster.map_shared_rank(Po + i, leader + r));
        } else {
          pm[r] = -INFINITY;
          pl[r] = 0.f;
          po[r] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int r = 0; r < kTcMaxCluster; ++r) mx = fmaxf(mx, pm[r]);
      const float bse = (mx == -INFINITY) ? 0.f : mx;
      float ls = 0.f;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int r = 0; r < kTcMaxCluster; ++r) {
        const float f = ex2(pm[r] - bse);
        fma4(acc, po[r], f);
        ls += pl[r] * f;
      }
      if (!to_part) {
        attn_store4<T, D, G>(p, seg, i, mx, ls, acc);
      } else {
        PartIO<D, G>::st(part_out + i, acc);
        if (i % D == 0) {
          part_out[G * D + g] = mx;
          part_out[G * D + G + g] = ls;
        }
      }
    }
  }
  cluster_arrive();  // keep this CTA's shared memory until every rank has read it
  cluster_wait();
  // ---- a segment spanning several clusters: each cluster's leader arrives
  // at the segment's counter once its partial is out; the last to arrive
  // merges the segment's partials in order (no second kernel, no wait)
  if (spans) {
    __shared__ int s_last, s_first, s_n;
    __syncthreads();  // this cluster's partial stores are ordered before (cluster barrier, CTA barrier) ...
    if (tid == 0) {
      int last = 0;
      if (cok) {
        // ... and released at gpu scope by the arrival, which acquires the
        // earlier arrivals' partials for the last one
        last = (atom_add_acq_rel_gpu(p.counters + seg, 1) == cn - 1) ? 1 : 0;
        if (last) p.counters[seg] = 0;  // every partial of this launch has arrived; the next use is a later launch
      } else {
        atomicOr(p.err, WNW_DEVERR_BAD_INDEX);
      }
      s_last = last;
      s_first = cfirst;
      s_n = nact;
    }
    __syncthreads();
    if (s_last) {
      const int n_act = s_n;
      const float* base = p.partials + int64_t(s_first) * PartIO<D, G>::kStride;
      for (int i = 4 * tid; i < G * D; i += 4 * kTcThreads) {
        const int g = i / D;
        float mx = -INFINITY, ls = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c0 = 0; c0 < n_act; c0 += kTcMaxCluster) {
          float bm[kTcMaxCluster], bl[kTcMaxCluster];
          float4 bo[kTcMaxCluster];
#pragma unroll
          for (int u = 0; u < kTcMaxCluster; ++u) {
            const int c = c0 + u;
            if (c < n_act) {
              const float* pc = base + int64_t(c) * PartIO<D, G>::kStride;
              bm[u] = __ldcg(pc + G * D + g);
              bl[u] = __ldcg(pc + G * D + G + g);
              bo[u] = PartIO<D, G>::ld(pc + i);
            } else {
              bm[u] = -INFINITY;
              bl[u] = 0.f;
              bo[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
          }
          float mn = mx;
#pragma unroll
          for (int u = 0; u < kTcMaxCluster; ++u) mn = fmaxf(mn, bm[u]);
          const float bse = (mn == -INFINITY) ? 0.f : mn;
          const float a = ex2(mx - bse);
          scale4(acc, a);
          ls *= a;
#pragma unroll
          for (int u = 0; u < kTcMaxCluster; ++u) {
            const float f = ex2(bm[u] - bse);
            fma4(acc, bo[u], f);
            ls += bl[u] * f;
          }
          mx = mn;
        }
        attn_store4<T, D, G>(p, seg, i, mx, ls, acc);
      }
    }
  }
#ifdef WNW_ATTN_TRACE
  WNW_TR(5);
  if (tid == 0) {
    const int k = atomicAdd(&g_attn_trace_n, 1);
    if (k < kTraceCap) {
      unsigned smid;
      asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
      g_attn_trace[k][0] = uint64_t(blockIdx.x) | (uint64_t(smid) << 16) | (uint64_t(crank) << 24) |
                           (uint64_t(uint32_t(rows)) << 32);
      g_attn_trace[k][1] = reinterpret_cast<uint64_t>(pv.cta);
      for (int i = 0; i < 6; ++i) g_attn_trace[k][2 + i] = tr_[i];
    }
  }
#endif
}

// three stages of K + V 128-row tiles (192 KB at head_dim 128); the merge
// reuses them
constexpr int mma_smem_bytes(int D) { return kTcStages * 2 * (D / 64) * kTcTileRows * 128 + 1024; }

template <typename T, int D, int G>
wnw_status configure_attn_mma() {
  static bool configured = false;
  if (!configured) {
    auto kern = decode_attn_mma_kernel<T, D, G>;
    WNW_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, mma_smem_bytes(D)));
    WNW_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    configured = true;
  }
  return WNW_OK;
}

// Clusters of `cs` CTAs of the tensor-core kernel that fit the device at
// once (0 when none fit).
template <typename T, int D, int G>
wnw_status attn_mma_active_clusters(int cs, int* n) {
  const wnw_status st = configure_attn_mma<T, D, G>();
  if (st != WNW_OK) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cs, 1, 1);
  cfg.blockDim = dim3(kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = mma_smem_bytes(D);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  WNW_CUDA_TRY(cudaOccupancyMaxActiveClusters(n, decode_attn_mma_kernel<T, D, G>, &cfg));
  return WNW_OK;
}

template <typename T, int D, int G>
wnw_status launch_attn_mma(const wnw_decode_attn_args* a, cudaStream_t stream) {
  {
    const wnw_status st = configure_attn_mma<T, D, G>();
    if (st != WNW_OK) return st;
  }
  WNW_CHECK_ARG(a->plan != nullptr && a->plan_ctas > 0 && a->plan_parts >= 0 && a->plan_combine >= 0,
                "the tensor-core path needs a work plan (wnw_attn_plan): plan, plan_ctas, plan_parts, "
                "plan_combine");
  WNW_CHECK_ARG(a->cluster_size >= 1 && a->cluster_size <= kTcMaxCluster && a->plan_ctas % a->cluster_size == 0,
                "cluster_size %d must be the plan's (1..16, dividing its %d CTAs)", a->cluster_size, a->plan_ctas);
  WNW_CHECK_ARG(a->plan_combine == 0 || (a->plan_parts > 0 && a->partials && a->counters),
                "a plan with combine entries needs partials and per-segment counters (zero before first use)");
  WNW_CHECK_ARG(a->store_rows > 0 && a->store_rows < (int64_t(1) << 31), "store_rows must be in (0, 2^31)");
  WNW_CHECK_ARG(aligned16(a->plan), "plan must be 16-byte aligned");
  CUtensorMap tk, tv;
  if (!kv_tensor_map(&tk, a->k_store, a->store_rows, D, a->dtype, kTcWarpRows) ||
      !kv_tensor_map(&tv, a->v_store, a->store_rows, D, a->dtype, kTcWarpRows))
    return WNW_ERR_CUDA;
  AttnParams p = make_params(a);
  AttnPlanView pv;
  const int64_t cta_at = 8;
  const int64_t part_at = cta_at + 4 * int64_t(a->plan_ctas);
  const int64_t comb_at = part_at + (int64_t(a->plan_parts) + 3) / 4 * 4;
  pv.cta = reinterpret_cast<const int4*>(a->plan + cta_at);
  pv.part_r0 = a->plan + part_at;
  pv.comb = reinterpret_cast<const int4*>(a->plan + comb_at);
  pv.parts = a->plan_parts;
  pv.combine = a->plan_combine;
  pv.ready = (a->flags & WNW_ATTN_ROWS_READY) ? 1 : 0;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = a->cluster_size;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a->plan_ctas, 1, 1);
  cfg.blockDim = dim3(kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = mma_smem_bytes(D);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  WNW_CUDA_TRY(cudaLaunchKernelEx(&cfg, decode_attn_mma_kernel<T, D, G>, p, pv, tk, tv));
  return WNW_OK;
}

}  // namespace wnw
