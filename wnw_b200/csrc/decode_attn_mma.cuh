// Tensor-core variant of the decode-attention kernel for 16-bit K/V
// (bf16 / fp16, head_dim 64 or 128).
//
// Same work decomposition, fused append, class-A logits and merge tail as the
// CUDA-core kernel (decode_attn.cuh), but the two products run on the tensor
// cores with fp32 accumulation:
//   S^T[rows x g] = K[rows x D] . q^T[D x g]      (mma m16n8k16, A = K via ldmatrix)
//   O^T[D x g]   += V^T[D x rows] . P^T[rows x g]  (A = V^T via ldmatrix.trans,
//                                                   B = P^T via movmatrix.trans)
// with the GQA group (<= 8 heads) as the n = 8 dimension.  K / V tiles of 128
// rows are staged by 2-D TMA with 128-byte swizzle (conflict-free ldmatrix);
// a CTA streams `split_rows / 128` consecutive tiles of its segment through
// up to three stages, each warp owning 32 rows of every tile: it waits for
// its rows, keeps an online softmax across tiles and refills its rows of the
// stage with a later tile as soon as it is done with them.
#pragma once

#include "decode_attn.cuh"
#include "tma.cuh"

namespace wnw {

constexpr int kMmaTileRows = 128;  // rows per CTA = 4 warps x 32
constexpr int kMmaWarpRows = 32;

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ uint32_t movm_t(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

template <typename T>
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__half>(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                 uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// byte offset of (row, 16-byte chunk) inside a 128-byte-swizzled tile whose
// base is 1024-byte aligned
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return uint32_t(row) * 128u + (uint32_t(chunk ^ (row & 7)) << 4);
}

template <typename T, int D, int G>
__global__ void __launch_bounds__(kAttnThreads)
    decode_attn_mma_kernel(const AttnParams p, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const int tiles, const int nstages) {
  static_assert(D == 64 || D == 128, "tensor-core path covers head_dim 64 and 128");
  static_assert(G >= 1 && G <= 8, "GQA group is the mma n=8 dimension");
  constexpr int NH = D / 64;                   // 128-byte halves per row
  constexpr int HALF = kMmaTileRows * 128;     // bytes of one half tile
  constexpr int STAGE = 2 * NH * HALF;         // K + V of one 128-row tile
  constexpr int NS = D / 16;                   // k-steps over D / m-tiles of O^T
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t bars[kMmaMaxStages][kAttnWarps];

  cg::cluster_group cluster = cg::this_cluster();
  const int cs = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  const int cid = blockIdx.x / cs;
  // prologue that does not depend on the preceding kernel (work table and
  // slot bases are fixed per layout) overlaps its tail under PDL
  const int seg = __ldg(p.work + 2 * cid);
  const int j = __ldg(p.work + 2 * cid + 1);
  const int64_t base = __ldg(p.seg_base + seg);
  // L2 prefetch of this CTA's first tiles (up to the slot capacity): it needs
  // only layout constants, so it runs before the dependency wait and the rows
  // stream into L2 while the preceding kernel finishes.  L2 is the point of
  // coherence and nothing lands in shared memory, so rows the preceding
  // kernel still writes are read correctly after the wait.
  if (p.seg_cap != nullptr && threadIdx.x < 2 * kMmaMaxStages) {
    const int cap = __ldg(p.seg_cap + seg);
    const int i = threadIdx.x >> 1;
    const int r0 = (j * cs + rank) * tiles * kMmaTileRows + i * kMmaTileRows;
    const int r1 = min(min(r0 + kMmaTileRows, cap), (j * cs + rank + 1) * tiles * kMmaTileRows);
    if (i < tiles && r1 > r0) {
      const T* src = reinterpret_cast<const T*>((threadIdx.x & 1) ? p.v_store : p.k_store) + (base + r0) * D;
      prefetch_l2(src, uint32_t(r1 - r0) * D * sizeof(T));
    }
  }
  if (threadIdx.x == 0) {
#pragma unroll
    for (int st = 0; st < kMmaMaxStages; ++st)
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) mbar_init(&bars[st][w], 1);
    fence_mbar_init();
  }
  pdl_wait();  // seg_len, K/V rows and q may come from the preceding kernel
  const int len = p.seg_len[seg];
  const bool append = p.new_k != nullptr;
  const int total = len + (append ? 1 : 0);
  const int rows_per_cta = tiles * kMmaTileRows;
  const int nsplit = (total + rows_per_cta - 1) / rows_per_cta;
  const int ncl = max(1, (nsplit + cs - 1) / cs);
  if (j >= ncl) return;  // the whole cluster is idle at this length (uniform)

  const int row0 = (j * cs + rank) * rows_per_cta;
  const int nrows = max(0, min(rows_per_cta, total - row0));
  const int ntiles = (nrows + kMmaTileRows - 1) / kMmaTileRows;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int gid = lane >> 2;
  const int tig = lane & 3;
  __syncthreads();

  // ---- producer: warp w's 32 rows of tile i -> stage i % nstages, one 2-D
  // TMA box (32 rows x 64 columns) per half and tensor; each warp refills its
  // own rows of a stage as soon as it is done with them
  auto issue = [&](int i, int w) {
    const int st = i % nstages;
    uint8_t* sK = smem + st * STAGE;
    uint8_t* sV = sK + NH * HALF;
    const int trow0 = row0 + i * kMmaTileRows;
    const int lo = w * kMmaWarpRows;
    if (lo >= total - trow0) return;  // rows past the segment's end: no copy, no wait
    mbar_arrive_expect_tx(&bars[st][w], 2u * NH * kMmaWarpRows * 128u);
    const int y = static_cast<int>(base + trow0 + lo);
#pragma unroll
    for (int h = 0; h < NH; ++h) {
      tma_load_2d(sK + h * HALF + lo * 128, &tmK, h * 64, y, &bars[st][w]);
      tma_load_2d(sV + h * HALF + lo * 128, &tmV, h * 64, y, &bars[st][w]);
    }
  };
  if (tid == 0) {
    for (int i = 0; i < min(ntiles, nstages); ++i)
      for (int w = 0; w < kAttnWarps; ++w) issue(i, w);
  }
  pdl_launch_dependents();  // the next kernel may start its own prologue now

  // ---- q as the mma B operand: b[k = d][n = g], zero for padded heads
  const T* qs = reinterpret_cast<const T*>(p.q) + int64_t(seg) * G * D;
  uint32_t qb[NS][2];
#pragma unroll
  for (int s = 0; s < NS; ++s) {
    if (gid < G) {
      qb[s][0] = *reinterpret_cast<const uint32_t*>(qs + gid * D + 16 * s + 2 * tig);
      qb[s][1] = *reinterpret_cast<const uint32_t*>(qs + gid * D + 16 * s + 8 + 2 * tig);
    } else {
      qb[s][0] = qb[s][1] = 0u;
    }
  }

  int a0 = 0, a1 = 0;
  float* lg = nullptr;
  if (p.score_slot != nullptr) {
    const int slot = p.score_slot[seg];
    if (slot >= 0) {
      const int b = seg / p.num_kv_heads;
      a0 = p.audio_start[b];
      a1 = p.audio_end[b];
      lg = p.logits + p.logits_off[slot];
    }
  }

  // running softmax state of this warp; per lane heads g0 = 2*tig, g1 = 2*tig+1
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float o[NS][4];
#pragma unroll
  for (int t = 0; t < NS; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
  const int jm = lane >> 3;  // which 8x8 matrix this lane addresses in ldmatrix

  for (int i = 0; i < ntiles; ++i) {
    const int st = i % nstages;
    uint8_t* sK = smem + st * STAGE;
    uint8_t* sV = sK + NH * HALF;
    const int trow0 = row0 + i * kMmaTileRows;
    const int tv = min(kMmaTileRows, total - trow0);
    const int lo = warp * kMmaWarpRows;
    const int hi = min(lo + kMmaWarpRows, tv);
    if (hi > lo) {
      mbar_wait(&bars[st][warp], (i / nstages) & 1, p.err);
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
      if (hi - lo < kMmaWarpRows) {
        // rows past the segment's end are masked out of the softmax, but their
        // V bytes still enter the mma: zero them so stale or non-finite memory
        // (slack rows, a neighbouring slot) cannot reach the output
        const int n0 = (lo + kMmaWarpRows - hi) * NH * 8;
        for (int idx = lane; idx < n0; idx += 32) {
          const int r = hi + idx / (NH * 8);
          const int rem = idx % (NH * 8);
          *reinterpret_cast<uint4*>(sV + (rem >> 3) * HALF + swz(r, rem & 7)) = make_uint4(0u, 0u, 0u, 0u);
        }
        __syncwarp();
      }
      const uint32_t kbase = smem_u32(sK);
      const uint32_t vbase = smem_u32(sV);
      // S^T for the two 16-row blocks of this warp's chunk
      float sc[2][4];
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        sc[b][0] = sc[b][1] = sc[b][2] = sc[b][3] = 0.f;
        const int row = lo + 16 * b + (lane & 7) + 8 * (jm & 1);
#pragma unroll
        for (int s = 0; s < NS; ++s) {
          const int h = (16 * s) >> 6;
          const int c = ((16 * s) & 63) / 8 + (jm >> 1);
          uint32_t r0, r1, r2, r3;
          ldsm_x4(kbase + h * HALF + swz(row, c), r0, r1, r2, r3);
          mma16816<T>(sc[b], r0, r1, r2, r3, qb[s][0], qb[s][1]);
        }
      }
      // base-2 scaling, masking of rows past the end, class-A logits
#pragma unroll
      for (int b = 0; b < 2; ++b) {
#pragma unroll
        for (int hrow = 0; hrow < 2; ++hrow) {
          const int rw = lo + 16 * b + gid + 8 * hrow;
          const bool valid = rw < hi;
          float& x0 = sc[b][2 * hrow];
          float& x1 = sc[b][2 * hrow + 1];
          x0 = valid ? x0 * p.scale_log2 : -INFINITY;
          x1 = valid ? x1 * p.scale_log2 : -INFINITY;
          if (lg != nullptr && valid) {
            const int srow = trow0 + rw;
            if (srow >= a0 && srow < a1) {
              float* dst = lg + int64_t(srow - a0) * G;
              if (2 * tig < G) dst[2 * tig] = x0;
              if (2 * tig + 1 < G) dst[2 * tig + 1] = x1;
            }
          }
        }
      }
      // online softmax update over this chunk: lanes sharing tig hold the same heads
      float mx0 = fmaxf(fmaxf(sc[0][0], sc[0][2]), fmaxf(sc[1][0], sc[1][2]));
      float mx1 = fmaxf(fmaxf(sc[0][1], sc[0][3]), fmaxf(sc[1][1], sc[1][3]));
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
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        sc[b][0] = ex2(sc[b][0] - b0s);
        sc[b][1] = ex2(sc[b][1] - b1s);
        sc[b][2] = ex2(sc[b][2] - b0s);
        sc[b][3] = ex2(sc[b][3] - b1s);
        s0 += sc[b][0] + sc[b][2];
        s1 += sc[b][1] + sc[b][3];
      }
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        s0 += __shfl_xor_sync(0xffffffffu, s0, off);
        s1 += __shfl_xor_sync(0xffffffffu, s1, off);
      }
      m0 = mx0;
      m1 = mx1;
      l0 = l0 * al0 + s0;
      l1 = l1 * al1 + s1;
#pragma unroll
      for (int t = 0; t < NS; ++t) {
        o[t][0] *= al0;
        o[t][2] *= al0;
        o[t][1] *= al1;
        o[t][3] *= al1;
      }
      // O^T += V^T . P^T
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        const uint32_t pb0 = movm_t(pack2<T>(sc[b][0], sc[b][1]));  // rows 0-7 of the block
        const uint32_t pb1 = movm_t(pack2<T>(sc[b][2], sc[b][3]));  // rows 8-15
        const int row = lo + 16 * b + (lane & 7) + 8 * (jm >> 1);
#pragma unroll
        for (int t = 0; t < NS; ++t) {
          const int h = (16 * t) >> 6;
          const int c = ((16 * t) & 63) / 8 + (jm & 1);
          uint32_t r0, r1, r2, r3;
          ldsm_x4_t(vbase + h * HALF + swz(row, c), r0, r1, r2, r3);
          mma16816<T>(o[t], r0, r1, r2, r3, pb0, pb1);
        }
      }
    }
    __syncwarp();  // the warp is done with its rows of this stage
    if (lane == 0 && i + nstages < ntiles) issue(i + nstages, warp);
  }

  // ---- hand the warp partials to the shared merge (tile region reused once
  // every warp is done with its last tile)
  __syncthreads();
  float* wm = reinterpret_cast<float*>(smem);
  float* wl = wm + kAttnWarps * G;
  float* wo = wl + kAttnWarps * G;
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
  for (int t = 0; t < NS; ++t) {
    const int d0 = 16 * t + gid, d1 = d0 + 8;
    if (g0 < G) {
      wo[(warp * G + g0) * D + d0] = o[t][0];
      wo[(warp * G + g0) * D + d1] = o[t][2];
    }
    if (g1 < G) {
      wo[(warp * G + g1) * D + d0] = o[t][1];
      wo[(warp * G + g1) * D + d1] = o[t][3];
    }
  }
  __syncthreads();
  attn_finish<T, D, G>(p, smem, seg, j, cid, ncl);
}

// one stage = K + V of one 128-row tile; a CTA streaming several tiles keeps
// up to three stages (192 KB at head_dim 128) in flight
constexpr int kMmaStageBytes(int D) { return 2 * (D / 64) * kMmaTileRows * 128; }

constexpr int mma_smem_bytes(int D, int nstages) { return nstages * kMmaStageBytes(D) + 1024; }

template <typename T, int D, int G>
wnw_status configure_attn_mma() {
  auto kern = decode_attn_mma_kernel<T, D, G>;
  static bool configured = false;
  if (!configured) {
    WNW_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      mma_smem_bytes(D, kMmaMaxStages)));
    WNW_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    configured = true;
  }
  return WNW_OK;
}

// Clusters of `cs` CTAs of the kernel that can be resident at once with
// `nstages` stages of shared memory (0 when none fit).
template <typename T, int D, int G>
wnw_status attn_mma_active_clusters(int cs, int nstages, int* n) {
  const wnw_status st = configure_attn_mma<T, D, G>();
  if (st != WNW_OK) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cs, 1, 1);
  cfg.blockDim = dim3(kAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = mma_smem_bytes(D, nstages);
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
  auto kern = decode_attn_mma_kernel<T, D, G>;
  {
    const wnw_status st = configure_attn_mma<T, D, G>();
    if (st != WNW_OK) return st;
  }
  WNW_CHECK_ARG(a->split_rows >= kMmaTileRows && a->split_rows % kMmaTileRows == 0,
                "split_rows %d must be a positive multiple of the tensor-core tile (%d rows)", a->split_rows,
                kMmaTileRows);
  const int tiles = a->split_rows / kMmaTileRows;
  const int nstages = mma_stages(tiles);
  const int smem = mma_smem_bytes(D, nstages);
  WNW_CHECK_ARG(a->store_rows > 0 && a->store_rows < (int64_t(1) << 31), "store_rows must be in (0, 2^31)");
  CUtensorMap tk, tv;
  if (!kv_tensor_map(&tk, a->k_store, a->store_rows, D, a->dtype, kMmaWarpRows) ||
      !kv_tensor_map(&tv, a->v_store, a->store_rows, D, a->dtype, kMmaWarpRows))
    return WNW_ERR_CUDA;
  AttnParams p = make_params(a);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a->n_clusters * a->cluster_size, 1, 1);
  cfg.blockDim = dim3(kAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a->cluster_size;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  WNW_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p, tk, tv, tiles, nstages));
  return WNW_OK;
}

}  // namespace wnw
