// Prefill audio scores: the per-layer class-A and class-B audio-token scores
// the session hands to prefill_after_attn (the reference computes them in
// src/algorithms/wnw/code/session.py:121-201 with a bf16 / fp16 matmul, a
// scale and a mask add in the model dtype, then an fp32 softmax over all
// keys).
//
// Two launches per layer.  Pass 1, one CTA per (task, 1,024-key chunk, 64
// query rows): for each of its rows, the running max and sum of exp over the
// chunk's keys (each K fragment loaded once for the 64 rows).  Pass 2, one
// CTA per (task, 256 audio keys): merges the chunks' statistics of every row
// (in chunk order), recomputes the audio keys' logits and adds
// exp(x - max) / sum over the rows, in a fixed order.
// Logits of 16-bit q / k with head_dim 64 or 128 come from the tensor cores
// (mma m16n8k16, keys as m, query rows as n, fp32 accumulation); fp32 ones
// and small head dims from CUDA-core FMAs.  They are rounded to the model
// dtype exactly where the reference rounds them (not at all for fp32).
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "mma.cuh"

namespace wnw {
namespace {

constexpr int kPfThreads = 256;
constexpr int kPfWarps = 8;
constexpr int kPfChunk = 1024;        // keys per pass-1 CTA
constexpr int kPfAudioChunk = 256;    // audio keys per pass-2 CTA
constexpr int kPfTilesPerWarp = kPfAudioChunk / (16 * kPfWarps);
constexpr int kPfRowsBlock = 256;     // query rows staged in shared memory at a time (pass 2)
constexpr int kPfRowTiles = 8;        // 8-row query tiles per pass-1 CTA (64 rows)

struct PfParams {
  const void* q;
  int64_t qsb, qsh, qss;
  const void* k;
  int64_t ksb, ksh, kss;
  const void* mask;
  int64_t msb, mss;
  int mask_kind;
  float scale;
  const wnw_prefill_task* tasks;
  const int32_t* heads;
  float* out;
  int64_t out_len;
  float2* stats;  // [task][max_rows][n_chunks]
  int B, Hq, Hkv, S, num_heads, max_rows, max_audio, n_chunks;
  int32_t* err;
};

template <typename T>
__device__ __forceinline__ float rnd(float x) {
  return DT<T>::to_f(DT<T>::from_f(x));
}

__device__ __forceinline__ uint32_t ld32(const void* p) { return __ldg(static_cast<const uint32_t*>(p)); }

__device__ __forceinline__ bool task_ok(const wnw_prefill_task& t, const PfParams& p) {
  return t.batch >= 0 && t.batch < p.B && t.kv_head >= 0 && t.kv_head < p.Hkv && t.n_heads >= 1 &&
         t.head_off >= 0 && int64_t(t.head_off) + t.n_heads <= p.num_heads && t.n_rows >= 1 && t.row0 >= 0 &&
         int64_t(t.row0) + t.n_rows <= p.S && int64_t(t.n_heads) * t.n_rows <= p.max_rows &&
         t.audio_start >= 0 && t.audio_start <= t.audio_end && t.audio_end <= p.S &&
         t.audio_end - t.audio_start <= p.max_audio && t.out_off >= 0 &&
         t.out_off + (t.audio_end - t.audio_start) <= p.out_len;
}

// first element of query row r (row-major over (head, position)); nullptr
// when r is past the task's rows or its head index is out of range
template <typename T>
__device__ __forceinline__ const T* q_row(const PfParams& p, const wnw_prefill_task& t, int r, int R) {
  if (r >= R) return nullptr;
  const int h = p.heads[t.head_off + r / t.n_rows];
  if (h < 0 || h >= p.Hq) return nullptr;
  return static_cast<const T*>(p.q) + t.batch * p.qsb + h * p.qsh + int64_t(t.row0 + r % t.n_rows) * p.qss;
}

__device__ __forceinline__ int row_pos(const wnw_prefill_task& t, int r, int R) {
  return r < R ? t.row0 + r % t.n_rows : -1;
}

// the reference's logit of (query position pos, key j) from the fp32 dot
// product; -inf where masked
template <typename T>
__device__ __forceinline__ float logit(const PfParams& p, const wnw_prefill_task& t, float dot, int pos, int j) {
  if (pos < 0) return -INFINITY;
  if (p.mask_kind == WNW_MASK_CAUSAL && j > pos) return -INFINITY;
  float x = rnd<T>(rnd<T>(dot) * p.scale);
  if (p.mask_kind == WNW_MASK_ADDITIVE)
    x = rnd<T>(x + DT<T>::to_f(static_cast<const T*>(p.mask)[t.batch * p.msb + int64_t(pos) * p.mss + j]));
  return x;
}

// The softmax runs in base 2 on x * log2(e) (MUFU ex2): row statistics are
// (max, sum of 2^(x' - max)) of the scaled logits x'.
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void online(float& m, float& l, float x) {
  x *= kLog2e;  // a masked logit near -FLT_MAX becomes -inf here
  if (!(x > -INFINITY)) return;
  if (x > m) {
    l = l * ex2(m - x) + 1.f;
    m = x;
  } else {
    l += ex2(x - m);
  }
}

__device__ __forceinline__ void merge(float& m, float& l, float m2, float l2) {
  if (!(m2 > -INFINITY)) return;
  if (!(m > -INFINITY)) {
    m = m2;
    l = l2;
    return;
  }
  const float mx = fmaxf(m, m2);
  l = l * ex2(m - mx) + l2 * ex2(m2 - mx);
  m = mx;
}

// two logits (natural units) into a row's statistics, without branches
// (ex2 of -inf is 0, so masked logits and a first update need no case)
__device__ __forceinline__ void online2(float& m, float& l, float x0, float x1) {
  x0 *= kLog2e;  // a masked logit near -FLT_MAX becomes -inf here
  x1 *= kLog2e;
  const float mn = fmaxf(m, fmaxf(x0, x1));
  if (mn == -INFINITY) return;
  l = l * ex2(m - mn) + ex2(x0 - mn) + ex2(x1 - mn);
  m = mn;
}

// softmax probability of logit x (natural units) under row statistics
// s = (max, 1 / sum)
__device__ __forceinline__ float prob(float x, float2 s) {
  x *= kLog2e;
  return x > -INFINITY ? ex2(x - s.x) * s.y : 0.f;
}

// K fragment (A operand, keys j0 + g and j0 + g + 8, head dims [16 kk, 16 kk + 16))
template <typename T, int D>
__device__ __forceinline__ void load_k(const T* kb, int64_t kss, int j0, int j1, int g, int tq,
                                       uint32_t (&a)[D / 16][4]) {
  const int r0 = j0 + g, r1 = j0 + g + 8;
  const T* p0 = kb + int64_t(r0) * kss + 2 * tq;
  const T* p1 = kb + int64_t(r1) * kss + 2 * tq;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    a[kk][0] = r0 < j1 ? ld32(p0 + 16 * kk) : 0u;
    a[kk][1] = r1 < j1 ? ld32(p1 + 16 * kk) : 0u;
    a[kk][2] = r0 < j1 ? ld32(p0 + 16 * kk + 8) : 0u;
    a[kk][3] = r1 < j1 ? ld32(p1 + 16 * kk + 8) : 0u;
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kPfThreads) prefill_stats_kernel(PfParams p) {
  const wnw_prefill_task t = p.tasks[blockIdx.y];
  if (!task_ok(t, p)) {
    if (blockIdx.x == 0 && blockIdx.z == 0 && threadIdx.x == 0) atomicOr(p.err, WNW_DEVERR_BAD_INDEX);
    return;
  }
  const int k0 = blockIdx.x * kPfChunk;
  const int R = t.n_heads * t.n_rows;
  const int rb = blockIdx.z * 8 * kPfRowTiles;  // this CTA's query rows: [rb, rb + 64)
  if (k0 >= p.S || rb >= R) return;
  const int k1 = min(p.S, k0 + kPfChunk);
  const int nt = min(kPfRowTiles, (R - rb + 7) / 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const T* kb = static_cast<const T*>(p.k) + t.batch * p.ksb + t.kv_head * p.ksh;
  constexpr int QS = D + 8;  // padded row: a fragment load's 8 rows fall in distinct banks
  __shared__ __align__(16) T qs[8 * kPfRowTiles][QS];
  __shared__ float2 red[kPfWarps][8 * kPfRowTiles];
  for (int i = threadIdx.x; i < 8 * kPfRowTiles * (D / 8); i += kPfThreads) {
    const int r = i / (D / 8), c = i % (D / 8);
    const T* qr = q_row<T>(p, t, rb + r, R);
    *reinterpret_cast<uint4*>(&qs[r][c * 8]) =
        qr ? __ldg(reinterpret_cast<const uint4*>(qr + c * 8)) : make_uint4(0u, 0u, 0u, 0u);
  }
  __syncthreads();
  // per lane: rows 8 ti + 2 tq (a) and + 1 (b) of each row tile, over this warp's keys
  float ma[kPfRowTiles], la[kPfRowTiles], mb[kPfRowTiles], lb[kPfRowTiles];
#pragma unroll
  for (int ti = 0; ti < kPfRowTiles; ++ti) ma[ti] = mb[ti] = -INFINITY, la[ti] = lb[ti] = 0.f;
  for (int j = k0 + warp * 16; j < k1; j += kPfWarps * 16) {
    uint32_t a[D / 16][4];  // the K fragment of keys j .. j + 15, reused by every row tile
    load_k<T, D>(kb, p.kss, j, k1, g, tq, a);
#pragma unroll
    for (int ti = 0; ti < kPfRowTiles; ++ti) {
      if (ti < nt) {
        const T* qr = &qs[8 * ti + g][2 * tq];
        float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          mma16816<T>(c, a[kk][0], a[kk][1], a[kk][2], a[kk][3], *reinterpret_cast<const uint32_t*>(qr + 16 * kk),
                      *reinterpret_cast<const uint32_t*>(qr + 16 * kk + 8));
        // c[0]: (key j+g, row 2tq), c[1]: (key j+g, row 2tq+1), c[2] / c[3]: key j+g+8
        const int pa = row_pos(t, rb + 8 * ti + 2 * tq, R), pb = row_pos(t, rb + 8 * ti + 2 * tq + 1, R);
        const bool v0 = j + g < k1, v1 = j + g + 8 < k1;
        online2(ma[ti], la[ti], v0 ? logit<T>(p, t, c[0], pa, j + g) : -INFINITY,
                v1 ? logit<T>(p, t, c[2], pa, j + g + 8) : -INFINITY);
        online2(mb[ti], lb[ti], v0 ? logit<T>(p, t, c[1], pb, j + g) : -INFINITY,
                v1 ? logit<T>(p, t, c[3], pb, j + g + 8) : -INFINITY);
      }
    }
  }
#pragma unroll
  for (int ti = 0; ti < kPfRowTiles; ++ti) {
    if (ti < nt) {
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) {
        const float m2a = __shfl_xor_sync(0xffffffffu, ma[ti], o), l2a = __shfl_xor_sync(0xffffffffu, la[ti], o);
        const float m2b = __shfl_xor_sync(0xffffffffu, mb[ti], o), l2b = __shfl_xor_sync(0xffffffffu, lb[ti], o);
        merge(ma[ti], la[ti], m2a, l2a);
        merge(mb[ti], lb[ti], m2b, l2b);
      }
      if (g == 0) {
        red[warp][8 * ti + 2 * tq] = make_float2(ma[ti], la[ti]);
        red[warp][8 * ti + 2 * tq + 1] = make_float2(mb[ti], lb[ti]);
      }
    }
  }
  __syncthreads();
  for (int r = threadIdx.x; r < min(8 * kPfRowTiles, R - rb); r += kPfThreads) {
    float m = -INFINITY, l = 0.f;
    for (int w = 0; w < kPfWarps; ++w) merge(m, l, red[w][r].x, red[w][r].y);
    p.stats[(int64_t(blockIdx.y) * p.max_rows + rb + r) * p.n_chunks + blockIdx.x] = make_float2(m, l);
  }
}

template <int D>
constexpr int pf_smem_bytes() {
  return kPfRowsBlock * (D + 8) * 2 + kPfRowsBlock * int(sizeof(float2));
}

template <typename T, int D>
__global__ void __launch_bounds__(kPfThreads) prefill_colsum_kernel(PfParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const wnw_prefill_task t = p.tasks[blockIdx.y];
  if (!task_ok(t, p)) return;  // flagged by pass 1
  const int j0 = t.audio_start + blockIdx.x * kPfAudioChunk;
  if (j0 >= t.audio_end) return;
  const int j1 = min(t.audio_end, j0 + kPfAudioChunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int R = t.n_heads * t.n_rows;
  const T* kb = static_cast<const T*>(p.k) + t.batch * p.ksb + t.kv_head * p.ksh;
  constexpr int QS = D + 8;  // padded row: the 8 rows a fragment load reads fall in distinct banks
  T* qs = reinterpret_cast<T*>(smem);
  float2* st = reinterpret_cast<float2*>(smem + kPfRowsBlock * QS * 2);
  float acc[kPfTilesPerWarp][2];
#pragma unroll
  for (int i = 0; i < kPfTilesPerWarp; ++i) acc[i][0] = acc[i][1] = 0.f;

  for (int rb = 0; rb < R; rb += kPfRowsBlock) {
    const int nr = min(kPfRowsBlock, R - rb);
    __syncthreads();  // the previous block's rows are no longer read
    for (int i = threadIdx.x; i < kPfRowsBlock * (D / 8); i += kPfThreads) {
      const int r = i / (D / 8), c = i % (D / 8);
      const T* qr = q_row<T>(p, t, rb + r, R);
      *reinterpret_cast<uint4*>(qs + r * QS + c * 8) =
          qr ? __ldg(reinterpret_cast<const uint4*>(qr + c * 8)) : make_uint4(0u, 0u, 0u, 0u);
    }
    for (int r = threadIdx.x; r < nr; r += kPfThreads) {
      float m = -INFINITY, l = 0.f;
      const float2* s = p.stats + (int64_t(blockIdx.y) * p.max_rows + rb + r) * p.n_chunks;
      for (int c = 0; c < p.n_chunks; ++c) {
        const float2 v = s[c];
        merge(m, l, v.x, v.y);
      }
      st[r] = make_float2(m, l > 0.f ? 1.f / l : 0.f);
    }
    __syncthreads();
#pragma unroll
    for (int ti = 0; ti < kPfTilesPerWarp; ++ti) {
      const int j = j0 + (ti * kPfWarps + warp) * 16;
      if (j < j1) {  // warp-uniform
        uint32_t a[D / 16][4];
        load_k<T, D>(kb, p.kss, j, j1, g, tq, a);
        for (int rt = 0; rt < nr; rt += 8) {
          const T* qr = qs + (rt + g) * QS + 2 * tq;
          float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma16816<T>(c, a[kk][0], a[kk][1], a[kk][2], a[kk][3], *reinterpret_cast<const uint32_t*>(qr + 16 * kk),
                        *reinterpret_cast<const uint32_t*>(qr + 16 * kk + 8));
#pragma unroll
          for (int e = 0; e < 2; ++e) {  // rows rt + 2tq + e (block-local)
            const int r = rt + 2 * tq + e;
            if (r < nr) {
              const int pos = row_pos(t, rb + r, R);
              const float2 s = st[r];
              const float x0 = logit<T>(p, t, c[e], pos, j + g);
              const float x1 = logit<T>(p, t, c[2 + e], pos, j + g + 8);
              acc[ti][0] += prob(x0, s);
              acc[ti][1] += prob(x1, s);
            }
          }
        }
      }
    }
  }
#pragma unroll
  for (int ti = 0; ti < kPfTilesPerWarp; ++ti) {
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
      acc[ti][0] += __shfl_xor_sync(0xffffffffu, acc[ti][0], o);
      acc[ti][1] += __shfl_xor_sync(0xffffffffu, acc[ti][1], o);
    }
    const int j = j0 + (ti * kPfWarps + warp) * 16 + g;
    if (tq == 0) {
      const float inv = t.n_rows;
      if (j < j1) p.out[t.out_off + j - t.audio_start] = t.n_rows > 1 ? acc[ti][0] / inv : acc[ti][0];
      if (j + 8 < j1) p.out[t.out_off + j + 8 - t.audio_start] = t.n_rows > 1 ? acc[ti][1] / inv : acc[ti][1];
    }
  }
}

// ---- CUDA-core variant: fp32 q / k, or 16-bit ones with head_dim 16 / 32.
// Same two passes, same statistics layout; dot products in fp32 FMAs, one key
// per lane, the 8 query rows of a tile (pass 1) or a block of rows (pass 2)
// staged in shared memory as fp32.
constexpr int kPfCcRows = 32;  // query rows staged at a time in pass 2

template <typename T, int D>
__device__ __forceinline__ void load_row_f(const T* src, float (&x)[D]) {
  constexpr int E = 16 / sizeof(T);  // elements per 16-byte load
#pragma unroll
  for (int c = 0; c < D / E; ++c) unpack16<T>(__ldg(reinterpret_cast<const uint4*>(src) + c), x + c * E);
}

template <typename T, int D>
__global__ void __launch_bounds__(kPfThreads) prefill_stats_cc_kernel(PfParams p) {
  const wnw_prefill_task t = p.tasks[blockIdx.y];
  if (!task_ok(t, p)) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(p.err, WNW_DEVERR_BAD_INDEX);
    return;
  }
  const int k0 = blockIdx.x * kPfChunk;
  if (k0 >= p.S) return;
  const int k1 = min(p.S, k0 + kPfChunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int R = t.n_heads * t.n_rows;
  const T* kb = static_cast<const T*>(p.k) + t.batch * p.ksb + t.kv_head * p.ksh;
  __shared__ float qs[8][D];
  __shared__ float2 red[kPfWarps][8];
  for (int rt = 0; rt < R; rt += 8) {
    __syncthreads();  // the previous tile's rows and partials are no longer read
    for (int i = threadIdx.x; i < 8 * D; i += kPfThreads) {
      const T* qr = q_row<T>(p, t, rt + i / D, R);
      qs[i / D][i % D] = qr ? DT<T>::to_f(qr[i % D]) : 0.f;
    }
    __syncthreads();
    float m[8], l[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) m[r] = -INFINITY, l[r] = 0.f;
    for (int j = k0 + warp * 32 + lane; j < k1; j += kPfThreads) {
      float kv[D];
      load_row_f<T, D>(kb + int64_t(j) * p.kss, kv);
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        float dot = 0.f;
#pragma unroll
        for (int d = 0; d < D; ++d) dot = fmaf(qs[r][d], kv[d], dot);
        online(m[r], l[r], logit<T>(p, t, dot, row_pos(t, rt + r, R), j));
      }
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m[r], o), l2 = __shfl_xor_sync(0xffffffffu, l[r], o);
        merge(m[r], l[r], m2, l2);
      }
      if (lane == 0) red[warp][r] = make_float2(m[r], l[r]);
    }
    __syncthreads();
    if (threadIdx.x < 8 && rt + int(threadIdx.x) < R) {
      float mm = -INFINITY, ll = 0.f;
      for (int w = 0; w < kPfWarps; ++w) merge(mm, ll, red[w][threadIdx.x].x, red[w][threadIdx.x].y);
      p.stats[(int64_t(blockIdx.y) * p.max_rows + rt + threadIdx.x) * p.n_chunks + blockIdx.x] = make_float2(mm, ll);
    }
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kPfThreads) prefill_colsum_cc_kernel(PfParams p) {
  const wnw_prefill_task t = p.tasks[blockIdx.y];
  if (!task_ok(t, p)) return;  // flagged by pass 1
  const int j = t.audio_start + blockIdx.x * kPfThreads + threadIdx.x;
  if (t.audio_start + int(blockIdx.x) * kPfThreads >= t.audio_end) return;  // CTA-uniform
  const bool valid = j < t.audio_end;
  const int R = t.n_heads * t.n_rows;
  const T* kb = static_cast<const T*>(p.k) + t.batch * p.ksb + t.kv_head * p.ksh;
  __shared__ float qs[kPfCcRows][D];
  __shared__ float2 st[kPfCcRows];
  float kv[D];
  if (valid) load_row_f<T, D>(kb + int64_t(j) * p.kss, kv);
  float acc = 0.f;
  for (int rb = 0; rb < R; rb += kPfCcRows) {
    const int nr = min(kPfCcRows, R - rb);
    __syncthreads();
    for (int i = threadIdx.x; i < kPfCcRows * D; i += kPfThreads) {
      const T* qr = q_row<T>(p, t, rb + i / D, R);
      qs[i / D][i % D] = qr ? DT<T>::to_f(qr[i % D]) : 0.f;
    }
    for (int r = threadIdx.x; r < nr; r += kPfThreads) {
      float m = -INFINITY, l = 0.f;
      const float2* sp = p.stats + (int64_t(blockIdx.y) * p.max_rows + rb + r) * p.n_chunks;
      for (int c = 0; c < p.n_chunks; ++c) {
        const float2 v = sp[c];
        merge(m, l, v.x, v.y);
      }
      st[r] = make_float2(m, l > 0.f ? 1.f / l : 0.f);
    }
    __syncthreads();
    if (valid) {
      for (int r = 0; r < nr; ++r) {
        float dot = 0.f;
#pragma unroll
        for (int d = 0; d < D; ++d) dot = fmaf(qs[r][d], kv[d], dot);
        const float x = logit<T>(p, t, dot, row_pos(t, rb + r, R), j);
        acc += prob(x, st[r]);
      }
    }
  }
  if (valid) p.out[t.out_off + j - t.audio_start] = t.n_rows > 1 ? acc / float(t.n_rows) : acc;
}

template <typename T, int D>
wnw_status launch_pf_cc(const PfParams& p, int num_tasks, cudaStream_t s) {
  prefill_stats_cc_kernel<T, D><<<dim3(p.n_chunks, num_tasks), kPfThreads, 0, s>>>(p);
  WNW_CUDA_TRY(cudaGetLastError());
  const int ax = std::max(1, (p.max_audio + kPfThreads - 1) / kPfThreads);
  prefill_colsum_cc_kernel<T, D><<<dim3(ax, num_tasks), kPfThreads, 0, s>>>(p);
  WNW_CUDA_TRY(cudaGetLastError());
  return WNW_OK;
}

template <typename T>
wnw_status launch_pf_cc_any(const PfParams& p, int head_dim, int num_tasks, cudaStream_t s) {
  switch (head_dim) {
    case 16: return launch_pf_cc<T, 16>(p, num_tasks, s);
    case 32: return launch_pf_cc<T, 32>(p, num_tasks, s);
    case 64: return launch_pf_cc<T, 64>(p, num_tasks, s);
    default: return launch_pf_cc<T, 128>(p, num_tasks, s);
  }
}

template <typename T, int D>
wnw_status launch_pf(const PfParams& p, int num_tasks, cudaStream_t s) {
  static bool configured = false;  // the dynamic shared memory opt-in, once per instantiation
  if (!configured) {
    WNW_CUDA_TRY(cudaFuncSetAttribute(prefill_colsum_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      pf_smem_bytes<D>()));
    configured = true;
  }
  prefill_stats_kernel<T, D><<<dim3(p.n_chunks, num_tasks, (p.max_rows + 8 * kPfRowTiles - 1) / (8 * kPfRowTiles)),
                                kPfThreads, 0, s>>>(p);
  WNW_CUDA_TRY(cudaGetLastError());
  const int ax = std::max(1, (p.max_audio + kPfAudioChunk - 1) / kPfAudioChunk);
  prefill_colsum_kernel<T, D><<<dim3(ax, num_tasks), kPfThreads, pf_smem_bytes<D>(), s>>>(p);
  WNW_CUDA_TRY(cudaGetLastError());
  return WNW_OK;
}

}  // namespace
}  // namespace wnw

extern "C" wnw_status wnw_prefill_scores_scratch_bytes(int num_tasks, int max_rows, int seq_len, int64_t* bytes) {
  using namespace wnw;
  WNW_CHECK_ARG(bytes, "null pointer argument");
  WNW_CHECK_ARG(num_tasks >= 0 && max_rows >= 1 && seq_len >= 1, "sizes must be positive");
  *bytes = int64_t(num_tasks) * max_rows * ((seq_len + kPfChunk - 1) / kPfChunk) * int64_t(sizeof(float2));
  return WNW_OK;
}

extern "C" wnw_status wnw_prefill_scores(const wnw_prefill_scores_args* a, void* stream) {
  using namespace wnw;
  WNW_CHECK_ARG(a, "null pointer argument");
  WNW_CHECK_ARG(a->dtype == WNW_BF16 || a->dtype == WNW_F16 || a->dtype == WNW_F32, "unknown dtype %d", a->dtype);
  WNW_CHECK_ARG(a->head_dim == 16 || a->head_dim == 32 || a->head_dim == 64 || a->head_dim == 128,
                "head_dim must be 16, 32, 64 or 128");
  WNW_CHECK_ARG(a->num_tasks >= 0 && a->num_tasks <= 65535, "num_tasks must be in 0..65535");
  if (a->num_tasks == 0) return WNW_OK;
  WNW_CHECK_ARG(a->batch > 0 && a->num_q_heads > 0 && a->num_kv_heads > 0 && a->seq_len > 0 && a->num_heads > 0 &&
                    a->max_rows > 0 && a->max_audio >= 0 && a->out_len >= 0,
                "sizes must be positive");
  WNW_CHECK_ARG(a->max_rows <= 65535 * 8 * kPfRowTiles, "max_rows above %d", 65535 * 8 * kPfRowTiles);
  WNW_CHECK_ARG(a->q && a->k && a->tasks && a->heads && a->out && a->scratch && a->err, "null pointer argument");
  WNW_CHECK_ARG(a->mask_kind == WNW_MASK_NONE || a->mask_kind == WNW_MASK_CAUSAL || a->mask_kind == WNW_MASK_ADDITIVE,
                "unknown mask kind %d", a->mask_kind);
  WNW_CHECK_ARG(a->mask_kind != WNW_MASK_ADDITIVE || a->mask, "an additive mask needs its pointer");
  WNW_CHECK_ARG(aligned16(a->q) && aligned16(a->k), "q and k must be 16-byte aligned");
  const int epc = a->dtype == WNW_F32 ? 4 : 8;  // elements per 16 bytes
  WNW_CHECK_ARG(a->q_stride_b % epc == 0 && a->q_stride_h % epc == 0 && a->q_stride_s % epc == 0 &&
                    a->k_stride_b % epc == 0 && a->k_stride_h % epc == 0 && a->k_stride_s % epc == 0,
                "q / k strides must be multiples of 16 bytes");
  int64_t need = 0;
  wnw_status st = wnw_prefill_scores_scratch_bytes(a->num_tasks, a->max_rows, a->seq_len, &need);
  if (st != WNW_OK) return st;
  if (a->scratch_bytes < need) {
    set_error("prefill scores need %lld scratch bytes, got %lld", static_cast<long long>(need),
              static_cast<long long>(a->scratch_bytes));
    return WNW_ERR_CAPACITY;
  }
  PfParams p;
  p.q = a->q;
  p.qsb = a->q_stride_b;
  p.qsh = a->q_stride_h;
  p.qss = a->q_stride_s;
  p.k = a->k;
  p.ksb = a->k_stride_b;
  p.ksh = a->k_stride_h;
  p.kss = a->k_stride_s;
  p.mask = a->mask;
  p.msb = a->mask_stride_b;
  p.mss = a->mask_stride_s;
  p.mask_kind = a->mask_kind;
  p.scale = a->scaling;
  p.tasks = a->tasks;
  p.heads = a->heads;
  p.out = a->out;
  p.out_len = a->out_len;
  p.stats = static_cast<float2*>(a->scratch);
  p.B = a->batch;
  p.Hq = a->num_q_heads;
  p.Hkv = a->num_kv_heads;
  p.S = a->seq_len;
  p.num_heads = a->num_heads;
  p.max_rows = a->max_rows;
  p.max_audio = a->max_audio;
  p.n_chunks = (a->seq_len + kPfChunk - 1) / kPfChunk;
  p.err = a->err;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a->dtype == WNW_F32) return launch_pf_cc_any<float>(p, a->head_dim, a->num_tasks, s);
  if (a->head_dim < 64)  // tensor-core tiles cover head_dim 64 and 128
    return a->dtype == WNW_BF16 ? launch_pf_cc_any<__nv_bfloat16>(p, a->head_dim, a->num_tasks, s)
                                : launch_pf_cc_any<__half>(p, a->head_dim, a->num_tasks, s);
  if (a->dtype == WNW_BF16)
    return a->head_dim == 128 ? launch_pf<__nv_bfloat16, 128>(p, a->num_tasks, s)
                              : launch_pf<__nv_bfloat16, 64>(p, a->num_tasks, s);
  return a->head_dim == 128 ? launch_pf<__half, 128>(p, a->num_tasks, s) : launch_pf<__half, 64>(p, a->num_tasks, s);
}
