/*
 * wnw_b200.h -- C ABI of the B200-native WnW decode hot path.
 *
 * One shared library (libwnw_b200.so, sm_100a) exports everything below.
 * All entry points take plain pointers, sizes and a cudaStream_t passed as
 * void*; none allocates device memory (the caller owns every buffer) and none
 * aborts: each returns a wnw_status, with a message from wnw_last_error().
 *
 * Every entry point names the reference interface it replaces
 * (paths relative to the XMUDeepLIT/WnW project root).
 */
#ifndef WNW_B200_H_
#define WNW_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WNW_ABI_VERSION 1

typedef enum wnw_status {
  WNW_OK = 0,
  WNW_ERR_INVALID = 1,     /* bad argument (size, alignment, dtype, null)   */
  WNW_ERR_CUDA = 2,        /* a CUDA runtime call failed                    */
  WNW_ERR_CAPACITY = 3,    /* a plan or buffer exceeds its stated capacity  */
  WNW_ERR_STATE = 4,       /* call out of order / inconsistent state        */
  WNW_ERR_TIMEOUT = 5,     /* a bounded wait ran out (device or host)       */
  WNW_ERR_UNSUPPORTED = 6  /* shape or dtype not compiled in                */
} wnw_status;

typedef enum wnw_dtype { WNW_F32 = 0, WNW_F16 = 1, WNW_BF16 = 2 } wnw_dtype;

/* Device error codes written by kernels into the caller's err word. */
#define WNW_DEVERR_MBAR_TIMEOUT 1   /* a TMA mbarrier wait ran out           */
#define WNW_DEVERR_LEN_MISMATCH 2   /* rebuild plan disagrees with seg_len   */
#define WNW_DEVERR_CAPACITY 4       /* a segment would exceed its slot       */
#define WNW_DEVERR_PEER_TIMEOUT 8   /* a tensor-parallel peer's partials did not arrive */
#define WNW_DEVERR_BAD_INDEX 16     /* a device-side table index out of range (device fetch plan, prefill score task) */

int wnw_abi_version(void);
const char* wnw_status_string(wnw_status s);
/* Last error message of the calling thread ("" when none). */
const char* wnw_last_error(void);

/* ------------------------------------------------------------------ *
 * Decode attention (replaces src/common/kv/fused_attn.py:9-156,
 * q1_decode_attn / q1_decode_attn_score, and the varlen_attn call of
 * src/algorithms/wnw/code/session.py:90-106).
 *
 * Segment s (= b * num_kv_heads + h) holds seg_len[s] rows starting at row
 * seg_base[s] of k_store / v_store ([rows, head_dim], row-major).  When
 * new_k/new_v are given, the step's new token is attended as row seg_len[s]
 * and written there (fused append; src/common/kv/kernels.py:7-73), so the
 * caller advances seg_len by one afterwards (wnw_advance_lengths).
 * Two launch layouts:
 *  - tensor-core path (16-bit K/V, head_dim 64 or 128): `plan` (device) is
 *    the layer's work plan from wnw_attn_plan -- every CTA attends one row
 *    range of one segment, a segment's CTAs share one thread-block cluster of
 *    `cluster_size` CTAs and merge through distributed shared memory, and a
 *    segment too long for one cluster spans several: each writes its partial,
 *    arrives at the segment's counter, and the last to arrive merges the
 *    partials in order -- with plan_ctas / cluster_size / plan_parts /
 *    plan_combine copied from its wnw_attn_plan_info.  work / n_clusters /
 *    split_rows are not used; counters only when plan_combine > 0.
 *  - CUDA-core path (fp32, or head_dim 16 / 32): work is split into
 *    `split_rows`-row pieces grouped into clusters of `cluster_size` CTAs;
 *    `work` lists (segment, cluster index within the segment) pairs covering
 *    every cluster a segment may need (wnw_build_work_table).
 * Outputs o[s, g, :] = softmax(q.K^T*scale).V in the
 * q dtype with fp32 accumulation.  For segments with score_slot[s] >= 0 the
 * kernel also stores the base-2 logits of the audio rows
 * [audio_start[b], audio_end[b]) into logits + logits_off[slot] ([t][g]) and
 * the merged per-head softmax statistics into stats[s] ([2][group]: max, sum),
 * from which wnw_score_finalize forms the class-A scores.
 * The layout inputs -- seg_base, seg_cap, the plan or work table and the
 * scoring tables (score_slot, audio_start / audio_end, logits_off) -- are
 * read before the kernel waits for the preceding kernel in the stream
 * (programmatic dependent launch): they must not be written by a kernel that
 * may still run when the launch starts.
 * ------------------------------------------------------------------ */
typedef struct wnw_decode_attn_args {
  int dtype;           /* wnw_dtype of q, k/v stores, new_k/new_v and out   */
  int head_dim;        /* 16, 32, 64 or 128                                  */
  int group;           /* q heads per kv head, 1..8                          */
  int num_segs;        /* batch * num_kv_heads                               */
  int num_kv_heads;
  const void* q;       /* [num_segs, group, head_dim]                        */
  const void* new_k;   /* [num_segs, head_dim] or NULL (no append)           */
  const void* new_v;
  void* k_store;       /* [rows, head_dim]                                   */
  void* v_store;
  const int64_t* seg_base;  /* [num_segs] first row of each segment          */
  const int32_t* seg_len;   /* [num_segs] rows stored before this step       */
  const int32_t* seg_cap;   /* [num_segs] slot capacity or NULL (unchecked)  */
  const int32_t* work;      /* [n_clusters][2] (segment, cluster-in-segment) */
  int n_clusters;
  int cluster_size;         /* 1, 2, 4, 8 or 16 (16: non-portable size); the
                               plan's cluster on the tensor-core path          */
  int split_rows;           /* rows per CTA; wnw_split_rows()                */
  void* out;                /* [num_segs, group, head_dim]                   */
  float scale;
  /* class-A scoring (all NULL when unused) */
  const int32_t* score_slot;     /* [num_segs] -1 or slot index              */
  const int32_t* audio_start;    /* [batch] audio rows within a segment      */
  const int32_t* audio_end;
  float* logits;                 /* base-2 logits, see above                 */
  const int64_t* logits_off;     /* [n_slots] element offset of each slot    */
  float* stats;                  /* [num_segs][2][group] or NULL             */
  /* scratch: partials [n_clusters, or plan_parts][group][head_dim + 2]
     fp32, counters [num_segs] int32 (CUDA-core path, and plans with combine
     entries; zero before first use, kernels leave them zero) */
  float* partials;
  int32_t* counters;
  int32_t* err;                  /* device error word (WNW_DEVERR_* bits)    */
  int64_t store_rows;            /* rows of k_store / v_store (the TMA extent) */
  /* tensor-core path: the layer's plan (see above) */
  const int32_t* plan;           /* wnw_attn_plan output, on the device      */
  int plan_ctas, plan_parts, plan_combine;
  int flags;                     /* WNW_ATTN_ROWS_READY or 0                 */
} wnw_decode_attn_args;

/* flags: the caller guarantees that seg_len and the stored K/V rows
 * [seg_base, seg_base + seg_len) are not being written by any kernel that may
 * still run when this launch starts (they were final before the preceding
 * kernels in the stream started; q, new_k and new_v may still come from
 * them).  The tensor-core kernel then reads the lengths and starts streaming
 * rows before it waits for the preceding kernel (programmatic dependent
 * launch). */
#define WNW_ATTN_ROWS_READY 1

wnw_status wnw_decode_attn(const wnw_decode_attn_args* a, void* stream);

/* wnw_decode_attn with the four per-step pointers given separately: `a`
 * holds the layer's constant part (layout, work table, scratch, scoring) and
 * is not modified.  No reference counterpart: saves the host from rewriting
 * the argument block every layer of every step. */
wnw_status wnw_decode_attn_step(const wnw_decode_attn_args* a, const void* q, const void* new_k,
                                const void* new_v, void* out, void* stream);

/* Allocation-free variant of wnw_decode_attn.  It has no counterpart in the
 * reference.  It is for callers that cannot allocate device memory because
 * their host owns every byte of it (a serving engine with a fixed, pre-split
 * memory budget; a plugin host that only hands in its own buffers), where a
 * cudaMalloc would fail or escape the host's accounting.  The partial-state
 * and counter scratch come from a file-scope device array of
 * WNW_NOALLOC_MAX_PARTIAL_FLOATS floats + WNW_NOALLOC_MAX_SEGS counters (about
 * 4.3 MB, held by every device that loads the library until exit); a->partials
 * and a->counters are ignored, every other field means what it means for
 * wnw_decode_attn, and a->err is required.  Larger requests return
 * WNW_ERR_CAPACITY.  Calls share the array: calls that overlap on the GPU race.
 * The first call in a CUDA context looks up the array's address there (make it
 * before any stream capture), and a call made after the device's context
 * changed (a cudaDeviceReset) looks it up again; each call clears the
 * counters it uses. */
#define WNW_NOALLOC_MAX_PARTIAL_FLOATS (1 << 20)
#define WNW_NOALLOC_MAX_SEGS (1 << 16)
wnw_status wnw_decode_attn_noalloc(const wnw_decode_attn_args* a, void* stream);

/* Rows per CTA of the CUDA-core decode attention for a dtype / head_dim;
 * 0 for the tensor-core path (16-bit K/V with head_dim 64 or 128), which
 * takes a plan instead (wnw_attn_plan). */
int wnw_split_rows(int dtype, int head_dim);

/* Work plan of the tensor-core decode attention for one layer (no reference
 * counterpart: the reference's kernels take one CTA per segment).  Segment s
 * may hold up to seg_cap[s] + 1 rows at a launch (its capacity plus the
 * step's token), counted in 32-row units.  Every CTA takes about the same
 * units -- an equal share of the CTA slots the device holds at once, raised
 * (to at most 1,536 rows) so the longest segment fits one cluster of
 * `max_cluster` CTAs -- and a segment needing k CTAs gets k consecutive
 * ranks of one cluster (clusters hold the smallest power of two >= the
 * largest such k, at most max_cluster; short segments share clusters), the
 * share raised further if needed so the clusters fit one wave of those the
 * device holds at once.  When the longest segment does not fit one cluster
 * that way, or the equal share itself exceeds 1,536 rows, clusters hold at
 * most 4 CTAs, the share is sized to whole waves of the resident slots (of 1
 * to 4 waves, the count whose waves x (share + 512 rows of fixed cost) is
 * least), and a segment needing more CTAs than a cluster holds takes whole
 * clusters, each writing a partial that the last of them to finish merges.
 * sm_count <= 0: the current device's SMs and its resident clusters of the
 * kernel (otherwise sm_count stands for the slots at every cluster size);
 * max_cluster <= 0: 16 when the device holds clusters of 16 of the kernel,
 * else 8.  Layout of `plan` (int32):
 *   [0..7]  ctas, cluster, parts, combine, 0, 0, 0, 0
 *   [8 ..]  ctas x {segment (-1: idle rank), row_begin, row_end, meta}
 *           meta = leader rank | ranks << 5 | writes a partial << 10 |
 *                  partial slot << 11
 *   then    parts x first row of the partial's range (padded to 4 ints)
 *   then    combine x {segment, first partial, partials, 0}
 * Writes info (sizes) always and the plan when max_ints >= info->ints; with
 * plan == NULL and max_ints == 0 it only sizes; otherwise a plan too small
 * returns WNW_ERR_CAPACITY. */
typedef struct {
  int ctas, cluster, parts, combine;
  int64_t ints;
} wnw_attn_plan_info;
wnw_status wnw_attn_plan(const int32_t* seg_cap, int num_segs, int sm_count, int max_cluster, int32_t* plan,
                         int64_t max_ints, wnw_attn_plan_info* info);
/* Clusters of `cluster` CTAs (1..16) of the tensor-core decode-attention
 * kernel (head_dim 64 or 128) the current device holds at once
 * (cudaOccupancyMaxActiveClusters); wnw_attn_plan sizes its waves by it. */
wnw_status wnw_attn_resident_clusters(int head_dim, int cluster, int* n);

/* Launch shape for one layer (no reference counterpart: the reference's
 * kernels take one CTA per segment).  From the per-segment row capacities,
 * gives the CUDA-core kernel's split_rows and the cluster size (the
 * smallest power of two, up to 8, covering the longest segment's splits);
 * the tensor-core path takes a plan instead (WNW_ERR_INVALID here). */
wnw_status wnw_attn_launch_shape(int dtype, int head_dim, const int32_t* seg_cap, int num_segs,
                                 int* split_rows, int* cluster_size);

/* Build the cluster work table on the host from per-segment row capacities
 * (a segment needs ceil((cap+1)/split_rows) splits).  Writes up to max_clusters
 * pairs and the count (work == NULL with max_clusters == 0 only counts);
 * WNW_ERR_CAPACITY when max_clusters is too small.  Segments that need
 * several clusters come first; each segment's clusters are consecutive. */
wnw_status wnw_build_work_table(const int32_t* seg_cap, int num_segs, int split_rows,
                                int cluster_size, int32_t* work, int max_clusters,
                                int* n_clusters);

/* seg_len[i] += 1 for i < n (device), after a step's fused appends. */
wnw_status wnw_advance_lengths(int32_t* seg_len, int64_t n, void* stream);

/* ------------------------------------------------------------------ *
 * Class-A score finalisation + chunk scoring + top-k
 * (replaces the accumulation of src/common/kv/fused_attn.py:107-121 and
 * src/algorithms/wnw/code/kernels.py:302-370, and the selection of
 * src/algorithms/wnw/code/cache.py:632-649 /
 * src/algorithms/wnw_cpp/code/cache.py:160-171).
 * ------------------------------------------------------------------ */
/* Term table: for sample b, terms [term_off[b], term_off[b+1]) in order;
 * term i reads logits at logits + logit_off[i] ([t][group]) and statistics at
 * stats + stat_off[i] ([2][group]) and sums heads set in qmask[i].
 * acc[score_off[b] + t] = sum_i sum_{g in qmask[i]} 2^(x - max_g) / sum_g. */
wnw_status wnw_score_finalize(const float* logits, const float* stats, const int64_t* logit_off,
                              const int64_t* stat_off, const uint32_t* qmask,
                              const int32_t* term_off, int group, int batch,
                              const int32_t* score_off, int max_audio, float* acc,
                              void* stream);

/* Chunk scores + top-k per sample from a class-A score vector.
 * Chunk c of sample b spans segments [c, min(c+segs_per_chunk, n_seg_b)) with
 * segments of `stride` rows over audio_len[b] = score_off[b+1]-score_off[b].
 * score = (P[end]-P[start]) / max(1, end-start) with P the fp32-rounded
 * prefix sum (accumulated in fp64, like torch's CPU cumsum).  Writes
 * topk[b*top_k + j] (descending score, ties -> lower index; -1 padding) and
 * chunk_scores (optional, [sum of chunk counts] at chunk_off[b]).  max_audio
 * bounds every sample's audio length (it sizes shared memory). */
wnw_status wnw_chunk_topk(const float* acc, const int32_t* score_off, int batch, int max_audio,
                          int stride, int segs_per_chunk, int top_k, int32_t* topk,
                          float* chunk_scores, const int32_t* chunk_off, void* stream);

/* ------------------------------------------------------------------ *
 * In-place layout maintenance
 * ------------------------------------------------------------------ */
/* Compaction + splice of the changed segments of one layer (replaces
 * rebuild_append_kv, src/algorithms/wnw/code/kernels.py:375-473, and
 * WnWCache._apply_chunk_update_to_layer, cache.py:891-1010).  `plan_blob` is
 * the blob written by wnw_planner_device_plan and `layer` selects its record.
 * Two grid-stride launches: the kept rows that move are gathered into
 * k_move/v_move (>= the record's moved_total rows) while every plan record is
 * validated against seg_len / seg_cap (status[n_chg] scratch); then moved and
 * fetched (`landing`) rows are written to their final slot rows and seg_len
 * is set.  A record that fails validation moves nothing and sets
 * WNW_DEVERR_LEN_MISMATCH (or _CAPACITY) in *err.  Every index the blob
 * holds is checked against the sizes given here before it is used: the
 * layer record against blob_ints (ints in plan_blob), segment numbers against
 * num_segs (the entries of seg_base / seg_len / seg_cap, and of status),
 * landing rows against land_rows (rows of k_landing / v_landing), moved rows
 * against move_rows -- a malformed layer record makes the whole call a no-op
 * with the error bit set. */
wnw_status wnw_rebuild_segments(int dtype, int head_dim, void* k_store, void* v_store,
                                const int64_t* seg_base, int32_t* seg_len, const int32_t* seg_cap,
                                int num_segs, const void* k_landing, const void* v_landing,
                                int64_t land_rows, const int32_t* plan_blob, int64_t blob_ints,
                                int layer, void* k_move, void* v_move, int64_t move_rows,
                                int32_t* status, int32_t* err, void* stream);
/* The rebuilds of one step's changed layers in one call (no reference
 * counterpart: the per-layer issue loop of wnw_rebuild_segments done
 * natively, so the host spends microseconds, not tens of them, per layer).
 * For each l < num_layers with layer_changed[l] != 0 (a host array): the
 * stream waits for wait_events[l] (cudaEvent_t; NULL entries or a NULL
 * array: no wait), layer l's rebuild runs with k_store[l], v_store[l],
 * seg_base[l], seg_len[l], seg_cap[l], num_segs[l] and the shared landing,
 * plan, move, status and error buffers, then record_events[l] is recorded
 * (same NULL rules).  Stops at the first failing call and returns its
 * status. */
wnw_status wnw_rebuild_layers(int dtype, int head_dim, int num_layers, const int32_t* layer_changed,
                              void* const* k_store, void* const* v_store, const int64_t* const* seg_base,
                              int32_t* const* seg_len, const int32_t* const* seg_cap, const int32_t* num_segs,
                              const void* k_landing, const void* v_landing, int64_t land_rows,
                              const int32_t* plan_blob, int64_t blob_ints, void* k_move, void* v_move,
                              int64_t move_rows, int32_t* status, int32_t* err, void* const* wait_events,
                              void* const* record_events, void* stream);
/* The same rebuilds as wnw_rebuild_layers in one gather and one scatter
 * launch for all the changed layers (per 48 changed layers), for steps whose
 * fetched rows are all in device memory before the first rebuild is needed
 * (no reference counterpart; the reference rebuilds each layer in its own
 * kernel, src/algorithms/wnw/code/cache.py:716-754).  The stream waits for
 * every changed layer's wait_events[l] first, and every changed layer's
 * record_events[l] is recorded after the last launch.  Layer l (the i-th
 * changed layer of its launch) keeps its moved rows in the move buffers from
 * the row that sums the moved-row totals of the launch's earlier changed
 * layers (read from their plan records), so move_rows must cover the sum of
 * the changed layers' moved rows; its status words start at the sum of the
 * earlier changed layers' num_segs, so status_len must be at least the sum
 * over all changed layers.  Every check of wnw_rebuild_segments applies per
 * layer; a layer whose moved rows do not fit sets WNW_DEVERR_CAPACITY and
 * moves nothing.  Layouts and lengths equal those of the per-layer calls. */
wnw_status wnw_rebuild_layers_fused(int dtype, int head_dim, int num_layers, const int32_t* layer_changed,
                                    void* const* k_store, void* const* v_store, const int64_t* const* seg_base,
                                    int32_t* const* seg_len, const int32_t* const* seg_cap, const int32_t* num_segs,
                                    const void* k_landing, const void* v_landing, int64_t land_rows,
                                    const int32_t* plan_blob, int64_t blob_ints, void* k_move, void* v_move,
                                    int64_t move_rows, int32_t* status, int64_t status_len, int32_t* err,
                                    void* const* wait_events, void* const* record_events, void* stream);

/* Copy rows [0, len[s]) of every segment from src (+src_base[s]) to dst
 * (+dst_base[s]); src and dst must not overlap.  Used to pack a slot layout
 * into the reference's flat layout and back, and to grow slots. */
wnw_status wnw_copy_segments(int dtype, int head_dim, const void* src_k, const void* src_v,
                             const int64_t* src_base, void* dst_k, void* dst_v,
                             const int64_t* dst_base, const int32_t* len, int num_segs,
                             void* stream);

/* Reference-layout append (out-of-place, src/common/kv/kernels.py:7-73):
 * out segment s = old[cu_old[s]:cu_old[s+1]] ++ new_tokens[s]. */
wnw_status wnw_interleave_append(int dtype, int head_dim, const void* old, const void* new_tokens,
                                 const int32_t* cu_old, int num_segs, void* out, void* stream);

/* ------------------------------------------------------------------ *
 * Planner (replaces the pybind11 class Planner,
 * src/algorithms/wnw_cpp/code/planner.cpp:19-341; same method names and
 * argument meaning, int32 host arrays instead of CPU tensors).
 * ------------------------------------------------------------------ */
typedef struct wnw_planner wnw_planner;

wnw_status wnw_planner_create(int num_layers, int num_kv_heads, int batch_size, int num_kv_groups,
                              wnw_planner** out);
void wnw_planner_destroy(wnw_planner* p);
wnw_status wnw_planner_set_config(wnw_planner* p, int top_k_chunks, int eviction_lag);
wnw_status wnw_planner_set_seg_count(wnw_planner* p, const int32_t* seg_count, int n);
wnw_status wnw_planner_set_chunk_to_segs(wnw_planner* p, int b, const int32_t* flat_segs, int n_flat,
                                         const int32_t* offsets, int n_offsets);
wnw_status wnw_planner_set_class_b(wnw_planner* p, int layer, const int32_t* kv_heads, int n);
/* Flattened [L][num_segs][seg_count[b]] (planner.cpp:53-80). */
wnw_status wnw_planner_set_restore_meta(wnw_planner* p, const int32_t* cpu_s, const int32_t* cpu_e,
                                        const int32_t* gpu_s, const int32_t* gpu_e, int64_t n);
wnw_status wnw_planner_set_loaded(wnw_planner* p, int b, const int32_t* segs, int n);
wnw_status wnw_planner_set_seq_lens(wnw_planner* p, const int32_t* seq_lens, int64_t n);
wnw_status wnw_planner_get_loaded_segments(const wnw_planner* p, int b, int32_t* out, int cap,
                                           int* n_out);
/* planner.cpp:124-306.  Output arrays as in the reference ([L,nseg],
 * [L,nseg+1], [L], [L+1]); they are written only when *any_change is 1. */
wnw_status wnw_planner_compute_and_prepare(wnw_planner* p, const int32_t* topk_idx,
                                           const int32_t* topk_off, int32_t* load_starts_2d,
                                           int32_t* load_lens_2d, int32_t* cu_new_2d,
                                           int32_t* new_lens_2d, int32_t* evict_offsets_2d,
                                           int32_t* evict_max, int32_t* evict_layer_ptr,
                                           int* any_change, int* total_tokens);
/* Results of the last compute_and_prepare (the tuple's ev_starts, ev_ends,
 * cpu_ranges).  *n receives the count; arrays are copied when cap suffices. */
wnw_status wnw_planner_get_evictions(const wnw_planner* p, int32_t* starts, int32_t* ends, int cap,
                                     int* n);
wnw_status wnw_planner_get_cpu_ranges(const wnw_planner* p, int32_t* ranges, int cap_pairs,
                                      int* n_pairs);
/* Transfer-row offset ([L+1]) and cpu-range offset ([L+1], may be NULL) of
 * each layer's loads in the gathered order. */
wnw_status wnw_planner_get_layer_transfer(const wnw_planner* p, int32_t* layer_rows,
                                          int32_t* layer_ranges);
/* Per-sample to_load / to_evict of the last call (sorted segment ids). */
wnw_status wnw_planner_get_changes(const wnw_planner* p, int b, int32_t* to_load, int cap_load,
                                   int* n_load, int32_t* to_evict, int cap_evict, int* n_evict);
/* Device-plan blob for wnw_rebuild_segments: int32 [L+1] layer offsets, then
 * per layer {n_chg, moved_total, out_total, seg[n], old_len[n], new_len[n],
 * load_src[n], load_len[n], mov_off[n+1], out_off[n+1], ev_off[n+1],
 * ev_s[m], ev_e[m]} with lengths EXCLUDING the step's new token; moved rows
 * of a segment = its kept rows after the first evicted range, output rows =
 * moved + loaded. */
wnw_status wnw_planner_device_plan(const wnw_planner* p, int32_t* blob, int64_t cap, int64_t* used);

/* Gather the planned CPU ranges (cpu_ranges order) of row_bytes-wide rows from
 * src_k/src_v into dst_k/dst_v (pinned staging), using up to n_threads host
 * threads (planner.cpp:104-122). */
wnw_status wnw_gather_rows(const void* src_k, const void* src_v, int64_t row_bytes,
                           const int32_t* ranges, int n_pairs, void* dst_k, void* dst_v,
                           int n_threads);

/* Device address of pinned (page-locked, mapped) host memory, for
 * wnw_fetch_rows; WNW_ERR_CUDA when the memory is not mapped. */
wnw_status wnw_host_device_pointer(const void* host_ptr, void** dev_ptr);

/* Zero-copy fetch (replaces the staging gather + H2D copy of
 * src/algorithms/wnw/code/cache.py:868-889 / planner.cpp:113-122): the GPU
 * reads rows [ranges[i][0], ranges[i][1]) of src_k/src_v (device addresses of
 * pinned host memory, row_bytes per row) and writes them to dst_k/dst_v at row
 * dst_row[i].  ranges and dst_row are device arrays; at most max_ctas CTAs. */
wnw_status wnw_fetch_rows(const void* src_k, const void* src_v, int64_t row_bytes,
                          const int32_t* ranges, const int64_t* dst_row, int n_ranges,
                          void* dst_k, void* dst_v, int max_ctas, void* stream);

/* All layers of a step's fetch: for layer l, wnw_fetch_rows over ranges
 * [layer_ranges[l], layer_ranges[l+1]) (host array, [num_layers+1]) followed
 * by cudaEventRecord(events[l]) on `stream` (events may be NULL), so the
 * consumer of layer l waits for its rows only. */
wnw_status wnw_fetch_layers(const void* src_k, const void* src_v, int64_t row_bytes,
                            const int32_t* ranges, const int64_t* dst_row, const int32_t* layer_ranges,
                            int num_layers, void* dst_k, void* dst_v, int max_ctas, void* stream,
                            void* const* events);

/* After wnw_planner_compute_and_prepare reported a change, hand the plan to
 * the device in one call (the reference's staging gather + side-stream copy,
 * src/algorithms/wnw/code/cache.py:868-889 and planner.cpp:104-122, as one
 * host call): writes the device-plan blob into plan_host (pinned) and copies
 * it to plan_dev; writes the host ranges and their landing rows into
 * ranges_host / dst_host (pinned) and copies them to ranges_dev / dst_dev;
 * then wnw_fetch_layers from src_k / src_v (device addresses of the pinned
 * restore store) into land_k / land_v, recording events[l] after layer l --
 * all on `stream`.  With all buffers given, the copies, the per-layer
 * fetches and the event records run as one CUDA graph built once per set of
 * buffers (one graph launch per call).  info receives the sizes and, per layer, whether it
 * changed; if a capacity (plan ints, range pairs, landing rows) is too small
 * nothing is issued and WNW_ERR_CAPACITY is returned with info filled.
 * The pinned buffers must not be read by copies still in flight from a
 * previous call (synchronize `stream` first). */
typedef struct {
  int64_t plan_ints, total_rows, n_ranges, max_moved_rows;
  int64_t fetch_launches; /* fetch kernels this call ran                   */
  int32_t* layer_changed; /* caller-owned [num_layers]                     */
} wnw_fetch_info;
wnw_status wnw_planner_issue_fetch(const wnw_planner* p, int32_t* plan_host, int32_t* plan_dev, int64_t plan_cap,
                                   int32_t* ranges_host, int32_t* ranges_dev, int64_t* dst_host, int64_t* dst_dev,
                                   int64_t ranges_cap, const void* src_k, const void* src_v, int64_t row_bytes,
                                   void* land_k, void* land_v, int64_t land_rows, int max_ctas, void* stream,
                                   void* const* events, wnw_fetch_info* info);

/* The step's rebuild plan only: after wnw_planner_compute_and_prepare
 * reported a change, write the device-plan blob into plan_host (pinned) and
 * copy it to plan_dev on `stream`; fill info (plan ints, landed rows, ranges,
 * moved rows, changed layers).  The fetch itself is not issued: this is the
 * host half of the device-planned step (wnw_dplan_step below).  Replaces the
 * plan-blob part of the reference's staging path
 * (src/algorithms/wnw/code/cache.py:868-889).  WNW_ERR_CAPACITY (nothing
 * copied, info filled) when plan_cap is too small. */
wnw_status wnw_planner_upload_plan(const wnw_planner* p, int32_t* plan_host, int32_t* plan_dev, int64_t plan_cap,
                                   void* stream, wnw_fetch_info* info);

/* Device mirror of the planner's selection state, so that a step's fetch is
 * planned on the GPU straight from the device top-k and starts with no host
 * round trip.  No reference counterpart as a call: it restates, on the
 * device, the selection diff and range emission of the reference planner
 * (src/algorithms/wnw_cpp/code/planner.cpp:124-306; the Python path's
 * cache.py:609-630 and 771-823) for the fetch only; the host planner still
 * plans the rebuild and checks the device's result (wnw_dplan_verify).
 *
 * create: copies the planner's tables and current loaded sets / eviction
 *   counters to the device (synchronous; call after the prefill state is
 *   handed to the planner).  WNW_ERR_UNSUPPORTED when the per-step state does
 *   not fit one thread block's shared memory (the caller keeps the host path).
 * step: on compute_stream, one kernel turns the top-k rows topk_dev
 *   ([B][topk_stride] chunk ids, -1 padded) into this step's loads (updating
 *   the mirrored loaded sets and counters exactly as the planner does) and
 *   their host ranges and landing rows; then copy_stream waits for it and runs
 *   the per-layer fetch (src_k / src_v -> land_k / land_v, events[l] after
 *   layer l) as one CUDA graph.  Bad indices or a landing overflow set
 *   WNW_DEVERR_BAD_INDEX / WNW_DEVERR_CAPACITY in *err and fetch nothing.
 * verify: after the host has waited for the step and run
 *   wnw_planner_compute_and_prepare on the same top-k, compare the device's
 *   per-layer landing rows, loaded sets and counters with the planner's;
 *   WNW_ERR_STATE on any difference. */
typedef struct wnw_dplan wnw_dplan;
wnw_status wnw_dplan_create(const wnw_planner* p, wnw_dplan** out);
void wnw_dplan_destroy(wnw_dplan* dp);
wnw_status wnw_dplan_step(wnw_dplan* dp, const int32_t* topk_dev, int topk_stride, int32_t* err,
                          const void* src_k, const void* src_v, int64_t row_bytes, void* land_k, void* land_v,
                          int64_t land_rows, int max_ctas, void* compute_stream, void* copy_stream,
                          void* const* events);
wnw_status wnw_dplan_verify(const wnw_dplan* dp, const wnw_planner* p);

/* Kernel copy of `bytes` (a multiple of 16, 16-byte aligned) from `src` --
 * typically the device address of pinned host memory (wnw_host_device_pointer)
 * -- to `dst`, on `stream`.  No reference counterpart: a host->device copy
 * made of SM loads, which share the host link with the zero-copy fetch instead
 * of queueing behind it as a copy-engine transfer can. */
wnw_status wnw_copy_mapped(void* dst, const void* src, int64_t bytes, int max_ctas, void* stream);

/* Async copy of n bytes in either direction (cudaMemcpyDefault: unified
 * addressing tells host from device) on `stream`.  No reference counterpart:
 * the step's small host<->device copies in one call each. */
wnw_status wnw_copy_async(void* dst, const void* src, int64_t bytes, void* stream);

/* Make `stream` wait for `event` (cudaStreamWaitEvent; both as void*).  No
 * reference counterpart: the per-layer "rows of layer l have landed" wait of
 * the decode loop in one call. */
wnw_status wnw_stream_wait_event(void* stream, void* event);

/* Async H2D copy of n bytes for K and V on `stream`, then record `event`
 * (cudaEvent_t as void*, may be NULL) -- one per layer. */
wnw_status wnw_h2d_async(void* dst_k, void* dst_v, const void* src_k, const void* src_v,
                         int64_t bytes, void* stream, void* event);

/* ------------------------------------------------------------------------
 * Tensor parallelism by kv head: the per-layer o_proj exchange (no reference
 * counterpart -- the reference runs one request per GPU; its o_proj is the
 * model's dense projection, src/algorithms/wnw/code/session.py drives it).
 *
 * y[B, N] = sum over ranks r of x_r[B, K] . W_r[N, K]^T, where x_r is rank
 * r's attention output (its query heads) and W_r the matching column slice of
 * o_proj, in one kernel per rank: each CTA computes its chunk of this rank's
 * partial sums, stores them into every rank's receive buffer over NVLink,
 * raises a per-chunk flag there, waits for every rank's flag in its own
 * memory and adds the partials in rank order (bit-identical y on every rank).
 * recv[p] / flags[p]: rank p's buffers as mapped in this process
 * (wnw_ipc_open; p == rank: this rank's own allocation), sized
 *   recv:  2 * world * recv_batch * n_out fp32,
 *   flags: world * wnw_oproj_allreduce_chunks(n_out) u32, zeroed once.
 * epoch: 1, 2, 3, ... per call, the same on every rank.  A peer whose flag
 * does not arrive within timeout_ns (0: 2 s) sets WNW_DEVERR_PEER_TIMEOUT in
 * *err and the kernel returns with zeros in y. */
#define WNW_TP_MAX_RANKS 8
typedef struct {
  int dtype;                            /* WNW_BF16 or WNW_F16 (x, W, y) */
  int batch, n_out, k_in;               /* B <= 8, N, K (K % 8 == 0)     */
  int recv_batch;                       /* rows per rank and parity the recv
                                           buffers were sized for (their
                                           layout stride); batch > recv_batch
                                           returns WNW_ERR_CAPACITY      */
  int rank, world;                      /* world <= WNW_TP_MAX_RANKS     */
  const void* x;                        /* [B, K]                        */
  const void* w;                        /* [N, K] row-major              */
  void* y;                              /* [B, N]                        */
  float* recv[WNW_TP_MAX_RANKS];
  uint32_t* flags[WNW_TP_MAX_RANKS];
  uint32_t epoch;
  uint64_t timeout_ns;
  int32_t* err;
} wnw_oproj_allreduce_args;
wnw_status wnw_oproj_allreduce(const wnw_oproj_allreduce_args* a, void* stream);
/* CTAs (and flag slots per rank) of wnw_oproj_allreduce for n_out outputs. */
int wnw_oproj_allreduce_chunks(int n_out);

/* Device buffers shared across processes (CUDA IPC): allocate + zero + export
 * a 64-byte handle; open a peer's handle; close (owned: cudaFree, else
 * cudaIpcCloseMemHandle). */
wnw_status wnw_ipc_alloc(int64_t bytes, void** ptr, void* handle);
wnw_status wnw_ipc_open(const void* handle, void** ptr);
wnw_status wnw_ipc_close(void* ptr, int owned);

/* ------------------------------------------------------------------------
 * Prefill audio scores (replaces _compute_prefill_scores and
 * _compute_head_scores, src/algorithms/wnw/code/session.py:121-201).
 *
 * Per task: the query rows are (head, position) pairs -- n_heads query heads
 * heads[head_off ...] at positions row0 .. row0 + n_rows - 1 of sample
 * `batch` -- scored against every key of kv head `kv_head`:
 *   x = rnd(rnd(rnd(q . k) * scaling) [+ mask])
 * with rnd the rounding to the model dtype (the reference's bf16 / fp16
 * matmul output, its scale and its mask add), then a softmax over all
 * seq_len keys in fp32, and
 *   out[out_off + j - audio_start] = sum over heads of the mean over
 *                                    positions of softmax[j]
 * for the audio keys j in [audio_start, audio_end).  The session's class-A
 * score is one task (the class-A query heads, the last position, the first
 * class-A head's kv head); each class-B kv head's score is one task (its
 * group of query heads, the last position or the post-audio text
 * positions).  Two launches: per-chunk row statistics, then the audio
 * columns.  Sums are taken in a fixed order, so results repeat bit for bit.
 * A task whose indices fall outside the given sizes sets
 * WNW_DEVERR_BAD_INDEX in *err and writes nothing. */
#define WNW_MASK_NONE 0      /* no mask added                              */
#define WNW_MASK_CAUSAL 1    /* keys after the query position get -inf     */
#define WNW_MASK_ADDITIVE 2  /* mask[b, position, key] added (model dtype) */
typedef struct {
  int32_t batch, kv_head;
  int32_t head_off, n_heads;      /* query heads: heads[head_off .. + n_heads) */
  int32_t row0, n_rows;           /* query positions                           */
  int32_t audio_start, audio_end; /* key columns written                       */
  int64_t out_off;
} wnw_prefill_task;
typedef struct {
  int dtype, head_dim;                  /* WNW_BF16 / WNW_F16; 64 or 128    */
  int batch, num_q_heads, num_kv_heads, seq_len;
  int num_tasks;                        /* <= 65535                         */
  int num_heads;                        /* entries of `heads`               */
  int max_rows;                         /* >= n_heads * n_rows of any task  */
  int max_audio;                        /* >= audio_end - audio_start       */
  const void* q;                        /* [B, Hq, S, D] by the strides     */
  int64_t q_stride_b, q_stride_h, q_stride_s;   /* elements, multiples of 8 */
  const void* k;                        /* [B, Hkv, S, D]                   */
  int64_t k_stride_b, k_stride_h, k_stride_s;
  int mask_kind;                        /* WNW_MASK_*                       */
  const void* mask;                     /* [B, S, S], keys contiguous       */
  int64_t mask_stride_b, mask_stride_s;
  float scaling;
  const wnw_prefill_task* tasks;        /* device                           */
  const int32_t* heads;                 /* device                           */
  float* out;                           /* device                           */
  int64_t out_len;                      /* floats at out                    */
  void* scratch;                        /* device, >= scratch_bytes         */
  int64_t scratch_bytes;
  int32_t* err;                         /* device error word                */
} wnw_prefill_scores_args;
wnw_status wnw_prefill_scores(const wnw_prefill_scores_args* a, void* stream);
/* Scratch bytes wnw_prefill_scores needs (per-chunk row statistics). */
wnw_status wnw_prefill_scores_scratch_bytes(int num_tasks, int max_rows, int seq_len, int64_t* bytes);

#ifdef __cplusplus
}
#endif
#endif /* WNW_B200_H_ */
