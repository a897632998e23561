"""``B200WnWCache``: drop-in replacement for the reference ``WnWCache`` /
``WnWCppCache`` (src/algorithms/wnw/code/cache.py, src/algorithms/wnw_cpp/
code/cache.py) whose decode path runs on the sm_100a kernels of
``libwnw_b200.so``.

Same constructor arguments, ``setup_audio`` and hook methods, so the
reference ``WnWSession`` (or ``wnw_b200.session.WnWSession``) and
``model.generate(past_key_values=cache)`` drive it unchanged.

Device layout (per layer): K and V stores ``[rows, head_dim]`` in the model
dtype; every (sample, kv head) segment ``s = b * num_kv_heads + h`` owns the
slot ``[seg_base[s], seg_base[s] + seg_cap[s])`` and its first ``seg_len[s]``
rows hold exactly the rows of the reference's flat segment, in the same
order.  Appends write one row into the slot; a chunk update moves rows only
inside the changed slots.  ``packed_layer`` materialises the reference's flat
``[total_tokens, head_dim]`` + ``cu_seqlens`` view.

Per decode step:
  layer l:  [wait for layer l's H2D rows] rebuild changed slots (if a plan is
            pending) -> one decode-attention launch (attention + append +
            class-A logits)
  end:      advance lengths -> class-A score finalisation -> chunk top-k ->
            (host) planner -> device plan + per-layer H2D of fetched rows on
            a copy stream, each layer with its own event.
"""
from __future__ import annotations

import ctypes as C
import math
import time
from itertools import accumulate

import numpy as np
import torch

from wnw_b200 import kernels as Kx
from wnw_b200 import native as N
from wnw_b200.flat_cache import FlatVarlenCache
from wnw_b200.planner import DevicePlan, Planner, gather_rows


def compute_segments(num_audio, stride):
    """Audio segments of ``stride`` tokens (cache.py:1092-1094)."""
    return [(i * stride, min(i * stride + stride, num_audio)) for i in range(math.ceil(num_audio / stride))]


def compute_chunks(segments, chunk_size, stride):
    """Chunk c = segments [c, c + ceil(chunk/stride)) (cache.py:1097-1101)."""
    spc = math.ceil(chunk_size / stride)
    n = len(segments)
    return [list(range(i, min(i + spc, n))) for i in range(n)]


def wait_event(event, timeout_s):
    """Wait for a CUDA event with a host deadline: WnwError(WNW_ERR_TIMEOUT)
    instead of blocking forever when the device never gets there."""
    if event.query():
        return
    deadline = time.perf_counter() + timeout_s
    n = 0
    while not event.query():  # a tight poll wakes as fast as a blocking sync
        n += 1
        if (n & 255) == 0 and time.perf_counter() > deadline:
            raise N.WnwError(5, "decode step", f"device work not finished after {timeout_s:g} s")


def keep_audio_indices(scores, seg_ranges, ratio, global_topk):
    """Kept audio tokens of a group of heads sharing one retention ratio:
    scores [n_heads, n_audio] -> int64 [n_heads, K], ascending per head.  Per
    segment (cache.py:1114-1138) every segment keeps its max(1, int(len *
    ratio)) best tokens; globally (cache.py:1141-1150) the span keeps the sum
    of those counts -- for all the heads in one batched top-k."""
    nh, n = scores.shape
    if not seg_ranges:  # a sample with no audio keeps (and offloads) nothing
        return torch.empty(nh, 0, dtype=torch.int64, device=scores.device)
    if global_topk:
        k = min(n, sum(max(1, int((b - a) * ratio)) for a, b in seg_ranges))
        return scores.topk(k, dim=1).indices.sort(dim=1).values
    stride = seg_ranges[0][1] - seg_ranges[0][0]
    full = len(seg_ranges) if seg_ranges[-1][1] - seg_ranges[-1][0] == stride else len(seg_ranges) - 1
    parts = []
    if full:
        k = max(1, int(stride * ratio))
        idx = scores[:, :full * stride].reshape(nh, full, stride).topk(k, dim=2).indices.sort(dim=2).values
        idx = idx + (torch.arange(full, device=scores.device) * stride).view(1, full, 1)
        parts.append(idx.reshape(nh, full * k))
    if full < len(seg_ranges):
        a, b = seg_ranges[-1]
        parts.append(scores[:, a:b].topk(max(1, int((b - a) * ratio)), dim=1).indices.sort(dim=1).values + a)
    return torch.cat(parts, dim=1) if len(parts) > 1 else parts[0]


def offload_counts(seg_ranges, ratio, global_topk):
    """Rows a class-B head offloads per segment (per-segment keep rule), or
    None per segment when the global rule makes them data-dependent; and
    the head's total."""
    if global_topk:
        n = seg_ranges[-1][1] if seg_ranges else 0
        k = min(n, sum(max(1, int((b - a) * ratio)) for a, b in seg_ranges))
        return None, n - k
    c = [(b - a) - max(1, int((b - a) * ratio)) for a, b in seg_ranges]
    return c, sum(c)


class B200WnWCache(FlatVarlenCache):
    """WnW KV cache on the B200 slot layout.

    Extra keyword arguments (all optional):
      max_decode_tokens -- decode rows reserved per slot (grown on demand);
      fetch_mode        -- "zerocopy" (default): a kernel on the copy stream
                           reads the offloaded rows straight from pinned host
                           memory; "dma": host threads gather them into pinned
                           staging and cudaMemcpyAsync copies each layer;
      fetch_threads     -- host threads of the "dma" gather;
      fetch_ctas        -- CTAs of the zero-copy fetch; by default 12 for
                           the host tier (~0.8 MB of host reads in flight
                           keep the link saturated; more only queue requests
                           in the memory system and slow the layer kernels
                           running beside the fetch) and 148 for the HBM tier
                           (a device-memory gather, one range per CTA);
      fetch_plan        -- "device" (default): each step's fetch is planned
                           on the GPU from the device top-k and starts at
                           once, while the host planner plans the rebuild and
                           checks the device's result; "host": the host plans
                           the fetch after reading the top-k back;
      wait_timeout_s    -- the step waits this long for its scores and
                           errors on the device, then raises a timeout error;
      offload_tier      -- where class-B offloaded rows live: "host" (pinned
                           host memory, the reference's CPU offload; default)
                           or "hbm" (device memory, for deployments whose HBM
                           budget holds them: the same gather then reads HBM
                           instead of crossing the host link, and with
                           rebuild_ahead each step's rebuilds run as one
                           launch pair for all layers);
      score_reduce      -- tensor parallelism by kv head (wnw_b200.tp): a
                           callable that sums the class-A score accumulator
                           over the ranks before every chunk selection.
    """

    def __init__(self, config, num_layers, num_kv_heads, num_q_heads, head_dim, device, adapter=None, *,
                 max_decode_tokens=256, fetch_mode="zerocopy", fetch_threads=8, fetch_ctas=None, score_reduce=None,
                 offload_tier="host", wait_timeout_s=60.0, fetch_plan="device", rebuild_ahead=True):
        super().__init__(num_layers, num_kv_heads, num_q_heads, head_dim, device, adapter)
        if self.device.type != "cuda":
            raise RuntimeError("B200WnWCache needs a CUDA device; the CPU oracle lives in the test suite")
        if head_dim not in (16, 32, 64, 128):
            raise ValueError(f"head_dim {head_dim} not supported (16, 32, 64 or 128)")
        if not 1 <= self.num_kv_groups <= 8:
            raise ValueError(f"GQA group {self.num_kv_groups} not supported (1..8)")
        self.config = config
        self.max_decode_tokens = int(max_decode_tokens)
        if fetch_mode not in ("zerocopy", "dma"):
            raise ValueError(f"fetch_mode must be 'zerocopy' or 'dma', not {fetch_mode!r}")
        self.fetch_mode = fetch_mode
        if offload_tier not in ("host", "hbm"):
            raise ValueError(f"offload_tier must be 'host' or 'hbm', not {offload_tier!r}")
        if offload_tier == "hbm" and fetch_mode != "zerocopy":
            raise ValueError("offload_tier='hbm' is fetched by the gather kernel (fetch_mode='zerocopy')")
        self.offload_tier = offload_tier
        if fetch_plan not in ("device", "host"):
            raise ValueError(f"fetch_plan must be 'device' or 'host', not {fetch_plan!r}")
        self.fetch_plan = fetch_plan
        # rebuild every changed layer on its own stream as soon as its rows
        # land (the next step's attention of layer l waits for layer l only),
        # instead of on the compute stream right before layer l's attention
        self.rebuild_ahead = bool(rebuild_ahead)
        # the HBM tier's fetch lands every layer's rows within microseconds:
        # its rebuilds run as one launch pair for the whole step instead of a
        # pair per layer (the host tier keeps per-layer rebuilds, each behind
        # its own layer's fetch over the host link)
        self._fused_rebuild = self.rebuild_ahead and offload_tier == "hbm"
        self._rb_stream = None
        self._rb_events = None
        self._fused_ev = 0  # the rebuild event the fused rebuild records (its first changed layer's)
        self._rebuilt = None
        self._dplan = None
        self._dplan_args = None
        self.wait_timeout_s = float(wait_timeout_s)
        # seconds the host spent blocked in the step's wait for its tail (a
        # small total means the host, not the device, paces the steps)
        self.host_wait_s = 0.0
        self.fetch_threads = int(fetch_threads)
        self.fetch_ctas = int(fetch_ctas) if fetch_ctas is not None else (148 if offload_tier == "hbm" else 12)
        self.score_reduce = score_reduce
        self._dev_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self._rb_args = [None] * num_layers
        self._tail_args = None
        self._class_b_heads_by_layer = [config.get_layer_class_b(l) for l in range(num_layers)]
        self.batch_size = 0
        self.prefilled = False
        self._copy_stream = None

    # ------------------------------------------------------------- set-up
    def setup_audio(self, audio_starts, audio_ends, attention_mask=None):
        """cache.py:144-250: segments, chunks, score buffers, fresh state."""
        if self._copy_stream is not None:
            # the previous request's last step fetched ahead for a step that
            # never came: let it land before its buffers and plan go away
            self._copy_stream.synchronize()
        if self._rb_stream is not None:  # likewise its rebuilds issued ahead
            self._rb_stream.synchronize()
        self._dplan = self._dplan_args = None
        self._seg_rows = None
        super().setup_audio(audio_starts, audio_ends, attention_mask)
        a_s = [int(x) for x in audio_starts.tolist()]
        a_e = [int(x) for x in audio_ends.tolist()]
        pad = [int(x) for x in self.pad_lens.tolist()]
        B = self.batch_size = len(a_s)
        self._raw_audio_starts, self._raw_audio_ends, self.pad_lens_list = a_s, a_e, pad
        self._audio_starts_list = [s - p for s, p in zip(a_s, pad)]
        self._audio_ends_list = [e - p for e, p in zip(a_e, pad)]
        stride = self.config.stride_tokens
        self.segment_ranges = [compute_segments(self._audio_ends_list[b] - self._audio_starts_list[b], stride)
                               for b in range(B)]
        self.chunk_to_segs = [compute_chunks(self.segment_ranges[b], self.config.chunk_size_tokens, stride)
                              for b in range(B)]
        self.segs_per_chunk = math.ceil(self.config.chunk_size_tokens / stride)
        audio_lens = [self._audio_ends_list[b] - self._audio_starts_list[b] for b in range(B)]
        self._score_offsets_list = [0] + list(accumulate(audio_lens))
        self.max_audio = max(audio_lens) if audio_lens else 0
        dev = self.device
        self.score_offsets = torch.tensor(self._score_offsets_list, dtype=torch.int32, device=dev)
        self.score_accumulator = torch.zeros(self._score_offsets_list[-1], dtype=torch.float32, device=dev)
        self._prefill_scores = [[] for _ in range(B)]
        self.loaded_segments = [set() for _ in range(B)]
        L = self.num_layers
        self._pk = [None] * L          # packed prefill K / V (until the slot layout is built)
        self._pv = [None] * L
        self.seq_lens = [None] * L     # reference semantics: rows incl. this step's token once appended
        self._store_planned = False    # pinned restore store sized at the first prefill layer
        self._nonaudio = {}
        self.restore_meta = None
        self._pending = False
        self._rebuilt = [False] * self.num_layers
        self._decode_step = 0
        self._rows_ready = [False] * self.num_layers
        self.prefilled = False

    # ------------------------------------------------------------ prefill
    def prefill_before_attn(self, layer_idx):
        self.stats.record_prefill_before(self._snapshot_cache_stats)

    def prefill_after_attn(self, layer_idx, class_a_scores, per_head_scores, key_states, value_states):
        """cache.py:257-349: class-A heads keep everything after the padding;
        other heads keep the non-audio rows plus a top-``ratio`` subset of every
        audio segment; class-B heads offload the rest to host memory.

        One layer = a batched top-k per retention ratio, one row gather into
        the packed layer and one into the offload rows, which are copied
        (asynchronously) straight into their place in the pinned host store."""
        cfg, l = self.config, layer_idx
        B, H, D = self.batch_size, self.num_kv_heads, self.head_dim
        for b in range(B):
            if class_a_scores[b] is not None:
                self._prefill_scores[b].append(class_a_scores[b].float())
        if not self._store_planned:
            self._plan_restore_store(key_states.dtype)
        Sq = key_states.shape[2]
        dev = key_states.device
        kflat = key_states.reshape(B * H * Sq, D)
        vflat = value_states.reshape(B * H * Sq, D)
        keep_rows = [None] * (B * H)   # source rows of each segment, reference order
        off_rows = []                  # class-B offload source rows, store order
        lens = [0] * (B * H)
        g2c = [0] * B
        for b in range(B):
            r0, r1, pad = self._raw_audio_starts[b], self._raw_audio_ends[b], self.pad_lens_list[b]
            segs = self.segment_ranges[b]
            key = (b, Sq)
            if key not in self._nonaudio:
                self._nonaudio[key] = torch.cat([torch.arange(pad, r0, device=dev),
                                                 torch.arange(r1, Sq, device=dev)])
            nonaudio = self._nonaudio[key]
            groups = {}
            for h in range(H):
                fi = b * H + h
                if cfg.is_class_a_kv_head(l, h):
                    keep_rows[fi] = torch.arange(fi * Sq + pad, fi * Sq + Sq, device=dev)
                    lens[fi] = Sq - pad
                else:
                    groups.setdefault(cfg.get_retention(l, h), []).append(h)
            off_head = {}
            for ratio, hs in groups.items():
                sc = torch.stack([per_head_scores[b][h] for h in hs]).to(dev)
                kept = keep_audio_indices(sc, segs, ratio, cfg.prefill_global_topk)
                bases = torch.tensor([(b * H + h) * Sq for h in hs], device=dev).unsqueeze(1)
                rows = torch.cat([nonaudio.unsqueeze(0).expand(len(hs), -1), kept + r0], dim=1) + bases
                n_keep = kept.shape[1]
                hb = [i for i, h in enumerate(hs) if cfg.is_class_b(l, h)]
                if hb and n_keep < sc.shape[1]:
                    mask = torch.ones(len(hb), sc.shape[1], dtype=torch.int8, device=dev)
                    mask.scatter_(1, kept[hb], 0)
                    # stable descending sort lists the offloaded tokens first, ascending
                    off = torch.argsort(mask, dim=1, descending=True, stable=True)[:, :sc.shape[1] - n_keep]
                    off = off + r0 + bases[hb]
                    if cfg.prefill_global_topk:
                        cnt = torch.stack([torch.bincount((off[i] - bases[hb[i]] - r0) // cfg.stride_tokens,
                                                          minlength=len(segs)) for i in range(len(hb))]).cpu()
                    for i, j in enumerate(hb):
                        off_head[hs[j]] = (off[i], cnt[i].tolist() if cfg.prefill_global_topk else None)
                for i, h in enumerate(hs):
                    keep_rows[b * H + h] = rows[i]
                    lens[b * H + h] = (r0 - pad) + (Sq - r1) + n_keep
            for h in sorted(off_head):
                fi = b * H + h
                rows_h, cnt = off_head[h]
                if cnt is None:
                    cnt = offload_counts(segs, cfg.get_retention(l, h), False)[0]
                o = int(self._store_off[l, fi])
                m0 = self._meta_base[l, fi]
                for si, n in enumerate(cnt):
                    if n:
                        self._meta["cpu_s"][m0 + si], self._meta["cpu_e"][m0 + si] = o, o + n
                        o += n
                off_rows.append(rows_h)
                g2c[b] += rows_h.shape[0]
        src = torch.cat(keep_rows)
        self._pk[l] = kflat.index_select(0, src)
        self._pv[l] = vflat.index_select(0, src)
        if off_rows:
            src = torch.cat(off_rows)
            o0 = int(self._store_layer_off[l])
            n = src.shape[0]
            self.cpu_restore_k[o0:o0 + n].copy_(kflat.index_select(0, src), non_blocking=True)
            self.cpu_restore_v[o0:o0 + n].copy_(vflat.index_select(0, src), non_blocking=True)
        for b in range(B):
            if g2c[b]:
                self.stats.record_cpu_gpu_transfer(b, g2c_tokens=g2c[b],
                                                   g2c_bytes=g2c[b] * D * 2 * key_states.element_size())
        self.seq_lens[l] = lens

    def _plan_restore_store(self, dtype):
        """Sizes of everything the prefill offloads, known from the config and
        the audio spans alone: the restore-metadata layout, each (layer,
        segment)'s place in the host store, and the store itself (pinned,
        allocated once; layer-major, then segment, then audio segment)."""
        cfg = self.config
        L, H, B, D = self.num_layers, self.num_kv_heads, self.batch_size, self.head_dim
        S = B * H
        self.seg_count = [len(self.segment_ranges[b]) for b in range(B)]
        per_fi = np.array([self.seg_count[fi // H] for fi in range(S)], np.int64)
        self._meta_base = (np.arange(L, dtype=np.int64)[:, None] * per_fi.sum()
                           + np.concatenate([[0], np.cumsum(per_fi)[:-1]])[None, :])
        acc = int(L * per_fi.sum())
        self._meta = {k: np.full(acc, -1, np.int32) for k in ("cpu_s", "cpu_e", "gpu_s", "gpu_e")}
        self._store_off = np.zeros((L, S), np.int64)
        self._store_layer_off = np.zeros(L + 1, np.int64)
        off = 0
        for l in range(L):
            self._store_layer_off[l] = off
            for fi in range(S):
                b, h = divmod(fi, H)
                self._store_off[l, fi] = off
                if cfg.is_class_b(l, h) and not cfg.is_class_a_kv_head(l, h):
                    off += offload_counts(self.segment_ranges[b], cfg.get_retention(l, h),
                                          cfg.prefill_global_topk)[1]
        self._store_layer_off[L] = off
        if off:
            if self.offload_tier == "hbm":
                self.cpu_restore_k = torch.empty(off, D, dtype=dtype, device=self.device)
                self.cpu_restore_v = torch.empty(off, D, dtype=dtype, device=self.device)
            else:
                self.cpu_restore_k = torch.empty(off, D, dtype=dtype, pin_memory=True)
                self.cpu_restore_v = torch.empty(off, D, dtype=dtype, pin_memory=True)
        else:
            self.cpu_restore_k = torch.empty(0, D, dtype=dtype)
            self.cpu_restore_v = torch.empty(0, D, dtype=dtype)
        self._restore_ptrs = None
        self._store_planned = True

    def prefill_all_layers_done(self):
        """cache.py:351-390: host restore store, initial chunk selection and
        load, then the slot layout, the scoring tables and the planner."""
        L, H, B, D, G = self.num_layers, self.num_kv_heads, self.batch_size, self.head_dim, self.num_kv_groups
        S = B * H
        dt = self._pk[0].dtype
        self.dtype = dt
        if not self._store_planned:  # no layer offloaded anything
            self._plan_restore_store(dt)
        # the offload copies into the pinned store were queued on this stream
        # --- scoring geometry (needed by the initial selection)
        self._setup_scoring()
        # --- initial chunk selection from the summed prefill class-A scores
        sel = torch.zeros(self._score_offsets_list[-1], dtype=torch.float32, device=self.device)
        for b in range(B):
            o0, o1 = self._score_offsets_list[b], self._score_offsets_list[b + 1]
            if self._prefill_scores[b]:
                sel[o0:o1] = torch.stack(self._prefill_scores[b]).sum(dim=0)
            else:
                sel[o0:o1] = 1.0
            self._prefill_scores[b] = []
        if self.score_reduce is not None:
            sel = self.score_reduce(sel)
        top = self._select_topk(sel)
        for b in range(B):
            needed = sorted({s for c in top[b] for s in self.chunk_to_segs[b][c]})
            if needed:
                self._initial_load(b, needed)
            self.loaded_segments[b] = set(needed)
        # --- slot layout, planner, per-step buffers
        self._build_slots()
        self._init_planner()
        self._tail_args = None
        self._plan_layer_checks()
        self.prefilled = True
        self.stats.record_prefill(self._snapshot_cache_stats)

    def _initial_load(self, b, segs):
        """cache.py:651-714: append the selected host rows to sample b's
        class-B segments, in ascending segment order -- per layer one copy of
        the packed rows to their new places and one zero-copy fetch of the
        selected rows from the pinned store."""
        H, D = self.num_kv_heads, self.head_dim
        dev = self.device
        c2g = 0
        for l in range(self.num_layers):
            lens = list(self.seq_lens[l])
            old = list(lens)
            ranges, dst = [], []
            for fi in range(b * H, (b + 1) * H):
                if not self.config.is_class_b(l, fi - b * H):
                    continue
                rel = lens[fi]
                m0 = self._meta_base[l, fi]
                for si in segs:
                    cs, ce = int(self._meta["cpu_s"][m0 + si]), int(self._meta["cpu_e"][m0 + si])
                    if cs < 0:
                        continue
                    ranges.append((cs, ce))
                    dst.append((fi, rel))
                    self._meta["gpu_s"][m0 + si], self._meta["gpu_e"][m0 + si] = rel, rel + ce - cs
                    rel += ce - cs
                lens[fi] = rel
            if not ranges:
                continue
            new_cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
            old_cu = np.concatenate([[0], np.cumsum(old)]).astype(np.int64)
            nk = torch.empty(int(new_cu[-1]), D, dtype=self._pk[l].dtype, device=dev)
            nv = torch.empty_like(nk)
            Kx.copy_segments(self._pk[l], self._pv[l], torch.from_numpy(old_cu[:-1]).to(dev), nk, nv,
                             torch.from_numpy(new_cu[:-1]).to(dev),
                             torch.from_numpy(np.asarray(old, np.int32)).to(dev))
            rng = torch.tensor(ranges, dtype=torch.int32, device=dev)
            drow = torch.tensor([int(new_cu[fi]) + r for fi, r in dst], dtype=torch.int64, device=dev)
            src_k, src_v = self._restore_dev_ptrs()
            Kx.fetch_rows(src_k, src_v, D * nk.element_size(), rng, drow, nk, nv, max_ctas=self.fetch_ctas)
            c2g += sum(e - s_ for s_, e in ranges)
            self._pk[l], self._pv[l] = nk, nv
            self.seq_lens[l] = lens
        if c2g:
            self.stats.record_cpu_gpu_transfer(b, c2g_tokens=c2g,
                                               c2g_bytes=c2g * D * 2 * self.cpu_restore_k.element_size())

    def _loaded_bound(self, l, fi):
        """Most host rows segment (l, fi) can hold at once: a segment stays
        loaded at most ``eviction_lag`` steps after it was last needed, so at
        most max(1, lag) * top_k * segs_per_chunk segments are resident."""
        b = fi // self.num_kv_heads
        m0 = self._meta_base[l, fi]
        n = self.seg_count[b]
        sizes = self._meta["cpu_e"][m0:m0 + n] - self._meta["cpu_s"][m0:m0 + n]
        sizes = np.sort(sizes[self._meta["cpu_s"][m0:m0 + n] >= 0])[::-1]
        m = max(1, self.config.eviction_lag) * self.config.top_k_chunks * self.segs_per_chunk
        return int(sizes[:m].sum())

    def _build_slots(self):
        L, S, D = self.num_layers, self.batch_size * self.num_kv_heads, self.head_dim
        dev = self.device
        self._len_host = np.zeros((L, S), np.int64)     # rows stored (device seg_len mirror)
        self._cap_host = np.zeros((L, S), np.int64)
        self._base_host = np.zeros((L, S), np.int64)
        self.k_store, self.v_store = [None] * L, [None] * L
        for l in range(L):
            lens = np.asarray(self.seq_lens[l], np.int64)
            loaded_now = np.zeros(S, np.int64)
            extra = np.zeros(S, np.int64)
            for fi in range(S):
                if self.config.is_class_b(l, fi % self.num_kv_heads):
                    m0 = self._meta_base[l, fi]
                    n = self.seg_count[fi // self.num_kv_heads]
                    gs, ge = self._meta["gpu_s"][m0:m0 + n], self._meta["gpu_e"][m0:m0 + n]
                    loaded_now[fi] = int((ge - gs)[gs >= 0].sum())
                    extra[fi] = self._loaded_bound(l, fi)
            cap = lens - loaded_now + extra + self.max_decode_tokens
            self._len_host[l], self._cap_host[l] = lens, cap
        self._alloc_stores(range(L), copy_from_packed=True)
        self._pk = self._pv = None
        self._seg_len = torch.from_numpy(self._len_host.astype(np.int32)).to(dev)
        self._refresh_layout_tensors()

    def _alloc_stores(self, layers, copy_from_packed=False):
        D, dev = self.head_dim, self.device
        for l in layers:
            cap = self._cap_host[l]
            # 16-row alignment keeps every slot start 16-byte aligned for any dtype
            cap_al = (cap + 15) // 16 * 16
            base = np.concatenate([[0], np.cumsum(cap_al)[:-1]]).astype(np.int64)
            rows = int(cap_al.sum())
            ks = torch.empty(rows, D, dtype=self.dtype, device=dev)
            vs = torch.empty(rows, D, dtype=self.dtype, device=dev)
            lens = torch.from_numpy(self._len_host[l].astype(np.int32)).to(dev)
            dst_base = torch.from_numpy(base).to(dev)
            if copy_from_packed:
                src_base = torch.from_numpy(np.concatenate([[0], np.cumsum(self._len_host[l])[:-1]]).astype(np.int64)).to(dev)
                Kx.copy_segments(self._pk[l], self._pv[l], src_base, ks, vs, dst_base, lens)
            else:
                src_base = torch.from_numpy(self._base_host[l]).to(dev)
                Kx.copy_segments(self.k_store[l], self.v_store[l], src_base, ks, vs, dst_base, lens)
            self.k_store[l], self.v_store[l] = ks, vs
            self._base_host[l] = base

    def _refresh_layout_tensors(self):
        L, S, D, G = self.num_layers, self.batch_size * self.num_kv_heads, self.head_dim, self.num_kv_groups
        dev = self.device
        self._seg_base = torch.from_numpy(self._base_host).to(dev)
        self._seg_cap = torch.from_numpy(self._cap_host.astype(np.int32)).to(dev)
        max_rows = int((self._len_host + self.max_decode_tokens).max()) if S else 0
        self._work = []
        n_max = 0
        for l in range(L):
            # the layer's launch layout, fitted to its capacities
            w = Kx.AttnWork(self.dtype, D, self._cap_host[l], dev)
            self._work.append(w)
            n_max = max(n_max, w.slots)
        if getattr(self, "_scratch", None) is None or not self._scratch.fits(n_max, G, D, S):
            self._scratch = Kx.AttnScratch(dev, n_max, G, D, S)
            self._tail_args = None  # the step tail copies the scratch's error word
        del max_rows
        self._attn_args = [None] * L  # launch arguments, built lazily per (layer, scale)
        self._rb_args = [None] * L    # rebuild arguments, likewise

    def _grow(self, l):
        """Give layer l another ``max_decode_tokens`` rows per slot."""
        self._cap_host[l] = self._cap_host[l] + self.max_decode_tokens
        self._alloc_stores([l])
        self._refresh_layout_tensors()

    def _setup_scoring(self):
        """Slots for the class-A logits of every (layer, class-A kv head,
        sample) and the per-sample term table (layer-major, ascending kv)."""
        L, H, B, G = self.num_layers, self.num_kv_heads, self.batch_size, self.num_kv_groups
        S = B * H
        dev = self.device
        audio = [self._audio_ends_list[b] - self._audio_starts_list[b] for b in range(B)]
        self._score_groups = []
        for l in range(L):
            by_kv = {}
            for qh in self.config.get_layer_class_a(l) if sum(audio) > 0 else ():  # no audio: nothing to score
                by_kv.setdefault(qh // G, []).append(qh % G)
            self._score_groups.append(sorted(by_kv.items()))
        self._has_scoring = any(self._score_groups)
        slot = np.full((L, S), -1, np.int32)
        logit_off = []
        terms = [[] for _ in range(B)]
        total = 0
        for l in range(L):
            for kv, qs in self._score_groups[l]:
                mask = sum(1 << g for g in qs)
                for b in range(B):
                    fi = b * H + kv
                    slot[l, fi] = len(logit_off)
                    terms[b].append((l, kv, total, mask))
                    logit_off.append(total)
                    total += audio[b] * G
        self._slot_host = slot
        self._score_slot = torch.from_numpy(slot).to(dev)
        self._logits = torch.zeros(max(1, total), dtype=torch.float32, device=dev)
        self._logits_off = torch.tensor(logit_off or [0], dtype=torch.int64, device=dev)
        self._stats = torch.zeros(L * S * 2 * G, dtype=torch.float32, device=dev)
        t_logit, t_stat, t_mask, t_off = [], [], [], [0]
        for b in range(B):
            for l, kv, off, mask in sorted(terms[b]):
                t_logit.append(off)
                t_stat.append((l * S + b * H + kv) * 2 * G)
                t_mask.append(mask)
            t_off.append(len(t_logit))
        self._t_logit = torch.tensor(t_logit or [0], dtype=torch.int64, device=dev)
        self._t_stat = torch.tensor(t_stat or [0], dtype=torch.int64, device=dev)
        self._t_mask = torch.tensor(t_mask or [0], dtype=torch.int64, device=dev).to(torch.int32)
        self._t_off = torch.tensor(t_off, dtype=torch.int32, device=dev)
        self._audio_start_dev = torch.tensor(self._audio_starts_list, dtype=torch.int32, device=dev)
        self._audio_end_dev = torch.tensor(self._audio_ends_list, dtype=torch.int32, device=dev)
        self._topk_dev = torch.full((max(1, B), max(1, self.config.top_k_chunks)), -1, dtype=torch.int32,
                                    device=dev)
        self._topk_host = torch.empty_like(self._topk_dev, device="cpu").pin_memory()
        self._err_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._ready = torch.cuda.Event()

    def _select_topk(self, scores):
        """Chunk means + top-k of a class-A score vector (device kernel), to
        host lists per sample (a sync point)."""
        if self.config.top_k_chunks <= 0 or self.max_audio <= 0:
            return [[] for _ in range(self.batch_size)]
        Kx.chunk_topk(scores, self.score_offsets, self.max_audio, self.config.stride_tokens,
                      self.segs_per_chunk, self.config.top_k_chunks, self._topk_dev)
        rows = self._topk_dev.cpu().tolist()
        return [[c for c in r if c >= 0] for r in rows[:self.batch_size]]

    def _init_planner(self):
        """Hand the prefill state to the native planner (wnw_cpp/code/cache.py:40-116)."""
        L, H, B = self.num_layers, self.num_kv_heads, self.batch_size
        P = self._planner = Planner(L, H, B, self.num_kv_groups)
        self._seg_rows = self._segment_host_rows()
        P.set_config(self.config.top_k_chunks, self.config.eviction_lag)
        P.set_seg_count(self.seg_count)
        for b in range(B):
            flat = [s for c in self.chunk_to_segs[b] for s in c]
            off = [0] + list(accumulate(len(c) for c in self.chunk_to_segs[b]))
            P.set_chunk_to_segs(b, flat, off)
        for l in range(L):
            P.set_class_b(l, self._class_b_heads_by_layer[l])
        P.set_restore_meta(self._meta["cpu_s"], self._meta["cpu_e"], self._meta["gpu_s"], self._meta["gpu_e"])
        for b in range(B):
            P.set_loaded(b, sorted(self.loaded_segments[b]))
        P.set_seq_lens(self._len_host.reshape(-1))
        S = B * H
        self._plan_bufs = [np.zeros((L, S), np.int32), np.zeros((L, S), np.int32), np.zeros((L, S + 1), np.int32),
                           np.zeros((L, S), np.int32), np.zeros((L, S + 1), np.int32), np.zeros(L, np.int32),
                           np.zeros(L + 1, np.int32)]
        self._plan_host = torch.zeros(1024, dtype=torch.int32).pin_memory()
        self._plan_dev = torch.zeros(1024, dtype=torch.int32, device=self.device)
        self._land_k = self._land_v = None
        self._stage_k = self._stage_v = None
        self._events = [torch.cuda.Event() for _ in range(L)]
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(device=self.device)
        for e in self._events:  # create the CUDA events now so their handles can be passed down
            e.record(self._copy_stream)
        import ctypes as _C
        self._event_handles = (_C.c_void_p * L)(*[e.cuda_event for e in self._events])
        self._restore_ptrs = None
        self._fetched_rows = 0
        self._move_k = self._move_v = None
        # status words: one layer's records, or every layer's for the fused
        # rebuild of the HBM tier
        self._rb_status = torch.zeros(max(1, S * (L if self._fused_rebuild else 1)), dtype=torch.int32,
                                      device=self.device)
        self._layer_chg = [0] * L
        self._chg_buf = None
        self._layer_rows = np.zeros(L + 1, np.int64)
        self._new_kv = [None] * L
        self._presize_step_buffers()
        self._dplan, self._dplan_args = None, None
        if (self.fetch_mode == "zerocopy" and self.fetch_plan == "device" and self.config.top_k_chunks > 0
                and self.max_audio > 0 and self.cpu_restore_k.shape[0] and self._land_k is not None):
            self._dplan = DevicePlan.create(P)

    def _presize_step_buffers(self):
        """Size the per-step fetch and rebuild buffers for the worst step the
        planner can produce, so the decode loop never allocates (a pinned
        allocation is a slow, synchronising driver call): one step loads at
        most every segment a slot can hold, moves at most those rows plus the
        decoded ones, and the plan blob holds at most one record per slot."""
        L, S = self.num_layers, self.batch_size * self.num_kv_heads
        lag = max(1, self.config.eviction_lag)
        segs = lag * self.config.top_k_chunks * self.segs_per_chunk
        bound = np.zeros((L, S), np.int64)
        for l in range(L):
            for fi in range(S):
                if self.config.is_class_b(l, fi % self.num_kv_heads):
                    bound[l, fi] = self._loaded_bound(l, fi)
        rows = int(bound.sum())
        if rows == 0:
            return
        n_ranges = L * S * segs
        self._ensure_fetch_capacity(rows, n_ranges)
        moved = (bound + self.max_decode_tokens * (bound > 0)).sum(axis=1)
        # the fused rebuild keeps every changed layer's moved rows at once
        self._ensure_move_capacity(int(moved.sum() if self._fused_rebuild else moved.max()))
        plan_ints = (L + 1) + L * (6 + 8 * S) + 2 * n_ranges
        if plan_ints > self._plan_host.numel():
            n = 1 << (plan_ints - 1).bit_length()
            self._plan_host = torch.zeros(n, dtype=torch.int32).pin_memory()
            self._plan_dev = torch.zeros(n, dtype=torch.int32, device=self.device)
            self._rb_args = [None] * L

    # ------------------------------------------------------------- decode
    def decode_before_attn(self, layer_idx, new_k, new_v):
        """Rebuild the layer's changed slots if a plan is pending, check slot
        capacity, and stash the step's new K/V rows for the fused append.
        Returns (k_store, v_store, seg_len, max_seqlen_k); seg_len counts the
        rows stored before this step's token (cache.py:487-515 contract)."""
        l = layer_idx
        # rows and lengths of layer l stay as the last step left them (the
        # host waited for that step's end) unless this step grows or rebuilds
        # its slots
        self._rows_ready[l] = self._decode_step > 0
        if self._grow_flags[l]:
            self._grow(l)
            self._grow_flags[l] = False
            self._rows_ready[l] = False
        if self._rebuilt[l]:
            # rebuilt ahead on the rebuild stream: the compute stream waits
            # for this layer's rebuild, so its rows and lengths are final
            # before the attention launches (a stream wait holds back every
            # later launch, whatever its programmatic-dependency attribute).
            # The fused rebuild finishes every layer at once and records one
            # event: the first rebuilt layer's wait covers the step.
            if self._fused_rebuild:
                ev = self._rb_events[self._fused_ev]
                self._rebuilt = [False] * self.num_layers
            else:
                ev = self._rb_events[l]
                self._rebuilt[l] = False
            st = N.lib.wnw_stream_wait_event(self._raw_stream(), ev.cuda_event)
            if st:
                N.check(st, "wnw_stream_wait_event")
        if self._pending and self._layer_chg[l]:
            self._rows_ready[l] = False
            stream = self._raw_stream()
            st = N.lib.wnw_stream_wait_event(stream, self._event_handles[l])
            if st == 0:
                st = N.lib.wnw_rebuild_segments(*self._rebuild_args(l), stream)
            if st:
                N.check(st, "wnw_rebuild_segments")
            Kx.LAUNCHES[0] += 2
            self._len_host[l] = self._next_lens[l]
        if l == self.num_layers - 1:
            self._pending = False
        # the kernel reads the step's rows as [S, head_dim]: any contiguous
        # [B, Hkv, 1, D] (or [S, D]) tensor is that already
        self._new_kv[l] = (new_k if new_k.is_contiguous() else new_k.contiguous(),
                           new_v if new_v.is_contiguous() else new_v.contiguous())
        self.seq_lens[l] = self._step_seq[l]
        return self.k_store[l], self.v_store[l], self._seg_len[l], self._step_max[l]

    def decode_after_attn(self, layer_idx, q):
        """Not supported: this hook belongs to the reference session's
        non-fused branch (session.py:90-112), which attends with torch's
        varlen_attn over packed K/V and then scores here (cache.py:517-544).
        This cache attends, appends and scores in fused_decode_attention
        (the session's WNW_FUSED_ATTN=1 branch); reaching this hook means the
        session just attended over the slot stores as if they were packed,
        so it raises instead of returning a wrong result."""
        from wnw_b200.integration import NonFusedSessionError
        raise NonFusedSessionError(
            "B200WnWCache supports the fused-attention session path only (WNW_FUSED_ATTN=1): "
            "decode_after_attn was called, so the session attended with varlen_attn over K/V this cache "
            "does not pack")

    def _plan_layer_checks(self):
        """Per-layer facts of the coming step, computed once for all layers:
        the rows each slot will hold before this step's token (after any
        rebuild), whether a slot would overflow (grow first), the reference's
        seq_lens (rows including the token) and their maximum."""
        eff = self._len_host
        if self._pending:
            chg = np.asarray(self._layer_chg, bool)
            if chg.any():
                eff = eff.copy()
                eff[chg] = self._next_lens[chg]
        self._grow_flags = ((eff + 1) > self._cap_host).any(axis=1).tolist()
        self._step_seq = eff + 1
        self._step_max = (eff.max(axis=1) + 1).tolist() if eff.shape[1] else [1] * self.num_layers

    def _raw_stream(self):
        """cudaStream_t of the current torch stream on this cache's device."""
        return torch._C._cuda_getCurrentRawStream(self._dev_index)

    def _rebuild_args(self, l):
        """wnw_rebuild_segments arguments of layer l (all but the stream);
        rebuilt whenever a buffer they point at is reallocated."""
        a = self._rb_args[l]
        if a is None:
            mk, mv = self._move_k, self._move_v
            a = self._rb_args[l] = (
                N.dtype_code(self.dtype), self.head_dim, self.k_store[l].data_ptr(), self.v_store[l].data_ptr(),
                self._seg_base[l].data_ptr(), self._seg_len[l].data_ptr(), self._seg_cap[l].data_ptr(),
                int(self._seg_len[l].numel()),
                self._land_k.data_ptr() if self._land_k is not None else None,
                self._land_v.data_ptr() if self._land_v is not None else None,
                int(self._land_k.shape[0]) if self._land_k is not None else 0,
                self._plan_dev.data_ptr(), int(self._plan_dev.numel()), l,
                mk.data_ptr() if mk is not None else None, mv.data_ptr() if mv is not None else None,
                int(mk.shape[0]) if mk is not None else 0, self._rb_status.data_ptr(), self._scratch.err.data_ptr())
        return a

    def _score_args(self, l):
        if not self._score_groups[l]:
            return None
        S, G = self.batch_size * self.num_kv_heads, self.num_kv_groups
        return dict(slot=self._score_slot[l], audio_start=self._audio_start_dev, audio_end=self._audio_end_dev,
                    logits=self._logits, logits_off=self._logits_off,
                    stats=self._stats[l * S * 2 * G:(l + 1) * S * 2 * G])

    def fused_decode_attention(self, layer_idx, q_flat, q=None, k_flat=None, v_flat=None, cu_k=None,
                               scale=None):
        """cache.py:546-566: attention + append + class-A logits in one launch.
        Class-A probabilities use the attention scale, which is what the
        reference's fused kernel does; layers whose class-A set is not a
        whole kv group use 1/sqrt(d) in the reference (kernels.py:149), so a
        different attention scale triggers a separate scoring launch."""
        l = layer_idx
        G, D = self.num_kv_groups, self.head_dim
        qf = q_flat if q_flat.is_contiguous() else q_flat.contiguous()
        nk, nv = self._new_kv[l]
        cached = self._attn_args[l]
        if cached is None or cached[0] != scale:
            score = self._score_args(l)
            foldable = all(len(qs) == G for _, qs in self._score_groups[l])
            sep = score is not None and not foldable and not math.isclose(scale, D ** -0.5, rel_tol=0,
                                                                          abs_tol=1e-12)
            S = self.batch_size * self.num_kv_heads
            args = Kx.make_attn_args(self.dtype, S, G, D, self.k_store[l], self.v_store[l], self._seg_base[l],
                                     self._seg_len[l], self._work[l], scale, self._scratch,
                                     seg_cap=self._seg_cap[l], num_kv_heads=self.num_kv_heads,
                                     score=None if sep else score)
            cached = self._attn_args[l] = (scale, sep, args, C.byref(args))
        _, sep, args, ref = cached
        # the kernel may read this layer's lengths and rows before it waits
        # for the preceding kernel when nothing in this step has written them
        args.flags = N.ATTN_ROWS_READY if self._rows_ready[l] else 0
        out = torch.empty_like(qf)
        st = N.lib.wnw_decode_attn_step(ref, qf.data_ptr(), nk.data_ptr(), nv.data_ptr(), out.data_ptr(),
                                        self._raw_stream())
        if st:
            N.check(st, "wnw_decode_attn_step")
        Kx.LAUNCHES[0] += self._work[l].launches
        if sep:
            score = self._score_args(l)  # rescore with the reference's 1/sqrt(d) (the append is idempotent)
            Kx.decode_attention(qf, self.k_store[l], self.v_store[l], self._seg_base[l], self._seg_len[l],
                                self._work[l], D ** -0.5, self._scratch, new_k=nk, new_v=nv,
                                seg_cap=self._seg_cap[l], num_kv_heads=self.num_kv_heads, score=score,
                                out=torch.empty_like(qf))
        return out

    def decode_all_layers_done(self):
        """cache.py:568-600: advance lengths, score, select, plan, prefetch."""
        self._decode_step += 1
        self._fetched_rows = 0  # rows this step's plan fetches (set when it changes anything)
        self.stats.flush_decode_step(self._decode_step)
        if self.stats.enabled and self._decode_step % self.stats.interval == 0:
            self.stats.record_decode(self._decode_step, self._snapshot_cache_stats)
        B = self.batch_size
        st = self._raw_stream()
        a = self._tail_args if self._tail_args is not None else self._make_tail_args()
        select = self.config.top_k_chunks > 0 and self.max_audio > 0
        self._tail_call("wnw_advance_lengths", a["adv"], st)
        self._len_host += 1
        if self._has_scoring:
            self._tail_call("wnw_score_finalize", a["fin"], st)
        else:
            self.score_accumulator.zero_()
        if self.score_reduce is not None:
            self.score_accumulator.copy_(self.score_reduce(self.score_accumulator))
            st = self._raw_stream()
        if select:
            self._tail_call("wnw_chunk_topk", a["topk"], st)
        dplan = self._dplan if select else None
        if dplan is not None:  # the fetch starts now, planned on the device
            self._dplan_step(st)
        Kx.LAUNCHES[0] += 1 + int(self._has_scoring) + int(select)
        self._tail_call("wnw_copy_async", a["topk_d2h"], st)
        self._tail_call("wnw_copy_async", a["err_d2h"], st)
        self._ready.record()
        t_wait = time.perf_counter()
        wait_event(self._ready, self.wait_timeout_s)
        self.host_wait_s += time.perf_counter() - t_wait
        if int(a["err_np"][0]):
            Kx.check_device_error(self._scratch.err)
        if select:
            t = a["topk_np"]
            keep = t >= 0
            flat = np.ascontiguousarray(t[keep], np.int32)
            off = np.concatenate([[0], np.cumsum(keep.sum(axis=1))]).astype(np.int32)
        else:
            flat, off = np.zeros(0, np.int32), np.zeros(B + 1, np.int32)
        self.last_topk = [sorted(flat[off[b]:off[b + 1]].tolist()) for b in range(B)]
        if self.fetch_mode == "zerocopy":
            ch, total = self._planner.compute(flat, off, a["plan_ptrs"])
            ranges = None
        else:
            ch, total, _, _, ranges = self._planner.compute_and_prepare(flat, off, *self._plan_bufs)
        if dplan is not None:
            dplan.verify(self._planner)  # the fetch already in flight is the planner's
            if ch:
                self._upload_plan(st)
        elif ch:
            self._prepare_fetch(total, ranges)
        for b in range(B):
            now = set(self._planner.get_loaded_segments(b))
            if ch and self.stats.enabled:  # cache.py:816-820: each sample's loads
                new = sorted(now - self.loaded_segments[b])
                n = int(self._seg_rows[b][new].sum()) if new else 0
                if n:
                    row_bytes = self.head_dim * self.cpu_restore_k.element_size()
                    self.stats.record_cpu_gpu_transfer(b, c2g_tokens=n, c2g_bytes=n * row_bytes * 2)
            self.loaded_segments[b] = now
        self._plan_layer_checks()
        if self.rebuild_ahead and self._pending:
            self._issue_rebuilds()

    def _issue_rebuilds(self):
        """The step's rebuilds, issued now on the rebuild stream: after
        everything issued so far on the compute stream (the step's tail and
        the plan upload, and any slot growth, done here first), layer l's
        rebuild waits for layer l's fetched rows and records its own event,
        which the compute stream waits for before layer l's attention.  The
        next step's fetch reuses the landing rows only after the top-k,
        which comes after every attention, hence after every rebuild."""
        L = self.num_layers
        for l in range(L):  # growth copies the layer's rows into larger slots: before its rebuild
            if self._grow_flags[l]:
                self._grow(l)
                self._grow_flags[l] = False
        if self._rb_stream is None:
            self._rb_stream = torch.cuda.Stream(device=self.device)
            self._rb_events = [torch.cuda.Event() for _ in range(L)]
            for e in self._rb_events:  # create the CUDA events now: their handles are passed down
                e.record(self._rb_stream)
        rs = self._rb_stream
        chg = np.ascontiguousarray(self._layer_chg, np.int32)
        if self._fused_rebuild:  # every changed layer's moved rows at once (presized; grows only past that)
            ph = self._plan_host.numpy()
            self._ensure_move_capacity(int(sum(int(ph[int(ph[l]) + 1]) for l in np.nonzero(chg)[0])))
        start = torch.cuda.Event()
        start.record()
        rs.wait_event(start)
        b = self._rebuild_batch()
        if self._fused_rebuild:
            # the layers' fetch kernels run in order on the copy stream, so
            # the last changed layer's fetch event covers every earlier one;
            # one event, recorded in the first changed layer's slot, marks the
            # end of the launch pair (decode_before_attn waits for it once)
            idx = np.nonzero(chg)[0]
            if idx.size == 0:  # nothing to rebuild this step
                self._pending = False
                return
            first, last = int(idx[0]), int(idx[-1])
            P = C.c_void_p
            waits = (P * L)()
            waits[last] = self._event_handles[last]
            recs = (P * L)()
            recs[first] = b["record"][first]
            self._fused_ev = first
            sh = b["shared"]  # ... status, then its length, then err
            st = N.lib.wnw_rebuild_layers_fused(*b["head"], chg.ctypes.data, *b["layers"], *sh[:9],
                                                int(self._rb_status.numel()), sh[9], waits, recs, rs.cuda_stream)
            name = "wnw_rebuild_layers_fused"
        else:
            st = N.lib.wnw_rebuild_layers(*b["head"], chg.ctypes.data, *b["layers"], *b["shared"],
                                          self._event_handles, b["record"], rs.cuda_stream)
            name = "wnw_rebuild_layers"
        if st:
            N.check(st, name)
        changed = np.nonzero(chg)[0].tolist()
        Kx.LAUNCHES[0] += 2 * ((len(changed) + 47) // 48 if self._fused_rebuild else len(changed))
        for l in changed:
            self._len_host[l] = self._next_lens[l]
            self._rebuilt[l] = True
        self._pending = False

    def _rebuild_batch(self):
        """wnw_rebuild_layers arguments: per-layer pointer arrays and the
        shared buffers, from the per-layer rebuild arguments (rebuilt when
        those are: every invalidation assigns a new _rb_args list)."""
        if getattr(self, "_rb_batch_key", None) is self._rb_args:
            return self._rb_batch
        L = self.num_layers
        args = [self._rebuild_args(l) for l in range(L)]
        P = C.c_void_p
        arr = lambda i: (P * L)(*[a[i] for a in args])  # noqa: E731
        a0 = args[0]
        self._rb_batch = {
            "head": (a0[0], a0[1], L),
            "layers": (arr(2), arr(3), arr(4), arr(5), arr(6), (C.c_int32 * L)(*[a[7] for a in args])),
            # landing k / v, rows, plan blob, ints, move k / v, rows, status, err (layer index a[13] dropped)
            "shared": (a0[8], a0[9], a0[10], a0[11], a0[12], a0[14], a0[15], a0[16], a0[17], a0[18]),
            "record": (P * L)(*[e.cuda_event for e in self._rb_events]),
        }
        if not all(b for b in self._rb_batch["record"]):
            raise RuntimeError("rebuild events have no CUDA handle")
        self._rb_batch_key = self._rb_args
        return self._rb_batch

    def _tail_call(self, name, args, stream):
        st = getattr(N.lib, name)(*args, stream)
        if st:
            N.check(st, name)

    def _make_tail_args(self):
        """Launch arguments of the step's tail (length advance, score
        finalisation, chunk top-k, two small device-to-host copies), taken
        once: every buffer they name lives as long as the prefilled state."""
        B = self.batch_size
        a = {"adv": (self._seg_len.data_ptr(), self._seg_len.numel())}
        if self._has_scoring:
            a["fin"] = (self._logits.data_ptr(), self._stats.data_ptr(), self._t_logit.data_ptr(),
                        self._t_stat.data_ptr(), self._t_mask.data_ptr(), self._t_off.data_ptr(),
                        self.num_kv_groups, B, self.score_offsets.data_ptr(), int(self.max_audio),
                        self.score_accumulator.data_ptr())
        a["topk"] = (self.score_accumulator.data_ptr(), self.score_offsets.data_ptr(), B, int(self.max_audio),
                     int(self.config.stride_tokens), int(self.segs_per_chunk), int(self.config.top_k_chunks),
                     self._topk_dev.data_ptr(), None, None)
        a["topk_d2h"] = (self._topk_host.data_ptr(), self._topk_dev.data_ptr(),
                         self._topk_dev.numel() * self._topk_dev.element_size())
        a["err_d2h"] = (self._err_host.data_ptr(), self._scratch.err.data_ptr(), 4)
        a["topk_np"] = self._topk_host.numpy()
        a["err_np"] = self._err_host.numpy()
        a["plan_ptrs"] = [b.ctypes.data for b in self._plan_bufs]
        self._tail_args = a
        return a

    def _dplan_step(self, stream):
        """wnw_dplan_step: plan this step's loads on the device from the
        top-k just computed on `stream` and launch their fetch on the copy
        stream (per-layer events, as in _prepare_fetch)."""
        a = self._dplan_args
        if a is None:
            src_k, src_v = self._restore_dev_ptrs()
            a = self._dplan_args = (
                self._dplan._h, self._topk_dev.data_ptr(), int(self._topk_dev.shape[1]),
                self._scratch.err.data_ptr(), src_k, src_v, self.head_dim * self.cpu_restore_k.element_size(),
                self._land_k.data_ptr(), self._land_v.data_ptr(), int(self._land_k.shape[0]), self.fetch_ctas)
        st = N.lib.wnw_dplan_step(*a, stream, self._copy_stream.cuda_stream, self._event_handles)
        if st:
            N.check(st, "wnw_dplan_step")
        Kx.LAUNCHES[0] += 1 + self.num_layers

    def _upload_plan(self, stream):
        """The host half of a device-planned step: the rebuild plan blob to
        the device on `stream` (ahead of the next step's rebuilds)."""
        if self._chg_buf is None:
            self._chg_buf = np.zeros(self.num_layers, np.int32)
        info = N.FetchInfo()
        info.layer_changed = self._chg_buf.ctypes.data
        for _ in range(2):
            st = N.lib.wnw_planner_upload_plan(self._planner._h, self._plan_host.data_ptr(),
                                               self._plan_dev.data_ptr(), self._plan_host.numel(), stream,
                                               C.byref(info))
            if st != N.WNW_ERR_CAPACITY:
                N.check(st, "wnw_planner_upload_plan")
                break
            self._grow_plan(int(info.plan_ints))
        else:
            raise RuntimeError("wnw_planner_upload_plan: plan buffer still too small after growing it")
        self._layer_chg = self._chg_buf.tolist()
        self._after_plan(int(info.max_moved_rows), int(info.total_rows))

    def _grow_plan(self, ints):
        n = 1 << (ints - 1).bit_length()
        self._plan_host = torch.zeros(n, dtype=torch.int32).pin_memory()
        self._plan_dev = torch.zeros(n, dtype=torch.int32, device=self.device)
        self._rb_args = [None] * self.num_layers

    def _after_plan(self, moved, total):
        self._ensure_move_capacity(moved)
        # stored rows per slot after the rebuild: the planner's new lengths
        # (planner.cpp:278-357) count this step's token, every slot of every layer
        self._next_lens = self._plan_bufs[3].astype(np.int64) - 1
        self._fetched_rows = int(total)
        self._pending = True

    def _prepare_fetch(self, total, ranges):
        """Device plan + fetch of the newly needed host rows, per layer on the
        copy stream, each layer followed by its own event (the reference's
        staging cat + side-stream copy, cache.py:868-889)."""
        L = self.num_layers
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(device=self.device)
        cs = self._copy_stream
        cs.synchronize()  # the previous plan's copies no longer read the pinned buffers
        if self.fetch_mode == "zerocopy":
            info = self._issue_fetch(cs)
            moved, total = info.max_moved_rows, info.total_rows
            self._layer_chg = self._chg_buf.tolist()
            Kx.LAUNCHES[0] += int(info.fetch_launches)
        else:
            moved, total = self._prepare_fetch_dma(cs, total, ranges)
        self._after_plan(moved, total)

    def _issue_fetch(self, cs):
        """wnw_planner_issue_fetch; grows the plan / range / landing buffers
        and retries when it reports a capacity shortfall (nothing issued)."""
        row_bytes = self.head_dim * self.cpu_restore_k.element_size()
        if self._chg_buf is None:
            self._chg_buf = np.zeros(self.num_layers, np.int32)
        info = N.FetchInfo()
        info.layer_changed = self._chg_buf.ctypes.data
        for _ in range(3):
            rng_cap = self._rng_host.shape[0] if getattr(self, "_rng_host", None) is not None else 0
            land = self._land_k.shape[0] if self._land_k is not None else 0
            src_k, src_v = self._restore_dev_ptrs() if self.cpu_restore_k.shape[0] else (None, None)
            st = N.lib.wnw_planner_issue_fetch(
                self._planner._h, self._plan_host.data_ptr(), self._plan_dev.data_ptr(), self._plan_host.numel(),
                self._rng_host.data_ptr() if rng_cap else None, self._rng_dev.data_ptr() if rng_cap else None,
                self._dst_host.data_ptr() if rng_cap else None, self._dst_dev.data_ptr() if rng_cap else None,
                rng_cap, src_k, src_v, row_bytes, self._land_k.data_ptr() if land else None,
                self._land_v.data_ptr() if land else None, land, self.fetch_ctas, cs.cuda_stream,
                self._event_handles, C.byref(info))
            if st != N.WNW_ERR_CAPACITY:
                N.check(st, "wnw_planner_issue_fetch")
                return info
            if info.plan_ints > self._plan_host.numel():
                self._grow_plan(int(info.plan_ints))
            self._ensure_fetch_capacity(int(info.total_rows), int(info.n_ranges))
        raise RuntimeError("wnw_planner_issue_fetch: buffers still too small after growing them")

    def _prepare_fetch_dma(self, cs, total, ranges):
        """fetch_mode="dma": host threads gather the ranges into pinned
        staging, one cudaMemcpyAsync per layer and tensor."""
        L, D = self.num_layers, self.head_dim
        plan = self._planner.device_plan()
        if plan.size > self._plan_host.numel():
            n = 1 << (plan.size - 1).bit_length()
            self._plan_host = torch.zeros(n, dtype=torch.int32).pin_memory()
            self._plan_dev = torch.zeros(n, dtype=torch.int32, device=self.device)
            self._rb_args = [None] * L
        self._plan_host[:plan.size].copy_(torch.from_numpy(plan))
        moved = 0
        for l in range(L):
            self._layer_chg[l] = int(plan[int(plan[l])])
            moved = max(moved, int(plan[int(plan[l]) + 1]))
        rows, _ = self._planner.layer_transfer()
        self._layer_rows = rows.astype(np.int64)
        row_bytes = D * self.cpu_restore_k.element_size()
        with torch.cuda.stream(cs):
            self._plan_dev[:plan.size].copy_(self._plan_host[:plan.size], non_blocking=True)
            if total > 0:
                self._ensure_fetch_capacity(total, len(ranges))
                gather_rows(self.cpu_restore_k, self.cpu_restore_v, ranges, self._stage_k, self._stage_v,
                            self.fetch_threads)
                for l in range(L):
                    r0, r1 = int(self._layer_rows[l]), int(self._layer_rows[l + 1])
                    N.call("wnw_h2d_async", self._land_k[r0:].data_ptr(), self._land_v[r0:].data_ptr(),
                           self._stage_k[r0:].data_ptr(), self._stage_v[r0:].data_ptr(),
                           (r1 - r0) * row_bytes, cs.cuda_stream, None)
                    self._events[l].record(cs)
            else:
                for l in range(L):
                    self._events[l].record(cs)
        return moved, total

    def _ensure_move_capacity(self, rows):
        if self._move_k is None or self._move_k.shape[0] < max(1, rows):
            n = 1 << max(0, rows - 1).bit_length()
            self._move_k = torch.empty(n, self.head_dim, dtype=self.dtype, device=self.device)
            self._move_v = torch.empty(n, self.head_dim, dtype=self.dtype, device=self.device)
            self._rb_args = [None] * self.num_layers

    def _restore_dev_ptrs(self):
        if getattr(self, "_restore_ptrs", None) is None:
            if self.cpu_restore_k.is_cuda:  # offload_tier="hbm"
                self._restore_ptrs = (self.cpu_restore_k.data_ptr(), self.cpu_restore_v.data_ptr())
                return self._restore_ptrs
            if not self.cpu_restore_k.is_pinned():
                raise RuntimeError("zero-copy fetch needs the host restore store in pinned memory "
                                   "(use fetch_mode='dma')")
            self._restore_ptrs = (Kx.host_device_pointer(self.cpu_restore_k),
                                  Kx.host_device_pointer(self.cpu_restore_v))
        return self._restore_ptrs

    def _ensure_fetch_capacity(self, rows, n_ranges):
        D, dt = self.head_dim, self.dtype
        if self._land_k is None or self._land_k.shape[0] < rows:
            n = 1 << max(0, rows - 1).bit_length()
            self._land_k = torch.empty(n, D, dtype=dt, device=self.device)
            self._land_v = torch.empty(n, D, dtype=dt, device=self.device)
            if self._copy_stream is not None:  # written there: not reused until that work is done
                self._land_k.record_stream(self._copy_stream)
                self._land_v.record_stream(self._copy_stream)
            self._rb_args = [None] * self.num_layers
            self._dplan_args = None
            if self.fetch_mode == "dma":
                self._stage_k = torch.empty(n, D, dtype=dt).pin_memory()
                self._stage_v = torch.empty(n, D, dtype=dt).pin_memory()
        if self.fetch_mode == "zerocopy" and (getattr(self, "_rng_host", None) is None
                                              or self._rng_host.shape[0] < n_ranges):
            n = 1 << max(0, n_ranges - 1).bit_length()
            self._rng_host = torch.zeros(n, 2, dtype=torch.int32).pin_memory()
            self._dst_host = torch.zeros(n, dtype=torch.int64).pin_memory()
            self._rng_dev = torch.zeros(n, 2, dtype=torch.int32, device=self.device)
            self._dst_dev = torch.zeros(n, dtype=torch.int64, device=self.device)

    # ---------------------------------------------------------- inspection
    def packed_layer(self, layer_idx):
        """The reference's flat view of a layer: (K [T, D], V [T, D], cu int32)
        built by copying the slots (for checks and compatibility)."""
        l = layer_idx
        lens = self._seg_len[l]
        lens_host = self._len_host[l]
        cu = np.concatenate([[0], np.cumsum(lens_host)]).astype(np.int64)
        T = int(cu[-1])
        k = torch.empty(T, self.head_dim, dtype=self.dtype, device=self.device)
        v = torch.empty_like(k)
        Kx.copy_segments(self.k_store[l], self.v_store[l], self._seg_base[l], k, v,
                         torch.from_numpy(cu[:-1]).to(self.device), lens)
        return k, v, torch.from_numpy(cu.astype(np.int32)).to(self.device)

    def get_loaded_segments(self, b):
        return sorted(self._planner.get_loaded_segments(b)) if getattr(self, "_planner", None) else \
            sorted(self.loaded_segments[b])

    def _snapshot_cache_stats(self, step=-1):
        """Cache occupancy snapshot, the reference's fields and arithmetic
        (cache.py:1013-1080): GPU rows per sample (all, audio, per layer),
        retention against the full audio span of every (layer, kv head), and
        the host store (all rows, this sample's class-B rows, those loaded)."""
        out = []
        L, H = self.num_layers, self.num_kv_heads
        seg_rows = getattr(self, "_seg_rows", None)
        cpu_total = int(sum(int(r.sum()) for r in seg_rows)) if seg_rows is not None else 0
        dt = self._decode_step if self.prefilled else 0
        padded_prefill = (self._seq_lengths[0] - self._decode_step) if self._seq_lengths else 0
        for b in range(self.batch_size):
            n_audio = self._audio_ends_list[b] - self._audio_starts_list[b]
            full = L * H * n_audio
            post_text = max(0, max(0, padded_prefill - self.pad_lens_list[b]) - self._audio_ends_list[b])
            non_audio = self._audio_starts_list[b] + post_text
            tot, aud, per_layer = 0, 0, []
            for l in range(L):
                lens = self.seq_lens[l]
                if lens is None:
                    per_layer.append(0)
                    continue
                row = np.asarray(lens[b * H:(b + 1) * H], dtype=np.int64)
                a = int(np.maximum(row - non_audio - dt, 0).sum())
                tot += int(row.sum())
                aud += a
                per_layer.append(a)
            restore = int(seg_rows[b].sum()) if seg_rows is not None else 0
            loaded = 0
            if self.prefilled and seg_rows is not None and self.loaded_segments[b]:
                loaded = int(seg_rows[b][sorted(self.loaded_segments[b])].sum())
            out.append({"step": step, "num_audio": n_audio, "gpu_audio_tokens": aud, "gpu_total_tokens": tot,
                        "audio_retention": aud / full if full > 0 else 1.0, "per_layer_audio_tokens": per_layer,
                        "cpu_total_tokens": cpu_total, "cpu_loaded_tokens": loaded,
                        "cpu_restore_tokens": restore,
                        "gpu_plus_cpu_retention": (aud + restore) / full if full > 0 else 1.0})
        return out

    def get_snapshot_stats(self, step=-1):
        """The snapshot under its public name (cache.py:1082-1084)."""
        return self._snapshot_cache_stats(step=step)

    def get_compression_stats(self):
        """The snapshot at step -1 (cache.py:1086-1088)."""
        return self._snapshot_cache_stats(step=-1)

    def collect_stats(self, interval=20):
        """Collect InferenceStats every ``interval`` decode steps; 0 turns
        collection off (cache.py:136-138)."""
        self.stats.set_interval(interval)

    def get_all_stats(self):
        """Per-sample stats of the run (cache.py:140-142)."""
        return self.stats.get_all_stats()

    def _segment_host_rows(self):
        """Per sample, the host rows of each segment summed over every class-B
        (layer, kv head): what loading or evicting that segment moves."""
        L, H = self.num_layers, self.num_kv_heads
        cs, ce = self._meta["cpu_s"], self._meta["cpu_e"]
        rows = []
        for b in range(self.batch_size):
            n = self.seg_count[b]
            r = np.zeros(n, np.int64)
            for l in range(L):
                for h in range(H):
                    if self.config.is_class_b(l, h):
                        m0 = int(self._meta_base[l, b * H + h])
                        s, e = cs[m0:m0 + n].astype(np.int64), ce[m0:m0 + n].astype(np.int64)
                        r += np.where(s >= 0, e - s, 0)
            rows.append(r)
        return rows
