"""CPU restatement of the WnW cache state machine -- TEST INFRASTRUCTURE ONLY.

``OracleWnWCache`` follows ``src/algorithms/wnw/code/cache.py`` (class
``WnWCache``) hook by hook, on CPU torch tensors, so that the rebuilt GPU cache
can be driven with identical inputs and compared step by step:

* prefill compression and CPU offload      -- cache.py:257-390, 1092-1150
* decode append                            -- cache.py:487-515 (kernels.py:7-73)
* fused decode attention + class-A scoring -- cache.py:517-566 (fused_attn.py)
* chunk selection with eviction lag        -- cache.py:579-649
* rebuild planning and application         -- cache.py:716-889 (kernels.py:375-473)

Attention is computed in float64 from the stored rows; the score accumulator is
fp32 like the reference's, with per-segment contributions formed in float64
and added in layer-major, ascending-kv-head order (the reference's non-fused
order, cache.py:535-544).  Top-k ties go to the lower index.

The config object only needs the reference ``WnWConfig`` interface
(``src/algorithms/wnw/code/config.py``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from itertools import accumulate

import numpy as np
import torch

from oracle import kernels as K


@dataclass
class SegmentMeta:
    """cache.py:18-24."""
    cpu_start: int
    cpu_end: int
    gpu_rel_start: int = -1
    gpu_rel_end: int = -1


def compute_segments(num_audio, stride):
    """cache.py:1092-1094."""
    return [(i * stride, min(i * stride + stride, num_audio))
            for i in range(math.ceil(num_audio / stride))]


def compute_chunks(segments, chunk_size, stride):
    """cache.py:1097-1101."""
    spc = math.ceil(chunk_size / stride)
    n = len(segments)
    return [list(range(i, min(i + spc, n))) for i in range(n)]


def select_topk_per_segment(scores, seg_ranges, ratio):
    """cache.py:1114-1138 (torch CPU so tie handling equals the reference's CPU run)."""
    num_audio = scores.shape[0]
    kept = torch.zeros(num_audio, dtype=torch.bool)
    if not seg_ranges:
        return kept
    stride = seg_ranges[0][1] - seg_ranges[0][0]
    last_len = seg_ranges[-1][1] - seg_ranges[-1][0]
    n_full = len(seg_ranges) if last_len == stride else len(seg_ranges) - 1
    if n_full > 0:
        n_keep = max(1, int(stride * ratio))
        block = scores[:n_full * stride].reshape(n_full, stride)
        idx = block.topk(n_keep, dim=1).indices
        row_off = (torch.arange(n_full) * stride).unsqueeze(1)
        kept[(idx + row_off).reshape(-1)] = True
    if n_full < len(seg_ranges):
        s0, s1 = seg_ranges[-1]
        n_keep = max(1, int((s1 - s0) * ratio))
        kept[scores[s0:s1].topk(n_keep).indices + s0] = True
    return kept


def select_topk_global(scores, seg_ranges, ratio):
    """cache.py:1141-1150."""
    num_audio = scores.shape[0]
    n_keep = sum(max(1, int((e - s) * ratio)) for s, e in seg_ranges)
    n_keep = min(n_keep, num_audio)
    kept = torch.zeros(num_audio, dtype=torch.bool)
    kept[scores.topk(n_keep).indices] = True
    return kept


class OracleWnWCache:
    """Hook-compatible CPU restatement of ``WnWCache``."""

    def __init__(self, config, num_layers, num_kv_heads, num_q_heads, head_dim):
        self.config = config
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.num_q_heads = num_q_heads
        self.num_kv_groups = num_q_heads // num_kv_heads
        self.head_dim = head_dim
        self.prefilled = False
        self._class_b_heads_by_layer = [config.get_layer_class_b(l) for l in range(num_layers)]

    # ---------------------------------------------------------------- setup
    def setup_audio(self, audio_starts, audio_ends, pad_lens=None):
        """cache.py:144-250 (pad lens passed directly instead of a mask)."""
        a_s = [int(x) for x in audio_starts]
        a_e = [int(x) for x in audio_ends]
        pad = [0] * len(a_s) if pad_lens is None else [int(x) for x in pad_lens]
        self.batch_size = B = len(a_s)
        self._raw_audio_starts = a_s
        self._raw_audio_ends = a_e
        self.pad_lens_list = pad
        self._audio_starts_list = [s - p for s, p in zip(a_s, pad)]
        self._audio_ends_list = [e - p for e, p in zip(a_e, pad)]
        stride = self.config.stride_tokens
        self.segment_ranges = [compute_segments(self._audio_ends_list[b] - self._audio_starts_list[b], stride)
                               for b in range(B)]
        self.chunk_to_segs = [compute_chunks(self.segment_ranges[b], self.config.chunk_size_tokens, stride)
                              for b in range(B)]
        self.chunk_bounds = []
        for b in range(B):
            bounds = []
            for segs in self.chunk_to_segs[b]:
                bounds.append((self.segment_ranges[b][segs[0]][0], self.segment_ranges[b][segs[-1]][1])
                              if segs else (0, 0))
            self.chunk_bounds.append(bounds)
        audio_lens = [self._audio_ends_list[b] - self._audio_starts_list[b] for b in range(B)]
        self.score_offsets = [0] + list(accumulate(audio_lens))
        self.score_accumulator = np.zeros(self.score_offsets[-1], dtype=np.float32)
        self._prefill_scores = [[] for _ in range(B)]
        self.loaded_segments = [set() for _ in range(B)]
        self.eviction_counters = [{} for _ in range(B)]
        L = self.num_layers
        self.layer_k = [None] * L
        self.layer_v = [None] * L
        self.seq_lens = [None] * L
        self.restore_meta = [[[[None] * len(self.segment_ranges[b]) for _ in range(self.num_kv_heads)]
                              for b in range(B)] for _ in range(L)]
        self._cpu_k, self._cpu_v, self._cpu_metas = [], [], []
        self._seg_to_load = [set() for _ in range(B)]
        self._seg_to_evict = [set() for _ in range(B)]
        self._pending = None
        self.decode_step = 0
        self.prefilled = False
        # per-step records for comparisons
        self.last_scores = None
        self.last_topk = [[] for _ in range(B)]
        self.last_to_load = [[] for _ in range(B)]
        self.last_to_evict = [[] for _ in range(B)]

    def cu(self, layer):
        return np.asarray([0] + list(accumulate(self.seq_lens[layer])), dtype=np.int64)

    # -------------------------------------------------------------- prefill
    def prefill_after_attn(self, layer_idx, class_a_scores, per_head_scores, key_states, value_states):
        """cache.py:257-349."""
        cfg = self.config
        for b in range(self.batch_size):
            if class_a_scores[b] is not None:
                self._prefill_scores[b].append(torch.as_tensor(class_a_scores[b]).float().cpu())
        pk, pv, lens = [], [], []
        ks = torch.as_tensor(key_states).cpu()
        vs = torch.as_tensor(value_states).cpu()
        for b in range(self.batch_size):
            ra0, ra1 = self._raw_audio_starts[b], self._raw_audio_ends[b]
            pad = self.pad_lens_list[b]
            for h in range(self.num_kv_heads):
                kf, vf = ks[b, h], vs[b, h]
                if cfg.is_class_a_kv_head(layer_idx, h):
                    pk.append(kf[pad:]); pv.append(vf[pad:]); lens.append(kf.shape[0] - pad)
                    continue
                ratio = cfg.get_retention(layer_idx, h)
                hs = torch.as_tensor(per_head_scores[b][h]).float().cpu()
                if cfg.prefill_global_topk:
                    kept = select_topk_global(hs, self.segment_ranges[b], ratio)
                else:
                    kept = select_topk_per_segment(hs, self.segment_ranges[b], ratio)
                na_k = torch.cat([kf[pad:ra0], kf[ra1:]], 0)
                na_v = torch.cat([vf[pad:ra0], vf[ra1:]], 0)
                ak, av = kf[ra0:ra1], vf[ra0:ra1]
                pk.append(torch.cat([na_k, ak[kept]], 0))
                pv.append(torch.cat([na_v, av[kept]], 0))
                lens.append(na_k.shape[0] + int(kept.sum()))
                if cfg.is_class_b(layer_idx, h):
                    ridx = (~kept).nonzero(as_tuple=True)[0]
                    if ridx.numel() > 0:
                        rk, rv = ak.index_select(0, ridx), av.index_select(0, ridx)
                        nsegs = len(self.segment_ranges[b])
                        counts = torch.bincount(ridx // cfg.stride_tokens, minlength=nsegs)
                        off = 0
                        for si in range(nsegs):
                            n = int(counts[si])
                            if n > 0:
                                self._cpu_k.append(rk[off:off + n]); self._cpu_v.append(rv[off:off + n])
                                self._cpu_metas.append((layer_idx, b, h, si, n))
                                off += n
        self.layer_k[layer_idx] = torch.cat(pk, 0)
        self.layer_v[layer_idx] = torch.cat(pv, 0)
        self.seq_lens[layer_idx] = lens

    def prefill_all_layers_done(self):
        """cache.py:351-390 and the decode constants of cache.py:408-468."""
        if self._cpu_k:
            self.cpu_restore_k = torch.cat(self._cpu_k, 0)
            self.cpu_restore_v = torch.cat(self._cpu_v, 0)
            off = 0
            for l, b, h, si, n in self._cpu_metas:
                self.restore_meta[l][b][h][si] = SegmentMeta(off, off + n)
                off += n
        else:
            dt = self.layer_k[0].dtype
            self.cpu_restore_k = torch.empty(0, self.head_dim, dtype=dt)
            self.cpu_restore_v = torch.empty(0, self.head_dim, dtype=dt)
        self._cpu_k, self._cpu_v, self._cpu_metas = [], [], []
        for b in range(self.batch_size):
            if self._prefill_scores[b]:
                avg = torch.stack(self._prefill_scores[b]).sum(dim=0)
            else:
                avg = torch.ones(self._audio_ends_list[b] - self._audio_starts_list[b])
            to_load, _ = self._chunk_changes(b, avg.numpy().astype(np.float32))
            if to_load:
                self._load_segments_for_sample(b, to_load)
            self.loaded_segments[b] = to_load
            self._prefill_scores[b] = []
        self.prefilled = True
        self._precompute()

    def _precompute(self):
        cfg, G = self.config, self.num_kv_groups
        self.score_groups = []   # per layer: list of (kv_head, [local q offsets]) ascending kv
        self.foldable = []
        for l in range(self.num_layers):
            ca = cfg.get_layer_class_a(l)
            by_kv = {}
            for qh in ca:
                by_kv.setdefault(qh // G, []).append(qh)
            self.score_groups.append([(kv, [q - kv * G for q in qs]) for kv, qs in sorted(by_kv.items())])
            if not ca:
                self.foldable.append(False)
                continue
            cas = set(ca)
            self.foldable.append(all(set(range(kv * G, (kv + 1) * G)).issubset(cas) for kv in by_kv))
        self.any_class_a = any(self.score_groups[l] for l in range(self.num_layers))

    def _load_segments_for_sample(self, b, segs):
        """cache.py:651-714 (initial, synchronous chunk load)."""
        segs = sorted(segs)
        H = self.num_kv_heads
        for l in range(self.num_layers):
            cu = self.cu(l)
            pk, pv, lens = [], [], []
            for fi in range(self.batch_size * H):
                bb, h = divmod(fi, H)
                s, e = int(cu[fi]), int(cu[fi + 1])
                pk.append(self.layer_k[l][s:e]); pv.append(self.layer_v[l][s:e])
                rel = e - s
                extra = 0
                if bb == b and self.config.is_class_b(l, h):
                    for si in segs:
                        m = self.restore_meta[l][bb][h][si]
                        if m is None:
                            continue
                        n = m.cpu_end - m.cpu_start
                        pk.append(self.cpu_restore_k[m.cpu_start:m.cpu_end])
                        pv.append(self.cpu_restore_v[m.cpu_start:m.cpu_end])
                        m.gpu_rel_start, m.gpu_rel_end = rel, rel + n
                        rel += n
                        extra += n
                lens.append(e - s + extra)
            self.layer_k[l] = torch.cat(pk, 0)
            self.layer_v[l] = torch.cat(pv, 0)
            self.seq_lens[l] = lens

    # --------------------------------------------------------------- decode
    def decode_before_attn(self, layer_idx, new_k, new_v):
        """cache.py:487-515 / 716-754: rebuild (if pending) or append."""
        # rows are moved as fp32 numpy (exact for fp16 / bf16) and cast back
        dt = self.layer_k[layer_idx].dtype
        nk = torch.as_tensor(new_k).cpu().reshape(-1, self.head_dim).float()
        nv = torch.as_tensor(new_v).cpu().reshape(-1, self.head_dim).float()
        cu_old = self.cu(layer_idx)
        if self._pending is not None:
            p = self._pending[layer_idx]
            out_k = K.rebuild_append(self.layer_k[layer_idx].float().numpy(), nk.numpy(), p["load_k"],
                                     cu_old, p["cu_new"], p["load_starts"], p["load_lens"],
                                     p["ev_off"], p["ev_s"], p["ev_e"])
            out_v = K.rebuild_append(self.layer_v[layer_idx].float().numpy(), nv.numpy(), p["load_v"],
                                     cu_old, p["cu_new"], p["load_starts"], p["load_lens"],
                                     p["ev_off"], p["ev_s"], p["ev_e"])
            self.layer_k[layer_idx] = torch.from_numpy(out_k).to(dt)
            self.layer_v[layer_idx] = torch.from_numpy(out_v).to(dt)
            self.seq_lens[layer_idx] = list(p["new_lens"])
            if layer_idx == self.num_layers - 1:
                self._pending = None
        else:
            ok, _ = K.interleave_append(self.layer_k[layer_idx].float().numpy(), nk.numpy(), cu_old)
            ov, _ = K.interleave_append(self.layer_v[layer_idx].float().numpy(), nv.numpy(), cu_old)
            self.layer_k[layer_idx] = torch.from_numpy(ok).to(dt)
            self.layer_v[layer_idx] = torch.from_numpy(ov).to(dt)
            self.seq_lens[layer_idx] = [x + 1 for x in self.seq_lens[layer_idx]]
        return self.layer_k[layer_idx], self.layer_v[layer_idx], self.cu(layer_idx), max(self.seq_lens[layer_idx])

    def _score_layer(self, layer_idx, q_groups, scale_fn):
        """Class-A scoring of one layer: per kv group, full-segment softmax over the
        group's class-A q heads, audio range summed over heads (fp64), then added
        to the fp32 accumulator in ascending kv order (cache.py:517-544)."""
        if not self.any_class_a:
            return
        cu = self.cu(layer_idx)
        kk = self.layer_k[layer_idx].double().numpy()
        for kv, qoffs in self.score_groups[layer_idx]:
            for b in range(self.batch_size):
                fi = b * self.num_kv_heads + kv
                s, e = int(cu[fi]), int(cu[fi + 1])
                a0, a1 = self._audio_starts_list[b], self._audio_ends_list[b]
                q = q_groups[fi][qoffs]                       # [nh, D] float64
                logits = q @ kk[s:e].T * scale_fn(q.shape[-1])
                m = logits.max(axis=1, keepdims=True)
                p = np.exp(logits - m)
                p = p / p.sum(axis=1, keepdims=True)
                contrib = p[:, a0:a1].sum(axis=0).astype(np.float32)
                off = self.score_offsets[b]
                self.score_accumulator[off:off + (a1 - a0)] += contrib

    def fused_decode_attention(self, layer_idx, q_flat, q=None, k_flat=None, v_flat=None, cu_k=None,
                               scale=None):
        """cache.py:546-566: attention over the current layer; class-A scoring
        with the attention scale for foldable layers, else with 1/sqrt(d)
        (kernels.py:149, 354)."""
        qt = torch.as_tensor(q_flat)
        qf = qt.cpu().double().numpy()
        out, _, _ = K.decode_attn(qf, self.layer_k[layer_idx].double().numpy(),
                                  self.layer_v[layer_idx].double().numpy(), self.cu(layer_idx), scale)
        if self.score_groups and self.score_groups[layer_idx]:
            if self.foldable[layer_idx]:
                self._score_layer(layer_idx, qf, lambda d: scale)
            else:
                self._score_layer(layer_idx, qf, lambda d: 1.0 / math.sqrt(d))
        self.last_out64 = out
        return torch.from_numpy(out).to(qt.dtype)

    def decode_all_layers_done(self):
        """cache.py:568-600, 756-889."""
        self.decode_step += 1
        self.last_scores = self.score_accumulator.copy()
        any_change = False
        for b in range(self.batch_size):
            o0, o1 = self.score_offsets[b], self.score_offsets[b + 1]
            tl_, te_ = self._chunk_changes(b, self.score_accumulator[o0:o1])
            self._seg_to_load[b], self._seg_to_evict[b] = tl_, te_
            self.last_to_load[b], self.last_to_evict[b] = sorted(tl_), sorted(te_)
            any_change |= bool(tl_ or te_)
        if any_change:
            self._prepare_pending()
        self.score_accumulator[:] = 0

    def _select(self, b, cs, k):
        """The k chunks of sample b to keep loaded (cache.py:641-642)."""
        return K.topk_lower_index(cs, k)

    def _chunk_changes(self, b, scores):
        """cache.py:632-649 then 609-630."""
        bounds = self.chunk_bounds[b]
        if not bounds:
            self.last_topk[b] = []
            return set(), set()
        cs = K.chunk_scores(scores, [x for x, _ in bounds], [y for _, y in bounds])
        k = min(self.config.top_k_chunks, len(cs))
        if k == 0:
            self.last_topk[b] = []
            return set(), set()
        top = self._select(b, cs, k)
        self.last_topk[b] = sorted(top)
        needed = {si for ci in top for si in self.chunk_to_segs[b][ci]}
        loaded = self.loaded_segments[b]
        counters = self.eviction_counters[b]
        to_load = needed - loaded
        to_evict = set()
        for si in loaded:
            if si not in needed:
                counters[si] = counters.get(si, 0) + 1
                if counters[si] >= self.config.eviction_lag:
                    to_evict.add(si)
            else:
                counters.pop(si, None)
        self.loaded_segments[b] = (loaded | to_load) - to_evict
        for si in to_evict:
            counters.pop(si, None)
        return to_load, to_evict

    def _prepare_pending(self):
        """cache.py:756-889: per-layer evict ranges, loads and new lengths."""
        H = self.num_kv_heads
        S = self.batch_size * H
        changed = [b for b in range(self.batch_size) if self._seg_to_load[b] or self._seg_to_evict[b]]
        ranges = []
        pend = []
        gts = 0
        for l in range(self.num_layers):
            lens = self.seq_lens[l]
            new_lens = [x + 1 for x in lens]
            ev_by_seg = [[] for _ in range(S)]
            loads = []
            for b in changed:
                for h in self._class_b_heads_by_layer[l]:
                    fi = b * H + h
                    seg_len = lens[fi]
                    evicted = 0
                    metas = self.restore_meta[l][b][h]
                    if self._seg_to_evict[b]:
                        ev = []
                        for si in self._seg_to_evict[b]:
                            m = metas[si]
                            if m is not None and m.gpu_rel_start >= 0:
                                ev.append((m.gpu_rel_start, m.gpu_rel_end))
                                m.gpu_rel_start = m.gpu_rel_end = -1
                        ev.sort()
                        ev_by_seg[fi] = ev
                        evicted = sum(e - s for s, e in ev)
                        if ev:
                            for si, m in enumerate(metas):
                                if m is None or m.gpu_rel_start < 0 or si in self._seg_to_evict[b]:
                                    continue
                                sh = sum(e - s for s, e in ev if e <= m.gpu_rel_start)
                                m.gpu_rel_start -= sh
                                m.gpu_rel_end -= sh
                    rel = seg_len - evicted
                    loaded = 0
                    for si in sorted(self._seg_to_load[b]):
                        m = metas[si]
                        if m is None:
                            continue
                        n = m.cpu_end - m.cpu_start
                        ranges.append((m.cpu_start, m.cpu_end))
                        loads.append((fi, gts, n))
                        m.gpu_rel_start, m.gpu_rel_end = rel, rel + n
                        rel += n
                        loaded += n
                        gts += n
                    new_lens[fi] = seg_len - evicted + loaded + 1
            ls = np.full(S, -1, np.int64)
            ll = np.zeros(S, np.int64)
            for fi, ts, n in loads:
                if ls[fi] < 0:
                    ls[fi] = ts
                ll[fi] += n
            ev_off = [0]
            ev_s, ev_e = [], []
            for fi in range(S):
                for s_, e_ in ev_by_seg[fi]:
                    ev_s.append(s_); ev_e.append(e_)
                ev_off.append(len(ev_s))
            pend.append(dict(load_starts=ls, load_lens=ll, new_lens=new_lens,
                             cu_new=np.asarray([0] + list(accumulate(new_lens)), np.int64),
                             ev_off=np.asarray(ev_off), ev_s=np.asarray(ev_s, np.int64),
                             ev_e=np.asarray(ev_e, np.int64)))
        lk, lv = K.gather_restore(self.cpu_restore_k.float().numpy(), self.cpu_restore_v.float().numpy(), ranges)
        for p in pend:
            p["load_k"], p["load_v"] = lk, lv
        self.last_ranges = ranges
        self._pending = pend

    # ----------------------------------------------------------- utilities
    def packed(self, layer):
        return self.layer_k[layer], self.layer_v[layer], self.cu(layer)
