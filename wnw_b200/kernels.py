"""Torch-tensor wrappers over the C ABI kernels (all launches go through
``libwnw_b200.so``; nothing here computes on its own)."""
from __future__ import annotations

import ctypes as C
import math

import numpy as np
import torch

from wnw_b200 import native as N

#: kernel launches issued through these wrappers (bench.py reports it)
LAUNCHES = [0]


def _count(n=1):
    LAUNCHES[0] += n


def split_rows(dtype, head_dim):
    """Rows per CTA of the CUDA-core kernel (0 for the tensor-core path)."""
    return N.lib.wnw_split_rows(N.dtype_code(dtype), int(head_dim))


def uses_plan(dtype, head_dim):
    """True when 16-bit K/V with this head_dim take the tensor-core kernel,
    which is launched from a work plan (``attn_plan``)."""
    return dtype in (torch.bfloat16, torch.float16) and int(head_dim) in (64, 128)


def attn_launch_shape(dtype, head_dim, seg_cap):
    """(split_rows, cluster_size) of the CUDA-core kernel for one layer's
    capacities (``wnw_attn_launch_shape``)."""
    cap = np.ascontiguousarray(np.asarray(seg_cap, dtype=np.int32))
    split, cs = C.c_int(), C.c_int()
    N.call("wnw_attn_launch_shape", N.dtype_code(dtype), int(head_dim), N.ptr(cap), cap.size, C.byref(split),
           C.byref(cs))
    return split.value, cs.value


def choose_cluster_size(max_rows, split):
    """Clusters of up to 8 CTAs; smaller when even the longest segment needs
    fewer splits (idle cluster members only cost a barrier)."""
    nsplit = max(1, math.ceil((int(max_rows) + 1) / split))
    cs = 1
    while cs < nsplit and cs < 8:
        cs *= 2
    return cs


def build_work_table(seg_cap, split, cluster_size):
    """numpy int32 [n_clusters, 2] (segment, cluster index) from capacities."""
    cap = np.ascontiguousarray(np.asarray(seg_cap, dtype=np.int32))
    n = C.c_int()
    N.lib.wnw_build_work_table(N.ptr(cap), cap.size, split, cluster_size, None, 0, C.byref(n))
    work = np.zeros((max(1, n.value), 2), np.int32)
    N.call("wnw_build_work_table", N.ptr(cap), cap.size, split, cluster_size, N.ptr(work), n.value, C.byref(n))
    return work[:n.value]


def attn_plan(seg_cap, sm_count=None, max_cluster=None):
    """(numpy int32 plan, info) of the tensor-core kernel for one layer's
    capacities (``wnw_attn_plan``; None: the current device's SMs and
    largest cluster).  info = dict(ctas, cluster, parts, combine)."""
    cap = np.ascontiguousarray(np.asarray(seg_cap, dtype=np.int32))
    info = N.AttnPlanInfo()
    args = (N.ptr(cap), cap.size, int(sm_count or 0), int(max_cluster or 0))
    N.call("wnw_attn_plan", *args, None, 0, C.byref(info))
    plan = np.zeros(int(info.ints), np.int32)
    N.call("wnw_attn_plan", *args, N.ptr(plan), plan.size, C.byref(info))
    return plan, dict(ctas=info.ctas, cluster=info.cluster, parts=info.parts, combine=info.combine)


class AttnWork:
    """Launch layout of one layer's decode attention, from its slot
    capacities: the work plan of the tensor-core kernel, or the cluster work
    table (rows per CTA ``split``, ``cluster_size``) of the CUDA-core kernel.
    ``slots`` = partial states the layout can write (the scratch size),
    ``table`` = the device tensor the launch reads."""

    def __init__(self, dtype, head_dim, seg_cap, device, sm_count=None, max_cluster=None, split=None,
                 cluster_size=None):
        self.plan = uses_plan(dtype, head_dim)
        if self.plan:
            p, info = attn_plan(seg_cap, sm_count, max_cluster)
            self.table = torch.from_numpy(p).to(device)
            self.ctas, self.cluster_size = info["ctas"], info["cluster"]
            self.parts, self.combine = info["parts"], info["combine"]
            self.slots, self.split = max(1, self.parts), 0
        else:
            if split is None or cluster_size is None:
                split, cluster_size = attn_launch_shape(dtype, head_dim, seg_cap)
            w = build_work_table(seg_cap, split, cluster_size)
            self.table = torch.from_numpy(w).to(device)
            self.split, self.cluster_size = split, cluster_size
            self.slots = self.n_clusters = w.shape[0]
            self.ctas, self.parts, self.combine = 0, 0, 0

    @property
    def launches(self):
        """Kernel launches of one attention call with this layout."""
        return 1

    def fill(self, a):
        """Write the layout fields of a ``DecodeAttnArgs``."""
        if self.plan:
            a.plan = self.table.data_ptr()
            a.plan_ctas, a.plan_parts, a.plan_combine = self.ctas, self.parts, self.combine
            a.work, a.n_clusters, a.cluster_size, a.split_rows = None, 0, self.cluster_size, 0
        else:
            a.plan, a.plan_ctas, a.plan_parts, a.plan_combine = None, 0, 0, 0
            a.work = self.table.data_ptr()
            a.n_clusters, a.cluster_size, a.split_rows = self.slots, self.cluster_size, self.split


class AttnScratch:
    """Scratch of the decode-attention kernel: per-cluster partial states and
    per-segment arrival counters (zeroed once; the kernel leaves them zero),
    plus the device error word."""

    def __init__(self, device, n_clusters, group, head_dim, num_segs):
        self.partials = torch.empty(max(1, n_clusters) * group * (head_dim + 2), dtype=torch.float32,
                                    device=device)
        self.counters = torch.zeros(max(1, num_segs), dtype=torch.int32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)
        self.n_clusters, self.group, self.head_dim, self.num_segs = n_clusters, group, head_dim, num_segs

    def fits(self, n_clusters, group, head_dim, num_segs):
        return (n_clusters * group * (head_dim + 2) <= self.partials.numel() and num_segs <= self.counters.numel())


def make_attn_args(dtype, S, G, D, k_store, v_store, seg_base, seg_len, work, scale, scratch,
                   seg_cap=None, num_kv_heads=None, score=None, flags=0):
    """A reusable ``wnw_decode_attn_args`` with everything but q / new rows /
    out filled in (the per-layer constant part of a decode step); ``work`` is
    the layer's ``AttnWork``.  The struct keeps references to every tensor it
    points at, so temporaries passed in stay alive as long as the arguments
    do."""
    a = N.DecodeAttnArgs()
    a._keep = (k_store, v_store, seg_base, seg_len, work, scratch, seg_cap, score)
    a.dtype = N.dtype_code(dtype)
    a.head_dim, a.group, a.num_segs = D, G, S
    a.num_kv_heads = num_kv_heads if num_kv_heads is not None else S
    a.k_store, a.v_store = k_store.data_ptr(), v_store.data_ptr()
    a.seg_base, a.seg_len = seg_base.data_ptr(), seg_len.data_ptr()
    a.seg_cap = seg_cap.data_ptr() if seg_cap is not None else None
    work.fill(a)
    a.scale = float(scale)
    if score is not None:
        a.score_slot = score["slot"].data_ptr()
        a.audio_start = score["audio_start"].data_ptr()
        a.audio_end = score["audio_end"].data_ptr()
        a.logits = score["logits"].data_ptr()
        a.logits_off = score["logits_off"].data_ptr()
        a.stats = score["stats"].data_ptr() if score.get("stats") is not None else None
    a.partials = scratch.partials.data_ptr()
    a.counters = scratch.counters.data_ptr()
    a.err = scratch.err.data_ptr()
    a.store_rows = k_store.shape[0]
    a.flags = int(flags)
    return a


def launch_attn(args, q, new_k, new_v, out, stream_handle):
    """Fill the per-step pointers of a prepared args struct and launch."""
    args.q = q.data_ptr()
    args.new_k = new_k.data_ptr() if new_k is not None else None
    args.new_v = new_v.data_ptr() if new_v is not None else None
    args.out = out.data_ptr()
    st = N.lib.wnw_decode_attn(C.byref(args), stream_handle)
    if st:
        N.check(st, "wnw_decode_attn")
    LAUNCHES[0] += 1
    return out


def fetch_rows(src_k_dev, src_v_dev, row_bytes, ranges, dst_row, dst_k, dst_v, max_ctas=256, stream=None):
    """Zero-copy gather of host rows (device addresses of pinned memory)."""
    n = ranges.shape[0]
    if n == 0:
        return
    N.call("wnw_fetch_rows", src_k_dev, src_v_dev, int(row_bytes), ranges.data_ptr(), dst_row.data_ptr(), int(n),
           dst_k.data_ptr(), dst_v.data_ptr(), int(max_ctas), N.stream_ptr(stream))
    _count()


def host_device_pointer(t):
    """Device address of a pinned host tensor (raises if it is not mapped)."""
    out = C.c_void_p()
    N.call("wnw_host_device_pointer", t.data_ptr(), C.byref(out))
    return out.value


def decode_attention(q, k_store, v_store, seg_base, seg_len, work, scale, scratch,
                     new_k=None, new_v=None, seg_cap=None, out=None, num_kv_heads=None, score=None,
                     stream=None, flags=0):
    """Launch ``wnw_decode_attn``.  q: [S, G, D]; ``work``: the layer's
    ``AttnWork`` (built from capacities >= every segment's rows).
    ``score`` (optional) = dict(slot=int32[S], audio_start=int32[B], audio_end=int32[B],
    logits=fp32 buffer, logits_off=int64[n_slots], stats=fp32 [S, 2, G])."""
    S, G, D = q.shape
    if out is None:
        out = torch.empty_like(q)
    a = make_attn_args(q.dtype, S, G, D, k_store, v_store, seg_base, seg_len, work, scale, scratch,
                       seg_cap=seg_cap, num_kv_heads=num_kv_heads, score=score, flags=flags)
    a.q = q.data_ptr()
    a.new_k = new_k.data_ptr() if new_k is not None else None
    a.new_v = new_v.data_ptr() if new_v is not None else None
    a.out = out.data_ptr()
    N.check(N.lib.wnw_decode_attn(C.byref(a), N.stream_ptr(stream)), "wnw_decode_attn")
    _count(work.launches)
    return out


def advance_lengths(seg_len, stream=None):
    N.call("wnw_advance_lengths", seg_len.data_ptr(), seg_len.numel(), N.stream_ptr(stream))
    _count()


def score_finalize(logits, stats, logit_off, stat_off, qmask, term_off, group, score_off, max_audio, acc,
                   stream=None):
    batch = score_off.numel() - 1
    N.call("wnw_score_finalize", logits.data_ptr(), stats.data_ptr(), logit_off.data_ptr(),
           stat_off.data_ptr(), qmask.data_ptr(), term_off.data_ptr(), int(group), int(batch),
           score_off.data_ptr(), int(max_audio), acc.data_ptr(), N.stream_ptr(stream))
    _count()


def chunk_topk(acc, score_off, max_audio, stride, segs_per_chunk, top_k, topk_out, chunk_scores=None,
               chunk_off=None, stream=None):
    batch = score_off.numel() - 1
    N.call("wnw_chunk_topk", acc.data_ptr(), score_off.data_ptr(), int(batch), int(max_audio), int(stride),
           int(segs_per_chunk), int(top_k), topk_out.data_ptr(),
           chunk_scores.data_ptr() if chunk_scores is not None else None,
           chunk_off.data_ptr() if chunk_off is not None else None, N.stream_ptr(stream))
    _count()


def rebuild_layer(k_store, v_store, seg_base, seg_len, seg_cap, k_landing, v_landing, plan_blob, layer,
                  k_move, v_move, status, err, stream=None):
    """Compaction + splice of one layer's changed slots (two launches)."""
    N.call("wnw_rebuild_segments", N.dtype_code(k_store.dtype), k_store.shape[1], k_store.data_ptr(),
           v_store.data_ptr(), seg_base.data_ptr(), seg_len.data_ptr(), seg_cap.data_ptr(), int(seg_len.numel()),
           k_landing.data_ptr() if k_landing is not None else None,
           v_landing.data_ptr() if v_landing is not None else None,
           int(k_landing.shape[0]) if k_landing is not None else 0, plan_blob.data_ptr(), int(plan_blob.numel()),
           int(layer), k_move.data_ptr() if k_move is not None else None,
           v_move.data_ptr() if v_move is not None else None,
           int(k_move.shape[0]) if k_move is not None else 0, status.data_ptr(), err.data_ptr(),
           N.stream_ptr(stream))
    _count(2)


def rebuild_layers_fused(layers, changed, k_landing, v_landing, plan_blob, k_move, v_move, status, err,
                         stream=None):
    """Every changed layer's compaction + splice in one gather and one scatter
    launch.  ``layers``: per layer (k_store, v_store, seg_base, seg_len,
    seg_cap); ``changed``: per layer 0 / 1."""
    L = len(layers)
    P = C.c_void_p
    arr = lambda i: (P * L)(*[t[i].data_ptr() for t in layers])  # noqa: E731
    chg = np.ascontiguousarray(changed, np.int32)
    nsegs = (C.c_int32 * L)(*[int(t[3].numel()) for t in layers])
    k0 = layers[0][0]
    N.call("wnw_rebuild_layers_fused", N.dtype_code(k0.dtype), k0.shape[1], L, chg.ctypes.data, arr(0), arr(1),
           arr(2), arr(3), arr(4), nsegs, k_landing.data_ptr() if k_landing is not None else None,
           v_landing.data_ptr() if v_landing is not None else None,
           int(k_landing.shape[0]) if k_landing is not None else 0, plan_blob.data_ptr(), int(plan_blob.numel()),
           k_move.data_ptr() if k_move is not None else None, v_move.data_ptr() if v_move is not None else None,
           int(k_move.shape[0]) if k_move is not None else 0, status.data_ptr(), int(status.numel()),
           err.data_ptr(), None, None, N.stream_ptr(stream))
    _count(2 * ((int(chg.astype(bool).sum()) + 47) // 48))


def plan_record(blob, layer):
    """Host-side view of one layer record of a device-plan blob (numpy int32)."""
    o = int(blob[layer])
    n, moved, out = (int(x) for x in blob[o:o + 3])
    f = o + 3
    rec = {"n": n, "moved_total": moved, "out_total": out}
    for name in ("seg", "old_len", "new_len", "load_src", "load_len"):
        rec[name] = blob[f:f + n]
        f += n
    for name in ("mov_off", "out_off", "ev_off"):
        rec[name] = blob[f:f + n + 1]
        f += n + 1
    ne = int(rec["ev_off"][-1]) if n else 0
    rec["ev_s"] = blob[f:f + ne]
    rec["ev_e"] = blob[f + ne:f + 2 * ne]
    return rec


def pack_plan(layers):
    """Build a device-plan blob from per-layer lists of records
    (seg, old_len, new_len, load_src, load_len, [(ev_s, ev_e), ...]); the same
    format wnw_planner_device_plan writes (used by tests)."""
    L = len(layers)
    out = [0] * (L + 1)
    for l, recs in enumerate(layers):
        out[l] = len(out)
        n = len(recs)
        mov, outo, evo = [0], [0], [0]
        es, ee = [], []
        for seg, old, new, ls, ll, ev in recs:
            moved = (new - ll) - ev[0][0] if ev else 0
            mov.append(mov[-1] + moved)
            outo.append(outo[-1] + moved + ll)
            evo.append(evo[-1] + len(ev))
            es += [a for a, _ in ev]
            ee += [b for _, b in ev]
        out += [n, mov[-1], outo[-1]]
        for k in range(5):
            out += [r[k] for r in recs]
        out += mov + outo + evo + es + ee
    out[L] = len(out)
    return np.asarray(out, np.int32)


def copy_segments(src_k, src_v, src_base, dst_k, dst_v, dst_base, lens, stream=None):
    n = lens.numel()
    for lo in range(0, n, 65535):
        hi = min(n, lo + 65535)
        N.call("wnw_copy_segments", N.dtype_code(src_k.dtype), src_k.shape[1], src_k.data_ptr(),
               src_v.data_ptr(), src_base[lo:hi].data_ptr(), dst_k.data_ptr(), dst_v.data_ptr(),
               dst_base[lo:hi].data_ptr(), lens[lo:hi].data_ptr(), hi - lo, N.stream_ptr(stream))
        _count()


def interleave_append(old, new_tokens, cu_old, stream=None):
    """Reference-layout append (src/common/kv/kernels.py:76-97): returns
    (out [T + S, D], cu_new)."""
    S = new_tokens.shape[0]
    out = torch.empty(old.shape[0] + S, old.shape[1], dtype=old.dtype, device=old.device)
    N.call("wnw_interleave_append", N.dtype_code(old.dtype), old.shape[1],
           old.data_ptr() if old.numel() else None, new_tokens.data_ptr(), cu_old.data_ptr(), S,
           out.data_ptr(), N.stream_ptr(stream))
    _count()
    return out, cu_old + torch.arange(S + 1, dtype=cu_old.dtype, device=cu_old.device)


def check_device_error(err_tensor):
    """Raise on a non-zero device error word (reads it back: a sync point)."""
    v = int(err_tensor.item())
    if v:
        names = [n for bit, n in ((N.DEVERR_MBAR_TIMEOUT, "mbarrier wait timed out"),
                                  (N.DEVERR_LEN_MISMATCH, "segment length disagrees with the plan"),
                                  (N.DEVERR_CAPACITY, "segment exceeds its slot capacity"),
                                  (N.DEVERR_PEER_TIMEOUT, "tensor-parallel peer timed out"),
                                  (N.DEVERR_BAD_INDEX, "device plan, attention plan or prefill score task: "
                                                       "index out of range")) if v & bit]
        raise N.WnwError(5 if v & N.DEVERR_MBAR_TIMEOUT else 4, "device", ", ".join(names))


def packed_attention(q, k, v, cu, scale, scratch=None):
    """Attention over a reference-layout packed buffer ([T, D] + cu): the slot
    kernel with seg_base = cu[:-1], seg_len = diff(cu) and no append."""
    S, G, D = q.shape
    cu64 = cu.to(torch.int64)
    lens = (cu64[1:] - cu64[:-1]).to(torch.int32)
    lens_host = lens.cpu().numpy()
    # capacity = length - 1: the layout then covers exactly len rows
    work = AttnWork(q.dtype, D, np.maximum(lens_host - 1, 0), q.device)
    if scratch is None or not scratch.fits(work.slots, G, D, S):
        scratch = AttnScratch(q.device, work.slots, G, D, S)
    return decode_attention(q.contiguous(), k, v, cu64[:-1].contiguous(), lens, work, scale, scratch)


class PrefillScorer:
    """``wnw_prefill_scores`` for one device: the audio-token scores of a
    prefill layer for a list of tasks (see the header), with the scratch
    (per-chunk row statistics) grown on demand and a device error word that
    ``check()`` reads back (a sync point; call it once, after the last
    layer)."""

    def __init__(self, device):
        self.device = torch.device(device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.scratch = torch.empty(0, dtype=torch.uint8, device=self.device)

    def __call__(self, q, k, tasks, heads, scaling, out_len, mask_kind, mask=None, stream=None):
        """q [B, Hq, S, D] and k [B, Hkv, S, D] (bf16 / fp16, head dims
        contiguous); tasks: (batch, kv_head, head_off, n_heads, row0, n_rows,
        audio_start, audio_end, out_off) tuples; heads: query head indices;
        mask: [B, S, S] additive (mask_kind MASK_ADDITIVE), keys contiguous.
        Returns the fp32 scores [out_len]."""
        if q.device != self.device or k.device != self.device or q.device.type != "cuda":
            raise ValueError(f"q and k must be on {self.device} (a CUDA device)")
        if q.dim() != 4 or k.dim() != 4 or q.dtype != k.dtype or q.shape[0] != k.shape[0] \
                or q.shape[2] != k.shape[2] or q.shape[3] != k.shape[3]:
            raise ValueError(f"q {tuple(q.shape)} / k {tuple(k.shape)}: expected [B, Hq, S, D] and [B, Hkv, S, D] "
                             "of one dtype")
        if q.stride(3) != 1 or k.stride(3) != 1:
            raise ValueError("q and k need contiguous head dimensions")
        B, Hq, S, D = q.shape
        out = torch.zeros(max(1, int(out_len)), dtype=torch.float32, device=self.device)
        if not tasks:
            return out[:out_len]
        n = len(tasks)
        tab = np.zeros((n, 10), np.int32)
        tab[:, :8] = np.asarray([t[:8] for t in tasks], np.int32)
        tab.view(np.int64)[:, 4] = np.asarray([t[8] for t in tasks], np.int64)
        blob = np.concatenate([tab.reshape(-1), np.asarray(heads, np.int32)])
        dev_blob = torch.from_numpy(blob).pin_memory().to(self.device, non_blocking=True)
        max_rows = int(max(t[3] * t[5] for t in tasks))
        max_audio = int(max(t[7] - t[6] for t in tasks))
        need = C.c_int64()
        N.call("wnw_prefill_scores_scratch_bytes", n, max_rows, S, C.byref(need))
        if self.scratch.numel() < need.value:
            self.scratch = torch.empty(need.value, dtype=torch.uint8, device=self.device)
        if mask_kind == N.MASK_ADDITIVE:
            if mask is None or mask.dtype != q.dtype or mask.dim() != 3 or mask.stride(2) != 1:
                raise ValueError("an additive mask must be [B, S, S] in q's dtype with contiguous keys")
        a = N.PrefillScoresArgs(
            dtype=N.dtype_code(q.dtype), head_dim=D, batch=B, num_q_heads=Hq, num_kv_heads=k.shape[1], seq_len=S,
            num_tasks=n, num_heads=len(heads), max_rows=max_rows, max_audio=max_audio,
            q=q.data_ptr(), q_stride_b=q.stride(0), q_stride_h=q.stride(1), q_stride_s=q.stride(2),
            k=k.data_ptr(), k_stride_b=k.stride(0), k_stride_h=k.stride(1), k_stride_s=k.stride(2),
            mask_kind=int(mask_kind), mask=mask.data_ptr() if mask_kind == N.MASK_ADDITIVE else None,
            mask_stride_b=mask.stride(0) if mask_kind == N.MASK_ADDITIVE else 0,
            mask_stride_s=mask.stride(1) if mask_kind == N.MASK_ADDITIVE else 0,
            scaling=float(scaling), tasks=dev_blob.data_ptr(), heads=dev_blob.data_ptr() + tab.nbytes,
            out=out.data_ptr(), out_len=out.numel(), scratch=self.scratch.data_ptr(), scratch_bytes=self.scratch.numel(),
            err=self.err.data_ptr())
        N.check(N.lib.wnw_prefill_scores(C.byref(a), N.stream_ptr(stream)), "wnw_prefill_scores")
        _count(2)
        if stream is not None:  # buffers freed on the current stream must outlive the launches on `stream`
            for t in (dev_blob, out, self.scratch):
                t.record_stream(stream)
        self._keep = dev_blob  # alive until the launches have read it (stream order)
        return out[:out_len]

    def check(self):
        check_device_error(self.err)
