"""CPU restatements of the WnW decode-path kernels -- TEST INFRASTRUCTURE ONLY.

Each function restates one reference kernel's semantics in numpy.  Floating
point work is done in float64 (a strictly more accurate stand-in for the
reference's fp32 accumulation); integer and copy work is exact.

Paths are relative to the XMUDeepLIT/WnW project root.
"""
from __future__ import annotations

import numpy as np


def _f64(x):
    return np.asarray(x, dtype=np.float64)


def decode_attn(q, k, v, cu, scale):
    """q_len=1 GQA decode attention over packed varlen segments.

    Restates ``src/common/kv/fused_attn.py:9-44`` (``_q1_decode_attn_kernel``):
    for segment ``s`` the G query heads ``q[s]`` attend to rows
    ``k[cu[s]:cu[s+1]]`` with ``softmax(q . k^T * scale) @ v``.

    q: [nseg, G, D]; k, v: [T, D]; cu: int [nseg+1].  Returns float64 [nseg, G, D]
    and the per-(segment, head) softmax max ``m`` and sum ``l`` (natural-exp domain).
    """
    q = _f64(q)
    k = _f64(k)
    v = _f64(v)
    cu = np.asarray(cu, dtype=np.int64)
    nseg, G, D = q.shape
    out = np.zeros((nseg, G, D), dtype=np.float64)
    m_all = np.full((nseg, G), -np.inf)
    l_all = np.zeros((nseg, G))
    for s in range(nseg):
        a, b = int(cu[s]), int(cu[s + 1])
        if b <= a:
            continue
        logits = q[s] @ k[a:b].T * scale  # [G, n]
        m = logits.max(axis=1, keepdims=True)
        p = np.exp(logits - m)
        l = p.sum(axis=1, keepdims=True)
        out[s] = (p @ v[a:b]) / l
        m_all[s] = m[:, 0]
        l_all[s] = l[:, 0]
    return out, m_all, l_all


def decode_attn_score(q, k, v, cu, scale, ca_kv_mask, num_kv_heads,
                      audio_starts, audio_ends, score_acc, score_offsets):
    """Decode attention plus fused class-A audio-token scoring.

    Restates ``src/common/kv/fused_attn.py:68-121``
    (``_q1_decode_attn_score_kernel``): segments whose kv head is flagged in
    ``ca_kv_mask`` add ``sum_g softmax_full_segment(q_g . K)[audio_start + t]``
    into ``score_acc[score_offsets[b] + t]`` for t in [0, audio_len_b).
    Segments are visited in ascending index (the reference uses atomics, so its
    order is unspecified); the head sum runs in ascending head order.

    ``score_acc`` (float64 or float32 ndarray) is updated in place.
    Returns the attention output [nseg, G, D] (float64).
    """
    out, m_all, l_all = decode_attn(q, k, v, cu, scale)
    q = _f64(q)
    k = _f64(k)
    cu = np.asarray(cu, dtype=np.int64)
    nseg = q.shape[0]
    for s in range(nseg):
        kv = s % num_kv_heads
        if int(ca_kv_mask[kv]) == 0:
            continue
        b = s // num_kv_heads
        a0, a1 = int(audio_starts[b]), int(audio_ends[b])
        base = int(cu[s])
        off = int(score_offsets[b])
        logits = q[s] @ k[base + a0:base + a1].T * scale  # [G, na]
        w = np.exp(logits - m_all[s][:, None]) / l_all[s][:, None]
        score_acc[off:off + (a1 - a0)] += w.sum(axis=0)
    return out


def fused_score_accumulate(Q, K, seg_starts, seg_ends, audio_starts, audio_ends,
                           acc, acc_offsets):
    """Non-fused class-A scoring of one kv group.

    Restates ``src/algorithms/wnw/code/kernels.py:302-370``
    (``_fused_score_kernel_h1/_h4`` and ``_fused_score_pytorch``): full-segment
    softmax with scale ``1/sqrt(d)``; the audio-range probabilities summed over
    the group's heads are added to ``acc[acc_offsets[s]:]``.
    """
    Q = _f64(Q)
    K = _f64(K)
    n, nh, d = Q.shape
    scale = 1.0 / np.sqrt(d)
    for s in range(n):
        a, b = int(seg_starts[s]), int(seg_ends[s])
        a0, a1 = int(audio_starts[s]), int(audio_ends[s])
        off = int(acc_offsets[s])
        logits = Q[s] @ K[a:b].T * scale
        m = logits.max(axis=1, keepdims=True)
        p = np.exp(logits - m)
        p = p / p.sum(axis=1, keepdims=True)
        acc[off:off + (a1 - a0)] += p[:, a0:a1].sum(axis=0)


def interleave_append(old, new_tokens, cu_old):
    """Append one row per segment into a packed varlen buffer.

    Restates ``src/common/kv/kernels.py:7-73`` (``interleave_append``): output
    segment ``s`` is ``old[cu_old[s]:cu_old[s+1]]`` followed by
    ``new_tokens[s]``.  (The reference's fixed 10-step binary search mis-places
    rows once ``nseg >= 1024``; this restatement is exact for every size.)
    Returns (out, cu_new).
    """
    old = np.asarray(old)
    new_tokens = np.asarray(new_tokens)
    cu_old = np.asarray(cu_old, dtype=np.int64)
    n = new_tokens.shape[0]
    pieces = []
    for s in range(n):
        pieces.append(old[cu_old[s]:cu_old[s + 1]])
        pieces.append(new_tokens[s:s + 1])
    out = np.concatenate(pieces, axis=0) if pieces else old[:0]
    cu_new = cu_old + np.arange(n + 1, dtype=np.int64)
    return out, cu_new


def rebuild_append(old, new_tokens, load, cu_old, cu_new, load_starts, load_lens,
                   evict_offsets, evict_starts, evict_ends):
    """Evict + splice-load + append rebuild of one layer's packed buffer.

    Restates ``src/algorithms/wnw/code/kernels.py:375-473``
    (``rebuild_append_kv``): output segment ``s`` = the old segment's rows with
    the (sorted, segment-relative) evict ranges removed, then
    ``load[load_starts[s] : load_starts[s] + load_lens[s]]``, then
    ``new_tokens[s]``.  ``cu_new`` is trusted to describe the result.
    """
    old = np.asarray(old)
    cu_old = np.asarray(cu_old, dtype=np.int64)
    n = new_tokens.shape[0]
    pieces = []
    for s in range(n):
        seg = old[cu_old[s]:cu_old[s + 1]]
        e0, e1 = int(evict_offsets[s]), int(evict_offsets[s + 1])
        keep = np.ones(seg.shape[0], dtype=bool)
        for i in range(e0, e1):
            keep[int(evict_starts[i]):int(evict_ends[i])] = False
        pieces.append(seg[keep])
        ln = int(load_lens[s])
        if ln > 0:
            ls = int(load_starts[s])
            pieces.append(np.asarray(load)[ls:ls + ln])
        pieces.append(np.asarray(new_tokens)[s:s + 1])
    out = np.concatenate(pieces, axis=0)
    assert out.shape[0] == int(cu_new[-1]), (out.shape, cu_new[-1])
    return out


def prefix_sum_f32(scores):
    """fp32 prefix sum with a zero prepended, as the reference computes it.

    ``cache.py:636-637`` runs ``torch.cumsum`` on an fp32 vector; torch's CPU
    kernel accumulates in float64 and rounds each output to fp32.
    """
    s = np.asarray(scores, dtype=np.float32).astype(np.float64)
    p = np.zeros(s.shape[0] + 1, dtype=np.float64)
    np.cumsum(s, out=p[1:])
    return p.astype(np.float32)


def chunk_scores(scores, chunk_starts, chunk_ends):
    """Mean class-A score per chunk.

    Restates ``src/algorithms/wnw/code/cache.py:632-640`` and the lens of
    ``cache.py:203-205``: ``(P[end] - P[start]) / max(1, end - start)`` with
    fp32 subtraction and division.
    """
    p = prefix_sum_f32(scores)
    cs = np.asarray(chunk_starts, dtype=np.int64)
    ce = np.asarray(chunk_ends, dtype=np.int64)
    lens = np.maximum(ce - cs, 1).astype(np.float32)
    return (p[ce] - p[cs]).astype(np.float32) / lens


def topk_lower_index(values, k):
    """Indices of the k largest values, ties broken by the lower index.

    ``torch.topk`` (``cache.py:648``) leaves the order of equal values
    unspecified; the rebuilt path fixes it to "lower index wins".  Only the SET
    of selected indices matters to the planner (``cache.py:611``).
    """
    v = np.asarray(values, dtype=np.float32)
    k = min(int(k), v.shape[0])
    order = sorted(range(v.shape[0]), key=lambda i: (-float(v[i]), i))
    return order[:k]


def topk_gap(values, k):
    """Gap between the k-th and (k+1)-th largest value (inf when no (k+1)-th)."""
    v = np.sort(np.asarray(values, dtype=np.float64))[::-1]
    if k <= 0 or k >= v.shape[0]:
        return np.inf
    return float(v[k - 1] - v[k])


def gather_restore(cpu_k, cpu_v, ranges):
    """Concatenate host rows ``[s, e)`` of each range, in order.

    Restates ``src/algorithms/wnw_cpp/code/planner.cpp:113-122`` and the staging
    ``torch.cat`` of ``src/algorithms/wnw/code/cache.py:868-875``.
    """
    ranges = [(int(s), int(e)) for s, e in ranges]
    if not ranges:
        return cpu_k[:0].copy(), cpu_v[:0].copy()
    ks = np.concatenate([cpu_k[s:e] for s, e in ranges], axis=0)
    vs = np.concatenate([cpu_v[s:e] for s, e in ranges], axis=0)
    return ks, vs
