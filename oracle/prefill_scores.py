"""Prefill audio scores in plain torch -- TEST INFRASTRUCTURE ONLY.

A restatement of the reference session's ``_compute_prefill_scores`` and
``_compute_head_scores`` (src/algorithms/wnw/code/session.py:121-201): the
logits come from a matmul in the model dtype, are scaled and masked in that
dtype, then softmaxed in fp32.  The shipped session computes the same scores
with ``wnw_prefill_scores`` on the GPU; CPU tests hand this function to
``wnw_b200.session.WnWSession(prefill_scores=...)`` to drive the oracle cache,
and the GPU tests compare the kernel with it.
"""
from __future__ import annotations

import torch


def compute_prefill_scores(q, k, attention_mask, cache, layer_idx, B, S, H, G, scaling):
    """Per-sample class-A audio scores and per-kv-head audio scores from the
    last prefill query (or the mean over the post-audio text queries), as in
    src/algorithms/wnw/code/session.py:121-201 -- including the reference's
    choice of the FIRST class-A q head's kv head for all class-A heads of the
    layer (session.py:144-147)."""
    if attention_mask is not None and attention_mask.dim() == 4 and attention_mask.dtype == torch.bool:
        attention_mask = torch.where(attention_mask, 0.0, float("-inf")).to(q.dtype)
    if attention_mask is None:
        # the causal mask's rows the scores read -- the last query, or the
        # post-audio text queries -- instead of the whole S x S matrix
        attention_mask = _CausalRows(S, q.device, q.dtype)
    cfg = cache.config
    ca_heads = cfg.get_layer_class_a(layer_idx)
    class_a, per_head = [], []
    for b in range(B):
        a0, a1 = cache._raw_audio_starts[b], cache._raw_audio_ends[b]
        if ca_heads:
            kv = ca_heads[0] // G
            s = torch.matmul(q[b, ca_heads, -1:, :], k[b, kv:kv + 1].transpose(-1, -2)) * scaling
            if attention_mask.dim() == 4:
                s = s + attention_mask[b, :, -1:, :]
            class_a.append(s.float().softmax(dim=-1)[:, 0, a0:a1].sum(dim=0).detach())
        else:
            class_a.append(None)
        heads = []
        for h in range(H):
            if cfg.is_class_a_kv_head(layer_idx, h):
                heads.append(None)
                continue
            heads.append(_head_scores(q[b], k[b, h], attention_mask, b, S, h * G, h * G + G, a0, a1, scaling,
                                      cfg.prefill_score_mode))
        per_head.append(heads)
    return class_a, per_head


class _CausalRows:
    """Stand-in for a [B, 1, S, S] causal mask: indexing [b, :, rows, :]
    builds only the requested rows (0 on and below the diagonal, -inf above)."""

    def __init__(self, S, device, dtype):
        self.S, self.device, self.dtype = S, device, dtype

    def dim(self):
        return 4

    def __getitem__(self, idx):
        _, _, rows, _ = idx
        r = torch.arange(self.S, device=self.device)[rows]
        cols = torch.arange(self.S, device=self.device)
        m = torch.zeros(r.numel(), self.S, device=self.device, dtype=self.dtype)
        m.masked_fill_(cols.unsqueeze(0) > r.unsqueeze(1), float("-inf"))
        return m.unsqueeze(0)


def _head_scores(q_all, k_one, mask, b, S, q0, q1, a0, a1, scaling, mode):
    k = k_one.unsqueeze(0)
    if mode == "last":
        s = torch.matmul(q_all[q0:q1, -1:, :], k.transpose(-1, -2)) * scaling
        if mask is not None and mask.dim() == 4:
            s = s + mask[b, :, -1:, :]
        return s.float().softmax(dim=-1)[:, 0, a0:a1].sum(dim=0)
    if mode == "mean_text":
        if S - a1 == 0:
            return torch.zeros(a1 - a0, device=q_all.device, dtype=torch.float32)
        s = torch.matmul(q_all[q0:q1, a1:, :], k.transpose(-1, -2)) * scaling
        if mask is not None and mask.dim() == 4:
            s = s + mask[b, :, a1:, :]
        return s.float().softmax(dim=-1)[:, :, a0:a1].mean(dim=1).sum(dim=0)
    raise ValueError(f"unknown prefill_score_mode {mode!r}")
