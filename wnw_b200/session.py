"""``AlgorithmSession`` / ``WnWSession``: attention patching that drives the cache hooks.

Mirrors the reference session (src/common/session.py:15-90 and
src/algorithms/wnw/code/session.py:21-201) call for call, so either session
can drive either cache:

* prefill: SDPA over the GQA-expanded K/V, per-head audio scores,
  ``cache.prefill_after_attn``, and ``prefill_all_layers_done`` after the last
  layer;
* decode: ``cache.update`` -> ``decode_before_attn`` -> ``fused_decode_attention``
  -> ``o_proj``, and ``decode_all_layers_done`` after the last layer.

The decode step always takes the fused hook (the reference's
``WNW_FUSED_ATTN=1`` path, session.py:85-88).
"""
from __future__ import annotations

import types

import torch
import torch.nn.functional as F


class AlgorithmSession:
    """Context manager that installs and removes the patched attention forwards
    (src/common/session.py:15-90); the model is untouched outside the block."""

    def __init__(self, model, adapter, cache, processor=None):
        self.model, self.adapter, self.cache, self.processor = model, adapter, cache, processor
        self._state = None
        self._orig = []

    def __enter__(self):
        self.cache.reset()
        self.adapter.assert_compatible(self.model)
        self._state = self.adapter.prepare_for_inference(self.model)
        for layer in self.adapter.get_decoder_layers(self.model):
            attn = layer.self_attn
            self._orig.append((attn, attn.forward))
            attn.forward = types.MethodType(self._make_patched_forward(attn), attn)
        return self

    def __exit__(self, *exc):
        for attn, fwd in self._orig:
            attn.forward = fwd
        self._orig.clear()
        self.adapter.restore_after_inference(self.model, self._state)
        self._state = None

    def setup_audio(self, input_ids, attention_mask=None):
        starts, ends = self.adapter.locate_audio_tokens(input_ids, attention_mask, self.processor)
        self.cache.setup_audio(starts, ends, attention_mask)

    def generate(self, inputs, **gen_kwargs):
        gen_kwargs["past_key_values"] = self.cache
        return self.adapter.generate(self.model, inputs, **gen_kwargs)

    def get_stats(self):
        stats = getattr(self.cache, "stats", None)
        return stats.get_all_stats() if stats is not None else []

    def _make_patched_forward(self, attn_module):
        raise NotImplementedError


class WnWSession(AlgorithmSession):
    def _make_patched_forward(self, attn_module):
        cache, adapter = self.cache, self.adapter
        meta = adapter.attention_meta(attn_module)
        H, G, D = meta["num_kv_heads"], meta["num_kv_groups"], meta["head_dim"]
        scaling, layer_idx = meta["scaling"], meta["layer_idx"]
        last = layer_idx == cache.num_layers - 1

        def patched_forward(self_attn, hidden_states, position_embeddings=None, attention_mask=None,
                            past_key_values=None, **kwargs):
            B, S, _ = hidden_states.shape
            q, k, v = adapter.compute_qkv(self_attn, hidden_states)
            q, k = adapter.apply_rope(q, k, position_embeddings, self_attn)
            if not cache.prefilled:
                cache.prefill_before_attn(layer_idx)
                cache.update(k, v, layer_idx)
                kg = k.repeat_interleave(G, dim=1)
                vg = v.repeat_interleave(G, dim=1)
                out = F.scaled_dot_product_attention(q, kg, vg, attn_mask=attention_mask, scale=scaling,
                                                     is_causal=attention_mask is None)
                del kg, vg
                ca, ph = compute_prefill_scores(q, k, attention_mask, cache, layer_idx, B, S, H, G, scaling)
                cache.prefill_after_attn(layer_idx, ca, ph, k, v)
                if last:
                    cache.prefill_all_layers_done()
                out = out.transpose(1, 2).reshape(B, S, -1).contiguous()
                return self_attn.o_proj(out), None
            cache.update(k, v, layer_idx)
            k_flat, v_flat, cu_k, _ = cache.decode_before_attn(layer_idx, k, v)
            q_flat = q.squeeze(2).view(B, H, G, D).reshape(B * H, G, D)
            out = cache.fused_decode_attention(layer_idx, q_flat, q, k_flat, v_flat, cu_k, scaling)
            out = out.reshape(B, 1, H * G * D)
            if last:
                cache.decode_all_layers_done()
            return self_attn.o_proj(out), None

        return patched_forward


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
