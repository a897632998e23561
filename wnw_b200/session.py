"""``AlgorithmSession`` / ``WnWSession``: attention patching that drives the cache hooks.

Mirrors the reference session (src/common/session.py:15-90 and
src/algorithms/wnw/code/session.py:21-201) call for call, so either session
can drive either cache:

* prefill: SDPA over the GQA-expanded K/V, per-head audio scores
  (``wnw_prefill_scores`` on the GPU), ``cache.prefill_after_attn``, and
  ``prefill_all_layers_done`` after the last layer;
* decode: ``cache.update`` -> ``decode_before_attn`` -> ``fused_decode_attention``
  -> ``o_proj``, and ``decode_all_layers_done`` after the last layer.

The decode step always takes the fused hook (the reference's
``WNW_FUSED_ATTN=1`` path, session.py:85-88).
"""
from __future__ import annotations

import types

import torch
import torch.nn.functional as F

from wnw_b200 import native as N
from wnw_b200.kernels import PrefillScorer


class AlgorithmSession:
    """Context manager that installs and removes the patched attention forwards
    (src/common/session.py:15-90); the model is untouched outside the block."""

    def __init__(self, model, adapter, cache, processor=None, prefill_scores=None):
        self.model, self.adapter, self.cache, self.processor = model, adapter, cache, processor
        # prefill audio scores: the GPU kernel by default; a callable with the
        # signature of compute_prefill_scores minus ``scorer`` replaces it
        self.prefill_scores = prefill_scores
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
        scores_fn, scorer = self.prefill_scores, None
        if scores_fn is None:
            scorer = self._scorer = getattr(self, "_scorer", None) or PrefillScorer(cache.device)

            def scores_fn(*args):
                return compute_prefill_scores(*args, scorer=scorer)

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
                ca, ph = scores_fn(q, k, attention_mask, cache, layer_idx, B, S, H, G, scaling)
                cache.prefill_after_attn(layer_idx, ca, ph, k, v)
                if last:
                    if scorer is not None:
                        scorer.check()  # the score tasks' device error word, once per prefill
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


def compute_prefill_scores(q, k, attention_mask, cache, layer_idx, B, S, H, G, scaling, scorer):
    """Per-sample class-A audio scores and per-kv-head audio scores from the
    last prefill query (or the mean over the post-audio text queries), as in
    src/algorithms/wnw/code/session.py:121-201 -- including the reference's
    choice of the FIRST class-A q head's kv head for all class-A heads of the
    layer (session.py:144-147) -- in one ``wnw_prefill_scores`` call (two
    launches) per layer.  Returns views of one fp32 buffer."""
    mask_kind, mask = _score_mask(attention_mask, q.dtype)
    cfg = cache.config
    ca_heads = list(cfg.get_layer_class_a(layer_idx))
    mode = cfg.prefill_score_mode
    if mode not in ("last", "mean_text"):
        raise ValueError(f"unknown prefill_score_mode {mode!r}")
    tasks, heads, spans, off = [], [], [], 0
    for b in range(B):
        a0, a1 = int(cache._raw_audio_starts[b]), int(cache._raw_audio_ends[b])
        n = a1 - a0
        ca = None
        if ca_heads:  # the class-A query heads against the first one's kv head, last query
            tasks.append((b, ca_heads[0] // G, len(heads), len(ca_heads), S - 1, 1, a0, a1, off))
            heads.extend(ca_heads)
            ca, off = (off, n), off + n
        hs = []
        for h in range(H):
            if cfg.is_class_a_kv_head(layer_idx, h):
                hs.append(None)
                continue
            if mode == "last":
                row0, rows = S - 1, 1
            elif S - a1 == 0:  # no text after the audio: zero scores
                hs.append((off, n))
                off += n
                continue
            else:
                row0, rows = a1, S - a1
            tasks.append((b, h, len(heads), G, row0, rows, a0, a1, off))
            heads.extend(range(h * G, h * G + G))
            hs.append((off, n))
            off += n
        spans.append((ca, hs))
    out = scorer(q, k, [t for t in tasks if t[7] > t[6]], heads, scaling, off, mask_kind, mask)
    class_a = [out[s[0]:s[0] + s[1]] if s is not None else None for s, _ in spans]
    per_head = [[out[s[0]:s[0] + s[1]] if s is not None else None for s in hs] for _, hs in spans]
    return class_a, per_head


def _score_mask(attention_mask, dtype):
    """(mask kind, [B, S, S] additive mask) the reference's score path uses:
    a causal mask when none is given, nothing for a mask that is not 4-D,
    else the mask (a boolean one turned into 0 / -inf in the model dtype)."""
    if attention_mask is None:
        return N.MASK_CAUSAL, None
    if attention_mask.dim() != 4:
        return N.MASK_NONE, None
    if attention_mask.dtype == torch.bool:
        attention_mask = torch.where(attention_mask, 0.0, float("-inf")).to(dtype)
    m = attention_mask[:, 0]
    if m.dtype != dtype or m.stride(2) != 1:
        m = m.to(dtype).contiguous()
    return N.MASK_ADDITIVE, m
