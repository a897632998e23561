"""``FlatVarlenCache``: the HuggingFace ``Cache`` subclass the WnW session talks to.

Same constructor, HF-facing methods and WnW hook API as the reference
(src/common/kv/flat_cache.py:45-186): ``update`` only counts tokens (the hooks
own the storage), beam search / crop / batch re-indexing raise, and the
prefill / decode hooks are implemented by subclasses.
"""
from __future__ import annotations

from functools import partial

import torch
from transformers.cache_utils import Cache, CacheLayerMixin

from wnw_b200.stats import InferenceStats


class _SeqLengthStub(CacheLayerMixin):
    """Per-layer stub that reports the cache's token count to HF internals."""

    is_compileable = False
    is_sliding = False

    def __init__(self, get_len):
        super().__init__()
        self._get_len = get_len
        self.is_initialized = True

    def lazy_initialization(self, *args, **kwargs):
        pass

    def update(self, key_states, value_states, *args, **kwargs):
        raise RuntimeError("FlatVarlenCache: layers[].update must not be called directly")

    def get_seq_length(self):
        return self._get_len()

    def get_max_cache_shape(self):
        return -1

    def get_mask_sizes(self, query_length):
        n = self._get_len()
        return n + query_length, n

    def reset(self):
        pass

    def reorder_cache(self, beam_idx):
        raise NotImplementedError("the flat varlen layout cannot be reordered for beam search")


class FlatVarlenCache(Cache):
    is_compileable = False

    def __init__(self, num_layers, num_kv_heads, num_q_heads, head_dim, device, adapter=None):
        super().__init__(layers=[_SeqLengthStub(partial(self._layer_len, i)) for i in range(num_layers)])
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.num_q_heads = num_q_heads
        self.num_kv_groups = num_q_heads // num_kv_heads
        self.head_dim = head_dim
        self.device = torch.device(device)
        self.adapter = adapter
        self._seq_lengths = [0] * num_layers
        self.prefilled = False
        self.audio_starts = self.audio_ends = self.pad_lens = None
        self.stats = InferenceStats(self.device, interval=5)

    def setup_audio(self, audio_starts, audio_ends, attention_mask=None):
        self.audio_starts, self.audio_ends = audio_starts, audio_ends
        self.prefilled = False
        self._seq_lengths = [0] * self.num_layers
        self.stats.reset(audio_starts.shape[0])
        # left padding per sample: the first position whose mask is 1 (0 for
        # a row without one, and without a mask)
        if attention_mask is None:
            self.pad_lens = torch.zeros(audio_starts.shape[0], dtype=torch.int64, device=self.device)
        else:
            valid = attention_mask == 1
            first = valid.to(torch.int8).argmax(dim=-1)  # the first maximum
            self.pad_lens = torch.where(valid.any(dim=-1), first, 0).to(device=self.device, dtype=torch.int64)

    def _layer_len(self, i):
        """Tokens seen by layer i (0 before any), for the per-layer stubs."""
        lens = getattr(self, "_seq_lengths", None)
        return lens[i] if lens is not None and i < len(lens) else 0

    def update(self, key_states, value_states, layer_idx, *args, **kwargs):
        self._seq_lengths[layer_idx] += key_states.shape[-2]
        return key_states, value_states

    def get_seq_length(self, layer_idx=0):
        return self._seq_lengths[layer_idx] if layer_idx < self.num_layers else 0

    def get_max_cache_shape(self, layer_idx=0):
        return -1

    def get_mask_sizes(self, query_length, layer_idx):
        n = self.get_seq_length(layer_idx)
        return n + query_length, n

    def reset(self):
        self.prefilled = False
        self._seq_lengths = [0] * self.num_layers
        self.audio_starts = self.audio_ends = self.pad_lens = None
        self.stats.reset(0)

    # the flat varlen layout keeps one ragged segment per (sample, kv head):
    # HF's reordering and cropping operations have no meaning for it
    def reorder_cache(self, beam_idx):
        raise NotImplementedError("the flat varlen layout cannot be reordered for beam search")

    def crop(self, max_length):
        raise NotImplementedError("the flat varlen layout cannot be cropped (assisted decoding)")

    def batch_repeat_interleave(self, repeats):
        raise NotImplementedError("the flat varlen layout cannot repeat samples of its batch")

    def batch_select_indices(self, indices):
        raise NotImplementedError("the flat varlen layout cannot select samples of its batch")

    # WnW hooks (flat_cache.py:161-186)
    def prefill_before_attn(self, layer_idx):
        pass

    def prefill_after_attn(self, layer_idx, *args, **kwargs):
        pass

    def prefill_all_layers_done(self):
        self.prefilled = True

    def decode_before_attn(self, layer_idx, k_new, v_new):
        raise NotImplementedError(f"{type(self).__name__} defines no decode_before_attn storage")

    def decode_after_attn(self, layer_idx, q):
        pass

    def decode_all_layers_done(self):
        pass

    def _snapshot_cache_stats(self, step=-1):
        raise NotImplementedError(f"{type(self).__name__} defines no cache statistics snapshot")
