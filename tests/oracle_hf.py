"""Test helpers: wrap the CPU oracle cache in the HF ``Cache`` interface so a
session can drive it, and record hook calls like the golden session trace."""
import torch

from oracle.cache import OracleWnWCache
from wnw_b200.flat_cache import FlatVarlenCache


class OracleHFCache(FlatVarlenCache):
    """FlatVarlenCache whose hooks are served by ``OracleWnWCache`` (CPU)."""

    def __init__(self, config, num_layers, num_kv_heads, num_q_heads, head_dim):
        super().__init__(num_layers, num_kv_heads, num_q_heads, head_dim, torch.device("cpu"))
        self.config = config
        self.oracle = OracleWnWCache(config, num_layers, num_kv_heads, num_q_heads, head_dim)

    def setup_audio(self, audio_starts, audio_ends, attention_mask=None):
        super().setup_audio(audio_starts, audio_ends, attention_mask)
        self.oracle.setup_audio(audio_starts.tolist(), audio_ends.tolist(), self.pad_lens.tolist())
        self._raw_audio_starts = self.oracle._raw_audio_starts
        self._raw_audio_ends = self.oracle._raw_audio_ends

    def prefill_after_attn(self, layer_idx, class_a_scores, per_head_scores, k, v):
        self.oracle.prefill_after_attn(layer_idx, class_a_scores, per_head_scores, k, v)

    def prefill_all_layers_done(self):
        self.oracle.prefill_all_layers_done()
        self.prefilled = True

    def decode_before_attn(self, layer_idx, k, v):
        return self.oracle.decode_before_attn(layer_idx, k, v)

    def fused_decode_attention(self, layer_idx, q_flat, q, k_flat, v_flat, cu_k, scale):
        return self.oracle.fused_decode_attention(layer_idx, q_flat, scale=scale)

    def decode_all_layers_done(self):
        self.oracle.decode_all_layers_done()

    def _snapshot_cache_stats(self, step=-1):
        return [{} for _ in range(self.oracle.batch_size)]


class TracingMixin:
    """Records hook calls in the format of tests/golden/session_trace.json."""

    @property
    def calls(self):
        if not hasattr(self, "_calls"):
            self._calls = []
        return self._calls

    def prefill_after_attn(self, l, a, p, k, v):
        self.calls.append(["prefill_after_attn", l, list(k.shape)])
        return super().prefill_after_attn(l, a, p, k, v)

    def prefill_all_layers_done(self):
        self.calls.append(["prefill_all_layers_done"])
        return super().prefill_all_layers_done()

    def decode_before_attn(self, l, k, v):
        self.calls.append(["decode_before_attn", l, list(k.shape)])
        return super().decode_before_attn(l, k, v)

    def fused_decode_attention(self, l, q_flat, q, k_flat, v_flat, cu_k, scale):
        self.calls.append(["fused_decode_attention", l, list(q_flat.shape), list(q.shape), float(scale)])
        return super().fused_decode_attention(l, q_flat, q, k_flat, v_flat, cu_k, scale)

    def decode_all_layers_done(self):
        self.calls.append(["decode_all_layers_done"])
        return super().decode_all_layers_done()
