"""Model adapter for HF Llama-family text decoders (the Voxtral text decoder
is one), with the methods the session needs from the reference's
``BaseModelAdapter`` (src/common/adapters/base.py:9-163,
src/common/adapters/voxtral.py:98-140).  The audio span is given
explicitly because the build runs random-init decoders on synthetic
embeddings rather than real audio encoders."""
from __future__ import annotations

import torch
from transformers.models.llama.modeling_llama import apply_rotary_pos_emb


class LlamaFamilyAdapter:
    name = "llama_family"

    def __init__(self, audio_start=None, audio_end=None):
        self.audio_start, self.audio_end = audio_start, audio_end

    def get_decoder_layers(self, model):
        inner = getattr(model, "model", model)
        return inner.layers

    def get_text_config(self, model):
        return model.config

    def locate_audio_tokens(self, input_ids, attention_mask, processor=None):
        B = input_ids.shape[0]
        s = torch.as_tensor(self.audio_start, dtype=torch.int64).expand(B).clone()
        e = torch.as_tensor(self.audio_end, dtype=torch.int64).expand(B).clone()
        return s.to(input_ids.device), e.to(input_ids.device)

    def compute_qkv(self, attn, hidden_states):
        B, S, _ = hidden_states.shape
        hd = attn.head_dim
        q = attn.q_proj(hidden_states).view(B, S, -1, hd).transpose(1, 2)
        k = attn.k_proj(hidden_states).view(B, S, -1, hd).transpose(1, 2)
        v = attn.v_proj(hidden_states).view(B, S, -1, hd).transpose(1, 2)
        return q, k, v

    def apply_rope(self, q, k, position_embeddings, attn):
        cos, sin = position_embeddings
        return apply_rotary_pos_emb(q, k, cos, sin)

    def attention_meta(self, attn):
        c = attn.config
        return {"head_dim": attn.head_dim, "num_kv_heads": c.num_key_value_heads,
                "num_kv_groups": c.num_attention_heads // c.num_key_value_heads,
                "scaling": attn.scaling, "layer_idx": attn.layer_idx}

    def assert_compatible(self, model):
        cfg = self.get_text_config(model)
        hd = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        if hd & (hd - 1):
            raise AssertionError(f"head_dim={hd} must be a power of 2")
        layers = self.get_decoder_layers(model)
        if not len(layers) or not hasattr(layers[0].self_attn, "layer_idx"):
            raise AssertionError("decoder layers with layer_idx expected")

    def prepare_for_inference(self, model):
        return {}

    def restore_after_inference(self, model, state):
        pass

    def generate(self, model, inputs, **kwargs):
        return model.generate(**inputs, **kwargs)
