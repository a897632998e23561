"""The reference's own WnWSession from its offline install (baseline/_ref),
for drop-in tests of this package's caches under it; the tests skip when the
install is absent.  The adapter is the reference's BaseModelAdapter completed
for a tiny random-init Llama whose audio span the scenario fixes (the same
adapter the golden session trace was recorded with)."""
import importlib
import os
import sys

import pytest
import torch

REF_ROOT = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


def reference_session_or_skip(ss):
    """(the reference session module, an adapter instance)."""
    if not os.path.isdir(os.path.join(REF_ROOT, "algorithms")):
        pytest.skip("the reference is not installed in baseline/_ref")
    os.environ["WNW_FUSED_ATTN"] = "1"
    if REF_ROOT not in sys.path:
        sys.path.insert(0, REF_ROOT)
    rsess = importlib.import_module("algorithms.wnw.code.session")
    rsess._FUSED_ATTN = True  # read at import time by the reference (session.py:18)
    from wnw_b200.integration import accept_in_reference_session
    accept_in_reference_session(rsess)
    from common.adapters.base import BaseModelAdapter
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb

    class TinyAdapter(BaseModelAdapter):
        name = "tiny"

        def load(self, *a, **k): raise NotImplementedError
        def _build_inputs(self, *a, **k): raise NotImplementedError
        def get_decoder_layers(self, model): return model.model.layers
        def get_text_config(self, model): return model.config

        def locate_audio_tokens(self, input_ids, attention_mask, processor):
            B = input_ids.shape[0]
            return (torch.full((B,), ss["audio_start"], dtype=torch.int64, device=input_ids.device),
                    torch.full((B,), ss["audio_end"], dtype=torch.int64, device=input_ids.device))

        def compute_qkv(self, attn, h):
            B, S, _ = h.shape
            hd = attn.head_dim
            return (attn.q_proj(h).view(B, S, -1, hd).transpose(1, 2),
                    attn.k_proj(h).view(B, S, -1, hd).transpose(1, 2),
                    attn.v_proj(h).view(B, S, -1, hd).transpose(1, 2))

        def apply_rope(self, q, k, pe, attn): return apply_rotary_pos_emb(q, k, *pe)

        def attention_meta(self, attn):
            c = attn.config
            return {"head_dim": attn.head_dim, "num_kv_heads": c.num_key_value_heads,
                    "num_kv_groups": c.num_attention_heads // c.num_key_value_heads,
                    "scaling": attn.scaling, "layer_idx": attn.layer_idx}

        def prepare_for_inference(self, model): return {}
        def restore_after_inference(self, model, state): pass
        def generate(self, model, inputs, **kw): return model.generate(**inputs, **kw)
        def get_logits(self, model, outputs): return outputs.logits
        def get_text_model(self, model): return model
        def get_audio_token_id(self, model): return 0
        def build_analysis_inputs(self, *a, **k): raise NotImplementedError

    return rsess, TinyAdapter()
