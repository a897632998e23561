"""GQA -> MHA conversion of a model and of its WnW configuration.

The reference runs some models (its Qwen2.5-Omni adapter, by default) with
grouped-query attention expanded to one kv head per query head, and expands
the head-class configuration to match:

* ``degqa_model`` restates ``src/common/adapters/degqa.py:7-86``: every
  decoder layer's k_proj / v_proj output rows (and biases) are repeated
  ``group`` times per kv head, so kv head h becomes kv heads h*g .. h*g+g-1,
  each identical to the original; the attention modules and the text config
  then report num_key_value_heads = num_attention_heads, groups = 1.  The
  model computes exactly what it did before (each query head attends to a
  copy of its own kv head).
* ``expand_wnw_config`` restates
  ``src/analysis/wnw_config/scripts/expand_wnw_config.py:5-36``: per (layer,
  kv head) retention ratios are repeated per query head of the group, class-B
  kv-head ids become the ids of the group's query heads, class-A ids (already
  query heads) stay, and the result records the original kv-head count.

The decode path needs neither (its kernels take GQA groups of 1 to 8 as they
are); they exist so that configurations and checkpoints prepared for the
reference's MHA mode load unchanged.
"""
from __future__ import annotations

import torch
from torch import nn


def degqa_model(model, adapter):
    """Expand a GQA model to MHA in place (not reversible)."""
    cfg = adapter.get_text_config(model)
    n_kv, n_q = cfg.num_key_value_heads, cfg.num_attention_heads
    if n_kv == n_q:
        return
    if n_q % n_kv:
        raise ValueError(f"num_attention_heads ({n_q}) must be divisible by num_key_value_heads ({n_kv})")
    group = n_q // n_kv
    head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // n_q
    for layer in adapter.get_decoder_layers(model):
        attn = layer.self_attn
        _repeat_heads(attn.k_proj, head_dim, group)
        _repeat_heads(attn.v_proj, head_dim, group)
        for obj in (attn, getattr(attn, "config", None)):
            if obj is None:
                continue
            if hasattr(obj, "num_key_value_heads"):
                obj.num_key_value_heads = n_q
            if hasattr(obj, "num_key_value_groups"):
                obj.num_key_value_groups = 1
    cfg.num_key_value_heads = n_q
    if hasattr(cfg, "num_key_value_groups"):
        cfg.num_key_value_groups = 1
    if torch.cuda.is_available():
        torch.cuda.empty_cache()


def _repeat_heads(proj: nn.Linear, head_dim: int, group: int):
    out_f, in_f = proj.weight.shape
    if out_f % head_dim:
        raise ValueError(f"projection with {out_f} outputs is not a whole number of {head_dim}-wide heads")
    n = out_f // head_dim
    w = proj.weight.data.reshape(n, 1, head_dim, in_f).expand(n, group, head_dim, in_f)
    proj.weight = nn.Parameter(w.reshape(n * group * head_dim, in_f).contiguous(), requires_grad=False)
    if proj.bias is not None:
        b = proj.bias.data.reshape(n, 1, head_dim).expand(n, group, head_dim)
        proj.bias = nn.Parameter(b.reshape(n * group * head_dim).contiguous(), requires_grad=False)
    proj.out_features = n * group * head_dim


def expand_wnw_config(cfg: dict, num_layers: int, orig_kv_heads: int, num_q_heads: int) -> dict:
    """The WnW config JSON (dict) of a GQA model, rewritten for its MHA form."""
    if num_q_heads % orig_kv_heads:
        raise ValueError(f"num_q_heads ({num_q_heads}) must be divisible by orig_kv_heads ({orig_kv_heads})")
    g = num_q_heads // orig_kv_heads
    heads = cfg["heads"]
    rr = heads["retention_ratios"]
    if len(rr) != num_layers * orig_kv_heads:
        raise ValueError(f"retention_ratios has {len(rr)} entries, expected {num_layers * orig_kv_heads}")
    out = dict(cfg)
    out["heads"] = dict(heads)
    out["heads"]["retention_ratios"] = [r for r in rr for _ in range(g)]
    out["heads"]["class_b"] = [(gid // orig_kv_heads) * num_q_heads + (gid % orig_kv_heads) * g + j
                               for gid in heads["class_b"] for j in range(g)]
    out["heads"]["_orig_kv_heads"] = orig_kv_heads
    out["heads"]["_expanded_from_gqa"] = True
    return out
