"""GQA -> MHA mode (wnw_b200.degqa) on CPU, against the reference's own
outputs (tests/golden/session_degqa_trace.json, made by executing the
reference's expand_config, degqa_model and session):

* the config expansion equals the reference's, field for field;
* the expanded model computes what the GQA model computed;
* our session and the CPU oracle cache in MHA mode (one kv head per q head,
  the expanded config) reproduce the reference's hook calls, greedy tokens
  and loaded sets.
"""
import json
import os

import pytest
import torch

from tests.golden.scenario import SESSION_SCENARIO as ss, make_config_dict, make_tiny_llama_config, session_inputs
from wnw_b200.adapters import LlamaFamilyAdapter
from wnw_b200.config import WnWConfig
from wnw_b200.degqa import degqa_model, expand_wnw_config


@pytest.fixture(scope="module")
def ref(golden_dir):
    with open(os.path.join(golden_dir, "session_degqa_trace.json")) as f:
        return json.load(f)


def _tiny_llama():
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(ss["seed"])
    return LlamaForCausalLM(LlamaConfig(**make_tiny_llama_config(ss))).eval()


def test_expand_config_matches_reference(ref):
    out = expand_wnw_config(ref["config_in"], ss["L"], ss["Hkv"], ss["Hq"])
    assert out == ref["config_out"]
    with pytest.raises(ValueError):
        expand_wnw_config(ref["config_in"], ss["L"], 3, ss["Hq"])


def test_degqa_keeps_the_model_function():
    model = _tiny_llama()
    adapter = LlamaFamilyAdapter(ss["audio_start"], ss["audio_end"])
    ids = session_inputs(ss)
    with torch.no_grad():
        before = model(ids).logits
        degqa_model(model, adapter)
        after = model(ids).logits
    assert model.config.num_key_value_heads == ss["Hq"]
    assert model.model.layers[0].self_attn.k_proj.out_features == ss["Hq"] * ss["D"]
    torch.testing.assert_close(after, before, atol=1e-5, rtol=1e-5)


def test_mha_session_matches_reference(ref):
    from tests.oracle_hf import OracleHFCache, TracingMixin
    from oracle.prefill_scores import compute_prefill_scores
    from wnw_b200.session import WnWSession
    model = _tiny_llama()
    adapter = LlamaFamilyAdapter(ss["audio_start"], ss["audio_end"])
    degqa_model(model, adapter)
    heads = expand_wnw_config(WnWConfig(**make_config_dict(ss)).to_dict(), ss["L"], ss["Hkv"], ss["Hq"])["heads"]
    cfg = WnWConfig(**dict(make_config_dict(ss), class_b=heads["class_b"],
                           retention_ratios=heads["retention_ratios"], num_kv_heads=ss["Hq"]))

    class Tracing(TracingMixin, OracleHFCache):
        pass

    cache = Tracing(cfg, ss["L"], ss["Hq"], ss["Hq"], ss["D"])
    ids = session_inputs(ss)
    with WnWSession(model, adapter, cache, prefill_scores=compute_prefill_scores) as sess:
        sess.setup_audio(ids)
        with torch.no_grad():
            out = sess.generate({"input_ids": ids}, max_new_tokens=ss["new_tokens"], do_sample=False)
    calls = [c for c in cache.calls if c[0] in ("decode_before_attn", "decode_all_layers_done")]
    assert calls == ref["calls"]
    assert out.tolist() == ref["tokens"]
    assert [sorted(s) for s in cache.oracle.loaded_segments] == ref["loaded"]
