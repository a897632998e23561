"""The reference's own session (baseline/_ref) driving this package's CPU
oracle cache through the HF Cache interface reproduces the reference
session + reference cache trace: the session boundary is the reference's,
unchanged (wnw_b200.integration widens its cache type check only)."""
import json
import os

import torch

from tests.golden.scenario import SESSION_SCENARIO as ss, make_config_dict, make_tiny_llama_config, session_inputs
from tests.oracle_hf import OracleHFCache, TracingMixin
from tests.reference_session import reference_session_or_skip
from wnw_b200.config import WnWConfig


def test_reference_session_drives_the_oracle_cache(golden_dir):
    from transformers import LlamaConfig, LlamaForCausalLM
    rsess, adapter = reference_session_or_skip(ss)
    with open(os.path.join(golden_dir, "session_trace.json")) as f:
        ref = json.load(f)
    torch.manual_seed(ss["seed"])
    model = LlamaForCausalLM(LlamaConfig(**make_tiny_llama_config(ss))).eval()

    class Tracing(TracingMixin, OracleHFCache):
        pass

    cache = Tracing(WnWConfig(**make_config_dict(ss)), ss["L"], ss["Hkv"], ss["Hq"], ss["D"])
    ids = session_inputs(ss)
    with rsess.WnWSession(model, adapter, cache) as sess:
        sess.setup_audio(ids)
        with torch.no_grad():
            out = sess.generate({"input_ids": ids}, max_new_tokens=ss["new_tokens"], do_sample=False)
    assert cache.calls == ref["calls"]
    assert out.tolist() == ref["tokens"]
    assert [sorted(s) for s in cache.oracle.loaded_segments] == ref["loaded"]


def test_non_fused_reference_session_is_refused():
    """The reference session's default branch (WNW_FUSED_ATTN unset) would
    attend with varlen_attn over packed K/V the B200 cache does not build:
    the integration refuses such a module instead of running it wrong, and
    switches it to the fused branch only when asked to."""
    import pytest

    from wnw_b200.integration import NonFusedSessionError, accept_in_reference_session
    rsess, _ = reference_session_or_skip(ss)
    try:
        rsess._FUSED_ATTN = False
        with pytest.raises(NonFusedSessionError, match="non-fused mode"):
            accept_in_reference_session(rsess)
        accept_in_reference_session(rsess, enable_fused=True)
        assert rsess._FUSED_ATTN is True
    finally:
        rsess._FUSED_ATTN = True
