"""End-to-end parity of ``B200WnWCache`` on the GPU against outputs recorded
from the reference itself (tests/golden) and against the CPU oracle.

* the cache, driven hook by hook with the seeded scenario, reproduces the
  reference's flat K/V layouts bit for bit (SHA-256 of every layer at every
  step), its cu_seqlens and loaded-segment sets exactly, and its attention
  outputs / class-A scores within fp32 tolerance;
* the session, driving a tiny random-init Llama through model.generate,
  reproduces the reference session's hook sequence and greedy tokens.
"""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from tests.golden.scenario import CACHE_SCENARIO, make_cache_inputs, make_config_dict

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda:0")


def _digest(t):
    return hashlib.sha256(np.ascontiguousarray(t.float().cpu().numpy(), dtype=np.float32).tobytes()).hexdigest()


def _packed_with_token(cache, l):
    """Flat view of layer l after this step's attention (token included)."""
    from wnw_b200 import kernels as Kx
    lens = cache._len_host[l] + 1
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int64)
    k = torch.empty(int(cu[-1]), cache.head_dim, dtype=cache.dtype, device=cache.device)
    v = torch.empty_like(k)
    Kx.copy_segments(cache.k_store[l], cache.v_store[l], cache._seg_base[l], k, v,
                     torch.from_numpy(cu[:-1]).to(cache.device),
                     torch.from_numpy(lens.astype(np.int32)).to(cache.device))
    return k, v, cu


def _drive(dev, trace_rec=None, **kw):
    from wnw_b200.cache import B200WnWCache
    from wnw_b200.config import WnWConfig
    sc = CACHE_SCENARIO
    cfg = WnWConfig(**make_config_dict(sc))
    inp = make_cache_inputs(sc)
    cache = B200WnWCache(cfg, sc["L"], sc["Hkv"], sc["Hq"], sc["D"], dev, max_decode_tokens=3, **kw)
    cache.setup_audio(torch.tensor(inp["audio_starts"]), torch.tensor(inp["audio_ends"]),
                      torch.tensor(inp["attention_mask"]))
    for l in range(sc["L"]):
        cache.prefill_after_attn(l, [x.to(dev) if x is not None else None for x in inp["class_a_scores"][l]],
                                 [[x.to(dev) if x is not None else None for x in row] for row in inp["per_head_scores"][l]],
                                 torch.from_numpy(inp["prefill_k"][l]).to(dev),
                                 torch.from_numpy(inp["prefill_v"][l]).to(dev))
    cache.prefill_all_layers_done()
    return cache, inp, sc


@pytest.mark.parametrize("tier,fetch,plan", [("host", "zerocopy", "device"), ("hbm", "zerocopy", "device"),
                                             ("host", "zerocopy", "host"), ("host", "dma", "host")])
def test_cache_reproduces_reference_trace(dev, golden_dir, tier, fetch, plan):
    """offload_tier "hbm" keeps the offloaded rows in device memory, fetch_mode
    "dma" gathers them on the host and copies them with the copy engine, and
    fetch_plan "host" plans the fetch on the host instead of the device; the
    layouts, selections and outputs must not change."""
    tz = np.load(os.path.join(golden_dir, "cache_trace.npz"), allow_pickle=True)
    cache, inp, sc = _drive(dev, offload_tier=tier, fetch_mode=fetch, fetch_plan=plan)
    assert (cache._dplan is not None) == (plan == "device")
    G = sc["Hq"] // sc["Hkv"]
    for l in range(sc["L"]):
        k, v, cu = cache.packed_layer(l)
        assert np.array_equal(cu.cpu().numpy(), tz["prefill_cu"][l])
        assert np.array_equal(k.cpu().numpy(), tz[f"prefill_k{l}"])
    assert [sorted(s) for s in cache.loaded_segments] == [list(x) for x in tz["prefill_loaded"]]
    for t in range(sc["steps"]):
        for l in range(sc["L"]):
            q = torch.from_numpy(inp["dec_q"][t][l]).to(dev)
            kk, vv, cu, mk = cache.decode_before_attn(l, torch.from_numpy(inp["dec_k"][t][l]).to(dev),
                                                      torch.from_numpy(inp["dec_v"][t][l]).to(dev))
            qf = q.squeeze(2).reshape(sc["B"], sc["Hkv"], G, sc["D"]).reshape(-1, G, sc["D"])
            out = cache.fused_decode_attention(l, qf, q, kk, vv, cu, sc["D"] ** -0.5)
            pk, pv, pcu = _packed_with_token(cache, l)
            assert np.array_equal(pcu, tz[f"s{t}_l{l}_cu"]), (t, l)
            assert mk == int(np.diff(pcu).max())
            assert _digest(pk) == str(tz[f"s{t}_l{l}_khash"]), (t, l)
            assert _digest(pv) == str(tz[f"s{t}_l{l}_vhash"]), (t, l)
            np.testing.assert_allclose(out.cpu().numpy(), tz[f"s{t}_l{l}_out"], atol=1e-5, rtol=1e-5)
        cache.decode_all_layers_done()
        np.testing.assert_allclose(cache.score_accumulator.cpu().numpy(), tz[f"s{t}_scores"], atol=1e-5, rtol=1e-4)
        assert [sorted(s) for s in cache.loaded_segments] == [list(x) for x in tz[f"s{t}_loaded"]], t
    # slots grew past the initial decode reservation (3 rows) without losing rows
    assert (cache._cap_host >= cache._len_host + 1).all()
    # InferenceStats: the reference's snapshots and per-sample transfer events
    from tests.stats_compare import normalise
    with open(os.path.join(golden_dir, "stats.json")) as f:
        want = json.load(f)["cache_trace"]
    assert normalise(cache.get_all_stats()) == normalise(want)
    assert cache.get_compression_stats()[0]["step"] == -1
    assert cache.get_snapshot_stats(7)[1]["num_audio"] == want[1]["prefill"]["num_audio"]


def test_cache_matches_oracle_in_bf16(dev):
    """bf16 run of the same scenario: layouts exact vs the oracle fed the same
    bf16 rows; outputs within 2e-2; selections equal up to a near tie, on
    which the oracle follows the GPU (tests/follow_oracle.py)."""
    from tests.follow_oracle import FollowOracle, sync_selection
    from wnw_b200.cache import B200WnWCache
    from wnw_b200.config import WnWConfig
    sc = dict(CACHE_SCENARIO)
    sc["D"] = 64
    sc["steps"] = 6
    cfg = WnWConfig(**make_config_dict(sc))
    inp = make_cache_inputs(sc)
    bf = lambda a: torch.from_numpy(a).to(torch.bfloat16)  # noqa: E731
    cache = B200WnWCache(cfg, sc["L"], sc["Hkv"], sc["Hq"], sc["D"], dev, max_decode_tokens=2)
    orc = FollowOracle(cfg, sc["L"], sc["Hkv"], sc["Hq"], sc["D"])
    cache.setup_audio(torch.tensor(inp["audio_starts"]), torch.tensor(inp["audio_ends"]),
                      torch.tensor(inp["attention_mask"]))
    orc.setup_audio(inp["audio_starts"], inp["audio_ends"], inp["pad"])
    for l in range(sc["L"]):
        ca = inp["class_a_scores"][l]
        ph = inp["per_head_scores"][l]
        cache.prefill_after_attn(l, [x.to(dev) if x is not None else None for x in ca],
                                 [[x.to(dev) if x is not None else None for x in r] for r in ph],
                                 bf(inp["prefill_k"][l]).to(dev), bf(inp["prefill_v"][l]).to(dev))
        orc.prefill_after_attn(l, ca, ph, bf(inp["prefill_k"][l]), bf(inp["prefill_v"][l]))
    cache.prefill_all_layers_done()
    orc.prefill_all_layers_done()
    G = sc["Hq"] // sc["Hkv"]
    for t in range(sc["steps"]):
        for l in range(sc["L"]):
            q = bf(inp["dec_q"][t][l])
            k, v = bf(inp["dec_k"][t][l]), bf(inp["dec_v"][t][l])
            kk, vv, cu, _ = cache.decode_before_attn(l, k.to(dev), v.to(dev))
            orc.decode_before_attn(l, k, v)
            qf = q.squeeze(2).reshape(sc["B"], sc["Hkv"], G, sc["D"]).reshape(-1, G, sc["D"])
            out = cache.fused_decode_attention(l, qf.to(dev), q.to(dev), kk, vv, cu, sc["D"] ** -0.5)
            ref = orc.fused_decode_attention(l, qf, scale=sc["D"] ** -0.5)
            np.testing.assert_allclose(out.float().cpu().numpy(), orc.last_out64, atol=2e-2, rtol=2e-2)
            pk, _, pcu = _packed_with_token(cache, l)
            assert np.array_equal(pcu, orc.cu(l))
            assert torch.equal(pk.cpu(), orc.layer_k[l])
            del ref
        cache.decode_all_layers_done()  # scores are formed here
        sync_selection(orc, cache.last_topk)
        orc.decode_all_layers_done()
        np.testing.assert_allclose(cache.score_accumulator.cpu().numpy(), orc.last_scores, atol=1e-4, rtol=1e-3)
        assert cache.last_topk == orc.last_topk, t
        assert [sorted(s) for s in cache.loaded_segments] == [sorted(s) for s in orc.loaded_segments], t


@pytest.mark.parametrize("mode", ["last", "mean_text"])
def test_session_reproduces_reference_generation(dev, golden_dir, mode):
    """Tiny random-init Llama in fp32 on the GPU: model.generate through our
    session and B200WnWCache gives the reference session's hook calls,
    prefill layouts (under either prefill score mode), greedy tokens and
    stats."""
    from transformers import LlamaConfig, LlamaForCausalLM
    from tests.golden.scenario import (MEAN_TEXT_SESSION_SCENARIO, SESSION_SCENARIO, make_tiny_llama_config,
                                       session_inputs)
    from tests.oracle_hf import TracingMixin
    from wnw_b200.adapters import LlamaFamilyAdapter
    from wnw_b200.cache import B200WnWCache
    from wnw_b200.config import WnWConfig
    from wnw_b200.session import WnWSession

    ss = SESSION_SCENARIO if mode == "last" else MEAN_TEXT_SESSION_SCENARIO
    name = "session_trace.json" if mode == "last" else "session_mean_text_trace.json"
    with open(os.path.join(golden_dir, name)) as f:
        ref = json.load(f)
    torch.manual_seed(ss["seed"])
    model = LlamaForCausalLM(LlamaConfig(**make_tiny_llama_config(ss))).eval().to(dev)
    prefill_k = []  # prefill K layouts, per layer

    class Tracing(TracingMixin, B200WnWCache):
        def prefill_all_layers_done(self):
            super().prefill_all_layers_done()
            prefill_k.extend(self.packed_layer(l)[0].float().cpu().numpy() for l in range(ss["L"]))

    cache = Tracing(WnWConfig(**make_config_dict(ss)), ss["L"], ss["Hkv"], ss["Hq"], ss["D"], dev,
                    max_decode_tokens=4)
    ids = session_inputs(ss).to(dev)
    with WnWSession(model, LlamaFamilyAdapter(ss["audio_start"], ss["audio_end"]), cache) as sess:
        sess.setup_audio(ids)
        with torch.no_grad():
            out = sess.generate({"input_ids": ids}, max_new_tokens=ss["new_tokens"], do_sample=False)
    assert cache.calls == ref["calls"]
    # the model's K on the GPU differs from the reference's CPU run in the low
    # bits, so the kept rows are compared by value within fp32 tolerance (a
    # different choice of kept rows differs by O(1))
    want = np.load(os.path.join(golden_dir, name.replace(".json", "_prefill_k.npz")))
    for l, k in enumerate(prefill_k):
        assert k.shape == want[f"l{l}"].shape, l
        np.testing.assert_allclose(k, want[f"l{l}"], atol=1e-4, rtol=1e-4)
    assert out.cpu().tolist() == ref["tokens"]
    assert [sorted(s) for s in cache.loaded_segments] == ref["loaded"]
    from tests.stats_compare import normalise
    assert normalise(sess.get_stats()) == normalise(ref["stats"])


@pytest.mark.parametrize("variant", [dict(lag=0), dict(lag=1), dict(lag=3, top_k=1),
                                     dict(top_k=5, chunk_size_s=16.0, overlap_s=0.0), dict(steps=12, top_k=2),
                                     dict(audio_starts=[5, 305], audio_ends=[305, 305])])
def test_device_fetch_plan_follows_planner(dev, variant):
    """The device fetch plan mirrors the planner's selection diff (eviction
    lag, chunks of one or two segments, several loads per step, a sample
    with no audio at all): every step
    the cache checks its landing rows, loaded maps and counters against the
    host planner's (a difference raises), and the fp32 run must match the
    oracle's layouts, loaded sets and outputs."""
    from tests.follow_oracle import FollowOracle, sync_selection
    from wnw_b200.cache import B200WnWCache
    from wnw_b200.config import WnWConfig
    sc = dict(CACHE_SCENARIO, **variant)
    cfg = WnWConfig(**make_config_dict(sc))
    inp = make_cache_inputs(sc)
    G = sc["Hq"] // sc["Hkv"]
    cache = B200WnWCache(cfg, sc["L"], sc["Hkv"], sc["Hq"], sc["D"], dev, max_decode_tokens=2, fetch_plan="device")
    orc = FollowOracle(cfg, sc["L"], sc["Hkv"], sc["Hq"], sc["D"])
    cache.setup_audio(torch.tensor(inp["audio_starts"]), torch.tensor(inp["audio_ends"]),
                      torch.tensor(inp["attention_mask"]))
    orc.setup_audio(inp["audio_starts"], inp["audio_ends"], inp["pad"])
    for l in range(sc["L"]):
        ca, ph = inp["class_a_scores"][l], inp["per_head_scores"][l]
        k, v = torch.from_numpy(inp["prefill_k"][l]), torch.from_numpy(inp["prefill_v"][l])
        cache.prefill_after_attn(l, [x.to(dev) if x is not None else None for x in ca],
                                 [[x.to(dev) if x is not None else None for x in r] for r in ph], k.to(dev), v.to(dev))
        orc.prefill_after_attn(l, ca, ph, k, v)
    cache.prefill_all_layers_done()
    orc.prefill_all_layers_done()
    assert cache._dplan is not None
    loads = evicts = 0
    for t in range(sc["steps"]):
        for l in range(sc["L"]):
            q = torch.from_numpy(inp["dec_q"][t][l])
            k, v = torch.from_numpy(inp["dec_k"][t][l]), torch.from_numpy(inp["dec_v"][t][l])
            kk, vv, cu, _ = cache.decode_before_attn(l, k.to(dev), v.to(dev))
            orc.decode_before_attn(l, k, v)
            qf = q.squeeze(2).reshape(sc["B"], sc["Hkv"], G, sc["D"]).reshape(-1, G, sc["D"])
            out = cache.fused_decode_attention(l, qf.to(dev), q.to(dev), kk, vv, cu, sc["D"] ** -0.5)
            orc.fused_decode_attention(l, qf, scale=sc["D"] ** -0.5)
            np.testing.assert_allclose(out.cpu().numpy(), orc.last_out64, atol=1e-5, rtol=1e-5)
            pk, _, pcu = _packed_with_token(cache, l)
            assert np.array_equal(pcu, orc.cu(l)), (t, l)
            assert torch.equal(pk.cpu(), orc.layer_k[l]), (t, l)
        cache.decode_all_layers_done()
        sync_selection(orc, cache.last_topk)
        orc.decode_all_layers_done()
        assert cache.last_topk == orc.last_topk, t
        assert [sorted(s) for s in cache.loaded_segments] == [sorted(s) for s in orc.loaded_segments], t
        loads += sum(len(x) for x in orc.last_to_load)
        evicts += sum(len(x) for x in orc.last_to_evict)
    assert loads > 0 and (evicts > 0 or sc["lag"] > sc["steps"])


def test_cache_serves_a_second_request(dev, golden_dir):
    """One cache, two requests back to back: the first request's last step
    has already fetched ahead for a step that never comes; the second
    request's prefill waits for that fetch, replans from scratch and must
    reproduce the reference trace exactly as a fresh cache does."""
    from wnw_b200.cache import B200WnWCache
    from wnw_b200.config import WnWConfig
    tz = np.load(os.path.join(golden_dir, "cache_trace.npz"), allow_pickle=True)
    sc = CACHE_SCENARIO
    inp = make_cache_inputs(sc)
    G = sc["Hq"] // sc["Hkv"]
    cache = B200WnWCache(WnWConfig(**make_config_dict(sc)), sc["L"], sc["Hkv"], sc["Hq"], sc["D"], dev,
                         max_decode_tokens=3)
    for _ in range(2):
        cache.setup_audio(torch.tensor(inp["audio_starts"]), torch.tensor(inp["audio_ends"]),
                          torch.tensor(inp["attention_mask"]))
        for l in range(sc["L"]):
            cache.prefill_after_attn(l, [x.to(dev) if x is not None else None for x in inp["class_a_scores"][l]],
                                     [[x.to(dev) if x is not None else None for x in row]
                                      for row in inp["per_head_scores"][l]],
                                     torch.from_numpy(inp["prefill_k"][l]).to(dev),
                                     torch.from_numpy(inp["prefill_v"][l]).to(dev))
        cache.prefill_all_layers_done()
        assert [sorted(s) for s in cache.loaded_segments] == [list(x) for x in tz["prefill_loaded"]]
        for t in range(4):
            for l in range(sc["L"]):
                q = torch.from_numpy(inp["dec_q"][t][l]).to(dev)
                kk, vv, cu, _ = cache.decode_before_attn(l, torch.from_numpy(inp["dec_k"][t][l]).to(dev),
                                                         torch.from_numpy(inp["dec_v"][t][l]).to(dev))
                qf = q.squeeze(2).reshape(sc["B"], sc["Hkv"], G, sc["D"]).reshape(-1, G, sc["D"])
                out = cache.fused_decode_attention(l, qf, q, kk, vv, cu, sc["D"] ** -0.5)
                pk, pv, pcu = _packed_with_token(cache, l)
                assert np.array_equal(pcu, tz[f"s{t}_l{l}_cu"]), (t, l)
                assert _digest(pk) == str(tz[f"s{t}_l{l}_khash"]), (t, l)
                np.testing.assert_allclose(out.cpu().numpy(), tz[f"s{t}_l{l}_out"], atol=1e-5, rtol=1e-5)
            cache.decode_all_layers_done()
            assert [sorted(s) for s in cache.loaded_segments] == [list(x) for x in tz[f"s{t}_loaded"]], t


def test_mha_mode_session_reproduces_reference_generation(dev, golden_dir):
    """GQA -> MHA mode (wnw_b200.degqa: the expanded model and config, one kv
    head per q head) through our session and B200WnWCache on the GPU gives
    the reference's MHA-mode hook calls, greedy tokens and loaded sets."""
    from transformers import LlamaConfig, LlamaForCausalLM
    from tests.golden.scenario import SESSION_SCENARIO as ss, make_tiny_llama_config, session_inputs
    from tests.oracle_hf import TracingMixin
    from wnw_b200.adapters import LlamaFamilyAdapter
    from wnw_b200.cache import B200WnWCache
    from wnw_b200.config import WnWConfig
    from wnw_b200.degqa import degqa_model, expand_wnw_config
    from wnw_b200.session import WnWSession

    with open(os.path.join(golden_dir, "session_degqa_trace.json")) as f:
        ref = json.load(f)
    torch.manual_seed(ss["seed"])
    model = LlamaForCausalLM(LlamaConfig(**make_tiny_llama_config(ss))).eval().to(dev)
    adapter = LlamaFamilyAdapter(ss["audio_start"], ss["audio_end"])
    degqa_model(model, adapter)
    heads = expand_wnw_config(WnWConfig(**make_config_dict(ss)).to_dict(), ss["L"], ss["Hkv"], ss["Hq"])["heads"]
    cfg = WnWConfig(**dict(make_config_dict(ss), class_b=heads["class_b"],
                           retention_ratios=heads["retention_ratios"], num_kv_heads=ss["Hq"]))

    class Tracing(TracingMixin, B200WnWCache):
        pass

    cache = Tracing(cfg, ss["L"], ss["Hq"], ss["Hq"], ss["D"], dev, max_decode_tokens=4)
    ids = session_inputs(ss).to(dev)
    with WnWSession(model, adapter, cache) as sess:
        sess.setup_audio(ids)
        with torch.no_grad():
            out = sess.generate({"input_ids": ids}, max_new_tokens=ss["new_tokens"], do_sample=False)
    calls = [c for c in cache.calls if c[0] in ("decode_before_attn", "decode_all_layers_done")]
    assert calls == ref["calls"]
    assert out.cpu().tolist() == ref["tokens"]
    assert [sorted(s) for s in cache.loaded_segments] == ref["loaded"]


def test_reference_session_drives_our_cache(dev, golden_dir):
    """Drop-in check at the session boundary: the reference's OWN session
    (the offline install in baseline/_ref, fused-attention path) driving
    B200WnWCache on the GPU gives the reference session + reference cache's
    hook calls, greedy tokens, loaded sets and stats."""
    from transformers import LlamaConfig, LlamaForCausalLM
    from tests.golden.scenario import SESSION_SCENARIO as ss, make_tiny_llama_config, session_inputs
    from tests.oracle_hf import TracingMixin
    from tests.reference_session import reference_session_or_skip
    from tests.stats_compare import normalise
    from wnw_b200.cache import B200WnWCache
    from wnw_b200.config import WnWConfig

    rsess, adapter = reference_session_or_skip(ss)
    with open(os.path.join(golden_dir, "session_trace.json")) as f:
        ref = json.load(f)
    torch.manual_seed(ss["seed"])
    model = LlamaForCausalLM(LlamaConfig(**make_tiny_llama_config(ss))).eval().to(dev)

    class Tracing(TracingMixin, B200WnWCache):
        pass

    cache = Tracing(WnWConfig(**make_config_dict(ss)), ss["L"], ss["Hkv"], ss["Hq"], ss["D"], dev,
                    max_decode_tokens=4)
    ids = session_inputs(ss).to(dev)
    with rsess.WnWSession(model, adapter, cache) as sess:
        sess.setup_audio(ids)
        with torch.no_grad():
            out = sess.generate({"input_ids": ids}, max_new_tokens=ss["new_tokens"], do_sample=False)
    assert cache.calls == ref["calls"]
    assert out.cpu().tolist() == ref["tokens"]
    assert [sorted(s) for s in cache.loaded_segments] == ref["loaded"]
    assert normalise(sess.get_stats()) == normalise(ref["stats"])


@pytest.mark.parametrize("variant", [dict(audio_starts=[305, 305], audio_ends=[305, 305]),  # no audio at all
                                     dict(top_k=40),                   # top-k covers every chunk
                                     dict(lag=50, steps=10)])          # nothing is ever evicted
def test_cache_edge_cases_match_oracle(dev, variant):
    """Edge cases of the selection: a batch without audio (no scoring, no
    selection), a top-k that covers every chunk (everything loaded at
    prefill, nothing moves), an eviction lag longer than the run (loads
    only, slots grow): layouts, loaded sets and outputs as the oracle's."""
    from tests.follow_oracle import FollowOracle, sync_selection
    from wnw_b200.cache import B200WnWCache
    from wnw_b200.config import WnWConfig
    sc = dict(CACHE_SCENARIO, **variant)
    cfg = WnWConfig(**make_config_dict(sc))
    inp = make_cache_inputs(sc)
    G = sc["Hq"] // sc["Hkv"]
    cache = B200WnWCache(cfg, sc["L"], sc["Hkv"], sc["Hq"], sc["D"], dev, max_decode_tokens=2)
    orc = FollowOracle(cfg, sc["L"], sc["Hkv"], sc["Hq"], sc["D"])
    cache.setup_audio(torch.tensor(inp["audio_starts"]), torch.tensor(inp["audio_ends"]),
                      torch.tensor(inp["attention_mask"]))
    orc.setup_audio(inp["audio_starts"], inp["audio_ends"], inp["pad"])
    for l in range(sc["L"]):
        ca, ph = inp["class_a_scores"][l], inp["per_head_scores"][l]
        k, v = torch.from_numpy(inp["prefill_k"][l]), torch.from_numpy(inp["prefill_v"][l])
        cache.prefill_after_attn(l, [x.to(dev) if x is not None else None for x in ca],
                                 [[x.to(dev) if x is not None else None for x in r] for r in ph], k.to(dev), v.to(dev))
        orc.prefill_after_attn(l, ca, ph, k, v)
    cache.prefill_all_layers_done()
    orc.prefill_all_layers_done()
    assert [sorted(s) for s in cache.loaded_segments] == [sorted(s) for s in orc.loaded_segments]
    for t in range(sc["steps"]):
        for l in range(sc["L"]):
            q = torch.from_numpy(inp["dec_q"][t][l])
            k, v = torch.from_numpy(inp["dec_k"][t][l]), torch.from_numpy(inp["dec_v"][t][l])
            kk, vv, cu, _ = cache.decode_before_attn(l, k.to(dev), v.to(dev))
            orc.decode_before_attn(l, k, v)
            qf = q.squeeze(2).reshape(sc["B"], sc["Hkv"], G, sc["D"]).reshape(-1, G, sc["D"])
            out = cache.fused_decode_attention(l, qf.to(dev), q.to(dev), kk, vv, cu, sc["D"] ** -0.5)
            orc.fused_decode_attention(l, qf, scale=sc["D"] ** -0.5)
            np.testing.assert_allclose(out.cpu().numpy(), orc.last_out64, atol=1e-5, rtol=1e-5)
            pk, _, pcu = _packed_with_token(cache, l)
            assert np.array_equal(pcu, orc.cu(l)), (t, l)
            assert torch.equal(pk.cpu(), orc.layer_k[l]), (t, l)
        cache.decode_all_layers_done()
        sync_selection(orc, cache.last_topk)
        orc.decode_all_layers_done()
        assert cache.last_topk == orc.last_topk, t
        assert [sorted(s) for s in cache.loaded_segments] == [sorted(s) for s in orc.loaded_segments], t


def test_cache_reproduces_reference_trace_global_prefill_topk(dev, golden_dir):
    """The global per-head prefill top-k (cache.py:1141-1150): the B200 cache
    reproduces the reference's trace recorded with it (layout digests,
    cu_seqlens, loaded sets; outputs and class-A scores within fp32
    tolerance)."""
    from tests.golden.scenario import GLOBAL_TOPK_SCENARIO as sc
    from wnw_b200.cache import B200WnWCache
    from wnw_b200.config import WnWConfig
    tz = np.load(os.path.join(golden_dir, "cache_trace_global.npz"), allow_pickle=True)
    inp = make_cache_inputs(sc)
    G = sc["Hq"] // sc["Hkv"]
    cache = B200WnWCache(WnWConfig(**make_config_dict(sc)), sc["L"], sc["Hkv"], sc["Hq"], sc["D"], dev,
                         max_decode_tokens=3)
    cache.setup_audio(torch.tensor(inp["audio_starts"]), torch.tensor(inp["audio_ends"]),
                      torch.tensor(inp["attention_mask"]))
    for l in range(sc["L"]):
        cache.prefill_after_attn(l, [x.to(dev) if x is not None else None for x in inp["class_a_scores"][l]],
                                 [[x.to(dev) if x is not None else None for x in row]
                                  for row in inp["per_head_scores"][l]],
                                 torch.from_numpy(inp["prefill_k"][l]).to(dev),
                                 torch.from_numpy(inp["prefill_v"][l]).to(dev))
    cache.prefill_all_layers_done()
    for l in range(sc["L"]):
        k, _, cu = cache.packed_layer(l)
        assert np.array_equal(cu.cpu().numpy(), tz["prefill_cu"][l])
        assert _digest(k) == str(tz[f"prefill_khash{l}"])
    assert [sorted(s) for s in cache.loaded_segments] == [list(x) for x in tz["prefill_loaded"]]
    for t in range(sc["steps"]):
        for l in range(sc["L"]):
            q = torch.from_numpy(inp["dec_q"][t][l]).to(dev)
            kk, vv, cu, _ = cache.decode_before_attn(l, torch.from_numpy(inp["dec_k"][t][l]).to(dev),
                                                     torch.from_numpy(inp["dec_v"][t][l]).to(dev))
            qf = q.squeeze(2).reshape(sc["B"], sc["Hkv"], G, sc["D"]).reshape(-1, G, sc["D"])
            out = cache.fused_decode_attention(l, qf, q, kk, vv, cu, sc["D"] ** -0.5)
            pk, pv, pcu = _packed_with_token(cache, l)
            assert np.array_equal(pcu, tz[f"s{t}_l{l}_cu"]), (t, l)
            assert _digest(pk) == str(tz[f"s{t}_l{l}_khash"]), (t, l)
            assert _digest(pv) == str(tz[f"s{t}_l{l}_vhash"]), (t, l)
            np.testing.assert_allclose(out.cpu().numpy(), tz[f"s{t}_l{l}_out"], atol=1e-5, rtol=1e-5)
        cache.decode_all_layers_done()
        np.testing.assert_allclose(cache.score_accumulator.cpu().numpy(), tz[f"s{t}_scores"], atol=1e-5, rtol=1e-4)
        assert [sorted(s) for s in cache.loaded_segments] == [list(x) for x in tz[f"s{t}_loaded"]], t
