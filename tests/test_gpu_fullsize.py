"""Parity at the benchmark's full size: BASELINE config 2's shapes (30 layers,
8 kv heads / 32 q heads, head_dim 128, a 15,064-token prompt with 15,000
audio tokens, bf16, the bench's head classes and chunk settings), seeded
random prefill K/V and scores and decode q/k/v, run through ``B200WnWCache``
on the GPU and the CPU oracle side by side for a few decode steps (each with
chunk loads and evictions): flat layouts bit for bit, loaded sets exactly,
attention within bf16 tolerance, class-A scores within fp32 tolerance, chunk
selections equal up to a near tie (``tests/follow_oracle.py``: where the
oracle's k-th / (k+1)-th chunk-score gap is within fp32 rounding the oracle
follows the GPU's choice; a wider disagreement fails)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

STEPS = 3


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda:0")


def _inputs(seed, L, H, Hq, D, S0, a0, a1, cfg):
    rng = np.random.default_rng(seed)
    bf = lambda a: torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16)  # noqa: E731
    G = Hq // H
    n_audio = a1 - a0
    prefill = []
    for l in range(L):
        k = bf(rng.standard_normal((1, H, S0, D), np.float32))
        v = bf(rng.standard_normal((1, H, S0, D), np.float32))
        has_a = bool(cfg.get_layer_class_a(l))
        ca = [torch.from_numpy(rng.random(n_audio, np.float32)) if has_a else None]
        ph = [[None if cfg.is_class_a_kv_head(l, h) else torch.from_numpy(rng.random(n_audio, np.float32))
               for h in range(H)]]
        prefill.append((ca, ph, k, v))
    steps = [[(bf(rng.standard_normal((H, G, D), np.float32)), bf(rng.standard_normal((1, H, 1, D), np.float32)),
               bf(rng.standard_normal((1, H, 1, D), np.float32))) for _ in range(L)] for _ in range(STEPS)]
    return prefill, steps


def test_config2_full_size_matches_oracle(dev):
    from bench import MODEL, PROMPT, wnw_config
    from tests.follow_oracle import FollowOracle, sync_selection
    from tests.test_gpu_cache import _packed_with_token
    from wnw_b200.cache import B200WnWCache

    L, H, Hq, D = MODEL["L"], MODEL["Hkv"], MODEL["Hq"], MODEL["D"]
    a0 = PROMPT["sink"]
    a1 = a0 + PROMPT["audio"]
    S0 = a1 + PROMPT["tail"]
    cfg = wnw_config()
    prefill, steps = _inputs(2024, L, H, Hq, D, S0, a0, a1, cfg)
    cache = B200WnWCache(cfg, L, H, Hq, D, dev, max_decode_tokens=STEPS + 4)
    orc = FollowOracle(cfg, L, H, Hq, D)
    cache.setup_audio(torch.tensor([a0]), torch.tensor([a1]), None)
    orc.setup_audio([a0], [a1], [0])
    for l, (ca, ph, k, v) in enumerate(prefill):
        cache.prefill_after_attn(l, [x.to(dev) if x is not None else None for x in ca],
                                 [[x.to(dev) if x is not None else None for x in r] for r in ph], k.to(dev), v.to(dev))
        orc.prefill_after_attn(l, ca, ph, k, v)
    cache.prefill_all_layers_done()
    orc.prefill_all_layers_done()
    assert [sorted(s) for s in cache.loaded_segments] == [sorted(s) for s in orc.loaded_segments]
    changes, near_ties = 0, 0
    for t, step in enumerate(steps):
        for l, (q, k, v) in enumerate(step):
            kk, vv, cu, _ = cache.decode_before_attn(l, k.to(dev), v.to(dev))
            orc.decode_before_attn(l, k, v)
            out = cache.fused_decode_attention(l, q.to(dev), None, kk, vv, cu, D ** -0.5)
            orc.fused_decode_attention(l, q, scale=D ** -0.5)
            np.testing.assert_allclose(out.float().cpu().numpy(), orc.last_out64, atol=2e-2, rtol=2e-2)
            pk, _, pcu = _packed_with_token(cache, l)
            assert np.array_equal(pcu, orc.cu(l)), (t, l)
            assert torch.equal(pk.cpu(), orc.layer_k[l]), (t, l)
        cache.decode_all_layers_done()
        near_ties += sync_selection(orc, cache.last_topk)
        orc.decode_all_layers_done()
        np.testing.assert_allclose(cache.score_accumulator.cpu().numpy(), orc.last_scores, atol=1e-4, rtol=1e-3)
        assert cache.last_topk[0] == orc.last_topk[0], t
        assert [sorted(s) for s in cache.loaded_segments] == [sorted(s) for s in orc.loaded_segments], t
        changes += bool(orc.last_to_load[0] or orc.last_to_evict[0])
    assert changes >= 2
    assert near_ties < STEPS  # at least one step agreed on its own


def _config3_scenario(seed=31):
    """BASELINE config 3's shape, reduced to 2 layers: Qwen2.5-Omni-7B-like
    heads (4 kv / 28 q, GQA 7, head_dim 128), batch 8 with seeded lognormal
    prompt lengths (median 3k, clipped to [1k, 6k]) left-padded to the
    longest, 50 % class-A kv heads, class-B retention 0.25 (~60 % of the KV
    kept), chunks of 128 tokens, top-8, lag 1."""
    rng = np.random.default_rng(seed)
    B, L, H, Hq = 8, 2, 4, 28
    lens = np.clip(np.round(np.exp(rng.normal(np.log(3000), 0.5, B))), 1000, 6000).astype(int)
    S = int(lens.max())
    pad = [int(S - n) for n in lens]
    G = Hq // H
    return dict(seed=seed, L=L, Hkv=H, Hq=Hq, D=128, B=B, steps=3, S=S,
                audio_starts=[p + 4 for p in pad], audio_ends=[S - 30] * B, pad=pad,
                chunk_size_s=128.0, overlap_s=0.0, token_rate=1.0,
                class_a=[l * Hq + q for l in range(L) for q in range(2 * G)],
                class_b=[l * H + h for l in range(L) for h in (2, 3)],
                retention={(l, h): 0.25 for l in range(L) for h in (2, 3)},
                top_k=8, lag=1, prefill_mode="last")


def test_config3_shape_matches_oracle(dev):
    """Batch 8 with ragged, left-padded prompts and GQA 7 through the whole
    decode path (device fetch plan, fetch, rebuild, attention with scoring,
    top-k) against the oracle: layouts bit for bit, loaded sets exactly,
    attention within bf16 tolerance, class-A scores within fp32 tolerance."""
    from tests.follow_oracle import FollowOracle, sync_selection
    from tests.golden.scenario import make_cache_inputs, make_config_dict
    from tests.test_gpu_cache import _packed_with_token
    from wnw_b200.cache import B200WnWCache
    from wnw_b200.config import WnWConfig

    sc = _config3_scenario()
    cfg = WnWConfig(**make_config_dict(sc))
    inp = make_cache_inputs(sc)
    L, H, Hq, D, B = sc["L"], sc["Hkv"], sc["Hq"], sc["D"], sc["B"]
    G = Hq // H
    bf = lambda a: torch.from_numpy(a).to(torch.bfloat16)  # noqa: E731
    cache = B200WnWCache(cfg, L, H, Hq, D, dev, max_decode_tokens=sc["steps"] + 2)
    orc = FollowOracle(cfg, L, H, Hq, D)
    cache.setup_audio(torch.tensor(inp["audio_starts"]), torch.tensor(inp["audio_ends"]),
                      torch.tensor(inp["attention_mask"]))
    orc.setup_audio(inp["audio_starts"], inp["audio_ends"], inp["pad"])
    for l in range(L):
        ca, ph = inp["class_a_scores"][l], inp["per_head_scores"][l]
        k, v = bf(inp["prefill_k"][l]), bf(inp["prefill_v"][l])
        cache.prefill_after_attn(l, [x.to(dev) if x is not None else None for x in ca],
                                 [[x.to(dev) if x is not None else None for x in r] for r in ph], k.to(dev), v.to(dev))
        orc.prefill_after_attn(l, ca, ph, k, v)
    cache.prefill_all_layers_done()
    orc.prefill_all_layers_done()
    assert cache._dplan is not None
    assert [sorted(s) for s in cache.loaded_segments] == [sorted(s) for s in orc.loaded_segments]
    loads = 0
    for t in range(sc["steps"]):
        for l in range(L):
            q = bf(inp["dec_q"][t][l])
            k, v = bf(inp["dec_k"][t][l]), bf(inp["dec_v"][t][l])
            kk, vv, cu, _ = cache.decode_before_attn(l, k.to(dev), v.to(dev))
            orc.decode_before_attn(l, k, v)
            qf = q.squeeze(2).reshape(B, H, G, D).reshape(-1, G, D)
            out = cache.fused_decode_attention(l, qf.to(dev), q.to(dev), kk, vv, cu, D ** -0.5)
            orc.fused_decode_attention(l, qf, scale=D ** -0.5)
            np.testing.assert_allclose(out.float().cpu().numpy(), orc.last_out64, atol=2e-2, rtol=2e-2)
            pk, _, pcu = _packed_with_token(cache, l)
            assert np.array_equal(pcu, orc.cu(l)), (t, l)
            assert torch.equal(pk.cpu(), orc.layer_k[l]), (t, l)
        cache.decode_all_layers_done()
        sync_selection(orc, cache.last_topk)
        orc.decode_all_layers_done()
        np.testing.assert_allclose(cache.score_accumulator.cpu().numpy(), orc.last_scores, atol=1e-4, rtol=1e-3)
        assert cache.last_topk == orc.last_topk, t
        assert [sorted(s) for s in cache.loaded_segments] == [sorted(s) for s in orc.loaded_segments], t
        loads += sum(len(x) for x in orc.last_to_load)
    assert loads > 0


def _config4_scenario(seed=41):
    """BASELINE config 4's per-layer shape, reduced to one layer:
    Voxtral-Small-24B-like heads (8 kv / 32 q, head_dim 128), batch 2 at a
    120k-token context (a 119,900-token audio span), class-B chunks of 128
    tokens offloaded to pinned host memory, top-32; a quarter of the kv heads
    class A (full 120k context, scored), the rest class B at retention 0.05."""
    B, L, H, Hq = 2, 1, 8, 32
    S = 120064
    G = Hq // H
    return dict(seed=seed, L=L, Hkv=H, Hq=Hq, D=128, B=B, steps=3, S=S,
                audio_starts=[4, 4], audio_ends=[S - 160, S - 160], pad=[0, 0],
                chunk_size_s=128.0, overlap_s=0.0, token_rate=1.0,
                class_a=[q for q in range(2 * G)], class_b=list(range(2, H)),
                retention={(0, h): 0.05 for h in range(2, H)},
                top_k=32, lag=1, prefill_mode="last", torch_kv=True)


def test_config4_long_context_layer_matches_oracle(dev):
    """120k-token context through the whole decode path: ~940 chunks per
    sample, top-32 loads per step fetched from pinned host memory, two
    120k-row class-A segments per sample attended and scored."""
    from tests.follow_oracle import FollowOracle, sync_selection
    from tests.golden.scenario import make_cache_inputs, make_config_dict
    from tests.test_gpu_cache import _packed_with_token
    from wnw_b200.cache import B200WnWCache
    from wnw_b200.config import WnWConfig

    sc = _config4_scenario()
    cfg = WnWConfig(**make_config_dict(sc))
    inp = make_cache_inputs(sc)
    L, H, Hq, D, B = sc["L"], sc["Hkv"], sc["Hq"], sc["D"], sc["B"]
    G = Hq // H
    bf = lambda a: torch.from_numpy(a).to(torch.bfloat16)  # noqa: E731
    pk16 = [bf(x) for x in inp.pop("prefill_k")]
    pv16 = [bf(x) for x in inp.pop("prefill_v")]
    cache = B200WnWCache(cfg, L, H, Hq, D, dev, max_decode_tokens=sc["steps"] + 2)
    orc = FollowOracle(cfg, L, H, Hq, D)
    cache.setup_audio(torch.tensor(inp["audio_starts"]), torch.tensor(inp["audio_ends"]),
                      torch.tensor(inp["attention_mask"]))
    orc.setup_audio(inp["audio_starts"], inp["audio_ends"], inp["pad"])
    for l in range(L):
        ca, ph = inp["class_a_scores"][l], inp["per_head_scores"][l]
        cache.prefill_after_attn(l, [x.to(dev) if x is not None else None for x in ca],
                                 [[x.to(dev) if x is not None else None for x in r] for r in ph],
                                 pk16[l].to(dev), pv16[l].to(dev))
        orc.prefill_after_attn(l, ca, ph, pk16[l], pv16[l])
    del pk16, pv16
    cache.prefill_all_layers_done()
    orc.prefill_all_layers_done()
    assert cache._dplan is not None
    assert [sorted(s) for s in cache.loaded_segments] == [sorted(s) for s in orc.loaded_segments]
    loads = 0
    for t in range(sc["steps"]):
        for l in range(L):
            q = bf(inp["dec_q"][t][l])
            k, v = bf(inp["dec_k"][t][l]), bf(inp["dec_v"][t][l])
            kk, vv, cu, _ = cache.decode_before_attn(l, k.to(dev), v.to(dev))
            orc.decode_before_attn(l, k, v)
            qf = q.squeeze(2).reshape(B, H, G, D).reshape(-1, G, D)
            out = cache.fused_decode_attention(l, qf.to(dev), q.to(dev), kk, vv, cu, D ** -0.5)
            orc.fused_decode_attention(l, qf, scale=D ** -0.5)
            np.testing.assert_allclose(out.float().cpu().numpy(), orc.last_out64, atol=2e-2, rtol=2e-2)
            pk, _, pcu = _packed_with_token(cache, l)
            assert np.array_equal(pcu, orc.cu(l)), (t, l)
            assert torch.equal(pk.cpu(), orc.layer_k[l]), (t, l)
        cache.decode_all_layers_done()
        sync_selection(orc, cache.last_topk)
        orc.decode_all_layers_done()
        np.testing.assert_allclose(cache.score_accumulator.cpu().numpy(), orc.last_scores, atol=1e-4, rtol=1e-3)
        assert cache.last_topk == orc.last_topk, t
        assert [sorted(s) for s in cache.loaded_segments] == [sorted(s) for s in orc.loaded_segments], t
        loads += sum(len(x) for x in orc.last_to_load)
    assert loads > 0


def _config1_scenario(seed=0):
    """BASELINE config 1 (the reference's CPU-runnable case): one layer, batch
    4, 8 kv / 32 q heads, head_dim 128, fp32, context lengths U[512, 4096]
    per request (left-padded), layout [4 sink][audio][256 window], chunks of
    64 tokens, top-8, kv heads 0 and 1 class A (all 8 of their q heads), the
    other 6 class B at a small retention (the reference keeps >= 1 audio row
    per segment)."""
    rng = np.random.default_rng(seed)
    B, L, H, Hq = 4, 1, 8, 32
    lens = rng.integers(512, 4097, B)
    S = int(lens.max())
    pad = [int(S - n) for n in lens]
    G = Hq // H
    return dict(seed=seed, L=L, Hkv=H, Hq=Hq, D=128, B=B, steps=4, S=S,
                audio_starts=[p + 4 for p in pad], audio_ends=[S - 256] * B, pad=pad,
                chunk_size_s=64.0, overlap_s=0.0, token_rate=1.0,
                class_a=list(range(2 * G)), class_b=list(range(2, H)),
                retention={(0, h): 0.02 for h in range(2, H)},
                top_k=8, lag=1, prefill_mode="last")


def test_config1_matches_oracle_fp32(dev):
    """fp32 at config 1's shape: attention and class-A scores within 1e-5 of
    the oracle, layouts bit for bit, loaded sets exactly."""
    from tests.follow_oracle import FollowOracle, sync_selection
    from tests.golden.scenario import make_cache_inputs, make_config_dict
    from tests.test_gpu_cache import _packed_with_token
    from wnw_b200.cache import B200WnWCache
    from wnw_b200.config import WnWConfig

    sc = _config1_scenario()
    cfg = WnWConfig(**make_config_dict(sc))
    inp = make_cache_inputs(sc)
    L, H, Hq, D, B = sc["L"], sc["Hkv"], sc["Hq"], sc["D"], sc["B"]
    G = Hq // H
    t32 = torch.from_numpy
    cache = B200WnWCache(cfg, L, H, Hq, D, dev, max_decode_tokens=sc["steps"] + 2)
    orc = FollowOracle(cfg, L, H, Hq, D)
    cache.setup_audio(torch.tensor(inp["audio_starts"]), torch.tensor(inp["audio_ends"]),
                      torch.tensor(inp["attention_mask"]))
    orc.setup_audio(inp["audio_starts"], inp["audio_ends"], inp["pad"])
    ca, ph = inp["class_a_scores"][0], inp["per_head_scores"][0]
    k, v = t32(inp["prefill_k"][0]), t32(inp["prefill_v"][0])
    cache.prefill_after_attn(0, [x.to(dev) if x is not None else None for x in ca],
                             [[x.to(dev) if x is not None else None for x in r] for r in ph], k.to(dev), v.to(dev))
    orc.prefill_after_attn(0, ca, ph, k, v)
    cache.prefill_all_layers_done()
    orc.prefill_all_layers_done()
    assert [sorted(s) for s in cache.loaded_segments] == [sorted(s) for s in orc.loaded_segments]
    loads = 0
    for t in range(sc["steps"]):
        q = t32(inp["dec_q"][t][0])
        k, v = t32(inp["dec_k"][t][0]), t32(inp["dec_v"][t][0])
        kk, vv, cu, _ = cache.decode_before_attn(0, k.to(dev), v.to(dev))
        orc.decode_before_attn(0, k, v)
        qf = q.squeeze(2).reshape(B, H, G, D).reshape(-1, G, D)
        out = cache.fused_decode_attention(0, qf.to(dev), q.to(dev), kk, vv, cu, D ** -0.5)
        orc.fused_decode_attention(0, qf, scale=D ** -0.5)
        np.testing.assert_allclose(out.cpu().numpy(), orc.last_out64, atol=1e-5, rtol=1e-5)
        pk, _, pcu = _packed_with_token(cache, 0)
        assert np.array_equal(pcu, orc.cu(0)), t
        assert torch.equal(pk.cpu(), orc.layer_k[0]), t
        cache.decode_all_layers_done()
        sync_selection(orc, cache.last_topk)
        orc.decode_all_layers_done()
        np.testing.assert_allclose(cache.score_accumulator.cpu().numpy(), orc.last_scores, atol=1e-5, rtol=1e-4)
        assert cache.last_topk == orc.last_topk, t
        assert [sorted(s) for s in cache.loaded_segments] == [sorted(s) for s in orc.loaded_segments], t
        loads += sum(len(x) for x in orc.last_to_load)
    assert loads > 0


def _stream_full_shape(dev, sc, steps, max_follow=1):
    """Prefill and ``steps`` decode steps of scenario ``sc`` through
    ``B200WnWCache`` and the oracle side by side, with the inputs drawn one
    layer at a time (torch generator, bf16) and freed after use, so that the
    full-size prompt never sits in host memory as a whole.  Checks per layer
    and step: packed K layout and cu_seqlens bit for bit, attention within
    bf16 tolerance; per step: class-A scores, top-k and loaded sets.  At most
    ``max_follow`` steps may follow the GPU's selection on a near tie."""
    from tests.follow_oracle import FollowOracle, sync_selection
    from tests.golden.scenario import make_config_dict
    from tests.test_gpu_cache import _packed_with_token
    from wnw_b200.cache import B200WnWCache
    from wnw_b200.config import WnWConfig

    cfg = WnWConfig(**make_config_dict(sc))
    L, H, Hq, D, B, S = sc["L"], sc["Hkv"], sc["Hq"], sc["D"], sc["B"], sc["S"]
    G = Hq // H
    g = torch.Generator().manual_seed(sc["seed"])
    mask = torch.ones(B, S, dtype=torch.int64)
    for b in range(B):
        mask[b, :sc["pad"][b]] = 0
    n_audio = [e - s for s, e in zip(sc["audio_starts"], sc["audio_ends"])]

    def distinct(n):
        # prefill scores without exact ties: which of two equal scores the
        # reference keeps is unspecified (torch.topk), so tied inputs would
        # make the expected layout ambiguous (uniform floats on a 2^-24 grid
        # tie often at this size)
        return torch.randperm(n, generator=g).to(torch.float32) / n

    cache = B200WnWCache(cfg, L, H, Hq, D, dev, max_decode_tokens=steps + 2)
    orc = FollowOracle(cfg, L, H, Hq, D)
    cache.setup_audio(torch.tensor(sc["audio_starts"]), torch.tensor(sc["audio_ends"]), mask)
    orc.setup_audio(sc["audio_starts"], sc["audio_ends"], sc["pad"])
    for l in range(L):
        k = torch.randn(B, H, S, D, generator=g).to(torch.bfloat16)
        v = torch.randn(B, H, S, D, generator=g).to(torch.bfloat16)
        ca_kv = bool(cfg.get_layer_class_a(l))
        ca = [distinct(n_audio[b]) if ca_kv else None for b in range(B)]
        ph = [[None if cfg.is_class_a_kv_head(l, h) else distinct(n_audio[b]) for h in range(H)] for b in range(B)]
        cache.prefill_after_attn(l, [x.to(dev) if x is not None else None for x in ca],
                                 [[x.to(dev) if x is not None else None for x in r] for r in ph], k.to(dev), v.to(dev))
        orc.prefill_after_attn(l, ca, ph, k, v)
        del k, v
    cache.prefill_all_layers_done()
    orc.prefill_all_layers_done()
    assert cache._dplan is not None
    assert [sorted(s) for s in cache.loaded_segments] == [sorted(s) for s in orc.loaded_segments]
    loads = follows = 0
    for t in range(steps):
        for l in range(L):
            q = torch.randn(B, Hq, 1, D, generator=g).to(torch.bfloat16)
            k = torch.randn(B, H, 1, D, generator=g).to(torch.bfloat16)
            v = torch.randn(B, H, 1, D, generator=g).to(torch.bfloat16)
            kk, vv, cu, _ = cache.decode_before_attn(l, k.to(dev), v.to(dev))
            orc.decode_before_attn(l, k, v)
            qf = q.squeeze(2).reshape(B, H, G, D).reshape(-1, G, D)
            out = cache.fused_decode_attention(l, qf.to(dev), q.to(dev), kk, vv, cu, D ** -0.5)
            orc.fused_decode_attention(l, qf, scale=D ** -0.5)
            np.testing.assert_allclose(out.float().cpu().numpy(), orc.last_out64, atol=2e-2, rtol=2e-2)
            pk, _, pcu = _packed_with_token(cache, l)
            assert np.array_equal(pcu, orc.cu(l)), (t, l)
            assert torch.equal(pk.cpu(), orc.layer_k[l]), (t, l)
        cache.decode_all_layers_done()
        follows += bool(sync_selection(orc, cache.last_topk))
        orc.decode_all_layers_done()
        np.testing.assert_allclose(cache.score_accumulator.cpu().numpy(), orc.last_scores, atol=1e-4, rtol=1e-3)
        assert cache.last_topk == orc.last_topk, t
        assert [sorted(s) for s in cache.loaded_segments] == [sorted(s) for s in orc.loaded_segments], t
        loads += sum(len(x) for x in orc.last_to_load)
    assert loads > 0
    assert follows <= max_follow


def test_config3_full_shape_matches_oracle(dev):
    """BASELINE config 3 at its shape: 28 layers, Qwen2.5-Omni-7B heads (4 kv
    / 28 q, GQA 7, head_dim 128), batch 32 with seeded lognormal prompt
    lengths (median 6k, sigma 0.5, clipped to [1k, 30k]) left-padded to the
    longest, 50 % class-A kv heads, class-B retention 0.25, chunks of 128
    tokens, top-8, lag 1; two decode steps."""
    rng = np.random.default_rng(33)
    B, L, H, Hq = 32, 28, 4, 28
    lens = np.clip(np.round(np.exp(rng.normal(np.log(6000), 0.5, B))), 1000, 30000).astype(int)
    S = int(lens.max())
    pad = [int(S - n) for n in lens]
    G = Hq // H
    sc = dict(seed=33, L=L, Hkv=H, Hq=Hq, D=128, B=B, S=S, pad=pad,
              audio_starts=[p + 4 for p in pad], audio_ends=[S - 30] * B,
              chunk_size_s=128.0, overlap_s=0.0, token_rate=1.0,
              class_a=[l * Hq + q for l in range(L) for q in range(2 * G)],
              class_b=[l * H + h for l in range(L) for h in (2, 3)],
              retention={(l, h): 0.25 for l in range(L) for h in (2, 3)},
              top_k=8, lag=1, prefill_mode="last")
    _stream_full_shape(dev, sc, steps=2)


def test_config4_full_depth_matches_oracle(dev):
    """BASELINE config 4 at its depth: 40 layers of Voxtral-Small-24B heads
    (8 kv / 32 q, head_dim 128), batch 2 at a 120,064-token context, class-B
    chunks of 128 tokens offloaded to pinned host memory, top-32; a quarter
    of the kv heads class A (full context, scored), the rest at retention
    0.05; two decode steps."""
    B, L, H, Hq = 2, 40, 8, 32
    S = 120064
    G = Hq // H
    sc = dict(seed=44, L=L, Hkv=H, Hq=Hq, D=128, B=B, S=S, pad=[0, 0],
              audio_starts=[4, 4], audio_ends=[S - 160, S - 160],
              chunk_size_s=128.0, overlap_s=0.0, token_rate=1.0,
              class_a=[l * Hq + q for l in range(L) for q in range(2 * G)],
              class_b=[l * H + h for l in range(L) for h in range(2, H)],
              retention={(l, h): 0.05 for l in range(L) for h in range(2, H)},
              top_k=32, lag=1, prefill_mode="last")
    _stream_full_shape(dev, sc, steps=2)
