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
