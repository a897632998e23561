"""Prefill audio scores (``wnw_prefill_scores``) against the torch restatement
of the reference session's ``_compute_prefill_scores`` / ``_compute_head_scores``
(src/algorithms/wnw/code/session.py:121-201, ``oracle.prefill_scores``).

CPU: the session's task list (``wnw_b200.session.compute_prefill_scores``)
is executed task by task in torch and must equal the oracle bit for bit --
this pins what each task means (query heads, positions, kv head, audio
columns, mask) without a GPU.  GPU: the kernel against the oracle run on the
same GPU tensors, in both score modes, with causal, boolean and additive
masks, left-padded batches, GQA groups 4 and 8, head_dim 16 to 128, fp32,
bf16 and fp16, row counts above one shared-memory block; results repeat bit
for bit,
and a task with an out-of-range index raises instead of writing.
"""
import numpy as np
import pytest
import torch

from oracle.prefill_scores import compute_prefill_scores as oracle_scores
from wnw_b200 import native as N


class _Cfg:
    def __init__(self, class_a, Hq, G, mode):
        self.class_a, self.G, self.prefill_score_mode = class_a, G, mode

    def get_layer_class_a(self, layer_idx):
        return list(self.class_a)

    def is_class_a_kv_head(self, layer_idx, h):
        return any(q // self.G == h for q in self.class_a)


class _Cache:
    def __init__(self, cfg, a0, a1):
        self.config, self._raw_audio_starts, self._raw_audio_ends = cfg, a0, a1


def _task_scorer(q, k, tasks, heads, scaling, out_len, mask_kind, mask=None):
    """Each task in torch, as the header defines it."""
    out = torch.zeros(out_len, dtype=torch.float32, device=q.device)
    S = q.shape[2]
    for (b, kv, h0, nh, r0, nr, a0, a1, off) in tasks:
        hs = heads[h0:h0 + nh]
        s = torch.matmul(q[b, hs, r0:r0 + nr, :], k[b, kv:kv + 1].transpose(-1, -2)) * scaling
        if mask_kind == N.MASK_CAUSAL:
            pos = torch.arange(r0, r0 + nr, device=q.device)
            m = torch.zeros(nr, S, dtype=q.dtype, device=q.device)
            m.masked_fill_(torch.arange(S, device=q.device)[None, :] > pos[:, None], float("-inf"))
            s = s + m
        elif mask_kind == N.MASK_ADDITIVE:
            s = s + mask[b, r0:r0 + nr, :]
        p = s.float().softmax(dim=-1)[:, :, a0:a1]
        out[off:off + a1 - a0] = p.mean(dim=1).sum(dim=0) if nr > 1 else p[:, 0].sum(dim=0)
    return out


def _case(dev, dtype, B=2, Hkv=4, G=4, S=1500, D=128, class_a=(1, 2, 5), a0=(4, 30), a1=(1400, 1440),
          mask="none", seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = (torch.randn(B, S, Hkv * G, D, generator=g) * 0.5).to(dtype).to(dev).transpose(1, 2)  # model layout
    k = (torch.randn(B, S, Hkv, D, generator=g) * 0.5).to(dtype).to(dev).transpose(1, 2)
    pad = [0] + [int(a) for a in np.asarray(a0[1:]) - a0[0]]
    am = None
    if mask != "none":
        keep = torch.ones(B, 1, S, S, dtype=torch.bool).tril_()
        for b in range(B):
            keep[b, :, :, :pad[b]] = False
            keep[b, :, :pad[b], :] = torch.eye(S, dtype=torch.bool)[:pad[b]]  # padded queries see themselves
        am = keep.to(dev) if mask == "bool" else \
            torch.where(keep, 0.0, torch.finfo(dtype).min).to(dtype).to(dev)
        if mask == "2d":
            am = torch.ones(B, S, dtype=torch.long, device=dev)
    return q, k, am, list(class_a), list(a0), list(a1)


CASES = [
    dict(mode="last"), dict(mode="mean_text"), dict(mode="last", class_a=()),
    dict(mode="mean_text", mask="bool"), dict(mode="last", mask="additive"), dict(mode="mean_text", mask="2d"),
    dict(mode="mean_text", G=8, Hkv=2, class_a=(0, 3), a1=(1400, 1440)),  # 8 x 100 rows: several row blocks
    dict(mode="mean_text", a1=(1500, 1460)),  # sample 0 has no text after the audio
    dict(mode="last", D=64, S=2100, a1=(2050, 2090)),
]


def _run(fn, dev, dtype, p, **kw):
    q, k, am, ca, a0, a1 = _case(dev, dtype, **{x: v for x, v in p.items() if x != "mode"})
    G = p.get("G", 4)
    Hkv = p.get("Hkv", 4)
    cache = _Cache(_Cfg(ca, Hkv * G, G, p["mode"]), a0, a1)
    return fn(q, k, am, cache, 0, q.shape[0], q.shape[2], Hkv, G, q.shape[3] ** -0.5, **kw)


def _flat(res):
    ca, ph = res
    return [x for x in ca] + [x for row in ph for x in row]


@pytest.mark.parametrize("p", CASES)
def test_session_tasks_equal_oracle_cpu(p):
    from wnw_b200.session import compute_prefill_scores
    got = _flat(_run(compute_prefill_scores, "cpu", torch.bfloat16, p, scorer=_task_scorer))
    want = _flat(_run(oracle_scores, "cpu", torch.bfloat16, p))
    assert len(got) == len(want)
    for x, y in zip(got, want):
        assert (x is None) == (y is None)
        if x is not None:
            assert torch.equal(x, y)


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda:0")


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("p", CASES)
def test_prefill_scores_kernel_matches_oracle(dev, dtype, p):
    """Logits are rounded to the model dtype from an fp32 dot product whose
    summation order differs from cuBLAS's; a dot product within ~1e-7 of a
    rounding boundary can round one ulp the other way, so a few scores move
    by up to ~1 % of their value and the rest agree to fp32 summation
    order."""
    from wnw_b200.kernels import PrefillScorer
    from wnw_b200.session import compute_prefill_scores
    scorer = PrefillScorer(dev)
    got = _flat(_run(compute_prefill_scores, dev, dtype, p, scorer=scorer))
    again = _flat(_run(compute_prefill_scores, dev, dtype, p, scorer=scorer))
    want = _flat(_run(oracle_scores, dev, dtype, p))
    scorer.check()
    for x, x2, y in zip(got, again, want):
        assert (x is None) == (y is None)
        if x is None:
            continue
        assert bool(torch.isfinite(x).all())
        assert torch.equal(x, x2)  # fixed summation order
        y = y.float()
        assert x.shape == y.shape
        if x.numel() == 0:
            continue
        rel = (x - y).abs() / y.abs().clamp_min(1e-30)
        assert float(rel.max()) < 2e-2, float(rel.max())
        assert float((rel < 1e-4).float().mean()) > 0.99
        torch.testing.assert_close(x.sum(), y.sum(), rtol=1e-4, atol=1e-6)


CC_CASES = [(torch.float32, dict(mode="last", D=16)), (torch.float32, dict(mode="mean_text", D=16, mask="bool")),
            (torch.float32, dict(mode="mean_text", D=64)), (torch.float32, dict(mode="last", D=128, mask="additive")),
            (torch.bfloat16, dict(mode="mean_text", D=32)), (torch.float16, dict(mode="last", D=16, class_a=()))]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,p", CC_CASES)
def test_prefill_scores_cuda_core_path(dev, dtype, p):
    """fp32 q / k (the tiny session models) and 16-bit ones with head_dim
    16 / 32 take the CUDA-core kernels: fp32 logits agree with the oracle to
    summation order; 16-bit ones as on the tensor-core path."""
    from wnw_b200.kernels import PrefillScorer
    from wnw_b200.session import compute_prefill_scores
    scorer = PrefillScorer(dev)
    got = _flat(_run(compute_prefill_scores, dev, dtype, p, scorer=scorer))
    again = _flat(_run(compute_prefill_scores, dev, dtype, p, scorer=scorer))
    want = _flat(_run(oracle_scores, dev, dtype, p))
    scorer.check()
    for x, x2, y in zip(got, again, want):
        assert (x is None) == (y is None)
        if x is None or x.numel() == 0:
            continue
        assert bool(torch.isfinite(x).all())
        assert torch.equal(x, x2)
        rel = (x - y.float()).abs() / y.float().abs().clamp_min(1e-30)
        if dtype == torch.float32:
            assert float(rel.max()) < 1e-4, float(rel.max())
        else:
            assert float(rel.max()) < 2e-2 and float((rel < 1e-4).float().mean()) > 0.99


@pytest.mark.gpu
def test_prefill_scores_full_shape(dev):
    """Config 2's prefill layer: 15,064 tokens, 15,000 audio, 8 kv x 32 q
    heads, two class-A kv heads; the reference's default mean-over-text
    mode (60 text queries after the audio) and the last-query mode."""
    from wnw_b200.kernels import PrefillScorer
    from wnw_b200.session import compute_prefill_scores
    scorer = PrefillScorer(dev)
    for mode in ("mean_text", "last"):
        p = dict(mode=mode, B=1, Hkv=8, G=4, S=15064, class_a=tuple(range(8, 16)), a0=(4,), a1=(15004,))
        got = _flat(_run(compute_prefill_scores, dev, torch.bfloat16, p, scorer=scorer))
        want = _flat(_run(oracle_scores, dev, torch.bfloat16, p))
        for x, y in zip(got, want):
            if x is None:
                continue
            rel = (x - y.float()).abs() / y.float().abs().clamp_min(1e-30)
            assert float(rel.max()) < 2e-2 and float((rel < 1e-4).float().mean()) > 0.99
            # the rows the prefill keeps: the top-scoring audio rows agree
            n = x.numel() // 10
            top_x, top_y = set(torch.topk(x, n).indices.tolist()), set(torch.topk(y.float(), n).indices.tolist())
            assert len(top_x & top_y) >= n - 2
    scorer.check()


@pytest.mark.gpu
def test_prefill_scores_bad_task_raises(dev):
    from wnw_b200.kernels import PrefillScorer
    scorer = PrefillScorer(dev)
    q = torch.randn(1, 4, 64, 128, device=dev, dtype=torch.bfloat16)
    k = torch.randn(1, 2, 64, 128, device=dev, dtype=torch.bfloat16)
    out = scorer(q, k, [(0, 2, 0, 2, 63, 1, 4, 60, 0)], [0, 1], 0.1, 56, N.MASK_CAUSAL)  # kv head 2 of 2
    with pytest.raises(N.WnwError, match="prefill score task"):
        scorer.check()
    assert float(out.abs().sum()) == 0.0
