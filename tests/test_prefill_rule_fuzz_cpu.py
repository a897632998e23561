"""The prefill keep rule of the B200 cache (wnw_b200.cache.keep_audio_indices:
every head of a retention group in one batched top-k; offload_counts: rows
offloaded per segment) against the oracle's per-head restatement of the
reference (cache.py:1114-1150) on seeded random spans: audio lengths 0-700
(a short last segment or none), strides 1-128, retention 0-1, one to four
heads, per-segment and global rules.  Scores are distinct, so no tie order
is involved (tie order is not pinned across devices)."""
import numpy as np
import pytest
import torch

from oracle.cache import compute_segments, select_topk_global, select_topk_per_segment
from wnw_b200.cache import keep_audio_indices, offload_counts


@pytest.mark.parametrize("seed", range(60))
def test_keep_rule_matches_oracle(seed):
    rng = np.random.default_rng(500 + seed)
    n = int(rng.integers(0, 701))
    stride = int(rng.choice([1, 2, 7, 16, 64, 128]))
    ratio = float(rng.choice([0.0, 0.01, 0.1, 0.25, 0.5, 0.99, 1.0]))
    nh = int(rng.integers(1, 5))
    glob = bool(seed % 2)
    segs = compute_segments(n, stride)
    scores = torch.from_numpy(rng.permutation(nh * max(n, 1))[:nh * n].reshape(nh, n).astype(np.float32))
    kept = keep_audio_indices(scores, segs, ratio, glob)
    assert kept.shape[0] == nh
    counts, total = offload_counts(segs, ratio, glob)
    for h in range(nh):
        want = (select_topk_global if glob else select_topk_per_segment)(scores[h], segs, ratio)
        got = torch.zeros(n, dtype=torch.bool)
        got[kept[h]] = True
        assert torch.equal(got, want), (h, n, stride, ratio, glob)
        assert torch.equal(kept[h], kept[h].sort().values)  # ascending, as the layout needs
        assert total == n - int(want.sum())
        if counts is not None:
            assert counts == [(e - s) - int(want[s:e].sum()) for s, e in segs]
