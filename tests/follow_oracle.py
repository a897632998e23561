"""Near-tie resynchronisation for GPU-vs-oracle trajectory tests.

Chunk scores are means of sums over many layer x head terms; the GPU adds them
in a different order than the oracle, so two chunks whose scores sit within
fp32 rounding of each other may be ranked differently.  When that happens the
two runs would load different chunks from then on and every later comparison
would be meaningless.  ``FollowOracle`` lets a test make the oracle take the
GPU's selection for such a step, and ``sync_selection`` decides when that is
allowed: only when the oracle's own k-th / (k+1)-th chunk-score gap is below
``rel`` times the largest chunk score.  A wider disagreement is a failure.
"""
import numpy as np

from oracle import kernels as K
from oracle.cache import OracleWnWCache


class FollowOracle(OracleWnWCache):
    """Oracle whose top-k for sample b is ``follow[b]`` when that is set."""

    def __init__(self, *a, **kw):
        super().__init__(*a, **kw)
        self.follow = {}

    def _select(self, b, cs, k):
        if b in self.follow:
            return list(self.follow[b])
        return super()._select(b, cs, k)


def sync_selection(orc, gpu_topk, rel=1e-5):
    """Call after the GPU cache's ``decode_all_layers_done`` and before the
    oracle's.  Returns how many samples had to follow the GPU on a near tie;
    raises AssertionError on a disagreement that is not a near tie."""
    orc.follow = {}
    n = 0
    for b, bounds in enumerate(orc.chunk_bounds):
        if not bounds:
            continue
        o0, o1 = orc.score_offsets[b], orc.score_offsets[b + 1]
        cs = K.chunk_scores(orc.score_accumulator[o0:o1], [x for x, _ in bounds], [y for _, y in bounds])
        k = min(orc.config.top_k_chunks, len(cs))
        if sorted(K.topk_lower_index(cs, k)) == list(gpu_topk[b]):
            continue
        gap, tie = K.topk_gap(cs, k), rel * float(np.abs(cs).max())
        assert gap < tie, f"sample {b}: selections differ beyond a near tie (gap {gap:.3g}, bound {tie:.3g})"
        orc.follow[b] = list(gpu_topk[b])
        n += 1
    return n
