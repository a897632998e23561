"""Randomised planner states and top-k sequences (seeded): the native planner
(wnw_b200.planner.Planner), the reference's own planner compiled from its
source into oracle/_ref (skipped when that build is absent), the oracle
planner and the device fetch plan rule (oracle.planner.device_fetch_plan)
agree on every output of every step: change flag, transfer total, the seven
plan arrays, evictions, host ranges, loaded sets, per-layer landing offsets.
"""
import copy

import numpy as np
import pytest
import torch

from oracle.planner import OraclePlanner, device_fetch_plan
from tests.golden.scenario import make_planner_inputs
from tests.test_oracle_golden import _planner_from


def _scenario(seed):
    rng = np.random.default_rng(1000 + seed)
    B = int(rng.integers(1, 4))
    return dict(seed=2000 + seed, L=int(rng.integers(1, 5)), H=int(rng.integers(1, 5)), B=B,
                seg_count=[int(rng.integers(1, 25)) for _ in range(B)], spc=int(rng.integers(1, 4)),
                top_k=int(rng.integers(1, 9)), lag=int(rng.integers(0, 4)), steps=int(rng.integers(3, 10)))


def _reference_planner():
    from oracle.build_ref import load_prebuilt
    try:
        return load_prebuilt()
    except Exception:  # a stale or foreign build: treat as absent
        return None


@pytest.mark.parametrize("seed", range(40))
def test_planners_agree_on_random_states(seed):
    from wnw_b200.planner import Planner
    ps = _scenario(seed)
    inp = make_planner_inputs(ps)
    L, S = ps["L"], ps["B"] * ps["H"]
    shapes = [(L, S), (L, S), (L, S + 1), (L, S), (L, S + 1), (L,), (L + 1,)]
    ours, orc = _planner_from(ps, inp, Planner), _planner_from(ps, inp, OraclePlanner)
    dev_rule = copy.deepcopy(orc)
    ref_mod = _reference_planner()
    ref = None
    if ref_mod is not None:
        i32 = lambda x: torch.tensor(x, dtype=torch.int32)  # noqa: E731
        ref = ref_mod.Planner(L, ps["H"], ps["B"], 1)
        ref.set_config(ps["top_k"], ps["lag"])
        ref.set_seg_count(list(inp["seg_count"]))
        for b in range(ps["B"]):
            ref.set_chunk_to_segs(b, i32(inp["c2s_flat"][b]), i32(inp["c2s_off"][b]))
        for l in range(L):
            ref.set_class_b(l, i32(inp["class_b"][l]))
        ref.set_restore_meta(i32(inp["cpu_s"]), i32(inp["cpu_e"]), i32(inp["gpu_s"]), i32(inp["gpu_e"]))
        for b in range(ps["B"]):
            ref.set_loaded(b, i32(inp["loaded"][b]))
        ref.set_seq_lens(i32(inp["seq_lens"]))
    for tk, toff in inp["steps"]:
        a = [np.full(s, -7, np.int32) for s in shapes]
        ch, tot, evs, eve, rng = ours.compute_and_prepare(tk, toff, *a)
        o = orc.compute_and_prepare(tk, toff)
        d = device_fetch_plan(dev_rule, [tk[toff[b]:toff[b + 1]] for b in range(ps["B"])])
        assert ch == o["any_change"] and tot == o["total"]
        if ch:
            for name, buf in zip(("load_starts", "load_lens", "cu_new", "new_lens", "evict_offsets", "evict_max",
                                  "evict_layer_ptr"), a):
                assert np.array_equal(buf, o[name]), name
        assert np.array_equal(evs, o["ev_starts"]) and np.array_equal(eve, o["ev_ends"])
        assert np.array_equal(rng.reshape(-1, 2), o["cpu_ranges"].reshape(-1, 2))
        assert [ours.get_loaded_segments(b) for b in range(ps["B"])] == \
            [orc.get_loaded_segments(b) for b in range(ps["B"])]
        assert np.array_equal(np.asarray(d["ranges"], np.int32).reshape(-1, 2), rng.reshape(-1, 2))
        lrows, lranges = ours.layer_transfer()
        assert list(lrows) == d["layer_rows"] and list(lranges) == d["layer_ranges"]
        assert dev_rule.counters == orc.counters
        if ref is not None:
            t = [torch.full(s, -7, dtype=torch.int32) for s in shapes]
            rch, rtot, revs, reve, rrng = ref.compute_and_prepare(torch.tensor(tk, dtype=torch.int32),
                                                                  torch.tensor(toff, dtype=torch.int32), *t)
            assert (int(rch), int(rtot)) == (ch, tot)
            if ch:
                for x, y in zip(t, a):
                    assert np.array_equal(x.numpy(), y)
            assert np.array_equal(revs.numpy(), evs) and np.array_equal(reve.numpy(), eve)
            assert np.array_equal(rrng.numpy().reshape(-1, 2), rng.reshape(-1, 2))
            assert [sorted(ref.get_loaded_segments(b)) for b in range(ps["B"])] == \
                [ours.get_loaded_segments(b) for b in range(ps["B"])]
