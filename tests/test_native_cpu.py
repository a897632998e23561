"""CPU checks of libwnw_b200.so: it loads, exports every declared symbol, and
its host-side planner / gather match the oracle and the reference planner's
recorded outputs bit for bit (no GPU compute here)."""
import ctypes
import os
import re

import numpy as np
import pytest

from oracle import kernels as K
from oracle.planner import OraclePlanner
from tests.golden.scenario import PLANNER_SCENARIOS, make_planner_inputs
from tests.test_oracle_golden import _planner_from

N = pytest.importorskip("wnw_b200.native")


def test_library_exports_every_header_symbol():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    hdr = open(os.path.join(root, "include", "wnw_b200.h")).read()
    declared = set(re.findall(r"\b(wnw_[a-z0-9_]+)\s*\(", hdr)) - {"wnw_status", "wnw_dtype"}
    for name in declared:
        assert hasattr(N.lib, name), name
    assert declared == set(N.EXPORTS)
    assert N.lib.wnw_abi_version() == 1
    assert N.lib.wnw_split_rows(N.BF16, 128) == 0 and N.lib.wnw_split_rows(N.F32, 128) == 64


def test_ctypes_structs_match_the_header(tmp_path):
    """Every argument struct the ctypes binding declares has the C layout:
    size and each field's offset, from a program compiled against the
    header."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    structs = {"wnw_decode_attn_args": N.DecodeAttnArgs, "wnw_attn_plan_info": N.AttnPlanInfo,
               "wnw_oproj_allreduce_args": N.OprojAllReduceArgs, "wnw_fetch_info": N.FetchInfo,
               "wnw_prefill_task": N.PrefillTask, "wnw_prefill_scores_args": N.PrefillScoresArgs}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "wnw_b200.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'  printf("{cname} %zu\\n", sizeof({cname}));')
        for f, _ in py._fields_:
            lines.append(f'  printf("{cname}.{f} %zu\\n", offsetof({cname}, {f}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", os.path.join(root, "include"), str(src), "-o", str(exe)], check=True)
    got = dict(line.rsplit(" ", 1) for line in subprocess.run([str(exe)], check=True, capture_output=True,
                                                                 text=True).stdout.splitlines())
    for cname, py in structs.items():
        assert int(got[cname]) == ctypes.sizeof(py), cname
        for f, _ in py._fields_:
            assert int(got[f"{cname}.{f}"]) == getattr(py, f).offset, f"{cname}.{f}"


def test_status_and_error_reporting():
    from wnw_b200.planner import Planner
    assert N.lib.wnw_status_string(3) == b"capacity exceeded"
    with pytest.raises(N.WnwError, match="dimensions must be positive"):
        Planner(0, 1, 1)
    p = Planner(2, 2, 1)
    with pytest.raises(N.WnwError, match="set_seg_count must come first"):
        p.set_loaded(0, [1])
    with pytest.raises(N.WnwError, match="seg_count must have batch_size entries"):
        p.set_seg_count([3, 4])


@pytest.mark.parametrize("i", range(len(PLANNER_SCENARIOS)))
def test_native_planner_matches_reference_planner(golden_dir, i):
    from wnw_b200.planner import Planner
    pz = np.load(os.path.join(golden_dir, "planner.npz"), allow_pickle=True)
    ps = PLANNER_SCENARIOS[i]
    inp = make_planner_inputs(ps)
    P = _planner_from(ps, inp, Planner)
    O = _planner_from(ps, inp, OraclePlanner)
    L, S = ps["L"], ps["B"] * ps["H"]
    for step, (tk, toff) in enumerate(inp["steps"]):
        bufs = [np.full((L, S), -7, np.int32), np.full((L, S), -7, np.int32), np.full((L, S + 1), -7, np.int32),
                np.full((L, S), -7, np.int32), np.full((L, S + 1), -7, np.int32), np.full(L, -7, np.int32),
                np.full(L + 1, -7, np.int32)]
        ch, tot, evs, eve, rng = P.compute_and_prepare(tk, toff, *bufs)
        r = O.compute_and_prepare(tk, toff)
        pre = f"p{i}_s{step}_"
        assert ch == int(pz[pre + "change"]) == r["any_change"]
        assert tot == int(pz[pre + "total"])
        if ch:
            for name, buf in zip(("load_starts", "load_lens", "cu_new", "new_lens", "evict_offsets", "evict_max",
                                  "evict_layer_ptr"), bufs):
                assert np.array_equal(buf, pz[pre + name]), name
        assert np.array_equal(evs, pz[pre + "ev_starts"]) and np.array_equal(eve, pz[pre + "ev_ends"])
        assert np.array_equal(rng.reshape(-1, 2), pz[pre + "cpu_ranges"].reshape(-1, 2))
        for b in range(ps["B"]):
            assert P.get_loaded_segments(b) == list(pz[pre + "loaded"][b])
            assert P.changes(b) == (r["to_load"][b], r["to_evict"][b])
        if ch:
            _check_device_plan(P, bufs, evs, eve, L, S)


def _check_device_plan(P, bufs, evs, eve, L, S):
    """The rebuild blob restates the reference outputs per changed segment."""
    from wnw_b200.kernels import plan_record
    blob = P.device_plan()
    ls, ll, _, nl, eo, _, elp = bufs
    for l in range(L):
        r = plan_record(blob, l)
        for i, fi in enumerate(r["seg"]):
            assert r["new_len"][i] == nl[l, fi] - 1
            assert r["load_len"][i] == ll[l, fi]
            if r["load_len"][i]:
                assert r["load_src"][i] == ls[l, fi]
            r0, r1 = elp[l] + eo[l, fi], elp[l] + eo[l, fi + 1]
            e0, e1 = r["ev_off"][i], r["ev_off"][i + 1]
            assert list(r["ev_s"][e0:e1]) == list(evs[r0:r1])
            assert list(r["ev_e"][e0:e1]) == list(eve[r0:r1])
            kept = r["new_len"][i] - r["load_len"][i]
            moved = kept - r["ev_s"][e0] if e1 > e0 else 0
            assert r["mov_off"][i + 1] - r["mov_off"][i] == moved
            assert r["out_off"][i + 1] - r["out_off"][i] == moved + r["load_len"][i]
        assert r["moved_total"] == r["mov_off"][-1] and r["out_total"] == r["out_off"][-1]


@pytest.mark.parametrize("threads", [1, 4, 16])
def test_gather_rows_matches_oracle(threads):
    """The host gather of the pinned-copy fetch mode (any thread count, empty
    ranges included) copies the planned ranges in order, like the oracle."""
    from wnw_b200.planner import gather_rows
    rng = np.random.default_rng(threads)
    for rows, n_ranges, dtype in ((500, 40, np.float32), (70000, 300, np.float16)):
        ck = rng.standard_normal((rows, 64)).astype(dtype)
        cv = rng.standard_normal((rows, 64)).astype(dtype)
        starts = rng.integers(0, rows - 60, n_ranges)
        ranges = np.stack([starts, starts + rng.integers(0, 60, n_ranges)], 1).astype(np.int32)
        ek, ev = K.gather_restore(ck, cv, ranges)
        dk = np.zeros_like(ek)
        dv = np.zeros_like(ev)
        gather_rows(ck, cv, ranges, dk, dv, n_threads=threads)
        assert np.array_equal(dk, ek) and np.array_equal(dv, ev)


def test_work_table_covers_capacity():
    from wnw_b200.kernels import build_work_table
    cap = np.array([0, 127, 128, 1000, 5000], np.int32)
    w = build_work_table(cap, 128, 4)
    for s, c in enumerate(cap):
        nsplit = -(-(int(c) + 1) // 128)
        ncl = max(1, -(-nsplit // 4))
        assert sorted(j for seg, j in w.tolist() if seg == s) == list(range(ncl))
    n = ctypes.c_int()
    out = np.zeros((2, 2), np.int32)
    st = N.lib.wnw_build_work_table(N.ptr(cap), cap.size, 128, 4, N.ptr(out), 2, ctypes.byref(n))
    assert st == 3 and n.value == w.shape[0]


def test_launch_shape_cuda_core_kernel():
    """fp32 keeps the CUDA-core kernel's fixed split; clusters grow to 8 with
    the longest segment (no device query on this path)."""
    from wnw_b200.kernels import attn_launch_shape, split_rows
    import torch
    base = split_rows(torch.float32, 128)
    assert attn_launch_shape(torch.float32, 128, [10, 20]) == (base, 1)
    assert attn_launch_shape(torch.float32, 128, [3 * base]) == (base, 4)
    assert attn_launch_shape(torch.float32, 128, [100000, 5]) == (base, 8)
    with pytest.raises(N.WnwError, match="negative capacity"):
        attn_launch_shape(torch.float32, 128, [-1])
    with pytest.raises(N.WnwError, match="launched from a plan"):
        attn_launch_shape(torch.bfloat16, 128, [100])


def _parse_plan(plan):
    ctas, C, parts, ncomb = (int(x) for x in plan[:4])
    cta = plan[8:8 + 4 * ctas].reshape(-1, 4)
    at = 8 + 4 * ctas
    part_r0 = plan[at:at + parts]
    at += (parts + 3) // 4 * 4
    comb = plan[at:at + 4 * ncomb].reshape(-1, 4)
    assert plan.size == at + 4 * ncomb
    return C, cta, part_r0, comb


def _meta(m):
    m = int(m) & 0xFFFFFFFF
    return m & 31, (m >> 5) & 31, (m >> 10) & 1, m >> 11


@pytest.mark.parametrize("seed", range(40))
def test_attn_plan_properties_random(seed):
    """wnw_attn_plan on random capacities, SM counts and cluster limits:
    every segment's rows (capacity + the step's token, in 32-row units) are
    covered exactly once, by consecutive ranks of one cluster that name their
    leader and count -- or, for a segment longer than a cluster's CTAs take,
    by whole clusters in order, each with a partial slot and its first row,
    listed once in the combine table; the cluster size is a power of two no
    larger than allowed and divides the CTA count."""
    from wnw_b200.kernels import attn_plan
    rng = np.random.default_rng(900 + seed)
    nseg = int(rng.choice([1, 3, 8, 64, 700, 2048]))
    hi = int(rng.choice([40, 3000, 130000]))
    cap = rng.integers(0, hi, nseg).astype(np.int32)
    sm, mc = int(rng.choice([1, 7, 148, 600])), int(rng.choice([1, 2, 4, 8, 16]))
    plan, info = attn_plan(cap, sm, mc)
    C, cta, part_r0, comb = _parse_plan(plan)
    assert C == info["cluster"] and C <= mc and C & (C - 1) == 0
    assert len(cta) == info["ctas"] and len(cta) % C == 0
    assert len(part_r0) == info["parts"] and len(comb) == info["combine"]
    units = (cap.astype(np.int64) + 1 + 31) // 32
    covered = {s: [] for s in range(nseg)}
    parts_of = {}
    for c in range(0, len(cta), C):
        cl = cta[c:c + C]
        r = 0
        while r < C:
            seg = int(cl[r, 0])
            if seg < 0:
                r += 1
                continue
            leader, n, to_part, part = _meta(cl[r, 3])
            assert leader == r and 1 <= n <= C - r
            for i in range(n):  # the segment's ranks: consecutive, same leader and count
                assert int(cl[r + i, 0]) == seg and _meta(cl[r + i, 3]) == (leader, n, to_part, part)
                covered[seg].append((int(cl[r + i, 1]), int(cl[r + i, 2])))
            if to_part:
                assert n == C and part < len(part_r0) and part_r0[part] == cl[r, 1]
                parts_of.setdefault(seg, []).append(part)
            r += n
    for s in range(nseg):
        rngs = sorted(covered[s])
        assert rngs[0][0] == 0 and rngs[-1][1] == units[s] * 32
        assert all(a[1] == b[0] for a, b in zip(rngs, rngs[1:]))
        assert all(r0 % 32 == 0 and r1 >= r0 for r0, r1 in rngs)
    assert sorted(parts_of) == sorted(int(e[0]) for e in comb)
    for seg, first, n, _ in comb:
        assert parts_of[int(seg)] == list(range(int(first), int(first) + int(n)))
        assert list(part_r0[first:first + n]) == sorted(part_r0[first:first + n]) and part_r0[first] == 0


def test_attn_plan_config2_layer_spreads_over_half_the_sms():
    """The config-2 layer (two 15,100-row class-A and six 2,300-row class-B
    segments) on a 148-SM device with clusters of up to 16: one cluster of 16
    per class-A segment would stream each at one GPC's rate, so the plan
    takes clusters of 4 on at most half the SMs (the next layer's CTAs run
    beside it): the class-A segments span several clusters, merged through
    their partials, and each class-B segment stays inside one cluster."""
    from wnw_b200.kernels import attn_plan
    cap = np.array([15100 + 40] * 2 + [2300 + 40] * 6, np.int32)
    plan, info = attn_plan(cap, 148, 16)
    assert info["cluster"] == 4 and 64 <= info["ctas"] <= 74 and info["combine"] == 2
    C, cta, _, comb = _parse_plan(plan)
    assert sorted(int(e[0]) for e in comb) == [0, 1]
    for seg in range(2, 8):
        ranks = cta[cta[:, 0] == seg]
        assert len(ranks) <= 4 and all(_meta(m)[2] == 0 for m in ranks[:, 3])


@pytest.mark.parametrize("n_a,most", [(1, 74), (2, 74), (3, 98), (4, 98)])
def test_attn_plan_spreads_over_a_fraction_of_the_sms(n_a, most):
    """Layers of 1-4 long (15.1k-row) segments beside 2.3k-row ones: spread
    over clusters of 4 on half the SMs (1-2 long segments) or two thirds of
    them (3-4), the first fraction whose share is below the one-cluster
    plan's 960 rows -- the plans measured fastest back to back."""
    from wnw_b200.kernels import attn_plan
    lens = [15100 + 296] * n_a + [2300] * (8 - n_a)
    plan, info = attn_plan(np.array(lens, np.int32) + 40, 148, 16)
    assert info["cluster"] == 4 and info["combine"] == n_a
    assert most // 2 < info["ctas"] <= most
    C, cta, _, _ = _parse_plan(plan)
    rows = cta[cta[:, 0] >= 0, 2] - cta[cta[:, 0] >= 0, 1]
    assert rows.max() < 960


@pytest.mark.parametrize("lens", [[2300] * 8, [1, 2, 3, 300], [7000] * 4])
def test_attn_plan_short_shares_keep_one_cluster_per_segment(lens):
    """Layers whose one-cluster shares are at most 512 rows keep every
    segment inside one cluster (no partials)."""
    from wnw_b200.kernels import attn_plan
    plan, info = attn_plan(np.array(lens, np.int32) + 40, 148, 16)
    assert info["parts"] == 0 and info["combine"] == 0


@pytest.mark.parametrize("lens", [[120000] * 2 + [4000] * 6, [60000] * 8, [30000] * 2 + [3000] * 6])
def test_attn_plan_long_segments_fit_one_wave(lens):
    """Layers whose longest segment needs more CTAs than a cluster holds:
    clusters of at most 4 and no more CTAs than the (148) slots, so the
    launch runs in one wave; long segments are merged by the combine kernel."""
    from wnw_b200.kernels import attn_plan
    plan, info = attn_plan(np.array(lens, np.int32) + 64, 148, 16)
    assert info["cluster"] <= 4 and info["ctas"] <= 148 and info["combine"] >= 1


def test_attn_plan_balances_long_segments_among_many_short_ones():
    """16 long segments beside 112 short ones (batch 16, one class-A kv head
    of 8 at 131k rows): the plan spreads the long ones over several CTAs in
    a few waves rather than one lopsided wave."""
    from wnw_b200.kernels import attn_plan
    lens = [131072 if h == 0 else 13107 for _ in range(16) for h in range(8)]
    plan, info = attn_plan(np.array(lens, np.int32) + 16, 148, 16)
    C, cta, _, _ = _parse_plan(plan)
    per_seg = np.bincount(cta[cta[:, 0] >= 0, 0], minlength=128)
    assert per_seg[::8].min() >= 4 and info["ctas"] <= 4 * 148


def test_attn_plan_checks_arguments():
    from wnw_b200.kernels import attn_plan
    with pytest.raises(N.WnwError, match="out of range"):
        attn_plan([5, -1], 4, 4)
    with pytest.raises(N.WnwError, match="max_cluster"):
        attn_plan([5], 4, 17)
    info = N.AttnPlanInfo()
    cap = np.array([100, 200], np.int32)
    N.call("wnw_attn_plan", N.ptr(cap), 2, 4, 4, None, 0, ctypes.byref(info))
    small = np.zeros(int(info.ints) - 1, np.int32)
    st = N.lib.wnw_attn_plan(N.ptr(cap), 2, 4, 4, N.ptr(small), small.size, ctypes.byref(info))
    assert st == 3 and b"capacity" in N.lib.wnw_last_error()


@pytest.mark.parametrize("seed", range(12))
def test_attn_plan_semantics_restate_attention(seed):
    """The kernels' use of a plan, restated in numpy: every CTA attends rows
    [row_begin, min(row_end, total)) of its segment; the leader of a
    segment's ranks merges their (max, sum, o) states -- into the output, or,
    for a segment spanning clusters, into the cluster's partial unless the
    cluster starts at or past the segment's rows; the combine step merges a
    segment's partials whose ranges start below its row count (a prefix; the
    first always counts).  On random lengths at or below the capacities, with
    and without the step's token, the result equals the oracle's attention."""
    from wnw_b200.kernels import attn_plan
    rng = np.random.default_rng(40 + seed)
    S, G, D = int(rng.integers(1, 9)), int(rng.integers(1, 5)), 16
    cap = rng.integers(0, 700, S).astype(np.int32)
    append = bool(rng.integers(0, 2))
    lens = np.array([rng.integers(0, c + 1) if c else 0 for c in cap], np.int64)
    if append:
        lens = np.minimum(lens, cap)  # the token fits: len + 1 <= cap + 1
    total = lens + int(append)
    plan, _ = attn_plan(cap, int(rng.choice([1, 3, 9, 40])), int(rng.choice([1, 2, 4])))
    C, cta, part_r0, comb = _parse_plan(plan)
    q = rng.standard_normal((S, G, D))
    kv = [(rng.standard_normal((max(int(t), 1), D)), rng.standard_normal((max(int(t), 1), D))) for t in total]

    def attend(seg, r0, r1):
        rows = max(0, min(r1, int(total[seg])) - r0)
        k, v = kv[seg][0][r0:r0 + rows], kv[seg][1][r0:r0 + rows]
        x = q[seg] @ k.T / np.sqrt(D)
        m = x.max(axis=1) if rows else np.full(G, -np.inf)
        p = np.exp(x - m[:, None]) if rows else np.zeros((G, 0))
        return m, p.sum(axis=1), p @ v

    def merge(states):
        ms = np.stack([s[0] for s in states])
        mx = ms.max(axis=0)
        w = np.where(np.isinf(ms), 0.0, np.exp(ms - np.where(np.isinf(mx), 0.0, mx)))
        return mx, sum(w[j] * states[j][1] for j in range(len(states))), \
            sum(w[j][:, None] * states[j][2] for j in range(len(states)))

    out = np.full((S, G, D), np.nan)
    parts = {}
    for c in range(0, len(cta), C):
        cl = cta[c:c + C]
        for r in range(C):
            seg = int(cl[r, 0])
            if seg < 0:
                continue
            leader, n, to_part, part = _meta(cl[r, 3])
            if r != leader:
                continue
            mx, l, o = merge([attend(seg, int(cl[r + i, 1]), int(cl[r + i, 2])) for i in range(n)])
            if not to_part:
                out[seg] = np.where(l[:, None] > 0, o / np.where(l > 0, l, 1)[:, None], 0.0)
            elif not (cl[r, 1] >= total[seg] and cl[r, 1] > 0):
                parts[part] = (mx, l, o)
    for seg, first, n, _ in comb:
        act = 1
        while act < n and part_r0[first + act] < total[seg]:
            act += 1
        mx, l, o = merge([parts[first + j] for j in range(act)])
        out[seg] = np.where(l[:, None] > 0, o / np.where(l > 0, l, 1)[:, None], 0.0)
    cu = np.concatenate([[0], np.cumsum(total)])
    pk = np.concatenate([kv[s][0][:total[s]] for s in range(S)]) if total.sum() else np.zeros((0, D))
    pv = np.concatenate([kv[s][1][:total[s]] for s in range(S)]) if total.sum() else np.zeros((0, D))
    ref, _, _ = K.decode_attn(q.astype(np.float32), pk.astype(np.float32), pv.astype(np.float32), cu, D ** -0.5)
    nz = total > 0
    assert not np.isnan(out).any()
    np.testing.assert_allclose(out[nz], ref[nz], atol=1e-5, rtol=1e-5)
    assert np.all(out[~nz] == 0)


def test_issue_fetch_reports_sizes_without_issuing(golden_dir):
    """wnw_planner_issue_fetch checks every capacity before touching the
    device: with empty buffers it returns WNW_ERR_CAPACITY and reports the
    plan, range and row counts the step needs (equal to the planner's own
    outputs), so the caller can grow its buffers and retry."""
    from wnw_b200.planner import Planner
    ps = PLANNER_SCENARIOS[0]
    inp = make_planner_inputs(ps)
    P = _planner_from(ps, inp, Planner)
    L, S = ps["L"], ps["B"] * ps["H"]
    bufs = [np.zeros((L, S), np.int32), np.zeros((L, S), np.int32), np.zeros((L, S + 1), np.int32),
            np.zeros((L, S), np.int32), np.zeros((L, S + 1), np.int32), np.zeros(L, np.int32),
            np.zeros(L + 1, np.int32)]
    for tk, toff in inp["steps"]:
        ch, total, _, _, ranges = P.compute_and_prepare(tk, toff, *bufs)
        if ch and total:
            break
    assert ch and total
    chg = np.full(L, -1, np.int32)
    info = N.FetchInfo()
    info.layer_changed = chg.ctypes.data
    st = N.lib.wnw_planner_issue_fetch(P._h, None, None, 0, None, None, None, None, 0, None, None, 256, None, None,
                                       0, 32, None, None, ctypes.byref(info))
    assert st == N.WNW_ERR_CAPACITY
    assert info.total_rows == total and info.n_ranges == len(ranges)
    assert info.plan_ints == P.device_plan().size
    blob = P.device_plan()
    for l in range(L):
        assert chg[l] == (1 if blob[blob[l]] > 0 else 0)
    assert b"capacity" in N.lib.wnw_last_error()


def test_oproj_allreduce_rejects_bad_arguments():
    """Argument checks of the tensor-parallel exchange run before any launch."""
    a = N.OprojAllReduceArgs()
    a.dtype, a.batch, a.n_out, a.k_in, a.rank, a.world = N.BF16, 1, 64, 60, 0, 1
    st = N.lib.wnw_oproj_allreduce(ctypes.byref(a), None)
    assert st == 1 and b"multiple of 8" in N.lib.wnw_last_error()
    a.k_in, a.world, a.rank = 64, 9, 0
    assert N.lib.wnw_oproj_allreduce(ctypes.byref(a), None) == 1
    a.world, a.batch = 1, 9
    assert N.lib.wnw_oproj_allreduce(ctypes.byref(a), None) == 1
    assert N.lib.wnw_oproj_allreduce_chunks(3072) == 384
    assert N.lib.wnw_oproj_allreduce_chunks(0) == 0
    # a batch above the receive buffers' rows would store past a peer's buffer:
    # refused as a capacity error before anything is launched
    buf = (ctypes.c_uint8 * 4096)()
    base = (ctypes.addressof(buf) + 255) // 256 * 256
    a.x, a.w, a.y, a.err = base, base + 256, base + 512, base + 768
    a.recv[0], a.flags[0] = base + 1024, base + 2048
    a.batch, a.recv_batch = 2, 1
    assert N.lib.wnw_oproj_allreduce(ctypes.byref(a), None) == 3
    assert b"exceeds the receive buffers" in N.lib.wnw_last_error()
    a.recv_batch = 0
    assert N.lib.wnw_oproj_allreduce(ctypes.byref(a), None) == 1


def test_rebuild_layers_fused_rejects_bad_arguments():
    """Argument checks of the one-launch-pair rebuild run before any launch:
    null per-layer tables, misaligned stores, and a status buffer shorter than
    the changed layers' segments."""
    P = ctypes.c_void_p
    buf = (ctypes.c_uint8 * 8192)()
    base = (ctypes.addressof(buf) + 255) // 256 * 256
    L = 3
    ptrs = lambda off: (P * L)(*[base + off + 16 * i for i in range(L)])  # noqa: E731
    chg = np.array([1, 0, 1], np.int32)
    nsegs = (ctypes.c_int32 * L)(8, 8, 8)

    def call(k_store, status_len, changed=chg):
        return N.lib.wnw_rebuild_layers_fused(N.BF16, 128, L, changed.ctypes.data, k_store, ptrs(1024),
                                              ptrs(2048), ptrs(3072), ptrs(4096), nsegs, None, None, 0, base,
                                              64, None, None, 0, base + 5120, status_len, base + 6144, None, None,
                                              None)

    assert call(ptrs(0), 15) == 1 and b"status needs 16" in N.lib.wnw_last_error()
    bad = (P * L)(base, base, base + 8)
    assert call(bad, 16) == 1 and b"layer 2" in N.lib.wnw_last_error()
    bad = (P * L)(None, base, base)
    assert call(bad, 16) == 1 and b"layer 0" in N.lib.wnw_last_error()
    assert N.lib.wnw_rebuild_layers_fused(N.BF16, 128, 0, None, None, None, None, None, None, None, None, None, 0,
                                          None, 0, None, None, 0, None, 0, None, None, None, None) == 0


def test_oproj_exchange_refuses_shapes_it_was_not_built_for():
    """OprojAllReduce checks every call's tensors against the receive
    buffers it was built for before it launches anything."""
    import torch
    from wnw_b200.tp import OprojAllReduce

    ex = object.__new__(OprojAllReduce)  # the checks only, no IPC buffers
    ex.dev, ex.batch, ex.n_out, ex.dtype = torch.device("cpu"), 2, 16, torch.bfloat16
    x = torch.zeros(2, 32, dtype=torch.bfloat16)
    w = torch.zeros(16, 32, dtype=torch.bfloat16)
    ex._check_shapes(x, w, None)
    with pytest.raises(ValueError, match="batch 3 not in 1..2"):
        ex._check_shapes(torch.zeros(3, 32, dtype=torch.bfloat16), w, None)
    with pytest.raises(ValueError, match="w must be"):
        ex._check_shapes(x, torch.zeros(16, 24, dtype=torch.bfloat16), None)
    with pytest.raises(ValueError, match="w must be"):
        ex._check_shapes(x, torch.zeros(8, 32, dtype=torch.bfloat16), None)
    with pytest.raises(TypeError, match="must be torch.bfloat16"):
        ex._check_shapes(x.half(), w, None)
    with pytest.raises(ValueError, match="contiguous"):
        ex._check_shapes(torch.zeros(32, 2, dtype=torch.bfloat16).t(), w, None)
    with pytest.raises(ValueError, match="y must be"):
        ex._check_shapes(x, w, torch.zeros(2, 8, dtype=torch.bfloat16))


def test_step_wait_times_out_instead_of_blocking():
    """The decode step's host wait has a deadline: a device that never gets
    there (a fake event that never completes) raises a timeout error."""
    import time
    from wnw_b200.cache import wait_event

    class Never:
        def query(self):
            return False

    class Later:
        def __init__(self):
            self.t = time.perf_counter() + 0.05

        def query(self):
            return time.perf_counter() > self.t

    t0 = time.perf_counter()
    with pytest.raises(N.WnwError, match="timed out"):
        wait_event(Never(), 0.2)
    assert time.perf_counter() - t0 < 5
    wait_event(Later(), 5.0)  # completes in time: no error


def test_upload_plan_and_device_plan_argument_checks(golden_dir):
    """The device-planned step's host entry points refuse bad calls before
    any CUDA call: wnw_planner_upload_plan reports the plan size and
    WNW_ERR_CAPACITY for a too-small buffer; wnw_dplan_* reject null handles
    and an incomplete planner."""
    from wnw_b200.planner import Planner
    ps = PLANNER_SCENARIOS[0]
    inp = make_planner_inputs(ps)
    P = _planner_from(ps, inp, Planner)
    L, S = ps["L"], ps["B"] * ps["H"]
    bufs = [np.zeros((L, S), np.int32), np.zeros((L, S), np.int32), np.zeros((L, S + 1), np.int32),
            np.zeros((L, S), np.int32), np.zeros((L, S + 1), np.int32), np.zeros(L, np.int32),
            np.zeros(L + 1, np.int32)]
    for tk, toff in inp["steps"]:
        ch, total, _, _, _ = P.compute_and_prepare(tk, toff, *bufs)
        if ch and total:
            break
    chg = np.full(L, -1, np.int32)
    info = N.FetchInfo()
    info.layer_changed = chg.ctypes.data
    st = N.lib.wnw_planner_upload_plan(P._h, None, None, 0, None, ctypes.byref(info))
    assert st == N.WNW_ERR_CAPACITY
    assert info.plan_ints == P.device_plan().size and info.total_rows == total
    assert N.lib.wnw_planner_upload_plan(None, None, None, 0, None, ctypes.byref(info)) == N.WNW_ERR_INVALID
    h = ctypes.c_void_p()
    assert N.lib.wnw_dplan_create(None, ctypes.byref(h)) == N.WNW_ERR_INVALID
    bare = Planner(2, 2, 1)  # no segments or metadata yet
    assert N.lib.wnw_dplan_create(bare._h, ctypes.byref(h)) == N.WNW_ERR_INVALID
    assert b"incomplete" in N.lib.wnw_last_error()
    assert N.lib.wnw_dplan_step(None, None, 1, None, None, None, 256, None, None, 0, 12, None, None,
                                None) == N.WNW_ERR_INVALID
    assert N.lib.wnw_dplan_verify(None, P._h) == N.WNW_ERR_INVALID
    N.lib.wnw_dplan_destroy(None)  # a null handle is a no-op


def test_planner_gather_restore_matches_oracle(golden_dir):
    """Planner.set_restore_buffers / gather_restore (planner.cpp:104-122): the
    last plan's host ranges, in planner order, land at the front of the
    staging buffers; a staging buffer too small is refused."""
    import torch
    from oracle import kernels as K
    from wnw_b200.planner import Planner
    ps = PLANNER_SCENARIOS[0]
    inp = make_planner_inputs(ps)
    P = _planner_from(ps, inp, Planner)
    L, S = ps["L"], ps["B"] * ps["H"]
    bufs = [np.zeros((L, S), np.int32), np.zeros((L, S), np.int32), np.zeros((L, S + 1), np.int32),
            np.zeros((L, S), np.int32), np.zeros((L, S + 1), np.int32), np.zeros(L, np.int32),
            np.zeros(L + 1, np.int32)]
    for tk, toff in inp["steps"]:
        ch, total, _, _, ranges = P.compute_and_prepare(tk, toff, *bufs)
        if ch and total:
            break
    rows = int(np.max(ranges)) + 4
    g = torch.Generator().manual_seed(5)
    ck, cv = torch.randn(rows, 8, generator=g), torch.randn(rows, 8, generator=g)
    sk, sv = torch.full((total + 3, 8), -1.0), torch.full((total + 3, 8), -1.0)
    with pytest.raises(RuntimeError):
        P.gather_restore()
    P.set_restore_buffers(ck, cv, sk, sv)
    P.gather_restore()
    wk, wv = K.gather_restore(ck.numpy(), cv.numpy(), ranges)
    assert np.array_equal(sk[:total].numpy(), wk) and np.array_equal(sv[:total].numpy(), wv)
    assert (sk[total:] == -1).all()
    P.set_restore_buffers(ck, cv, sk[:total - 1], sv[:total - 1])
    with pytest.raises(N.WnwError):
        P.gather_restore()


def test_planner_returns_tensors_for_tensor_inputs(golden_dir):
    """The reference's C++ cache calls .to(device) / .numel() on the plan's
    evictions and ranges (wnw_cpp/code/cache.py:254-268): given torch inputs,
    compute_and_prepare returns int32 CPU tensors equal to the numpy path."""
    import torch
    from wnw_b200.planner import Planner
    ps = PLANNER_SCENARIOS[0]
    inp = make_planner_inputs(ps)
    L, S = ps["L"], ps["B"] * ps["H"]
    shapes = [(L, S), (L, S), (L, S + 1), (L, S), (L, S + 1), (L,), (L + 1,)]
    Pn, Pt = _planner_from(ps, inp, Planner), _planner_from(ps, inp, Planner)
    for tk, toff in inp["steps"]:
        rn = Pn.compute_and_prepare(tk, toff, *[np.zeros(s, np.int32) for s in shapes])
        outs = [torch.zeros(s, dtype=torch.int32) for s in shapes]
        rt = Pt.compute_and_prepare(torch.as_tensor(tk), torch.as_tensor(toff), *outs)
        assert rt[:2] == rn[:2]
        for a, b in zip(rt[2:], rn[2:]):
            assert isinstance(a, torch.Tensor) and a.dtype == torch.int32
            assert np.array_equal(a.numpy(), b)
        assert rt[4].dim() == 2 and rt[4].shape[1] == 2


def test_planner_is_a_drop_in_for_the_reference_cpp_cache(golden_dir):
    """tests/golden/cache_cpp_dropin_trace.npz was recorded by running the
    reference's own WnWCppCache with wnw_b200.planner.Planner in place of its
    pybind11 planner (make_golden.py dropin): every layout digest, cu_seqlens,
    output and loaded set equals the run with the reference's planner."""
    ours = np.load(os.path.join(golden_dir, "cache_cpp_dropin_trace.npz"), allow_pickle=True)
    ref = np.load(os.path.join(golden_dir, "cache_cpp_trace.npz"), allow_pickle=True)
    keys = [k for k in ours.files]
    assert any(k.endswith("_khash") for k in keys) and any(k.endswith("_loaded") for k in keys)
    for k in keys:
        a, b = ours[k], ref[k]
        if a.dtype == object:
            assert [list(x) for x in a] == [list(x) for x in b], k
        else:
            assert np.array_equal(a, b), k


@pytest.mark.parametrize("seed", range(30))
def test_work_table_properties_random(seed):
    """wnw_build_work_table on random capacities, splits and cluster sizes:
    every segment gets exactly the clusters its capacity (+1 appended row)
    needs, numbered 0..n-1 and consecutive; segments needing more clusters
    come first (a stable sort by decreasing cluster count), so the ones with
    a cross-cluster merge start earliest."""
    from wnw_b200.kernels import build_work_table
    rng = np.random.default_rng(700 + seed)
    cap = rng.integers(0, 40000, int(rng.integers(1, 70))).astype(np.int32)
    split = int(rng.choice([32, 64, 128, 256, 384, 512, 1024]))
    cs = int(rng.choice([1, 2, 4, 8, 16]))
    w = build_work_table(cap, split, cs).tolist()
    need = [max(1, -(-(-(-(int(c) + 1) // split)) // cs)) for c in cap]
    assert len(w) == sum(need)
    segs_in_order = []
    for seg, j in w:
        if not segs_in_order or segs_in_order[-1] != seg:
            segs_in_order.append(seg)
    assert sorted(segs_in_order) == list(range(len(cap)))  # each segment's clusters are consecutive
    for s in range(len(cap)):
        assert [j for seg, j in w if seg == s] == list(range(need[s]))
    assert segs_in_order == sorted(range(len(cap)), key=lambda s: -need[s])
