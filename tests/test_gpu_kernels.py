"""GPU parity of the sm_100a kernels against the CPU oracle (all launches go
through the C ABI of libwnw_b200.so).

Tolerances: fp32 1e-5 abs+rel, bf16/fp16 2e-2 abs+rel (fp32 accumulation);
copies, offsets and top-k selections bit-exact."""
import math
import os

import numpy as np
import pytest
import torch

from oracle import kernels as K

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 2e-2}


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from wnw_b200 import native  # noqa: F401  (fails loudly when the library is missing)
    return torch.device("cuda:0")


def _slots(lens, slack, D, dtype, dev, seed):
    """Slot layout with random rows: returns store K/V, base, cap, and the
    packed oracle copy of the stored rows."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    lens = np.asarray(lens, np.int64)
    cap = lens + slack
    cap_al = (cap + 15) // 16 * 16
    base = np.concatenate([[0], np.cumsum(cap_al)[:-1]]).astype(np.int64)
    rows = int(cap_al.sum())
    ks = torch.randn(rows, D, generator=g).to(dtype)
    vs = torch.randn(rows, D, generator=g).to(dtype)
    return ks.to(dev), vs.to(dev), base, cap


def _packed(store, base, lens):
    s = store.float().cpu().numpy()
    parts = [s[b:b + n] for b, n in zip(base, lens)]
    return np.concatenate(parts) if parts else s[:0]


def test_packed_attention_matches_reference_golden(dev, golden_dir):
    from wnw_b200 import kernels as Kx
    kz = np.load(os.path.join(golden_dir, "kernels.npz"))
    q = torch.from_numpy(kz["attn_q"]).to(dev)
    k = torch.from_numpy(kz["attn_k"]).to(dev)
    v = torch.from_numpy(kz["attn_v"]).to(dev)
    cu = torch.from_numpy(kz["attn_cu"]).to(dev)
    out = Kx.packed_attention(q, k, v, cu, float(kz["attn_scale"]))
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), kz["attn_out"], atol=1e-5, rtol=1e-5)


CASES = [
    # dtype, D, G, cluster, lens
    (torch.float32, 128, 4, 8, [0, 1, 63, 64, 65, 200, 3000, 20000]),
    (torch.bfloat16, 128, 4, 8, [1, 127, 128, 129, 1000, 15064, 2500, 7]),
    (torch.float16, 128, 4, 4, [5, 128, 777, 4096]),
    (torch.bfloat16, 128, 7, 8, [100, 6000, 1, 30000]),
    (torch.bfloat16, 128, 8, 2, [333, 256, 2]),
    (torch.bfloat16, 128, 1, 1, [10, 500, 129]),
    (torch.bfloat16, 128, 4, 1, [15064, 3, 2000, 129]),
    (torch.float32, 64, 2, 8, [3, 900, 4097]),
    (torch.bfloat16, 64, 3, 4, [1, 2, 3, 1000]),
    (torch.float32, 32, 2, 8, [400, 12]),
    (torch.float32, 16, 2, 2, [130, 9]),
]


@pytest.mark.parametrize("dtype,D,G,cs,lens", CASES)
@pytest.mark.parametrize("append", [True, False])
@pytest.mark.parametrize("sms,ready", [(None, False), ((4, 4), True), ((600, 2), True)])
def test_decode_attention_matches_oracle(dev, dtype, D, G, cs, lens, append, sms, ready):
    """Tensor-core path: ``sms`` = (SM count, largest cluster) the plan is cut
    for -- the device's own (the library default); 4 SMs with clusters of 4
    (long per-CTA shares, segments spanning several clusters, merged by the
    combine kernel); 600 SMs with clusters of 2 (32-row shares, dozens of
    cluster partials per long segment); ``ready`` lets the kernel read
    lengths and rows before its dependency wait.  The CUDA-core path (fp32,
    head_dim 16 / 32) takes its cluster table ``cs``."""
    from wnw_b200 import kernels as Kx
    S = len(lens)
    plan = Kx.uses_plan(dtype, D)
    if not plan and sms is not None:
        pytest.skip("the SM count of a plan is a tensor-core kernel mode")
    ks, vs, base, cap = _slots(lens, 40, D, dtype, dev, seed=sum(lens) + G)
    g = torch.Generator(device="cpu").manual_seed(7)
    q = torch.randn(S, G, D, generator=g).to(dtype).to(dev)
    nk = torch.randn(S, D, generator=g).to(dtype).to(dev) if append else None
    nv = torch.randn(S, D, generator=g).to(dtype).to(dev) if append else None
    work = Kx.AttnWork(dtype, D, cap, dev, sm_count=sms[0] if sms else None, max_cluster=sms[1] if sms else None,
                       split=None if plan else Kx.split_rows(dtype, D), cluster_size=None if plan else cs)
    scratch = Kx.AttnScratch(dev, work.slots, G, D, S)
    seg_len = torch.tensor(lens, dtype=torch.int32, device=dev)
    before_k = ks.clone()
    scale = D ** -0.5
    out = Kx.decode_attention(q, ks, vs, torch.from_numpy(base).to(dev), seg_len, work, scale, scratch,
                              new_k=nk, new_v=nv, seg_cap=torch.from_numpy(cap.astype(np.int32)).to(dev),
                              flags=1 if ready else 0)
    torch.cuda.synchronize()
    assert int(scratch.err.item()) == 0
    assert int(scratch.counters.abs().sum()) == 0  # left zero for the next launch
    # oracle over the packed rows (+ the appended token)
    lens_eff = np.asarray(lens) + (1 if append else 0)
    if append:
        ks_ref = before_k.clone()
        for s in range(S):
            ks_ref[base[s] + lens[s]] = nk[s]
        assert torch.equal(ks, ks_ref)  # exactly one new row per segment, slack untouched
    pk = _packed(ks, base, lens_eff)
    pv = _packed(vs, base, lens_eff)
    cu = np.concatenate([[0], np.cumsum(lens_eff)])
    ref, _, _ = K.decode_attn(q.float().cpu().numpy(), pk, pv, cu, scale)
    got = out.float().cpu().numpy()
    tol = TOL[dtype]
    nz = lens_eff > 0
    np.testing.assert_allclose(got[nz], ref[nz], atol=tol, rtol=tol)
    assert np.all(got[~nz] == 0)


@pytest.mark.parametrize("lens", [[15100, 15100, 2300, 2300, 2300, 2300, 2300, 2300], [120000, 4000, 3],
                                  [1, 2, 3, 300], [5000] * 64, [700] * 2048])
def test_library_plan_matches_oracle(dev, lens):
    """The library's default plan (this device's SMs and clusters) is valid
    and its output matches the oracle -- including 2,048 segments (batch 256
    x 8 kv heads, where the reference's row-gather kernels break down)."""
    from wnw_b200 import kernels as Kx
    dtype, D, G = torch.bfloat16, 128, 4
    S = len(lens)
    ks, vs, base, cap = _slots(lens, 64, D, dtype, dev, seed=len(lens))
    work = Kx.AttnWork(dtype, D, cap, dev)
    assert work.plan and work.ctas >= S and work.ctas % work.cluster_size == 0
    g = torch.Generator(device="cpu").manual_seed(5)
    q = torch.randn(S, G, D, generator=g).to(dtype).to(dev)
    scratch = Kx.AttnScratch(dev, work.slots, G, D, S)
    out = Kx.decode_attention(q, ks, vs, torch.from_numpy(base).to(dev),
                              torch.tensor(lens, dtype=torch.int32, device=dev), work, D ** -0.5, scratch,
                              seg_cap=torch.from_numpy(cap.astype(np.int32)).to(dev))
    torch.cuda.synchronize()
    assert int(scratch.err.item()) == 0
    pk, pv = _packed(ks, base, lens), _packed(vs, base, lens)
    ref, _, _ = K.decode_attn(q.float().cpu().numpy(), pk, pv, np.concatenate([[0], np.cumsum(lens)]), D ** -0.5)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=TOL[dtype], rtol=TOL[dtype])


@pytest.mark.parametrize("dtype,sms", [(torch.float32, None), (torch.bfloat16, None), (torch.bfloat16, (6, 2))])
def test_scoring_logits_and_finalize_match_oracle(dev, dtype, sms):
    """Fused class-A logits + stats, then wnw_score_finalize, equal the
    reference's per-token probabilities summed over kv heads and q heads
    (bf16: the same inputs as fp32 values, logits accumulated in fp32)."""
    from wnw_b200 import kernels as Kx
    B, H, G, D = 2, 4, 4, 128
    lens = [3000, 2900, 2700, 4100, 3500, 3300, 2900, 900]  # class-A kv 0, 2 cover the audio
    a_s, a_e = [10, 40], [2600, 2800]
    ks, vs, base, cap = _slots(lens, 16, D, dtype, dev, seed=3)
    g = torch.Generator(device="cpu").manual_seed(11)
    q = torch.randn(B * H, G, D, generator=g).to(dtype).to(dev)
    plan = Kx.uses_plan(dtype, D)
    work = Kx.AttnWork(dtype, D, cap, dev, sm_count=sms[0] if sms else None, max_cluster=sms[1] if sms else None,
                       split=None if plan else Kx.split_rows(dtype, D), cluster_size=None if plan else 8)
    scratch = Kx.AttnScratch(dev, work.slots, G, D, B * H)
    ca_kv = [0, 2]                       # class-A kv heads (all q heads of each)
    slot = np.full(B * H, -1, np.int32)
    offs, t_logit, t_stat, t_mask, t_off = [], [], [], [], [0]
    total = 0
    for b in range(B):
        for kv in ca_kv:
            slot[b * H + kv] = len(offs)
            offs.append(total)
            t_logit.append(total)
            t_stat.append((b * H + kv) * 2 * G)
            t_mask.append((1 << G) - 1)
            total += (a_e[b] - a_s[b]) * G
        t_off.append(len(t_logit))
    logits = torch.zeros(total, device=dev)
    stats = torch.zeros(B * H * 2 * G, device=dev)
    score = dict(slot=torch.from_numpy(slot).to(dev), audio_start=torch.tensor(a_s, dtype=torch.int32, device=dev),
                 audio_end=torch.tensor(a_e, dtype=torch.int32, device=dev), logits=logits,
                 logits_off=torch.tensor(offs, dtype=torch.int64, device=dev), stats=stats)
    Kx.decode_attention(q, ks, vs, torch.from_numpy(base).to(dev), torch.tensor(lens, dtype=torch.int32, device=dev),
                        work, D ** -0.5, scratch, num_kv_heads=H, score=score)
    n_audio = [e - s for s, e in zip(a_s, a_e)]
    score_off = torch.tensor([0, n_audio[0], sum(n_audio)], dtype=torch.int32, device=dev)
    acc = torch.full((sum(n_audio),), -1.0, device=dev)
    Kx.score_finalize(logits, stats, torch.tensor(t_logit, device=dev), torch.tensor(t_stat, device=dev),
                      torch.tensor(t_mask, dtype=torch.int32, device=dev), torch.tensor(t_off, dtype=torch.int32,
                                                                                         device=dev),
                      G, score_off, max(n_audio), acc)
    torch.cuda.synchronize()
    pk = _packed(ks, base, lens)
    pv = _packed(vs, base, lens)
    cu = np.concatenate([[0], np.cumsum(lens)])
    ref_acc = np.zeros(sum(n_audio))
    ca_mask = np.zeros(H, np.int32)
    ca_mask[ca_kv] = 1
    K.decode_attn_score(q.float().cpu().numpy(), pk, pv, cu, D ** -0.5, ca_mask, H, a_s, a_e, ref_acc,
                        [0, n_audio[0], sum(n_audio)])
    np.testing.assert_allclose(acc.cpu().numpy(), ref_acc, atol=1e-6, rtol=1e-5)


@pytest.mark.parametrize("stride,spc,top_k,n_audio", [(64, 1, 8, [3000, 5000, 64]), (16, 2, 3, [300, 250]),
                                                     (128, 1, 16, [15000]), (128, 1, 32, [120000, 90000]),
                                                     (7, 3, 5, [40, 0, 13])])
def test_chunk_topk_bit_exact(dev, stride, spc, top_k, n_audio):
    """Same accumulator in -> identical chunk scores and top-k (ties -> lower index)."""
    from wnw_b200 import kernels as Kx
    rng = np.random.default_rng(stride * 31 + top_k)
    acc = (rng.random(sum(n_audio)) ** 4).astype(np.float32)
    if n_audio[0] >= 4 * stride:  # plant exact ties: two identical chunks
        acc[stride:2 * stride] = acc[:stride]
        acc[2 * stride:3 * stride] = 1.0
        acc[3 * stride:4 * stride] = 1.0
    off = np.concatenate([[0], np.cumsum(n_audio)]).astype(np.int32)
    n_chunks = [math.ceil(n / stride) for n in n_audio]
    coff = np.concatenate([[0], np.cumsum(n_chunks)]).astype(np.int32)
    topk = torch.full((len(n_audio), top_k), -5, dtype=torch.int32, device=dev)
    cs = torch.zeros(max(1, int(coff[-1])), device=dev)
    Kx.chunk_topk(torch.from_numpy(acc).to(dev), torch.from_numpy(off).to(dev), max(n_audio), stride, spc, top_k,
                  topk, cs, torch.from_numpy(coff).to(dev))
    torch.cuda.synchronize()
    got = topk.cpu().numpy()
    for b, n in enumerate(n_audio):
        a = acc[off[b]:off[b + 1]]
        nseg = n_chunks[b]
        starts = [c * stride for c in range(nseg)]
        ends = [n if min(c + spc, nseg) == nseg else min(c + spc, nseg) * stride for c in range(nseg)]
        ref = K.chunk_scores(a, starts, ends)
        assert np.array_equal(cs.cpu().numpy()[coff[b]:coff[b + 1]], ref)
        want = K.topk_lower_index(ref, top_k)
        k = min(top_k, nseg)
        assert got[b, :k].tolist() == want
        assert np.all(got[b, k:] == -1)


def test_rebuild_matches_oracle(dev):
    """In-place compaction + splice per changed segment == the reference's
    rebuild semantics (without the step token), bit-exact; untouched slots
    keep their rows."""
    from wnw_b200 import kernels as Kx
    from wnw_b200 import native as N
    D, dtype = 128, torch.bfloat16
    rng = np.random.default_rng(5)
    S = 6
    lens = [700, 40, 3000, 0, 513, 1200]
    ks, vs, base, cap = _slots(lens, 2600, D, dtype, dev, seed=9)
    before_k, before_v = ks.clone(), vs.clone()
    recs = []  # (seg, evict ranges, n_load)
    recs.append((0, [(10, 130), (200, 328), (600, 700)], 500))
    recs.append((2, [(0, 1000), (1500, 1501)], 0))
    recs.append((3, [], 77))
    recs.append((5, [(1199, 1200)], 1024))
    land_rows = sum(r[2] for r in recs)
    g = torch.Generator(device="cpu").manual_seed(1)
    land_k = torch.randn(land_rows, D, generator=g).to(dtype).to(dev)
    land_v = torch.randn(land_rows, D, generator=g).to(dtype).to(dev)
    n = len(recs)
    new, lsrc = [], []
    cur = 0
    plan_recs = []
    for s_, ev, nl in recs:
        new.append(lens[s_] - sum(b - a for a, b in ev) + nl)
        lsrc.append(cur)
        plan_recs.append((s_, lens[s_], new[-1], cur, nl, ev))
        cur += nl
    blob = Kx.pack_plan([plan_recs, []])  # layer 1: no changes
    blob_d = torch.from_numpy(blob).to(dev)
    move_k = torch.empty(4096, D, dtype=dtype, device=dev)
    move_v = torch.empty_like(move_k)
    status = torch.zeros(8, dtype=torch.int32, device=dev)
    seg_len = torch.tensor(lens, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    cap_d = torch.from_numpy(cap.astype(np.int32)).to(dev)
    Kx.rebuild_layer(ks, vs, torch.from_numpy(base).to(dev), seg_len, cap_d, land_k, land_v, blob_d, 0,
                     move_k, move_v, status, err)
    Kx.rebuild_layer(ks, vs, torch.from_numpy(base).to(dev), seg_len, cap_d, land_k, land_v, blob_d, 1,
                     move_k, move_v, status, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    new_lens = list(lens)
    for i, (s, ev, nl) in enumerate(recs):
        new_lens[s] = new[i]
    assert seg_len.cpu().tolist() == new_lens
    lk, lv = land_k.float().cpu().numpy(), land_v.float().cpu().numpy()
    for i, (s, ev, nl) in enumerate(recs):
        old_rows = before_k[base[s]:base[s] + lens[s]].float().cpu().numpy()
        keep = np.ones(lens[s], bool)
        for a, b in ev:
            keep[a:b] = False
        want = np.concatenate([old_rows[keep], lk[lsrc[i]:lsrc[i] + nl]])
        got = ks[base[s]:base[s] + new[i]].float().cpu().numpy()
        assert np.array_equal(got, want), s
        old_v = before_v[base[s]:base[s] + lens[s]].float().cpu().numpy()
        assert np.array_equal(vs[base[s]:base[s] + new[i]].float().cpu().numpy(),
                              np.concatenate([old_v[keep], lv[lsrc[i]:lsrc[i] + nl]]))
    for s in (1, 4):  # untouched segments
        assert torch.equal(ks[base[s]:base[s] + cap[s]], before_k[base[s]:base[s] + cap[s]])
    # a stale plan (length mismatch) is refused on the device, not applied
    snap = ks.clone()
    Kx.rebuild_layer(ks, vs, torch.from_numpy(base).to(dev), seg_len, cap_d, land_k, land_v, blob_d, 0,
                     move_k, move_v, status, err)
    torch.cuda.synchronize()
    assert int(err.item()) & N.DEVERR_LEN_MISMATCH
    assert torch.equal(ks, snap)


def _rebuild_case(dev, D, dtype, L, seed):
    """L layers of six slots each with random changes (evictions, loads, some
    layers unchanged); returns the layers' tensors, the plan blob, the landing
    rows and the changed flags."""
    rng = np.random.default_rng(seed)
    layers, plans, changed = [], [], []
    cur = 0
    for l in range(L):
        lens = [int(x) for x in rng.integers(0, 1500, 6)]
        ks, vs, base, cap = _slots(lens, 1200, D, dtype, dev, seed=seed + l)
        recs = []
        if l % 4 != 3:  # every fourth layer unchanged
            for s in rng.permutation(6)[:int(rng.integers(1, 6))].tolist():
                n = lens[s]
                cuts = sorted(set(int(x) for x in rng.integers(0, n + 1, 2 * int(rng.integers(0, 4))))) if n else []
                ev = [(cuts[i], cuts[i + 1]) for i in range(0, len(cuts) - 1, 2) if cuts[i + 1] > cuts[i]]
                nl = int(rng.integers(0, 300))
                new = n - sum(b - a for a, b in ev) + nl
                recs.append((s, n, new, cur, nl, ev))
                cur += nl
        plans.append(recs)
        changed.append(1 if recs else 0)
        layers.append((ks, vs, torch.from_numpy(base).to(dev), torch.tensor(lens, dtype=torch.int32, device=dev),
                       torch.from_numpy(cap.astype(np.int32)).to(dev)))
    g = torch.Generator(device="cpu").manual_seed(seed)
    land_k = torch.randn(max(1, cur), D, generator=g).to(dtype).to(dev)
    land_v = torch.randn(max(1, cur), D, generator=g).to(dtype).to(dev)
    from wnw_b200 import kernels as Kx
    blob = Kx.pack_plan(plans)
    moved = [Kx.plan_record(blob, l)["moved_total"] for l in range(L)]
    return layers, torch.from_numpy(blob).to(dev), land_k, land_v, changed, moved


def test_rebuild_layers_fused_equals_per_layer(dev):
    """wnw_rebuild_layers_fused (one launch pair for every changed layer, each
    with its own region of the move buffers) leaves every store and length
    exactly as the per-layer wnw_rebuild_segments calls do; a move buffer too
    small for the step's moved rows is refused with the capacity bit."""
    from wnw_b200 import kernels as Kx
    from wnw_b200 import native as N
    D, dtype, L = 128, torch.bfloat16, 7
    layers, blob, land_k, land_v, changed, moved = _rebuild_case(dev, D, dtype, L, seed=31)
    assert sum(moved) > 0 and sum(changed) >= 4
    ref = [tuple(t.clone() for t in lay) for lay in layers]
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    mk = torch.empty(max(moved) + 1, D, dtype=dtype, device=dev)
    mv = torch.empty_like(mk)
    status = torch.zeros(8, dtype=torch.int32, device=dev)
    for l in range(L):
        ks, vs, base, slen, cap = ref[l]
        Kx.rebuild_layer(ks, vs, base, slen, cap, land_k, land_v, blob, l, mk, mv, status, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    mk2 = torch.empty(sum(moved), D, dtype=dtype, device=dev)
    mv2 = torch.empty_like(mk2)
    status2 = torch.zeros(6 * L, dtype=torch.int32, device=dev)
    Kx.rebuild_layers_fused(layers, changed, land_k, land_v, blob, mk2, mv2, status2, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for l in range(L):
        for a, b in zip(layers[l], ref[l]):
            assert torch.equal(a, b), l
    # the same step again from the original stores, with one row too few to
    # move: the last layer that moves rows does not fit and is left as it was
    layers, blob, land_k, land_v, changed, moved = _rebuild_case(dev, D, dtype, L, seed=31)
    last = max(l for l in range(L) if moved[l] > 0)
    before = [t.clone() for t in layers[last]]
    small = torch.empty(sum(moved) - 1, D, dtype=dtype, device=dev)
    Kx.rebuild_layers_fused(layers, changed, land_k, land_v, blob, small, torch.empty_like(small), status2, err)
    torch.cuda.synchronize()
    assert int(err.item()) & N.DEVERR_CAPACITY
    for a, b in zip(layers[last], before):
        assert torch.equal(a, b)


def test_rebuild_refuses_malformed_plans(dev):
    """Host-side fault injection: corrupted plan blobs (a layer offset past the
    blob, more records than segments, a segment number out of range, landing
    rows past the landing buffer, more moved rows than the move buffer) are
    refused by the kernels' own checks -- error bit set, nothing written."""
    from wnw_b200 import kernels as Kx
    from wnw_b200 import native as N
    D, dtype = 64, torch.bfloat16
    lens = [300, 50, 900]
    ks, vs, base, cap = _slots(lens, 400, D, dtype, dev, seed=21)
    base_d = torch.from_numpy(base).to(dev)
    cap_d = torch.from_numpy(cap.astype(np.int32)).to(dev)
    land_k = torch.randn(64, D, device=dev).to(dtype)
    land_v = torch.randn(64, D, device=dev).to(dtype)
    move_k = torch.empty(1024, D, dtype=dtype, device=dev)
    move_v = torch.empty_like(move_k)
    status = torch.zeros(len(lens), dtype=torch.int32, device=dev)

    def good(seg=0, ls=0, ll=10):
        return (seg, lens[0], lens[0] - 20 + ll, ls, ll, [(100, 120)])

    cases = {}
    b = Kx.pack_plan([[good()]]).copy()
    b[0] = 10 ** 6
    cases["layer offset past the blob"] = (b, 1024)
    b = Kx.pack_plan([[good()]]).copy()
    b[b[0]] = 1000
    cases["more records than segments"] = (b, 1024)
    cases["segment out of range"] = (Kx.pack_plan([[good(seg=99)]]), 1024)
    cases["landing rows past the buffer"] = (Kx.pack_plan([[good(ls=60, ll=10)]]), 1024)
    cases["moved rows past the move buffer"] = (Kx.pack_plan([[good()]]), 8)
    for name, (blob, move_rows) in cases.items():
        snap_k, snap_v = ks.clone(), vs.clone()
        seg_len = torch.tensor(lens, dtype=torch.int32, device=dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        N.call("wnw_rebuild_segments", N.BF16, D, ks.data_ptr(), vs.data_ptr(), base_d.data_ptr(),
               seg_len.data_ptr(), cap_d.data_ptr(), len(lens), land_k.data_ptr(), land_v.data_ptr(),
               land_k.shape[0], torch.from_numpy(blob).to(dev).data_ptr(), int(blob.size), 0, move_k.data_ptr(),
               move_v.data_ptr(), move_rows, status.data_ptr(), err.data_ptr(), N.stream_ptr(None))
        torch.cuda.synchronize()
        assert int(err.item()) & (N.DEVERR_LEN_MISMATCH | N.DEVERR_CAPACITY), name
        assert torch.equal(ks, snap_k) and torch.equal(vs, snap_v), name
        assert seg_len.cpu().tolist() == lens, name
    # the same record, well formed, is applied
    seg_len = torch.tensor(lens, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    blob = Kx.pack_plan([[good()]])
    Kx.rebuild_layer(ks, vs, base_d, seg_len, cap_d, land_k, land_v, torch.from_numpy(blob).to(dev), 0,
                     move_k, move_v, status, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0 and seg_len.cpu().tolist()[0] == lens[0] - 10


def test_copy_segments_and_interleave_append_exact(dev):
    from wnw_b200 import kernels as Kx
    rng = np.random.default_rng(2)
    lens = rng.integers(0, 300, 37).astype(np.int64)
    cu = np.concatenate([[0], np.cumsum(lens)])
    old = torch.randn(int(cu[-1]), 64, dtype=torch.float16, device=dev)
    new = torch.randn(37, 64, dtype=torch.float16, device=dev)
    cu_d = torch.from_numpy(cu.astype(np.int32)).to(dev)
    out, cu_new = Kx.interleave_append(old, new, cu_d)
    ref, ref_cu = K.interleave_append(old.cpu().numpy(), new.cpu().numpy(), cu)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), ref) and np.array_equal(cu_new.cpu().numpy(), ref_cu)
    # packed -> slots -> packed round trip
    cap_base = torch.from_numpy((np.arange(37) * 320).astype(np.int64)).to(dev)
    sk = torch.zeros(37 * 320, 64, dtype=torch.float16, device=dev)
    sv = torch.zeros_like(sk)
    lens_d = torch.from_numpy(lens.astype(np.int32)).to(dev)
    src_base = torch.from_numpy(cu[:-1].astype(np.int64)).to(dev)
    Kx.copy_segments(old, old, src_base, sk, sv, cap_base, lens_d)
    back = torch.empty_like(old)
    Kx.copy_segments(sk, sv, cap_base, back, back, src_base, lens_d)
    torch.cuda.synchronize()
    assert torch.equal(back, old)
