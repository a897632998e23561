"""GPU test of the allocation-free decode-attention entry point.

``wnw_decode_attn_noalloc`` serves callers whose host owns all device memory
(a serving engine with a fixed memory budget, a plugin host that passes in
only its own buffers) and therefore cannot let this library call cudaMalloc:
its scratch lives in a fixed device array inside the library.  These tests
call it through the C ABI, twice in a row and interleaved with calls of other
sizes and dtypes, and check every result against the regular entry point
(which takes caller-allocated scratch).  Both run the same kernels on the same
work layout, so the outputs -- and, with scoring on, the class-A logits and
softmax statistics -- must be bit-identical.  The size limits are checked too.

The file name makes pytest collect it last; it needs no state from other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda:0")


def _case(dev, dtype, lens, G=4, D=128, sms=None, cluster=8, score=False, seed=0):
    """One layer's arguments.  With ``score``, segment 0 of every sample (two
    kv heads per sample) is a class-A segment whose audio rows [4, len - 60)
    get their logits and softmax statistics stored."""
    from wnw_b200 import kernels as Kx
    g = torch.Generator(device="cpu").manual_seed(seed)
    S = len(lens)
    cap = np.asarray(lens, np.int64) + 32
    cap_al = (cap + 15) // 16 * 16
    base = np.concatenate([[0], np.cumsum(cap_al)[:-1]]).astype(np.int64)
    rows = int(cap_al.sum())
    t = dict(
        ks=torch.randn(rows, D, generator=g).to(dtype).to(dev),
        vs=torch.randn(rows, D, generator=g).to(dtype).to(dev),
        q=torch.randn(S, G, D, generator=g).to(dtype).to(dev),
        nk=torch.randn(S, D, generator=g).to(dtype).to(dev),
        nv=torch.randn(S, D, generator=g).to(dtype).to(dev),
        base=torch.from_numpy(base).to(dev),
        len=torch.tensor(lens, dtype=torch.int32, device=dev),
        cap=torch.from_numpy(cap.astype(np.int32)).to(dev),
    )
    plan = Kx.uses_plan(dtype, D)
    t["work"] = Kx.AttnWork(dtype, D, cap, dev, sm_count=sms[0] if sms else None,
                            max_cluster=sms[1] if sms else None, split=None if plan else Kx.split_rows(dtype, D),
                            cluster_size=None if plan else cluster)
    t["scratch"] = Kx.AttnScratch(dev, t["work"].slots, G, D, S)
    t["err"] = torch.zeros(1, dtype=torch.int32, device=dev)
    sc = None
    if score:
        H = 2
        B = S // H
        a0 = [4] * B
        a1 = [max(4, lens[b * H] - 60) for b in range(B)]
        slot = [-1] * S
        offs = []
        o = 0
        for b in range(B):
            slot[b * H] = b
            offs.append(o)
            o += (a1[b] - a0[b]) * G
        sc = dict(slot=torch.tensor(slot, dtype=torch.int32, device=dev),
                  audio_start=torch.tensor(a0, dtype=torch.int32, device=dev),
                  audio_end=torch.tensor(a1, dtype=torch.int32, device=dev),
                  logits=torch.zeros(max(o, 1), dtype=torch.float32, device=dev),
                  logits_off=torch.tensor(offs, dtype=torch.int64, device=dev),
                  stats=torch.zeros(S * 2 * G, dtype=torch.float32, device=dev))
    t["score"] = sc
    t["args"] = Kx.make_attn_args(dtype, S, G, D, t["ks"], t["vs"], t["base"], t["len"], t["work"],
                                  D ** -0.5, t["scratch"], seg_cap=t["cap"], num_kv_heads=2 if score else S,
                                  score=sc)
    return t


def _call(name, t, out):
    """Run one entry point; returns copies of (out, logits, stats)."""
    from wnw_b200 import native as N
    a = t["args"]
    a.q, a.new_k, a.new_v, a.out = t["q"].data_ptr(), t["nk"].data_ptr(), t["nv"].data_ptr(), out.data_ptr()
    err = t["err"] if name == "wnw_decode_attn_noalloc" else t["scratch"].err
    a.err = err.data_ptr()
    sc = t["score"]
    if sc is not None:
        sc["logits"].fill_(float("nan"))
        sc["stats"].fill_(float("nan"))
    st = getattr(N.lib, name)(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    N.check(st, name)
    torch.cuda.synchronize()
    assert int(err.item()) == 0, name
    return (out.clone(),) + ((sc["logits"].clone(), sc["stats"].clone()) if sc is not None else ())


def _check(t):
    """The regular entry point once, then the allocation-free one twice in a
    row (the static scratch keeps the last call's contents): bit-identical."""
    ref = _call("wnw_decode_attn", t, torch.empty_like(t["q"]))
    for _ in range(2):
        got = _call("wnw_decode_attn_noalloc", t, torch.full_like(t["q"], float("nan")))
        for r, x in zip(ref, got):
            assert torch.equal(r, x)


@pytest.mark.parametrize("dtype,lens,sms,cluster,score", [
    # tensor-core kernel, class-A scoring on: the device's plan (a cluster
    # per segment, merged in distributed shared memory); and a plan for 6 SMs
    # in clusters of 2, where long segments span several clusters whose
    # partials go through the scratch and the combine kernel
    (torch.bfloat16, [15100, 2300, 1, 700, 129, 4097, 2300, 60], None, 8, True),
    (torch.bfloat16, [15100, 2300, 1, 700, 129, 4097, 2300, 60], (6, 2), 8, True),
    # CUDA-core kernel: clusters of 8 and the global counter merge
    (torch.float32, [3000, 64, 65, 1], None, 8, False),
])
def test_noalloc_bit_identical_to_regular_entry_point(dev, dtype, lens, sms, cluster, score):
    _check(_case(dev, dtype, lens, sms=sms, cluster=cluster, score=score))


def test_noalloc_clears_the_counters_each_call_uses(dev):
    """Calls of growing and shrinking segment counts, alternating dtypes
    (bf16 plans whose long segments go through cluster partials, fp32
    cluster tables with arrival counters): each starts from the scratch the
    previous call left and must still merge every segment's partials
    correctly."""
    cases = [(torch.bfloat16, [9000, 17]), (torch.float32, [3000, 5, 1200, 2, 800, 64, 4000, 3]),
             (torch.bfloat16, [5000] * 12 + [130, 7]), (torch.float32, [2500]),
             (torch.bfloat16, [12000, 64, 3000, 1])]
    for i, (dtype, lens) in enumerate(cases):
        _check(_case(dev, dtype, lens, sms=(5, 2) if dtype == torch.bfloat16 else None, cluster=4, seed=i))


def test_noalloc_rejects_oversized_requests(dev):
    from wnw_b200 import native as N
    t = _case(dev, torch.bfloat16, [100, 100])
    a = t["args"]
    a.q, a.out, a.err = t["q"].data_ptr(), t["q"].data_ptr(), t["err"].data_ptr()
    parts = a.plan_parts
    a.plan_parts = (1 << 20) // (4 * 130) + 1  # one partial more than the static partial buffer holds
    st = N.lib.wnw_decode_attn_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert st == 3 and b"static scratch holds" in N.lib.wnw_last_error()
    a.plan_parts = parts
    a.num_segs = (1 << 16) + 1
    st = N.lib.wnw_decode_attn_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert st == 3 and b"counters for" in N.lib.wnw_last_error()
