"""GPU test of the allocation-free decode-attention entry point.

``wnw_decode_attn_noalloc`` serves callers whose host owns all device memory
(a serving engine with a fixed memory budget, a plugin host that passes in
only its own buffers) and therefore cannot let this library call cudaMalloc:
its scratch lives in a fixed device array inside the library.  This test
calls it through the C ABI twice in a row and checks both results against the
regular entry point (which takes caller-allocated scratch), with the same
tolerance as the other bf16 attention tests, and checks the size limit.

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


def _case(dev, dtype, lens, G=4, D=128, cluster=8, seed=0):
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
    split = Kx.split_rows(dtype, D)
    t["work"] = torch.from_numpy(Kx.build_work_table(cap, split, cluster)).to(dev)
    t["scratch"] = Kx.AttnScratch(dev, t["work"].shape[0], G, D, S)
    t["err"] = torch.zeros(1, dtype=torch.int32, device=dev)
    t["args"] = Kx.make_attn_args(dtype, S, G, D, t["ks"], t["vs"], t["base"], t["len"], t["work"], cluster,
                                  D ** -0.5, t["scratch"], seg_cap=t["cap"], num_kv_heads=S)
    return t


def _call(name, t, out):
    from wnw_b200 import native as N
    a = t["args"]
    a.q, a.new_k, a.new_v, a.out = t["q"].data_ptr(), t["nk"].data_ptr(), t["nv"].data_ptr(), out.data_ptr()
    if name == "wnw_decode_attn_noalloc":
        a.err = t["err"].data_ptr()
    st = getattr(N.lib, name)(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    N.check(st, name)


@pytest.mark.parametrize("dtype,lens", [(torch.bfloat16, [15100, 2300, 1, 700, 129, 4097, 2300, 60]),
                                        (torch.float32, [3000, 64, 65, 1])])
def test_noalloc_matches_regular_entry_point_twice(dev, dtype, lens):
    t = _case(dev, dtype, lens)
    ref = torch.empty_like(t["q"])
    _call("wnw_decode_attn", t, ref)
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
    for _ in range(2):  # the static scratch keeps the last call's contents
        out = torch.full_like(t["q"], float("nan"))
        _call("wnw_decode_attn_noalloc", t, out)
        torch.cuda.synchronize()
        assert int(t["err"].item()) == 0 and int(t["scratch"].err.item()) == 0
        np.testing.assert_allclose(out.float().cpu().numpy(), ref.float().cpu().numpy(), atol=tol, rtol=tol)


def test_noalloc_rejects_oversized_requests(dev):
    from wnw_b200 import native as N
    t = _case(dev, torch.bfloat16, [100, 100])
    a = t["args"]
    a.q, a.out, a.err = t["q"].data_ptr(), t["q"].data_ptr(), t["err"].data_ptr()
    a.n_clusters = (1 << 20) // (4 * 130) + 1  # one cluster more than the static partial buffer holds
    st = N.lib.wnw_decode_attn_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert st == 3 and b"static scratch holds" in N.lib.wnw_last_error()
    a.n_clusters = t["work"].shape[0]
    a.num_segs = (1 << 16) + 1
    st = N.lib.wnw_decode_attn_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream)
    assert st == 3 and b"counters for" in N.lib.wnw_last_error()
