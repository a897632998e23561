"""Tensor parallelism by kv head on two GPUs: each rank's ``B200WnWCache``
over its kv heads (NCCL score reduction) against the oracle cache over the
same heads (gloo score reduction), which the CPU suite already ties to the
single-process oracle and that to the reference's recorded trace: flat
layouts bit for bit, cu_seqlens and loaded sets exactly, attention outputs
within fp32 tolerance."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.golden.scenario import CACHE_SCENARIO, make_cache_inputs, make_config_dict

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device(f"cuda:{rank}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                           timeout=datetime.timedelta(seconds=120))
    try:
        q.put((rank, _checks(rank, world, dev)))
    except Exception as e:  # report; the other rank's next collective times out
        q.put((rank, repr(e)))
    finally:
        torch.cuda.synchronize()
        dist.destroy_process_group()


def _checks(rank, world, dev):
    from oracle.cache import OracleWnWCache
    from tests.test_gpu_cache import _packed_with_token
    from wnw_b200.cache import B200WnWCache
    from wnw_b200.config import WnWConfig
    from wnw_b200.tp import ScoreReducer, head_range, shard_config

    sc = CACHE_SCENARIO
    cfg = WnWConfig(**make_config_dict(sc))
    L, H, Hq, D, B = sc["L"], sc["Hkv"], sc["Hq"], sc["D"], sc["B"]
    G = Hq // H
    h0, h1 = head_range(rank, world, H)
    scfg = shard_config(cfg, rank, world, L, H, Hq)
    inp = make_cache_inputs(sc)
    gloo = dist.new_group(backend="gloo")
    ored = ScoreReducer(gloo)

    class TPOracle(OracleWnWCache):
        def decode_all_layers_done(self):
            self.score_accumulator[:] = ored(torch.from_numpy(self.score_accumulator.copy())).numpy()
            super().decode_all_layers_done()

    orc = TPOracle(scfg, L, h1 - h0, (h1 - h0) * G, D)
    gpu = B200WnWCache(scfg, L, h1 - h0, (h1 - h0) * G, D, dev, max_decode_tokens=3, score_reduce=ScoreReducer())
    orc.setup_audio(inp["audio_starts"], inp["audio_ends"], inp["pad"])
    gpu.setup_audio(torch.tensor(inp["audio_starts"]), torch.tensor(inp["audio_ends"]),
                    torch.tensor(inp["attention_mask"]))
    for l in range(L):
        ca = inp["class_a_scores"][l]
        ph = [r[h0:h1] for r in inp["per_head_scores"][l]]
        k = torch.from_numpy(inp["prefill_k"][l][:, h0:h1].copy())
        v = torch.from_numpy(inp["prefill_v"][l][:, h0:h1].copy())
        orc.prefill_after_attn(l, ca, ph, k, v)
        # the GPU cache sums the ranks' prefill scores: rank 0 carries the totals
        gca = [(x if rank == 0 else torch.zeros_like(x)).to(dev) if x is not None else None for x in ca]
        gpu.prefill_after_attn(l, gca, [[x.to(dev) if x is not None else None for x in r] for r in ph],
                               k.to(dev), v.to(dev))
    orc.prefill_all_layers_done()
    gpu.prefill_all_layers_done()
    assert [sorted(s) for s in gpu.loaded_segments] == [sorted(s) for s in orc.loaded_segments]
    changes = 0
    for t in range(sc["steps"]):
        for l in range(L):
            qf = torch.from_numpy(inp["dec_q"][t][l]).squeeze(2).reshape(B, H, G, D)[:, h0:h1].reshape(-1, G, D)
            k = torch.from_numpy(inp["dec_k"][t][l][:, h0:h1].copy())
            v = torch.from_numpy(inp["dec_v"][t][l][:, h0:h1].copy())
            orc.decode_before_attn(l, k, v)
            o_ref = orc.fused_decode_attention(l, qf, scale=D ** -0.5)
            kk, vv, cu, _ = gpu.decode_before_attn(l, k.to(dev), v.to(dev))
            o = gpu.fused_decode_attention(l, qf.to(dev), None, kk, vv, cu, D ** -0.5)
            np.testing.assert_allclose(o.cpu().numpy(), o_ref.numpy(), atol=1e-5, rtol=1e-5)
            pk, pv, pcu = _packed_with_token(gpu, l)
            assert np.array_equal(pcu, orc.cu(l)), (t, l)
            assert torch.equal(pk.cpu(), orc.layer_k[l]) and torch.equal(pv.cpu(), orc.layer_v[l]), (t, l)
        orc.decode_all_layers_done()
        gpu.decode_all_layers_done()
        assert gpu.last_topk == orc.last_topk, t
        assert [sorted(s) for s in gpu.loaded_segments] == [sorted(s) for s in orc.loaded_segments], t
        changes += bool(any(orc.last_to_load) or any(orc.last_to_evict))
    assert changes >= 3
    return "ok"


def test_two_gpu_tensor_parallel_cache_matches_oracle():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(world))
    for p in ps:
        p.join(timeout=120)
    assert res == {0: "ok", 1: "ok"}, res


def _oproj_ref(xs, ws):
    return sum(x.float().cpu() @ w.float().cpu().t() for x, w in zip(xs, ws))


def test_oproj_allreduce_single_rank():
    """world 1: the fused kernel is the o_proj GEMV (its own receive buffer)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from wnw_b200.tp import OprojAllReduce
    dev = torch.device("cuda:0")
    g = torch.Generator(device="cpu").manual_seed(3)
    for B, N, K in ((1, 3072, 1024), (3, 1000, 256), (8, 64, 4096)):
        x = torch.randn(B, K, generator=g).to(torch.bfloat16).to(dev)
        w = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16).to(dev)
        ex = OprojAllReduce(dev, N, batch=B)
        for _ in range(3):  # successive epochs reuse both receive parities
            y = ex(x, w)
        torch.cuda.synchronize()
        ex.check()
        ref = _oproj_ref([x], [w])
        np.testing.assert_allclose(y.float().cpu().numpy(), ref.numpy(), atol=2e-2, rtol=2e-2)
        ex.close()


def test_oproj_allreduce_reports_missing_peer():
    """A peer that never arrives: the wait runs out after its deadline, the
    kernel sets WNW_DEVERR_PEER_TIMEOUT and returns zeros, and the context
    stays usable (one GPU; the 'peer' is a second local buffer nobody fills)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    import ctypes as C
    from wnw_b200 import native as N
    dev = torch.device("cuda:0")
    B, Nout, K, world = 1, 512, 256, 2
    nch = N.lib.wnw_oproj_allreduce_chunks(Nout)
    bufs = [torch.zeros(2 * world * B * Nout + world * nch + 64, dtype=torch.float32, device=dev) for _ in range(2)]
    x = torch.ones(B, K, dtype=torch.bfloat16, device=dev)
    w = torch.ones(Nout, K, dtype=torch.bfloat16, device=dev)
    y = torch.full((B, Nout), 7.0, dtype=torch.bfloat16, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    a = N.OprojAllReduceArgs()
    a.dtype, a.batch, a.n_out, a.k_in, a.rank, a.world = N.BF16, B, Nout, K, 0, world
    a.recv_batch = B
    for p in range(world):
        a.recv[p] = bufs[p].data_ptr()
        a.flags[p] = bufs[p].data_ptr() + 4 * 2 * world * B * Nout
    a.x, a.w, a.y, a.epoch, a.timeout_ns, a.err = x.data_ptr(), w.data_ptr(), y.data_ptr(), 1, 20_000_000, err.data_ptr()
    N.check(N.lib.wnw_oproj_allreduce(C.byref(a), N.stream_ptr(None)))
    torch.cuda.synchronize()
    assert int(err.item()) & N.DEVERR_PEER_TIMEOUT
    assert torch.count_nonzero(y).item() == 0
    # the device is still usable
    z = torch.arange(10, device=dev).sum()
    assert int(z.item()) == 45


def _oproj_rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device(f"cuda:{rank}")
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                           timeout=datetime.timedelta(seconds=120))
    ex = None
    try:
        from wnw_b200.tp import OprojAllReduce
        B, Nout, K = 2, 3072, 512
        xs = [torch.randn(B, K, generator=torch.Generator().manual_seed(10 + r)).to(torch.bfloat16)
              for r in range(world)]
        ws = [(torch.randn(Nout, K, generator=torch.Generator().manual_seed(20 + r)) * 0.05).to(torch.bfloat16)
              for r in range(world)]
        ex = OprojAllReduce(dev, Nout, batch=B)
        x, w = xs[rank].to(dev), ws[rank].to(dev)
        for _ in range(5):
            y = ex(x, w)
        torch.cuda.synchronize()
        ex.check()
        ys = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(ys, y)
        assert all(torch.equal(ys[0], t) for t in ys), "ranks disagree"
        np.testing.assert_allclose(y.float().cpu().numpy(), _oproj_ref(xs, ws).numpy(), atol=3e-2, rtol=2e-2)
        q.put((rank, "ok"))
    except Exception as e:
        q.put((rank, repr(e)))
    finally:
        if ex is not None:
            ex.close()
        torch.cuda.synchronize()
        dist.destroy_process_group()


def test_two_gpu_oproj_allreduce():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_oproj_rank, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(world))
    for p in ps:
        p.join(timeout=120)
    assert res == {0: "ok", 1: "ok"}, res
