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
