"""Tensor parallelism by kv head, on CPU: head re-indexing of the config, the
rank-order score reduction (gloo, world size 2), and a 2-rank run of the
oracle cache whose per-rank outputs and chunk selections equal the
single-process run's."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from wnw_b200.config import WnWConfig
from wnw_b200.tp import ScoreReducer, head_range, shard_config, slice_flat, slice_kv
from tests.golden.scenario import CACHE_SCENARIO, make_cache_inputs, make_config_dict


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_config_reindexes_heads():
    sc = CACHE_SCENARIO
    cfg = WnWConfig(**make_config_dict(sc))
    L, H, Hq = sc["L"], sc["Hkv"], sc["Hq"]
    for world in (1, 2, 4):
        for r in range(world):
            h0, h1 = head_range(r, world, H)
            s = shard_config(cfg, r, world, L, H, Hq)
            assert (s.num_kv_heads, s.num_q_heads) == (h1 - h0, (h1 - h0) * (Hq // H))
            for l in range(L):
                for h in range(h0, h1):
                    assert s.is_class_b(l, h - h0) == cfg.is_class_b(l, h)
                    assert s.is_class_a_kv_head(l, h - h0) == cfg.is_class_a_kv_head(l, h)
                    assert s.get_retention(l, h - h0) == cfg.get_retention(l, h)
                G = Hq // H
                for q in range(h0 * G, h1 * G):
                    assert s.is_class_a(l, q - h0 * G) == cfg.is_class_a(l, q)
    with pytest.raises(ValueError):
        head_range(0, 3, 4)


def test_slices():
    x = torch.arange(2 * 4 * 3).reshape(2, 4, 3)
    assert torch.equal(slice_kv(x, 1, 3), x[:, 1:3])
    f = x.reshape(8, 3)
    assert torch.equal(slice_flat(f, 1, 3, 4), x[:, 1:3].reshape(-1, 3))


def _run(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q.put((rank, _tp_checks(rank, world)))
    except Exception as e:  # report, do not hang the other rank
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def _tp_checks(rank, world):
    from oracle.cache import OracleWnWCache
    red = ScoreReducer()
    # 1. rank-order sum, identical on every rank
    x = torch.full((5,), 0.1 * (rank + 1), dtype=torch.float32)
    y = red(x)
    ys = [torch.empty_like(y) for _ in range(world)]
    dist.all_gather(ys, y)
    assert all(torch.equal(ys[0], t) for t in ys)
    want = torch.full((5,), 0.1, dtype=torch.float32)
    for r in range(1, world):
        want = want + torch.full((5,), 0.1 * (r + 1), dtype=torch.float32)
    assert torch.equal(y, want)

    # 2. the 2-rank oracle run equals the single-process run head for head
    sc = CACHE_SCENARIO
    cfg = WnWConfig(**make_config_dict(sc))
    L, H, Hq, D, B = sc["L"], sc["Hkv"], sc["Hq"], sc["D"], sc["B"]
    G = Hq // H
    h0, h1 = head_range(rank, world, H)
    inp = make_cache_inputs(sc)

    class TPOracle(OracleWnWCache):
        def decode_all_layers_done(self):
            self.score_accumulator[:] = red(torch.from_numpy(self.score_accumulator.copy())).numpy()
            super().decode_all_layers_done()

    full = OracleWnWCache(cfg, L, H, Hq, D)
    part = TPOracle(shard_config(cfg, rank, world, L, H, Hq), L, h1 - h0, (h1 - h0) * G, D)
    for c, lo, hi in ((full, 0, H), (part, h0, h1)):
        c.setup_audio(inp["audio_starts"], inp["audio_ends"], inp["pad"])
        for l in range(L):
            # prefill class-A scores are the layer totals on every rank here
            c.prefill_after_attn(l, inp["class_a_scores"][l], [r[lo:hi] for r in inp["per_head_scores"][l]],
                                 torch.from_numpy(inp["prefill_k"][l][:, lo:hi].copy()),
                                 torch.from_numpy(inp["prefill_v"][l][:, lo:hi].copy()))
        c.prefill_all_layers_done()
    changes = 0
    for t in range(sc["steps"]):
        for l in range(L):
            qf = torch.from_numpy(inp["dec_q"][t][l]).squeeze(2).reshape(B, H, G, D)
            k = torch.from_numpy(inp["dec_k"][t][l])
            v = torch.from_numpy(inp["dec_v"][t][l])
            full.decode_before_attn(l, k, v)
            o_full = full.fused_decode_attention(l, qf.reshape(-1, G, D), scale=D ** -0.5)
            part.decode_before_attn(l, k[:, h0:h1].contiguous(), v[:, h0:h1].contiguous())
            o_part = part.fused_decode_attention(l, qf[:, h0:h1].reshape(-1, G, D), scale=D ** -0.5)
            assert torch.equal(o_part, slice_flat(o_full, h0, h1, H)), (t, l)
            assert np.array_equal(np.diff(part.cu(l)), slice_flat(torch.from_numpy(np.diff(full.cu(l))),
                                                                   h0, h1, H).numpy()), (t, l)
        full.decode_all_layers_done()
        part.decode_all_layers_done()
        assert part.last_topk == full.last_topk, t
        assert [sorted(s) for s in part.loaded_segments] == [sorted(s) for s in full.loaded_segments], t
        changes += bool(any(full.last_to_load) or any(full.last_to_evict))
    assert changes >= 3
    return "ok"


def test_two_rank_oracle_matches_single_process():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_run, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res


def _dead_peer(rank, world, port, q):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        q.put((1, "left"))
        q.close()
        q.join_thread()  # the message is out before the process dies
        os._exit(0)  # leaves between steps, before the score reduction
    t0 = __import__("time").perf_counter()
    try:
        ScoreReducer()(torch.ones(4))
        q.put((0, "no error"))
    except Exception:
        q.put((0, f"raised after {__import__('time').perf_counter() - t0:.1f} s"))


def test_dead_rank_fails_the_score_reduction():
    """Failure detection on the host: a tensor-parallel rank that leaves
    between steps makes the survivors' next score reduction raise (a closed
    peer or the process group's timeout) instead of hanging."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_dead_peer, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=60) for _ in range(world))
    for p in ps:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert res[1] == "left"
    assert res[0].startswith("raised"), res
