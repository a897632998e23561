"""Generate golden fixtures by EXECUTING the XMUDeepLIT/WnW reference on CPU.

Run in a container that has the reference checked out (its ``src``
directory named by ``WNW_REFERENCE_SRC``, by default ``reference/src`` beside
this repository)::

    python tests/golden/make_golden.py

The reference's Triton kernels run under ``TRITON_INTERPRET=1``.  Two shims
are needed to run its CUDA-oriented code on CPU (neither changes arithmetic):

* ``torch.cuda.device`` -> a null context (``src/common/kv/kernels.py:67``);
* ``pin_memory=True`` is dropped (``src/algorithms/wnw_cpp/code/cache.py:107``),
  and the C++ cache's planner output tensors are re-allocated before every plan,
  because on a CPU "device" ``.to(device)`` aliases them
  (``src/algorithms/wnw_cpp/code/cache.py:258-265``).

Outputs (all small, committed): ``kernels.npz``, ``cache_trace.npz``,
``cache_cpp_trace.npz``, ``planner.npz``, ``session_trace.json``,
``session_degqa_trace.json``, ``stats.json``, ``cache_cpp_dropin_trace.npz``, ``cache_trace_global.npz``,
``session_mean_text_trace.json`` (each session trace with its prefill K
layouts, ``*_prefill_k.npz``).
"""
from __future__ import annotations

import contextlib
import json
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"
os.environ["WNW_FUSED_ATTN"] = "1"
os.environ.setdefault("TORCH_EXTENSIONS_DIR", "/tmp/wnw_golden_ext")
REF = os.environ.get("WNW_REFERENCE_SRC", os.path.join(
    os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))), "reference", "src"))
sys.path.insert(0, REF)

import numpy as np  # noqa: E402
import torch  # noqa: E402

torch.cuda.device = lambda d: contextlib.nullcontext()
_orig_empty = torch.empty


def _empty_no_pin(*a, **kw):
    kw.pop("pin_memory", None)
    return _orig_empty(*a, **kw)


torch.empty = _empty_no_pin

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from tests.golden.scenario import (  # noqa: E402
    CACHE_SCENARIO, make_cache_inputs, make_config_dict, PLANNER_SCENARIOS,
    make_planner_inputs)


def gen_kernels():
    from common.kv.fused_attn import q1_decode_attn, q1_decode_attn_score
    from common.kv.kernels import interleave_append
    from algorithms.wnw.code.kernels import rebuild_append_kv, fused_score_accumulate
    g = torch.Generator().manual_seed(1234)
    out = {}
    # decode attention + fused scoring (fp32, B=2, Hkv=4, G=4, D=64)
    B, Hkv, G, D = 2, 4, 4, 64
    lens = torch.randint(40, 300, (B * Hkv,), generator=g)
    cu = torch.zeros(B * Hkv + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(lens, 0)
    T = int(cu[-1])
    q = torch.randn(B * Hkv, G, D, generator=g)
    k = torch.randn(T, D, generator=g)
    v = torch.randn(T, D, generator=g)
    scale = D ** -0.5
    o = q1_decode_attn(q, k, v, cu, scale)
    ca = torch.tensor([1, 0, 1, 0], dtype=torch.int32)
    a_s = torch.tensor([3, 10], dtype=torch.int32)
    a_e = torch.tensor([33, 38], dtype=torch.int32)
    off = torch.tensor([0, 30, 58], dtype=torch.int32)
    acc = torch.zeros(58)
    o2 = q1_decode_attn_score(q, k, v, cu, scale, ca, Hkv, a_s, a_e, acc, off)
    out.update(attn_q=q.numpy(), attn_k=k.numpy(), attn_v=v.numpy(), attn_cu=cu.numpy(),
               attn_scale=np.float64(scale), attn_out=o.numpy(), attn_score_out=o2.numpy(),
               attn_ca=ca.numpy(), attn_as=a_s.numpy(), attn_ae=a_e.numpy(), attn_off=off.numpy(),
               attn_acc=acc.numpy())
    # interleave append
    n = 6
    lens = torch.randint(0, 9, (n,), generator=g)
    cu_old = torch.zeros(n + 1, dtype=torch.int32)
    cu_old[1:] = torch.cumsum(lens, 0)
    old = torch.randn(int(cu_old[-1]), 16, generator=g)
    new = torch.randn(n, 16, generator=g)
    cu_new = cu_old + torch.arange(n + 1, dtype=torch.int32)
    app = interleave_append(old, new, cu_old, cu_new)
    out.update(app_old=old.numpy(), app_new=new.numpy(), app_cu_old=cu_old.numpy(),
               app_out=app.numpy())
    # rebuild (evict sorted ranges, splice loads, append)
    n = 5
    old_lens = [20, 12, 7, 30, 9]
    cu_old = torch.tensor([0] + list(np.cumsum(old_lens)), dtype=torch.int32)
    old_k = torch.randn(int(cu_old[-1]), 16, generator=g)
    old_v = torch.randn(int(cu_old[-1]), 16, generator=g)
    new_k = torch.randn(n, 16, generator=g)
    new_v = torch.randn(n, 16, generator=g)
    evicts = {0: [(4, 8), (12, 15)], 2: [(0, 7)], 3: [(10, 20)]}
    loads = {0: 5, 1: 3, 3: 6}
    ev_off, ev_s, ev_e = [0], [], []
    load_starts, load_lens, new_lens = [], [], []
    cursor = 0
    for s in range(n):
        for a, b in evicts.get(s, []):
            ev_s.append(a); ev_e.append(b)
        ev_off.append(len(ev_s))
        ln = loads.get(s, 0)
        load_starts.append(cursor if ln else -1)
        load_lens.append(ln)
        cursor += ln
        new_lens.append(old_lens[s] - sum(b - a for a, b in evicts.get(s, [])) + ln + 1)
    load_k = torch.randn(cursor, 16, generator=g)
    load_v = torch.randn(cursor, 16, generator=g)
    cu_new = torch.tensor([0] + list(np.cumsum(new_lens)), dtype=torch.int32)
    t = lambda x: torch.tensor(x, dtype=torch.int32)  # noqa: E731
    rk, rv = rebuild_append_kv(old_k, old_v, new_k, new_v, load_k, load_v, cu_old, cu_new,
                               t(load_starts), t(load_lens), t(ev_off), t(ev_s), t(ev_e), 2)
    out.update(rb_old_k=old_k.numpy(), rb_old_v=old_v.numpy(), rb_new_k=new_k.numpy(),
               rb_new_v=new_v.numpy(), rb_load_k=load_k.numpy(), rb_load_v=load_v.numpy(),
               rb_cu_old=cu_old.numpy(), rb_cu_new=cu_new.numpy(),
               rb_load_starts=np.array(load_starts, np.int32), rb_load_lens=np.array(load_lens, np.int32),
               rb_ev_off=np.array(ev_off, np.int32), rb_ev_s=np.array(ev_s, np.int32),
               rb_ev_e=np.array(ev_e, np.int32), rb_out_k=rk.numpy(), rb_out_v=rv.numpy())
    # non-fused scoring for group sizes 4 (h4), 1 (h1) and 3 (torch fallback)
    for nh in (4, 1, 3):
        ns, D = 3, 32
        lens = [50, 70, 40]
        cu = np.array([0] + list(np.cumsum(lens)))
        Kt = torch.randn(int(cu[-1]), D, generator=g)
        Q = torch.randn(ns, nh, D, generator=g)
        ss = t(cu[:-1].tolist()); se = t(cu[1:].tolist())
        a_s = t([2, 5, 0]); a_e = t([30, 60, 40])
        offs = t([0, 28, 83, 123])
        acc = torch.rand(123, generator=g)
        acc0 = acc.clone()
        fused_score_accumulate(Q, Kt, ss, se, a_s, a_e, acc, offs)
        out.update({f"fs{nh}_Q": Q.numpy(), f"fs{nh}_K": Kt.numpy(), f"fs{nh}_cu": cu,
                    f"fs{nh}_as": a_s.numpy(), f"fs{nh}_ae": a_e.numpy(), f"fs{nh}_off": offs.numpy(),
                    f"fs{nh}_acc0": acc0.numpy(), f"fs{nh}_acc": acc.numpy()})
    np.savez_compressed(os.path.join(HERE, "kernels.npz"), **out)


def _digest(a):
    """SHA-256 of a contiguous fp32 array's bytes (layouts are exact copies)."""
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(a, dtype=np.float32).tobytes()).hexdigest()


class _Adapter:
    """Minimal stand-in: the cache only stores its adapter."""


def run_cache_trace(cache_cls, cpp, sc=CACHE_SCENARIO):
    from algorithms.wnw.code.config import WnWConfig
    cfg = WnWConfig(**make_config_dict(sc))
    cache = cache_cls(config=cfg, num_layers=sc["L"], num_kv_heads=sc["Hkv"],
                      num_q_heads=sc["Hq"], head_dim=sc["D"], device=torch.device("cpu"),
                      adapter=_Adapter())
    inp = make_cache_inputs(sc)
    cache.setup_audio(torch.tensor(inp["audio_starts"]), torch.tensor(inp["audio_ends"]),
                      torch.tensor(inp["attention_mask"]))
    for l in range(sc["L"]):
        cache.prefill_after_attn(l, inp["class_a_scores"][l], inp["per_head_scores"][l],
                                 torch.from_numpy(inp["prefill_k"][l]), torch.from_numpy(inp["prefill_v"][l]))
    cache.prefill_all_layers_done()
    if cpp:
        orig = cache._finalize_pending_plan

        def _fin():
            L, S = sc["L"], sc["B"] * sc["Hkv"]
            cache._cpp_load_starts_2d = torch.empty(L, S, dtype=torch.int32)
            cache._cpp_load_lens_2d = torch.empty(L, S, dtype=torch.int32)
            cache._cpp_cu_new_2d = torch.empty(L, S + 1, dtype=torch.int32)
            cache._cpp_new_lens_2d = torch.empty(L, S, dtype=torch.int32)
            cache._cpp_evict_offsets_2d = torch.empty(L, S + 1, dtype=torch.int32)
            cache._cpp_evict_max = torch.empty(L, dtype=torch.int32)
            cache._cpp_evict_layer_ptr = torch.empty(L + 1, dtype=torch.int32)
            return orig()
        cache._finalize_pending_plan = _fin
    rec = {}
    rec["prefill_cu"] = np.stack([cache.cu_seqlens_k[l].numpy() for l in range(sc["L"])])
    rec["prefill_loaded"] = np.array([sorted(s) for s in cache.loaded_segments], dtype=object)
    for l in range(sc["L"]):
        rec[f"prefill_k{l}"] = cache.layer_k[l].numpy()
        rec[f"prefill_v{l}"] = cache.layer_v[l].numpy()
    G = sc["Hq"] // sc["Hkv"]
    for t in range(sc["steps"]):
        for l in range(sc["L"]):
            q, k, v = (torch.from_numpy(inp[n][t][l]) for n in ("dec_q", "dec_k", "dec_v"))
            K_, V_, cu, mk = cache.decode_before_attn(l, k, v)
            q_flat = q.squeeze(2).reshape(sc["B"], sc["Hkv"], G, sc["D"]).reshape(-1, G, sc["D"])
            o = cache.fused_decode_attention(l, q_flat, q, K_, V_, cu, sc["D"] ** -0.5)
            rec[f"s{t}_l{l}_out"] = o.numpy()
            rec[f"s{t}_l{l}_cu"] = cu.numpy().copy()
            rec[f"s{t}_l{l}_khash"] = np.array(_digest(K_.numpy()))
            rec[f"s{t}_l{l}_vhash"] = np.array(_digest(V_.numpy()))
            if t == sc["steps"] - 1:
                rec[f"s{t}_l{l}_k"] = K_.numpy().copy()
                rec[f"s{t}_l{l}_v"] = V_.numpy().copy()
        if not cpp:
            rec[f"s{t}_scores"] = cache.score_accumulator.numpy().copy()
        cache.decode_all_layers_done()
        if cpp:
            rec[f"s{t}_scores"] = np.zeros(0, np.float32)
        rec[f"s{t}_loaded"] = np.array(
            [sorted(cache._planner.get_loaded_segments(b)) if cpp else sorted(cache.loaded_segments[b])
             for b in range(sc["B"])], dtype=object)
    run_cache_trace.last_cache = cache
    return rec


def gen_cache_traces():
    from algorithms.wnw.code.cache import WnWCache
    rec = run_cache_trace(WnWCache, cpp=False)
    np.savez_compressed(os.path.join(HERE, "cache_trace.npz"), **rec)
    try:
        from algorithms.wnw_cpp.code.cache import WnWCppCache
        rec2 = run_cache_trace(WnWCppCache, cpp=True)
        np.savez_compressed(os.path.join(HERE, "cache_cpp_trace.npz"), **rec2)
    except Exception as e:  # the C++ JIT needs a compiler; report and continue
        print("C++ cache trace skipped:", e)


def _jsonable(x):
    if isinstance(x, dict):
        return {k: _jsonable(v) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return [_jsonable(v) for v in x]
    if isinstance(x, (np.integer,)):
        return int(x)
    if isinstance(x, (np.floating,)):
        return float(x)
    return x


def gen_stats():
    """InferenceStats as the reference records them: (1) its InferenceStats
    driven by a scripted call sequence, (2) its Python cache's stats after the
    seeded cache scenario (prefill offload, initial loads, per-step loads, the
    interval snapshots).  GPU-memory fields are None here (no CUDA)."""
    from common.monitoring.inference_stats import InferenceStats
    st = InferenceStats(torch.device("cpu"), interval=2)
    st.reset(3)

    def snap(step=-1):
        return [{"step": step, "b": b, "x": b * 10 + max(step, 0)} for b in range(3)]

    st.record_prefill_before(snap)
    st.record_prefill_before(snap)  # guarded: once
    st.record_cpu_gpu_transfer(0, g2c_tokens=7, g2c_bytes=70)
    st.record_cpu_gpu_transfer(2, c2g_tokens=3, c2g_bytes=30)
    st.record_prefill(snap)
    for step in range(1, 6):
        st.record_cpu_gpu_transfer(step % 3, c2g_tokens=step, c2g_bytes=step * 11)
        st.record_cpu_gpu_transfer(1, c2g_tokens=0)  # all-zero: no event
        st.flush_decode_step(step)
        if step % st.interval == 0:
            st.record_decode(step, snap)
    scripted = st.get_all_stats()
    from algorithms.wnw.code.cache import WnWCache
    run_cache_trace(WnWCache, cpp=False)
    cache_stats = run_cache_trace.last_cache.stats.get_all_stats()
    with open(os.path.join(HERE, "stats.json"), "w") as f:
        json.dump(_jsonable({"scripted": scripted, "cache_trace": cache_stats}), f)


def gen_dropin():
    """The reference's own C++-planner cache (WnWCppCache) run with OUR
    Planner class in place of its pybind11 module: the same seeded trace,
    recorded without the big layout arrays, to be compared with
    cache_cpp_trace.npz (the reference's planner) by the CPU tests."""
    import types
    import algorithms.wnw_cpp.code._ext as ext
    from algorithms.wnw_cpp.code.cache import WnWCppCache
    from wnw_b200.planner import Planner
    ext.get_planner_module = lambda: types.SimpleNamespace(Planner=Planner)
    rec = run_cache_trace(WnWCppCache, cpp=True)
    keep = {k: v for k, v in rec.items() if not (k.startswith("prefill_k") or k.startswith("prefill_v")
                                                  or k.endswith("_k") or k.endswith("_v"))}
    np.savez_compressed(os.path.join(HERE, "cache_cpp_dropin_trace.npz"), **keep)


def gen_global_trace():
    """The reference's Python cache on the seeded scenario with the global
    per-head prefill top-k (cache.py:1141-1150) instead of the per-segment
    rule; layouts as digests only (no raw arrays)."""
    from algorithms.wnw.code.cache import WnWCache
    from tests.golden.scenario import GLOBAL_TOPK_SCENARIO
    rec = run_cache_trace(WnWCache, cpp=False, sc=GLOBAL_TOPK_SCENARIO)
    for k in list(rec):
        if k.startswith("prefill_k") or k.startswith("prefill_v") or k.endswith("_k") or k.endswith("_v"):
            arr = rec.pop(k)
            if k.startswith("prefill_k"):
                rec[k.replace("prefill_k", "prefill_khash")] = np.array(_digest(arr))
    np.savez_compressed(os.path.join(HERE, "cache_trace_global.npz"), **rec)


def gen_planner():
    from algorithms.wnw_cpp.code._ext import get_planner_module
    mod = get_planner_module()
    out = {}
    for i, ps in enumerate(PLANNER_SCENARIOS):
        inp = make_planner_inputs(ps)
        P = mod.Planner(ps["L"], ps["H"], ps["B"], 1)
        P.set_config(ps["top_k"], ps["lag"])
        P.set_seg_count(inp["seg_count"])
        for b in range(ps["B"]):
            P.set_chunk_to_segs(b, torch.tensor(inp["c2s_flat"][b], dtype=torch.int32),
                                torch.tensor(inp["c2s_off"][b], dtype=torch.int32))
        for l in range(ps["L"]):
            P.set_class_b(l, torch.tensor(inp["class_b"][l], dtype=torch.int32))
        P.set_restore_meta(*(torch.tensor(inp[n], dtype=torch.int32) for n in ("cpu_s", "cpu_e", "gpu_s", "gpu_e")))
        for b in range(ps["B"]):
            P.set_loaded(b, torch.tensor(inp["loaded"][b], dtype=torch.int32))
        P.set_seq_lens(torch.tensor(inp["seq_lens"], dtype=torch.int32))
        L, S = ps["L"], ps["B"] * ps["H"]
        for step, (tk, toff) in enumerate(inp["steps"]):
            bufs = [torch.full((L, S), -7, dtype=torch.int32), torch.full((L, S), -7, dtype=torch.int32),
                    torch.full((L, S + 1), -7, dtype=torch.int32), torch.full((L, S), -7, dtype=torch.int32),
                    torch.full((L, S + 1), -7, dtype=torch.int32), torch.full((L,), -7, dtype=torch.int32),
                    torch.full((L + 1,), -7, dtype=torch.int32)]
            ch, tot, evs, eve, rng = P.compute_and_prepare(
                torch.tensor(tk, dtype=torch.int32), torch.tensor(toff, dtype=torch.int32), *bufs)
            pre = f"p{i}_s{step}_"
            out[pre + "change"] = np.int32(ch)
            out[pre + "total"] = np.int32(tot)
            for name, buf in zip(("load_starts", "load_lens", "cu_new", "new_lens", "evict_offsets",
                                  "evict_max", "evict_layer_ptr"), bufs):
                out[pre + name] = buf.numpy()
            out[pre + "ev_starts"] = evs.numpy()
            out[pre + "ev_ends"] = eve.numpy()
            out[pre + "cpu_ranges"] = rng.numpy()
            out[pre + "loaded"] = np.array([sorted(P.get_loaded_segments(b)) for b in range(ps["B"])],
                                           dtype=object)
    np.savez_compressed(os.path.join(HERE, "planner.npz"), **out)


def _tiny_adapter(ss):
    """The reference's BaseModelAdapter completed for a tiny random-init
    Llama whose audio span is fixed by the scenario."""
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    from common.adapters.base import BaseModelAdapter

    class TinyAdapter(BaseModelAdapter):
        name = "tiny"

        def load(self, *a, **k): raise NotImplementedError
        def _build_inputs(self, *a, **k): raise NotImplementedError
        def get_decoder_layers(self, model): return model.model.layers
        def get_text_config(self, model): return model.config
        def locate_audio_tokens(self, input_ids, attention_mask, processor):
            B = input_ids.shape[0]
            return (torch.full((B,), ss["audio_start"], dtype=torch.int64),
                    torch.full((B,), ss["audio_end"], dtype=torch.int64))
        def compute_qkv(self, attn, h):
            B, S, _ = h.shape
            hd = attn.head_dim
            return (attn.q_proj(h).view(B, S, -1, hd).transpose(1, 2),
                    attn.k_proj(h).view(B, S, -1, hd).transpose(1, 2),
                    attn.v_proj(h).view(B, S, -1, hd).transpose(1, 2))
        def apply_rope(self, q, k, pe, attn):
            return apply_rotary_pos_emb(q, k, *pe)
        def attention_meta(self, attn):
            c = attn.config
            return {"head_dim": attn.head_dim, "num_kv_heads": c.num_key_value_heads,
                    "num_kv_groups": c.num_attention_heads // c.num_key_value_heads,
                    "scaling": attn.scaling, "layer_idx": attn.layer_idx}
        def prepare_for_inference(self, model): return {}
        def restore_after_inference(self, model, state): pass
        def generate(self, model, inputs, **kw): return model.generate(**inputs, **kw)
        def get_logits(self, model, outputs): return outputs.logits
        def get_text_model(self, model): return model
        def get_audio_token_id(self, model): return 0
        def build_analysis_inputs(self, *a, **k): raise NotImplementedError

    return TinyAdapter()


def gen_session_trace(ss=None, name="session_trace.json"):
    """Drive the reference WnWSession over a tiny random-init Llama (fp32) and
    record the hook call sequence and the greedy tokens."""
    from transformers import LlamaConfig, LlamaForCausalLM
    from algorithms.wnw.code.config import WnWConfig
    from algorithms.wnw.code.cache import WnWCache
    from algorithms.wnw.code.session import WnWSession
    from tests.golden.scenario import SESSION_SCENARIO, make_tiny_llama_config, session_inputs
    ss = ss or SESSION_SCENARIO

    adapter = _tiny_adapter(ss)
    calls = []
    prefill_hash, prefill_k = [], []

    class TracingCache(WnWCache):
        def prefill_after_attn(self, l, a, p, k, v):
            calls.append(["prefill_after_attn", l, list(k.shape)])
            return super().prefill_after_attn(l, a, p, k, v)

        def prefill_all_layers_done(self):
            calls.append(["prefill_all_layers_done"])
            r = super().prefill_all_layers_done()
            prefill_hash.extend(_digest(self.layer_k[l].numpy()) for l in range(self.num_layers))
            prefill_k.extend(self.layer_k[l].numpy().copy() for l in range(self.num_layers))
            return r

        def decode_before_attn(self, l, k, v):
            calls.append(["decode_before_attn", l, list(k.shape)])
            return super().decode_before_attn(l, k, v)

        def fused_decode_attention(self, l, q_flat, q, k_flat, v_flat, cu_k, scale):
            calls.append(["fused_decode_attention", l, list(q_flat.shape), list(q.shape), float(scale)])
            return super().fused_decode_attention(l, q_flat, q, k_flat, v_flat, cu_k, scale)

        def decode_all_layers_done(self):
            calls.append(["decode_all_layers_done"])
            return super().decode_all_layers_done()

    torch.manual_seed(ss["seed"])
    mcfg = LlamaConfig(**make_tiny_llama_config(ss))
    model = LlamaForCausalLM(mcfg).eval()
    cfg = WnWConfig(**make_config_dict(ss))
    cache = TracingCache(config=cfg, num_layers=ss["L"], num_kv_heads=ss["Hkv"], num_q_heads=ss["Hq"],
                         head_dim=ss["D"], device=torch.device("cpu"), adapter=adapter)
    ids = session_inputs(ss)
    with WnWSession(model, adapter, cache) as sess:
        sess.setup_audio(ids)
        with torch.no_grad():
            out = sess.generate({"input_ids": ids}, max_new_tokens=ss["new_tokens"], do_sample=False)
    res = {"calls": calls, "tokens": out.tolist(),
           "loaded": [sorted(s) for s in cache.loaded_segments], "stats": _jsonable(sess.get_stats()),
           "prefill_khash": prefill_hash}
    np.savez_compressed(os.path.join(HERE, name.replace(".json", "_prefill_k.npz")),
                        **{f"l{l}": k for l, k in enumerate(prefill_k)})
    with open(os.path.join(HERE, name), "w") as f:
        json.dump(res, f)


def gen_degqa_trace():
    """The reference's GQA -> MHA path: its config expansion
    (analysis/wnw_config/scripts/expand_wnw_config.py) on the session
    scenario's config, then its degqa_model on the same tiny Llama and its
    session in MHA mode (one kv head per q head) with the expanded config:
    hook calls, greedy tokens, loaded sets."""
    from analysis.wnw_config.scripts.expand_wnw_config import expand_config
    from common.adapters.degqa import degqa_model
    from transformers import LlamaConfig, LlamaForCausalLM
    from algorithms.wnw.code.config import WnWConfig
    from algorithms.wnw.code.cache import WnWCache
    from algorithms.wnw.code.session import WnWSession
    from tests.golden.scenario import SESSION_SCENARIO as ss, make_tiny_llama_config, session_inputs
    from wnw_b200.config import WnWConfig as OurConfig

    cfg_in = OurConfig(**make_config_dict(ss)).to_dict()
    cfg_out = expand_config(cfg_in, ss["L"], ss["Hkv"], ss["Hq"])
    torch.manual_seed(ss["seed"])
    model = LlamaForCausalLM(LlamaConfig(**make_tiny_llama_config(ss))).eval()
    ad = _tiny_adapter(ss)
    degqa_model(model, ad)
    kw = dict(make_config_dict(ss), class_b=cfg_out["heads"]["class_b"],
              retention_ratios=cfg_out["heads"]["retention_ratios"], num_kv_heads=ss["Hq"])
    calls = []

    class TracingCache(WnWCache):
        def decode_before_attn(self, l, k, v):
            calls.append(["decode_before_attn", l, list(k.shape)])
            return super().decode_before_attn(l, k, v)

        def decode_all_layers_done(self):
            calls.append(["decode_all_layers_done"])
            return super().decode_all_layers_done()

    cache = TracingCache(config=WnWConfig(**kw), num_layers=ss["L"], num_kv_heads=ss["Hq"], num_q_heads=ss["Hq"],
                         head_dim=ss["D"], device=torch.device("cpu"), adapter=ad)
    ids = session_inputs(ss)
    with WnWSession(model, ad, cache) as sess:
        sess.setup_audio(ids)
        with torch.no_grad():
            out = sess.generate({"input_ids": ids}, max_new_tokens=ss["new_tokens"], do_sample=False)
    res = {"config_in": cfg_in, "config_out": cfg_out, "calls": calls, "tokens": out.tolist(),
           "loaded": [sorted(s) for s in cache.loaded_segments]}
    with open(os.path.join(HERE, "session_degqa_trace.json"), "w") as f:
        json.dump(res, f)


if __name__ == "__main__":
    which = sys.argv[1:] or ["kernels", "cache", "planner", "session", "degqa", "stats", "dropin", "global",
                             "mean_text"]
    if "kernels" in which:
        gen_kernels()
    if "cache" in which:
        gen_cache_traces()
    if "planner" in which:
        gen_planner()
    if "session" in which:
        gen_session_trace()
    if "mean_text" in which:
        from tests.golden.scenario import MEAN_TEXT_SESSION_SCENARIO
        gen_session_trace(MEAN_TEXT_SESSION_SCENARIO, "session_mean_text_trace.json")
    if "degqa" in which:
        gen_degqa_trace()
    if "stats" in which:
        gen_stats()
    if "dropin" in which:
        gen_dropin()
    if "global" in which:
        gen_global_trace()
    print("golden fixtures written to", HERE)
