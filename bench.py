#!/usr/bin/env python
"""Benchmark of the WnW decode hot path on B200 (one JSON line on rank 0).

Workload: Voxtral-Mini-3B-shaped decoder, random
init, bf16, batch 1 -- 30 layers, hidden 3072, 32 q / 8 kv heads, head_dim
128, RoPE theta 1e8 (MLP 8192 and vocab 131072: the installed transformers
Voxtral text-config defaults).  Prompt = 4 text tokens + 15,000 audio
embeddings ~ N(0, 0.02) + 60 text tokens; 30 % of the kv heads are class A
(seeded choice), the rest class B with chunk = segment = 128 tokens, top-16,
eviction lag 1; class B keeps the 64 non-audio tokens, one audio token per
segment (retention 0) and every decoded token.

A step is one decode step of the hot path over all 30 layers: per layer the
pending chunk rebuild and one fused decode-attention launch (attention +
append + class-A logits), then length advance, class-A score finalisation,
chunk top-k, the host planner and the per-layer H2D fetch of the chosen
chunks.  Its per-layer q/k/v inputs come from the random-init decoder itself:
the model is run once (untimed) through the session and every decode step's
q/k/v is recorded; the timed legs replay them into a freshly prefilled cache,
so they do exactly the work the model run did.

* value -- decode tokens/s with the inputs resident in HBM;
* e2e   -- the same through the Python hook API with each step's q/k/v copied
           from pinned host memory (one copy per step) and each step's
           attention outputs copied back (one copy; bytes per step reported);
* roofline -- the decode-attention kernel: algorithmic bytes (K+V rows
           attended + q in + o out + class-A logits) / CUDA-event time;
* cpu_baseline -- the CPU oracle (numpy/torch restatement of the reference's
           path) replaying a bounded sample of the same steps.

``--impl reference`` times that CPU path alone (rank 0; other ranks exit).
With torchrun, every rank runs its own replica (request sharding, weak
scaling); value = all ranks' tokens / max-over-ranks time.  ``--parallel tp``
instead shards the one request by kv head (wnw_b200.tp): rank r owns kv heads
[r*8/N, (r+1)*8/N) of every layer, the step adds each layer's o_proj partial
(the rank's query heads x its slice of a random o_proj weight) and its NCCL
all-reduce, and the class-A scores are summed over the ranks before top-k
(strong scaling; value = the request's tokens / max-over-ranks time).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

MODEL = dict(L=30, hidden=3072, Hq=32, Hkv=8, D=128, inter=8192, vocab=131072, theta=1e8)
PROMPT = dict(sink=4, audio=15000, tail=60)
WNW = dict(frac_a=0.30, chunk=128, top_k=16, lag=1, retention=0.0, seed=1234)
METRIC = "decode tokens/s and varlen-attn HBM GB/s (frac of peak) at 1/2/4/8 B200"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-steps", type=int, default=3, help="oracle steps in the bounded CPU sample")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--profile", action="store_true", help="short run for ncu (no clocks, no CPU leg)")
    ap.add_argument("--parallel", default="replicas", choices=["replicas", "tp"],
                    help="N>1: independent per-request replicas, or one request sharded by kv head")
    ap.add_argument("--tp-exchange", default="fused", choices=["fused", "nccl"],
                    help="tensor parallel: o_proj GEMV + all-reduce as one NVLink kernel, or cuBLAS + NCCL")
    ap.add_argument("--config", type=int, default=2, choices=[2, 3, 4],
                    help="BASELINE config of the step: 2 (the default line; q/k/v recorded from the random-init "
                         "decoder), 3 or 4 (their shapes with seeded synthetic q/k/v)")
    ap.add_argument("--synthetic", action="store_true",
                    help="config 2 with seeded synthetic inputs instead of the model run (as configs 3 and 4)")
    ap.add_argument("--depth", type=int, default=None, help="synthetic configs: only this many layers")
    ap.add_argument("--mode", default="step", choices=["step", "attn", "sweep"],
                    help="step: the decode hot path (the default line); attn: decode attention alone on "
                         "--class-a / --class-b segment lengths; sweep: the BASELINE config-5 kernel grid")
    ap.add_argument("--class-a", type=int, default=15100, help="attn mode: rows of each class-A segment")
    ap.add_argument("--class-b", type=int, default=2300, help="attn mode: rows of each class-B segment")
    ap.add_argument("--n-class-a", type=int, default=2, help="attn mode: class-A segments of the 8 kv heads")
    ap.add_argument("--layers", type=int, default=8, help="attn mode: distinct layers launched round-robin")
    ap.add_argument("--reps", type=int, default=20, help="attn / sweep modes: timed passes over the layers")
    ap.add_argument("--batch", default="1,16,64,256", help="sweep mode: batch sizes")
    ap.add_argument("--ctx", default="1024,8192,32768,131072", help="sweep mode: context lengths")
    ap.add_argument("--frac-a", default="0.1,0.3,0.5,1.0", help="sweep mode: class-A fractions of the kv heads")
    ap.add_argument("--retained", default="0.1,0.25,0.5,1.0", help="sweep mode: class-B retained fractions")
    ap.add_argument("--max-gb", type=float, default=48.0, help="sweep mode: skip cells above this many GB per GPU")
    ap.add_argument("--check", action="store_true", help="attn / sweep modes: compare sampled segments with "
                                                          "a torch fp32 reference")
    ap.add_argument("--max-cluster", type=int, default=None,
                    help="attn mode: plan with clusters of at most this many CTAs (default: the device's largest)")
    ap.add_argument("--sm-count", type=int, default=None,
                    help="attn mode: plan for this many CTA slots (default: the device's resident clusters)")
    ap.add_argument("--trace", action="store_true",
                    help="attn mode: load libwnw_b200_trace.so (python -m wnw_b200.build --trace) and report the "
                         "kernel's per-CTA phase timestamps")
    ap.add_argument("--isolated", action="store_true", help="attn mode --trace: one launch at a time")
    ap.add_argument("--no-rebuild-ahead", action="store_true",
                    help="rebuild each changed layer on the compute stream before its attention "
                         "(B200WnWCache(rebuild_ahead=False)) instead of ahead on its own stream")
    ap.add_argument("--tier", default="host", choices=["host", "hbm"],
                    help="step mode: where the timed legs keep the offloaded rows (host: pinned host memory, the "
                         "headline; hbm: device memory, to profile that tier)")
    ap.add_argument("--vs-reference", action="store_true",
                    help="attn mode: also time the reference's own GPU kernels (baseline/_ref) on the same layers")
    return ap.parse_args()


# ------------------------------------------------------------------ set-up
def wnw_config_fields():
    """The WnWConfig fields of the workload (the reference's config schema)."""
    L, H, Hq = MODEL["L"], MODEL["Hkv"], MODEL["Hq"]
    G = Hq // H
    rng = np.random.default_rng(WNW["seed"])
    n_a = round(WNW["frac_a"] * L * H)
    a_kv = sorted(rng.choice(L * H, size=n_a, replace=False).tolist())
    class_a = [(g // H) * Hq + (g % H) * G + j for g in a_kv for j in range(G)]
    class_b = [g for g in range(L * H) if g not in set(a_kv)]
    ret = [None if g in set(a_kv) else WNW["retention"] for g in range(L * H)]
    return dict(chunk_size_s=float(WNW["chunk"]), overlap_s=0.0, token_rate=1.0, class_a=class_a,
                class_b=class_b, retention_ratios=ret, top_k_chunks=WNW["top_k"], eviction_lag=WNW["lag"],
                prefill_score_mode="last", num_layers=L, num_kv_heads=H, num_q_heads=Hq)


def wnw_config():
    from wnw_b200.config import WnWConfig
    return WnWConfig(**wnw_config_fields())


def make_model(dev, seed):
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=MODEL["vocab"], hidden_size=MODEL["hidden"], intermediate_size=MODEL["inter"],
                      num_hidden_layers=MODEL["L"], num_attention_heads=MODEL["Hq"],
                      num_key_value_heads=MODEL["Hkv"], head_dim=MODEL["D"], max_position_embeddings=131072,
                      rope_parameters={"rope_theta": MODEL["theta"], "rope_type": "default"}, rms_norm_eps=1e-5)
    torch.manual_seed(seed)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(dev):
            model = LlamaForCausalLM(cfg).eval()
    finally:
        torch.set_default_dtype(prev)
    return model


class Recorder:
    """Cache mix-in that keeps the hook inputs of a model run."""

    def prefill_after_attn(self, l, ca, ph, k, v):
        self.rec_prefill.append((l, [x.clone() if x is not None else None for x in ca],
                                 [[x.clone() if x is not None else None for x in r] for r in ph], k.clone(),
                                 v.clone()))
        return super().prefill_after_attn(l, ca, ph, k, v)

    def decode_before_attn(self, l, k, v):
        if l == 0:
            self.rec_steps.append([None] * self.num_layers)
        self.rec_steps[-1][l] = [None, k.clone(), v.clone()]
        return super().decode_before_attn(l, k, v)

    def fused_decode_attention(self, l, q_flat, q, k_flat, v_flat, cu_k, scale):
        self.rec_steps[-1][l][0] = q_flat.clone()
        self.rec_scale = scale
        return super().fused_decode_attention(l, q_flat, q, k_flat, v_flat, cu_k, scale)


def reference_modules():
    """(session module, WnWCache, WnWConfig, BaseModelAdapter) of the
    reference's offline install in baseline/_ref, its session in the fused
    attention mode (WNW_FUSED_ATTN=1)."""
    import importlib
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "algorithms")):
        raise RuntimeError("baseline/_ref (offline install of the reference) not present")
    os.environ["WNW_FUSED_ATTN"] = "1"
    if ref not in sys.path:
        sys.path.insert(0, ref)
    sess = importlib.import_module("algorithms.wnw.code.session")
    sess._FUSED_ATTN = True  # read once, at the module's import
    return (sess, importlib.import_module("algorithms.wnw.code.cache").WnWCache,
            importlib.import_module("algorithms.wnw.code.config").WnWConfig,
            importlib.import_module("common.adapters.base").BaseModelAdapter)


def reference_adapter(base_cls, audio_start, audio_end):
    """The reference's BaseModelAdapter completed for the random-init Llama
    decoder, with the audio span given explicitly (no audio encoder)."""
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb

    class BenchLlamaAdapter(base_cls):
        name = "bench_llama"

        def load(self, *a, **k): raise NotImplementedError
        def _build_inputs(self, *a, **k): raise NotImplementedError
        def get_decoder_layers(self, model): return model.model.layers
        def get_text_config(self, model): return model.config

        def locate_audio_tokens(self, input_ids, attention_mask, processor):
            B = input_ids.shape[0]
            return (torch.full((B,), audio_start, dtype=torch.int64, device=input_ids.device),
                    torch.full((B,), audio_end, dtype=torch.int64, device=input_ids.device))

        def compute_qkv(self, attn, h):
            B, S, _ = h.shape
            hd = attn.head_dim
            return (attn.q_proj(h).view(B, S, -1, hd).transpose(1, 2),
                    attn.k_proj(h).view(B, S, -1, hd).transpose(1, 2),
                    attn.v_proj(h).view(B, S, -1, hd).transpose(1, 2))

        def apply_rope(self, q, k, pe, attn): return apply_rotary_pos_emb(q, k, *pe)

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

    return BenchLlamaAdapter()


def record(dev, n_steps, seed, reference=False):
    """Run the random-init decoder through the session: prefill + n_steps
    greedy decode steps; return the recorded hook inputs and model timing.
    ``reference``: through the reference's own session and cache (its
    offline install in baseline/_ref) instead of this package's, so that the
    reference arm runs none of this package's code."""
    if reference:
        sess_mod, CacheCls, CfgCls, base = reference_modules()
        cfg = CfgCls(**wnw_config_fields())
        Session = sess_mod.WnWSession
    else:
        from wnw_b200.cache import B200WnWCache as CacheCls
        from wnw_b200.session import WnWSession as Session
        cfg = wnw_config()

    class RecCache(Recorder, CacheCls):
        pass

    model = make_model(dev, seed)
    S0 = PROMPT["sink"] + PROMPT["audio"] + PROMPT["tail"]
    a0, a1 = PROMPT["sink"], PROMPT["sink"] + PROMPT["audio"]
    if reference:
        cache = RecCache(cfg, MODEL["L"], MODEL["Hkv"], MODEL["Hq"], MODEL["D"], dev, None)
    else:
        cache = RecCache(cfg, MODEL["L"], MODEL["Hkv"], MODEL["Hq"], MODEL["D"], dev, max_decode_tokens=n_steps + 8)
    cache.rec_prefill, cache.rec_steps = [], []
    g = torch.Generator(device=dev).manual_seed(seed)
    ids = torch.randint(1, MODEL["vocab"], (1, S0), device=dev, generator=g)
    with torch.no_grad():
        emb = model.get_input_embeddings()(ids)
        emb[:, a0:a1] = (torch.randn(1, a1 - a0, MODEL["hidden"], device=dev, generator=g) * 0.02).to(emb.dtype)
    if reference:
        adapter = reference_adapter(base, a0, a1)
    else:
        from wnw_b200.adapters import LlamaFamilyAdapter
        adapter = LlamaFamilyAdapter(a0, a1)
    times = []
    with Session(model, adapter, cache) as sess, torch.no_grad():
        sess.setup_audio(ids)
        out = model(inputs_embeds=emb, past_key_values=cache, use_cache=True, logits_to_keep=1)
        tok = out.logits[:, -1:].argmax(-1)
        for i in range(n_steps):
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record()
            out = model(input_ids=tok, past_key_values=cache, use_cache=True)
            tok = out.logits[:, -1:].argmax(-1)
            t1.record()
            times.append((t0, t1))
    torch.cuda.synchronize()
    ms = [a.elapsed_time(b) for a, b in times[2:]] or [float("nan")]
    rec = dict(cfg=cfg, prefill=cache.rec_prefill, steps=cache.rec_steps, scale=cache.rec_scale,
               audio=(a0, a1), S0=S0, model_ms=statistics.median(ms))
    del model, cache, out
    torch.cuda.empty_cache()
    return rec


# BASELINE configs 3 and 4: their shapes, with seeded synthetic inputs
SYNTH = {
    3: dict(name="qwen2.5-omni-7b-thinker-shaped", L=28, Hkv=4, Hq=28, D=128, hidden=3584, B=32, median=6000,
            sigma=0.5, clip=(1000, 30000), class_a_kv=(0, 1), retention=0.25, chunk=128, top_k=8, lag=1, seed=33,
            note="batch 32, lognormal prompts (median 6k, sigma 0.5, clipped [1k, 30k]) left-padded, 50 % class-A kv "
                 "heads, class-B retention 0.25"),
    2: dict(name="voxtral-mini-3b-shaped", L=30, Hkv=8, Hq=32, D=128, hidden=3072, B=1, S=15064, tail=60,
            class_a_kv=(0, 1), retention=0.0, chunk=128, top_k=16, lag=1, seed=22,
            note="batch 1, 15,064-token prompt (15,000 audio), 25 % class-A kv heads, class-B retention 0"),
    4: dict(name="voxtral-small-24b-shaped", L=40, Hkv=8, Hq=32, D=128, hidden=5120, B=2, S=120064,
            class_a_kv=(0, 1), retention=0.05, chunk=128, top_k=32, lag=1, seed=44,
            note="batch 2 at a 120,064-token context, 25 % class-A kv heads, class-B retention 0.05, class-B "
                 "chunks offloaded to pinned host memory, top-32"),
}


def use_config(n, synthetic=False, layers=None):
    """Point the workload globals at BASELINE config ``n`` (config 2 with
    ``synthetic``: its shapes with seeded inputs instead of a model run);
    ``layers`` shortens a synthetic config to that many layers."""
    if n in SYNTH and layers:
        SYNTH[n]["L"] = min(SYNTH[n]["L"], layers)
    if n in SYNTH and (n != 2 or synthetic):
        c = SYNTH[n]
        MODEL.update(L=c["L"], Hkv=c["Hkv"], Hq=c["Hq"], D=c["D"], hidden=c["hidden"])
        WNW.update(chunk=c["chunk"], top_k=c["top_k"], lag=c["lag"], retention=c["retention"])


def synthetic_record(dev, n_steps, n, cfg_cls=None):
    """Config 3 / 4 inputs, seeded: prefill K/V ~ N(0, 1) per layer (on the
    device), prefill scores without exact ties, and per step and layer q/k/v
    ~ N(0, 1).  Same structure as ``record``'s (no model run).  ``cfg_cls``:
    the WnWConfig class to build (this package's by default)."""
    if cfg_cls is None:
        from wnw_b200.config import WnWConfig as cfg_cls
    WnWConfig = cfg_cls
    c = SYNTH[n]
    L, H, Hq, D, B = c["L"], c["Hkv"], c["Hq"], c["D"], c["B"]
    G = Hq // H
    rng = np.random.default_rng(c["seed"])
    if n == 3:
        lens = np.clip(np.round(np.exp(rng.normal(np.log(c["median"]), c["sigma"], B))), *c["clip"]).astype(int)
        S = int(lens.max())
        pad = [int(S - x) for x in lens]
        starts, ends = [p + 4 for p in pad], [S - 30] * B
    else:
        S, pad = c["S"], [0] * B
        starts, ends = [4] * B, [S - c.get("tail", 160)] * B
    cfg = WnWConfig(chunk_size_s=float(c["chunk"]), overlap_s=0.0, token_rate=1.0,
                    class_a=[l * Hq + h * G + j for l in range(L) for h in c["class_a_kv"] for j in range(G)],
                    class_b=[l * H + h for l in range(L) for h in range(H) if h not in c["class_a_kv"]],
                    retention_ratios=[None if h in c["class_a_kv"] else c["retention"] for l in range(L)
                                      for h in range(H)],
                    top_k_chunks=c["top_k"], eviction_lag=c["lag"], prefill_score_mode="last", num_layers=L,
                    num_kv_heads=H, num_q_heads=Hq)
    g = torch.Generator(device=dev).manual_seed(c["seed"])
    n_audio = [e - b for b, e in zip(starts, ends)]
    distinct = lambda m: (torch.randperm(m, generator=g, device=dev).to(torch.float32) / m)  # noqa: E731
    prefill = []
    for l in range(L):
        k = torch.randn(B, H, S, D, generator=g, device=dev, dtype=torch.bfloat16)
        v = torch.randn(B, H, S, D, generator=g, device=dev, dtype=torch.bfloat16)
        ca = [distinct(n_audio[b]) for b in range(B)]
        ph = [[None if h in c["class_a_kv"] else distinct(n_audio[b]) for h in range(H)] for b in range(B)]
        prefill.append((l, ca, ph, k, v))
    steps = [[(torch.randn(B * H, G, D, generator=g, device=dev, dtype=torch.bfloat16),
               torch.randn(B, H, 1, D, generator=g, device=dev, dtype=torch.bfloat16),
               torch.randn(B, H, 1, D, generator=g, device=dev, dtype=torch.bfloat16)) for _ in range(L)]
             for _ in range(n_steps)]
    mask = torch.ones(B, S, dtype=torch.int64)
    for b in range(B):
        mask[b, :pad[b]] = 0
    return dict(cfg=cfg, prefill=prefill, steps=steps, scale=D ** -0.5, audio=(starts, ends, mask, pad), S0=S,
                model_ms=None, batch=B)


class Shard:
    """The slice of the hot path one rank runs: kv heads [h0, h1) of every
    layer (all of them for replicas), plus -- tensor parallel -- the o_proj
    slice of those heads' query heads and the NCCL group of the exchanges."""

    def __init__(self, dev, rank=0, world=1, tp=False, seed=0, exchange="fused", batch=1):
        from wnw_b200.tp import OprojAllReduce, head_range
        self.tp, self.rank, self.world = tp, rank, world
        H, G, D = MODEL["Hkv"], MODEL["Hq"] // MODEL["Hkv"], MODEL["D"]
        self.h0, self.h1 = head_range(rank, world, H) if tp else (0, H)
        self.Hkv = self.h1 - self.h0
        self.Hq = self.Hkv * G
        self.wo = None
        if tp:
            g = torch.Generator(device=dev).manual_seed(seed + 17 * rank)
            self.wo = [(torch.randn(MODEL["hidden"], self.Hq * D, device=dev, generator=g) * 0.02).to(torch.bfloat16)
                       for _ in range(MODEL["L"])]
        self.batch = batch
        self.ex = OprojAllReduce(dev, MODEL["hidden"], batch=batch) if tp and exchange == "fused" else None

    def close(self):
        if self.ex is not None:
            self.ex.close()
            self.ex = None

    def cfg(self, cfg):
        from wnw_b200.tp import shard_config
        if not self.tp:
            return cfg
        return shard_config(cfg, self.rank, self.world, MODEL["L"], MODEL["Hkv"], MODEL["Hq"])

    def score_reduce(self):
        from wnw_b200.tp import ScoreReducer
        return ScoreReducer() if self.tp and self.world > 1 else None

    def prefill(self, ca, ph, k, v):
        """This rank's prefill hook inputs.  The recorded class-A scores are
        the layer totals; under tensor parallelism the cache sums the ranks'
        prefill scores, so rank 0 carries the totals and the others zeros."""
        if not self.tp:
            return ca, ph, k, v
        if self.rank:
            ca = [torch.zeros_like(x) if x is not None else None for x in ca]
        return ca, [r[self.h0:self.h1] for r in ph], k[:, self.h0:self.h1], v[:, self.h0:self.h1]

    def step_inputs(self, steps):
        """Per step and layer (q_flat, k, v) of this rank's heads, contiguous."""
        from wnw_b200.tp import slice_flat
        if not self.tp:
            return steps
        H = MODEL["Hkv"]
        return [[(slice_flat(q, self.h0, self.h1, H).contiguous(), k[:, self.h0:self.h1].contiguous(),
                  v[:, self.h0:self.h1].contiguous()) for q, k, v in st] for st in steps]

    def o_proj(self, l, out):
        """The layer's row-parallel o_proj: this rank's partial sum, all-reduced."""
        if not self.tp:
            return out
        if self.ex is not None:  # one kernel: GEMV + all-reduce over NVLink peer memory
            return self.ex(out.reshape(self.batch, -1), self.wo[l])
        y = out.reshape(self.batch, -1) @ self.wo[l].t()
        if self.world > 1:
            torch.distributed.all_reduce(y)
        return y


PREFILL_MS = []  # prefill-side compression time of every cache built (ms)
REBUILD_AHEAD = [True]  # B200WnWCache(rebuild_ahead=...); --no-rebuild-ahead for comparison


def fresh_cache(rec, dev, n_steps, shard=None, tier="host"):
    from wnw_b200.cache import B200WnWCache
    shard = shard or Shard(dev)
    c = B200WnWCache(shard.cfg(rec["cfg"]), MODEL["L"], shard.Hkv, shard.Hq, MODEL["D"], dev,
                     max_decode_tokens=n_steps + 8, score_reduce=shard.score_reduce(), offload_tier=tier,
                     rebuild_ahead=REBUILD_AHEAD[0])
    if len(rec["audio"]) == 2:
        a0, a1 = rec["audio"]
        c.setup_audio(torch.tensor([a0]), torch.tensor([a1]), None)
    else:
        c.setup_audio(torch.tensor(rec["audio"][0]), torch.tensor(rec["audio"][1]), rec["audio"][2])
    torch.cuda.synchronize()
    t = time.perf_counter()
    for l, ca, ph, k, v in rec["prefill"]:
        c.prefill_after_attn(l, *shard.prefill(ca, ph, k, v))
    c.prefill_all_layers_done()
    torch.cuda.synchronize()
    PREFILL_MS.append((time.perf_counter() - t) * 1e3)
    return c


def algorithmic_bytes(cache, l, extra_rows=1):
    """Per decode-attention launch: K+V rows attended, q in + o out, and the
    class-A logit traffic (8 B per audio token per class-A segment: fp32
    written here, read back by the score kernel)."""
    S = cache.batch_size * cache.num_kv_heads
    G, D, es = cache.num_kv_groups, cache.head_dim, 2
    rows = int((cache._len_host[l] + extra_rows).sum())
    H = cache.num_kv_heads
    audio = sum(cache._audio_ends_list[s // H] - cache._audio_starts_list[s // H]
                for s, slot in enumerate(cache._slot_host[l]) if slot >= 0)
    return rows * D * es * 2 + S * G * D * es * 2 + 8 * audio


def attention_replay(cache, qs, reps):
    """Decode-attention launches of all layers back to back on the final
    state of the timed run (no append), timed with CUDA events on the
    launching stream; the 30-layer working set (~770 MB) exceeds L2, so each
    launch reads its layer from HBM."""
    from wnw_b200 import kernels as Kx
    from wnw_b200 import native as N
    L = cache.num_layers
    torch.cuda.synchronize()  # the fetch and rebuilds issued ahead for the next step are done
    st = torch.cuda.current_stream()
    outs = [torch.empty_like(q) for q in qs]
    args = [cache._attn_args[l][2] for l in range(L)]
    for a in args:  # nothing between the launches writes a layer's rows or lengths
        a.flags = N.ATTN_ROWS_READY
    for l in range(L):
        Kx.launch_attn(args[l], qs[l], None, None, outs[l], st.cuda_stream)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        for l in range(L):
            Kx.launch_attn(args[l], qs[l], None, None, outs[l], st.cuda_stream)
    e1.record()
    torch.cuda.synchronize()
    n = reps * L
    us = e0.elapsed_time(e1) * 1e3 / n
    nbytes = sum(algorithmic_bytes(cache, l, extra_rows=0) for l in range(L)) / L
    return us, nbytes, n


def run_value(rec, dev, K, W, shard=None, tier="host"):
    """Timed replay with the inputs resident in HBM."""
    from wnw_b200 import kernels as Kx
    shard = shard or Shard(dev)
    cache = fresh_cache(rec, dev, K + W, shard, tier)
    steps, scale, L = shard.step_inputs(rec["steps"]), rec["scale"], MODEL["L"]

    selections = []  # per step: (top-k chunks, loaded segments) of sample 0

    def one(i):
        for l in range(L):
            q, k, v = steps[i][l]
            kk, vv, cu, _ = cache.decode_before_attn(l, k, v)
            shard.o_proj(l, cache.fused_decode_attention(l, q, None, kk, vv, cu, scale))
        cache.decode_all_layers_done()
        selections.append((list(cache.last_topk[0]), sorted(cache.loaded_segments[0])))

    for i in range(W):
        one(i)
    fetched = 0
    launches0 = Kx.LAUNCHES[0]
    wait0 = cache.host_wait_s
    torch.cuda.synchronize()
    if shard.world > 1:
        torch.distributed.barrier()
        torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    wall0 = time.time()
    t0.record()
    torch.cuda.nvtx.range_push("wnw_timed")
    for i in range(W, W + K):
        one(i)
        fetched += cache._fetched_rows
    torch.cuda.nvtx.range_pop()
    t1.record()
    torch.cuda.synchronize()
    wall1 = time.time()
    if shard.world > 1:
        torch.distributed.barrier()
        torch.cuda.synchronize()
    launches = Kx.LAUNCHES[0] - launches0
    host_wait_ms = (cache.host_wait_s - wait0) * 1e3
    total_ms = t0.elapsed_time(t1)
    us, nbytes, n = attention_replay(cache, [steps[W + K - 1][l][0] for l in range(L)], reps=10)
    return dict(ms=total_ms, attn_us=us, attn_bytes=nbytes, attn_n=n, launches=launches, fetched_rows=fetched,
                window=(wall0, wall1), selections=selections, host_wait_ms=host_wait_ms)


def run_e2e(rec, dev, K, W, shard=None, tier="host"):
    """Hook API with host buffers: per step one H2D copy of all layers' q/k/v
    from pinned memory and one D2H copy of all layers' outputs (attention
    outputs; under tensor parallelism the all-reduced o_proj rows)."""
    shard = shard or Shard(dev)
    cache = fresh_cache(rec, dev, K + W, shard, tier)
    steps, scale, L = shard.step_inputs(rec["steps"]), rec["scale"], MODEL["L"]
    shapes = [tuple(x.shape) for x in steps[0][0]]
    sizes = [math.prod(sh) for sh in shapes]
    per_layer = sum(sizes)
    host_in = [torch.empty(L * per_layer, dtype=torch.bfloat16).pin_memory() for _ in range(W + K)]
    for i in range(W + K):
        host_in[i].copy_(torch.cat([x.reshape(-1).cpu() for l in range(L) for x in steps[i][l]]))
    dev_in = torch.empty(L * per_layer, dtype=torch.bfloat16, device=dev)
    views = []
    for l in range(L):
        o, v = l * per_layer, []
        for sh, n in zip(shapes, sizes):
            v.append(dev_in[o:o + n].view(sh))
            o += n
        views.append(v)
    out_shape = (shard.batch, MODEL["hidden"]) if shard.tp else shapes[0]
    dev_out = torch.empty((L,) + tuple(out_shape), dtype=torch.bfloat16, device=dev)
    host_out = torch.empty_like(dev_out, device="cpu").pin_memory()
    in_bytes = host_in[0].numel() * host_in[0].element_size()
    out_bytes = host_out.numel() * host_out.element_size()

    from wnw_b200 import kernels as Kx
    from wnw_b200 import native as N
    host_ptr = [Kx.host_device_pointer(h) for h in host_in]

    def one(i):
        # the step's inputs: a kernel copy from mapped pinned memory (SM loads
        # share the host link with the zero-copy fetch; a copy-engine transfer
        # can queue behind it for the whole fetch)
        N.call("wnw_copy_mapped", dev_in.data_ptr(), host_ptr[i], in_bytes, 32,
               torch._C._cuda_getCurrentRawStream(dev.index if dev.index is not None else 0))
        Kx.LAUNCHES[0] += 1
        outs = []
        for l in range(L):
            q, k, v = views[l]
            kk, vv, cu, _ = cache.decode_before_attn(l, k, v)
            outs.append(shard.o_proj(l, cache.fused_decode_attention(l, q, None, kk, vv, cu, scale)))
        cache.decode_all_layers_done()
        torch.stack(outs, out=dev_out)
        host_out.copy_(dev_out, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    for i in range(W):
        one(i)
    torch.cuda.synchronize()
    if shard.world > 1:
        torch.distributed.barrier()
        torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(W, W + K):
        one(i)
    e1.record()
    torch.cuda.synchronize()
    if shard.world > 1:
        torch.distributed.barrier()
        torch.cuda.synchronize()
    return dict(ms=e0.elapsed_time(e1), in_bytes=in_bytes, out_bytes=out_bytes)


def run_reference_gpu(rec, dev, K, W):
    """The reference's own cache (its Python planner and Triton kernels, from
    the offline install in baseline/_ref) on this GPU, driven by the same
    replay -- for comparison only (the reference arm times its CPU path)."""
    import importlib
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "algorithms")):
        return {"unavailable": "baseline/_ref (offline install of the reference) not present"}
    sys.path.insert(0, ref)
    try:
        RefCache = importlib.import_module("algorithms.wnw.code.cache").WnWCache
        RefConfig = importlib.import_module("algorithms.wnw.code.config").WnWConfig
        c0 = rec["cfg"]
        rcfg = RefConfig(chunk_size_s=c0.chunk_size_s, overlap_s=c0.overlap_s, token_rate=c0.token_rate,
                         class_a=list(c0.class_a), class_b=list(c0.class_b),
                         retention_ratios=list(c0.retention_ratios), top_k_chunks=c0.top_k_chunks,
                         eviction_lag=c0.eviction_lag, prefill_score_mode=c0.prefill_score_mode,
                         prefill_global_topk=c0.prefill_global_topk, num_layers=c0.num_layers,
                         num_kv_heads=c0.num_kv_heads, num_q_heads=c0.num_q_heads)
        cache = RefCache(rcfg, MODEL["L"], MODEL["Hkv"], MODEL["Hq"], MODEL["D"], dev, None)
        # the reference's own selection each step (cache.py:632-649): its
        # chunk scores (fp32 cumsum on the GPU) and the top-k it takes
        picks = []
        orig = cache._compute_chunk_changes

        def capture(b, scores):
            if b == 0:  # its chunk scores, formed as it forms them (cache.py:636-640)
                prefix = torch.zeros(scores.shape[0] + 1, dtype=torch.float32, device=scores.device)
                torch.cumsum(scores, dim=0, out=prefix[1:])
                cs = (prefix[cache._chunk_ends_t[b]] - prefix[cache._chunk_starts_t[b]]) / cache._chunk_lens_t[b]
                picks.append((cs.float().cpu().numpy(), None))
            return orig(b, scores)

        orig_topk = cache._compute_chunk_changes_from_topk

        def capture_topk(b, topk_chunks):
            if b == 0 and picks and picks[-1][1] is None:
                picks[-1] = (picks[-1][0], sorted(int(c) for c in topk_chunks))
            return orig_topk(b, topk_chunks)

        cache._compute_chunk_changes = capture
        cache._compute_chunk_changes_from_topk = capture_topk
        ref_loaded = []
        a0, a1 = rec["audio"]
        cache.setup_audio(torch.tensor([a0]), torch.tensor([a1]), None)
        torch.cuda.synchronize()
        t = time.perf_counter()
        for l, ca, ph, k, v in rec["prefill"]:
            cache.prefill_after_attn(l, ca, ph, k, v)
        cache.prefill_all_layers_done()
        torch.cuda.synchronize()
        pre = (time.perf_counter() - t) * 1e3
        picks.clear()  # the prefill's own selection; decode steps from here
        steps, scale, L = rec["steps"], rec["scale"], MODEL["L"]

        def one(i):
            for l in range(L):
                q, k, v = steps[i][l]
                kk, vv, cu, _ = cache.decode_before_attn(l, k, v)
                cache.fused_decode_attention(l, q, None, kk, vv, cu, scale)
            cache.decode_all_layers_done()
            ref_loaded.append(sorted(cache.loaded_segments[0]))

        for i in range(W):
            one(i)
        n = min(K, 16)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(W, W + n):
            one(i)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / n
        for i in range(W + n, min(W + K, len(steps))):  # the rest of the replay, untimed, for the selections
            one(i)
        torch.cuda.synchronize()
        return {"value": 1e3 / ms, "unit": "tokens/s", "ms_per_step": ms, "steps": n, "prefill_compress_ms": pre,
                "how": "the reference's WnWCache (Python planner, Triton kernels; fused attention + scoring) "
                       "from baseline/_ref, same replay on this GPU; informational",
                "_picks": picks, "_loaded": ref_loaded}
    except Exception as e:  # report, never fail the bench on the comparison leg
        return {"unavailable": f"{type(e).__name__}: {e}"[:300]}


def selection_agreement(ours, ref_picks, ref_loaded, top_k, tie_rel=1e-5):
    """Step-by-step agreement of this cache's chunk selection with the
    reference's own GPU cache on the same replay: top-k sets and loaded
    segment sets, and, where the top-k differ, whether the reference's own
    scores have a near tie at the k-th place (gap between its k-th and
    (k+1)-th chunk score below tie_rel of its largest)."""
    n = min(len(ours), len(ref_picks), len(ref_loaded))
    eq_topk = eq_loaded = ties = 0
    first_diff = None
    diffs = []  # (step, the reference's k-th / (k+1)-th score gap relative to its largest score)
    for i in range(n):
        o_top, o_loaded = ours[i]
        r_scores, r_top = ref_picks[i]
        if o_top == r_top:
            eq_topk += 1
        else:
            srt = np.sort(np.asarray(r_scores, np.float64))[::-1]
            gap = srt[top_k - 1] - srt[top_k] if len(srt) > top_k else np.inf
            rel = float(gap / max(abs(srt[0]), 1e-30))
            diffs.append([i, rel, len(set(o_top) ^ set(r_top)) // 2])
            if rel <= tie_rel:
                ties += 1
            elif first_diff is None:
                first_diff = i
        if o_loaded == ref_loaded[i]:
            eq_loaded += 1
    return {"steps": n, "topk_equal_steps": eq_topk, "loaded_equal_steps": eq_loaded,
            "near_tie_steps": ties, "first_step_differing_beyond_ties": first_diff,
            "differing_steps": diffs[:8],  # [step, relative k-th gap, chunks swapped]
            "how": "per decode step, sample 0: this cache's top-k chunks and loaded segments against the "
                   "reference's own WnWCache (baseline/_ref, Triton + torch fp32 cumsum on the GPU) replaying "
                   "the same recorded q/k/v; a differing top-k counts as a near tie when the reference's k-th "
                   "and (k+1)-th chunk scores differ by < 1e-5 of its largest"}


def h2d_link_probe(dev, mb=128, reps=5):
    """H2D bandwidth of this GPU's host link right now, GB/s: (the fetch
    kernel reading 128-row ranges of a pinned buffer, a copy-engine copy of
    the same bytes from contiguous pinned memory).  The decode step fetches
    its offloaded rows over this link, so it bounds the step; the copy engine
    on contiguous memory is the link's practical ceiling."""
    from wnw_b200 import kernels as Kx
    D = MODEL["D"]
    rows = mb * (1 << 20) // (2 * D * 2)
    hk = torch.ones(rows, D, dtype=torch.bfloat16).pin_memory()
    hv = torch.ones(rows, D, dtype=torch.bfloat16).pin_memory()
    pk, pv = Kx.host_device_pointer(hk), Kx.host_device_pointer(hv)
    n = rows // 128
    perm = torch.randperm(n, generator=torch.Generator().manual_seed(0))
    st = (perm * 128).to(torch.int32)
    ranges = torch.stack([st, st + 128], 1).to(dev)
    dst = torch.arange(0, n * 128, 128, dtype=torch.int64, device=dev)
    dk = torch.empty(rows, D, dtype=torch.bfloat16, device=dev)
    dv = torch.empty_like(dk)
    Kx.fetch_rows(pk, pv, D * 2, ranges, dst, dk, dv, max_ctas=512)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        Kx.fetch_rows(pk, pv, D * 2, ranges, dst, dk, dv, max_ctas=512)
    e1.record()
    torch.cuda.synchronize()
    zero_copy = 2 * rows * D * 2 * reps / (e0.elapsed_time(e1) * 1e-3) / 1e9
    dk.copy_(hk, non_blocking=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        dk.copy_(hk, non_blocking=True)
        dv.copy_(hv, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    dma = 2 * rows * D * 2 * reps / (e0.elapsed_time(e1) * 1e-3) / 1e9
    return zero_copy, dma


def cpu_replay(rec, n_steps, start=0, layers=None):
    """The CPU oracle replaying steps [start, start+n_steps) after its own
    prefill from the same recorded inputs; returns seconds per step.
    ``layers``: only the first that many layers (a bounded sample of a deep
    workload; the caller scales the time to the full depth)."""
    from oracle.cache import OracleWnWCache
    cfg = rec["cfg"]
    nl = layers or MODEL["L"]
    c = OracleWnWCache(cfg, nl, MODEL["Hkv"], MODEL["Hq"], MODEL["D"])
    if len(rec["audio"]) == 2:
        a0, a1 = rec["audio"]
        c.setup_audio([a0], [a1], [0])
    else:
        c.setup_audio(list(rec["audio"][0]), list(rec["audio"][1]), list(rec["audio"][3]))
    for l, ca, ph, k, v in rec["prefill"][:nl]:
        c.prefill_after_attn(l, [x.cpu() if x is not None else None for x in ca],
                             [[x.cpu() if x is not None else None for x in r] for r in ph], k.cpu(), v.cpu())
    c.prefill_all_layers_done()
    steps, scale = rec["steps"], rec["scale"]
    for i in range(start):
        _cpu_step(c, steps[i][:nl], scale)
    t = time.perf_counter()
    for i in range(start, start + n_steps):
        _cpu_step(c, steps[i][:nl], scale)
    return (time.perf_counter() - t) / n_steps


def _cpu_step(c, step, scale):
    for l, (q, k, v) in enumerate(step):
        c.decode_before_attn(l, k.cpu(), v.cpu())
        c.fused_decode_attention(l, q.cpu(), scale=scale)
    c.decode_all_layers_done()


# ------------------------------------------------------------------ kernel modes
L2_BYTES = 126 << 20


def attn_layer(dev, lens, G, D, seed, n_score=0, a0=4, a1=None, sm_count=None, max_cluster=None):
    """One layer of decode attention over segments of ``lens`` rows, laid
    out as the cache lays a layer out (16-row aligned slots with slack),
    with the library's plan; the first ``n_score`` segments are class A with
    their audio rows [a0, a1) scored.  Returns the launch arguments and what
    they point at."""
    from wnw_b200 import kernels as Kx
    from wnw_b200 import native as N
    S = len(lens)
    dtype = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(seed)
    cap = np.asarray(lens, np.int64) + 16
    cap_al = (cap + 15) // 16 * 16
    base = np.concatenate([[0], np.cumsum(cap_al)[:-1]]).astype(np.int64)
    rows = int(cap_al.sum())
    ks = torch.randn(rows, D, device=dev, generator=g, dtype=dtype)
    vs = torch.randn(rows, D, device=dev, generator=g, dtype=dtype)
    q = torch.randn(S, G, D, device=dev, generator=g, dtype=dtype)
    work = Kx.AttnWork(dtype, D, cap, dev, sm_count=sm_count, max_cluster=max_cluster)
    scratch = Kx.AttnScratch(dev, work.slots, G, D, S)
    score = None
    a1 = min(lens) if a1 is None else a1
    n_audio = max(0, a1 - a0)
    if n_score and n_audio:
        slot = torch.full((S,), -1, dtype=torch.int32)
        slot[:n_score] = torch.arange(n_score, dtype=torch.int32)
        score = dict(slot=slot.to(dev), audio_start=torch.tensor([a0], dtype=torch.int32, device=dev),
                     audio_end=torch.tensor([a1], dtype=torch.int32, device=dev),
                     logits=torch.zeros(n_score * n_audio * G, device=dev),
                     logits_off=torch.arange(0, n_score * n_audio * G, n_audio * G, dtype=torch.int64, device=dev),
                     stats=torch.zeros(S * 2 * G, device=dev))
    args = Kx.make_attn_args(dtype, S, G, D, ks, vs, torch.from_numpy(base).to(dev),
                             torch.tensor(lens, dtype=torch.int32, device=dev), work, D ** -0.5, scratch,
                             seg_cap=torch.from_numpy(cap.astype(np.int32)).to(dev), num_kv_heads=S, score=score,
                             flags=N.ATTN_ROWS_READY)
    nbytes = int(np.sum(lens)) * D * 2 * 2 + S * G * D * 2 * 2 + 8 * (n_score if score else 0) * n_audio
    return dict(args=args, q=q, out=torch.empty_like(q), bytes=nbytes, work=work, lens=list(lens), base=base,
                ks=ks, vs=vs, n_score=n_score if score else 0, keep=(scratch, score))


def time_attn(layers, reps):
    """us per launch of the layers' decode attention, launched round-robin
    back to back (nothing between them writes a layer's rows, so each may
    load its rows before its dependency wait): replayed from a CUDA graph
    (the kernels' own time) and launched from the host."""
    from wnw_b200 import kernels as Kx
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for x in layers:
            Kx.launch_attn(x["args"], x["q"], None, None, x["out"], side.cuda_stream)
        torch.cuda.synchronize()
        per = max(1, math.ceil(32 / len(layers)))
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=side):
            for _ in range(per):
                for x in layers:
                    Kx.launch_attn(x["args"], x["q"], None, None, x["out"], side.cuda_stream)
    torch.cuda.synchronize()
    gr.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        gr.replay()
    e1.record()
    torch.cuda.synchronize()
    graph_us = e0.elapsed_time(e1) * 1e3 / (reps * per * len(layers))
    st = torch.cuda.current_stream().cuda_stream
    e0.record()
    for _ in range(reps):
        for x in layers:
            Kx.launch_attn(x["args"], x["q"], None, None, x["out"], st)
    e1.record()
    torch.cuda.synchronize()
    host_us = e0.elapsed_time(e1) * 1e3 / (reps * len(layers))
    del gr
    return graph_us, host_us


def check_attn(x, n=4):
    """Max |error| of up to ``n`` segments of a launched layer against
    softmax(q K^T / sqrt(d)) V in fp32 (torch)."""
    lens, base = x["lens"], x["base"]
    S, D = len(lens), x["ks"].shape[1]
    pick = sorted({0, S - 1, S // 2, max(0, S // 3)})[:n]
    err = 0.0
    for s in pick:
        if lens[s] == 0:
            continue
        k = x["ks"][base[s]:base[s] + lens[s]].float()
        v = x["vs"][base[s]:base[s] + lens[s]].float()
        p = torch.softmax(x["q"][s].float() @ k.t() * D ** -0.5, dim=-1)
        err = max(err, float((p @ v - x["out"][s].float()).abs().max()))
    return err


def reference_kernels(layers, a0, a1, reps):
    """The reference's own decode-attention GPU kernels from its offline
    install, on the same layers packed into its flat layout (``cu_seqlens``):
    ``q1_decode_attn_score`` (attention + class-A score accumulation,
    src/common/kv/fused_attn.py:124-156, what its session calls with
    WNW_FUSED_ATTN=1), ``q1_decode_attn`` (attention only, fused_attn.py:47-65)
    and torch's ``varlen_attn`` as its default session path calls it
    (src/algorithms/wnw/code/session.py:90-106).  us per launch, round-robin
    over the layers, CUDA events."""
    reference_modules()  # puts baseline/_ref on the path, or raises
    from common.kv.fused_attn import q1_decode_attn, q1_decode_attn_score
    from torch.nn.attention.varlen import varlen_attn
    x0 = layers[0]
    lens, dev = x0["lens"], x0["q"].device
    S, G, D = x0["q"].shape
    n_score = x0["n_score"]
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=dev)
    ca_mask = torch.tensor([1 if s < n_score else 0 for s in range(S)], dtype=torch.int32, device=dev)
    a_s = torch.tensor([a0], dtype=torch.int32, device=dev)
    a_e = torch.tensor([a1], dtype=torch.int32, device=dev)
    acc = torch.zeros(max(1, a1 - a0), dtype=torch.float32, device=dev)
    offs = torch.tensor([0, a1 - a0], dtype=torch.int32, device=dev)
    packed = []
    for x in layers:
        pk = torch.cat([x["ks"][int(b):int(b) + n] for b, n in zip(x["base"], lens)])
        pv = torch.cat([x["vs"][int(b):int(b) + n] for b, n in zip(x["base"], lens)])
        packed.append((x["q"], pk, pv))
    scale = D ** -0.5
    cu_q = torch.arange(S + 1, dtype=torch.int32, device=dev)

    def varlen(q, pk, pv):  # the session's call: K/V heads broadcast to the query heads
        T = pk.shape[0]
        ke = pk.unsqueeze(1).as_strided((T, G, D), (D, 0, 1))
        ve = pv.unsqueeze(1).as_strided((T, G, D), (D, 0, 1))
        return varlen_attn(q, ke, ve, cu_q, cu, max_q=1, max_k=int(max(lens)), scale=scale)

    def timed(fns):
        for f in fns:
            f()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            for f in fns:
                f()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / (reps * len(fns))

    out = {"q1_decode_attn_score_us": timed([lambda p=p: q1_decode_attn_score(
               p[0], p[1], p[2], cu, scale, ca_mask, S, a_s, a_e, acc, offs) for p in packed]),
           "q1_decode_attn_us": timed([lambda p=p: q1_decode_attn(p[0], p[1], p[2], cu, scale) for p in packed])}
    try:
        out["varlen_attn_us"] = timed([lambda p=p: varlen(*p) for p in packed])
    except Exception as e:  # the library kernel may not take this layout
        out["varlen_attn_us"] = f"failed: {type(e).__name__}: {e}"[:200]
    # both compute the same attention: ours (launched last by the timing) vs the reference's, layer 0
    ref_o = q1_decode_attn(packed[0][0], packed[0][1], packed[0][2], cu, scale)
    out["max_abs_diff_vs_ours"] = float((ref_o.float() - x0["out"].float()).abs().max())
    return out


def trace_phases(layers, reps=3, isolated=False):
    """Per-CTA phase timestamps (%globaltimer, ns) of ``reps`` passes of the
    layers' launches -- back to back, or (``isolated``) one launch at a time
    with the GPU idle before each -- from the trace build: per launch, the
    first CTA's start, the dependency wait's release, the last CTA's last
    tile, CTA merge, cluster merge and exit; medians over the launches after
    the first pass, in us relative to the launch's first CTA start."""
    import ctypes as C
    from wnw_b200 import kernels as Kx
    from wnw_b200 import native as N
    if not hasattr(N.lib, "wnw_attn_trace_reset"):
        raise RuntimeError(f"{N.LIB_PATH} has no phase trace: build libwnw_b200_trace.so with "
                           "`python -m wnw_b200.build --trace`")
    N.lib.wnw_attn_trace_reset.restype = C.c_int
    N.lib.wnw_attn_trace_read.restype = C.c_int

    def read():
        buf = np.zeros((16384, 8), np.uint64)
        n = C.c_int()
        N.check(N.lib.wnw_attn_trace_read(C.c_void_p(buf.ctypes.data), 16384, C.byref(n)), "wnw_attn_trace_read")
        return buf[:n.value].astype(np.int64)

    st = torch.cuda.current_stream().cuda_stream
    torch.cuda.synchronize()
    if isolated:
        parts = []
        for _ in range(reps):
            for x in layers:
                N.check(N.lib.wnw_attn_trace_reset(), "wnw_attn_trace_reset")
                torch.cuda.synchronize()
                Kx.launch_attn(x["args"], x["q"], None, None, x["out"], st)
                torch.cuda.synchronize()
                parts.append(read())
        rec = np.concatenate(parts)
    else:
        N.check(N.lib.wnw_attn_trace_reset(), "wnw_attn_trace_reset")
        for _ in range(reps):
            for x in layers:
                Kx.launch_attn(x["args"], x["q"], None, None, x["out"], st)
        torch.cuda.synchronize()
        rec = read()
    ctas = layers[0]["work"].ctas
    launches = []
    for pp in np.unique(rec[:, 1]):  # one plan (pointer) per layer
        r = rec[rec[:, 1] == pp]
        r = r[np.argsort(r[:, 2])]
        for k in range(len(r) // ctas):
            launches.append(r[k * ctas:(k + 1) * ctas])
    launches.sort(key=lambda r: r[:, 2].min())
    rows = []
    for i, r in enumerate(launches):
        t0 = r[:, 2].min()
        ph = [(r[:, 3].min() - t0), (r[:, 3].max() - t0), (r[:, 4].max() - t0), (r[:, 5].max() - t0),
              (r[:, 6].max() - t0), (r[:, 7].max() - t0)]
        gap = (r[:, 3].min() - launches[i - 1][:, 7].max()) if i else None
        rows.append(ph + [gap, t0 - (launches[i - 1][:, 2].min() if i else t0)])
    rows = rows[len(layers):] or rows
    med = lambda j: float(np.median([x[j] for x in rows if x[j] is not None])) / 1e3  # noqa: E731
    names = ["first_wait_release", "last_wait_release", "last_tile_done", "cta_merge_done", "cluster_barrier_done",
             "last_exit", "release_after_prev_exit", "launch_to_launch"]
    if isolated:
        names = names[:6]
    return {"launches": len(rows), "ctas_per_launch": ctas, "isolated": isolated,
            "median_us": {nm: med(j) for j, nm in enumerate(names)},
            "how": "%globaltimer per CTA (trace build), times from the launch's first CTA start; "
                   "release_after_prev_exit = this launch's first wait release - the previous launch's last exit"}


def mode_attn(a, dev):
    """Decode attention alone on one layer geometry (config 2's by default:
    two class-A segments of 15,100 rows, scored, and six class-B ones of
    2,300), ``--layers`` distinct layers launched round-robin so the working
    set exceeds L2."""
    H, G, D = MODEL["Hkv"], MODEL["Hq"] // MODEL["Hkv"], MODEL["D"]
    lens = [a.class_a] * a.n_class_a + [a.class_b] * (H - a.n_class_a)
    layers = [attn_layer(dev, lens, G, D, seed=l, n_score=a.n_class_a, a1=min(a.class_a, 15004),
                         sm_count=a.sm_count, max_cluster=a.max_cluster) for l in range(a.layers)]
    graph_us, host_us = time_attn(layers, a.reps)
    peak, kind = peaks()
    nb = layers[0]["bytes"]
    w = layers[0]["work"]
    line = {"mode": "attn", "lens": lens, "bytes_per_launch": nb, "us_per_launch": graph_us,
            "gbs": nb / (graph_us * 1e-6) / 1e9, "frac": nb / (graph_us * 1e-6) / 1e9 / peak, "peak_gbs": peak,
            "peak_source": kind, "host_launched_us": host_us, "ctas": w.ctas, "cluster": w.cluster_size,
            "partials": w.parts, "layers": len(layers),
            "how": "CUDA-graph replay of the layers' launches back to back, CUDA events"}
    if a.check:
        line["max_abs_err"] = max(check_attn(x) for x in layers[:2])
    if a.trace:
        line["trace"] = trace_phases(layers, isolated=a.isolated)
    if a.vs_reference:
        try:
            line["reference_kernels"] = reference_kernels(layers, 4, min(a.class_a, 15004),
                                                          max(1, a.reps // 4))
        except Exception as e:  # report, keep the line
            line["reference_kernels"] = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    print(json.dumps(line), flush=True)


def mode_sweep(a, dev, rank, world):
    """random bf16 K/V/q, 8 kv heads x head_dim 128, GQA
    4; per cell of batch x context x class-A fraction x retained fraction,
    the first round(frac_a * 8) kv heads of every sample are class A (the
    whole context) and the rest class B (retained * context rows).  Under
    torchrun the kv heads are sharded over the ranks (rank r attends heads
    [r*8/N, (r+1)*8/N) of every sample); value = all ranks' bytes / the
    slowest rank's time.  One JSON line per cell from rank 0."""
    from wnw_b200.tp import head_range
    H, G, D = MODEL["Hkv"], 4, MODEL["D"]
    h0, h1 = head_range(rank, world, H)
    ints = lambda t: [int(x) for x in t.split(",")]  # noqa: E731
    flts = lambda t: [float(x) for x in t.split(",")]  # noqa: E731
    peak, kind = peaks()
    for b in ints(a.batch):
        for c in ints(a.ctx):
            for fa in flts(a.frac_a):
                for r in flts(a.retained):
                    n_a = min(H, max(0, round(fa * H)))
                    lb = max(1, int(r * c))
                    lens = [c if h < n_a else lb for _ in range(b) for h in range(h0, h1)]
                    store = (sum(lens) + 16 * len(lens)) * D * 2 * 2
                    cell = {"mode": "sweep", "batch": b, "ctx": c, "frac_a": fa, "retained": r, "n_gpus": world}
                    t = torch.tensor([float(store > a.max_gb * 1e9)], device=dev)
                    if world > 1:
                        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
                    if t.item() > 0:
                        if rank == 0:
                            print(json.dumps(dict(cell, skipped=f"above --max-gb {a.max_gb} per GPU")), flush=True)
                        continue
                    n_layers = 1 if store > 8 * L2_BYTES else max(2, math.ceil(2 * L2_BYTES / store))
                    layers = [attn_layer(dev, lens, G, D, seed=l) for l in range(n_layers)]
                    if world > 1:
                        torch.distributed.barrier()
                    us, _ = time_attn(layers, max(2, a.reps // n_layers))
                    err = check_attn(layers[0]) if a.check else None
                    v = torch.tensor([us, layers[0]["bytes"], err or 0.0], device=dev, dtype=torch.float64)
                    if world > 1:
                        mx = v.clone()
                        torch.distributed.all_reduce(mx, op=torch.distributed.ReduceOp.MAX)
                        torch.distributed.all_reduce(v, op=torch.distributed.ReduceOp.SUM)
                        us, nb, err = float(mx[0]), float(v[1]), float(mx[2])
                    else:
                        nb = float(v[1])
                    if rank == 0:
                        gbs = nb / (us * 1e-6) / 1e9
                        cell.update(bytes=nb, us=us, gbs=gbs, frac=gbs / (peak * world), peak_gbs_per_gpu=peak,
                                    ctas=layers[0]["work"].ctas, cluster=layers[0]["work"].cluster_size)
                        if a.check:
                            cell["max_abs_err"] = err
                        print(json.dumps(cell), flush=True)
                    del layers
                    torch.cuda.empty_cache()


# ------------------------------------------------------------------ clocks
class Clocks:
    """nvidia-smi sampling during the timed region."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is None:
            return
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [x for x in out.splitlines() if x.strip()]
            self.proc = None

    def summary(self, window=None):
        """Median SM clock, max clock and active throttle reasons over the
        samples taken inside ``window`` = (t0, t1) in time.time() seconds
        (the timed region; all samples when None)."""
        import datetime
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            try:
                ts = datetime.datetime.strptime(p[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                clk, cmax = float(p[2]), float(p[3])
            except (ValueError, IndexError):
                continue
            if window is not None and not window[0] <= ts <= window[1]:
                continue
            sm.append(clk)
            mx.append(cmax)
            for n, v in zip(names, p[6:10]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm), "window": "timed region" if window is not None else "whole leg"}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def traffic_per_launch(algorithmic_bytes):
    """DRAM bytes per decode-attention launch: the committed ncu capture's
    DRAM/algorithmic ratio (profiles/decode_attn_traffic.json, a config-2
    layer geometry case) scaled to this launch's algorithmic bytes; None when
    no capture is committed."""
    try:
        with open(os.path.join(ROOT, "profiles", "decode_attn_traffic.json")) as f:
            return float(json.load(f)["ratio"]) * algorithmic_bytes
    except (OSError, ValueError, KeyError):
        return None


# ------------------------------------------------------------------ main
def main():
    a = parse()
    REBUILD_AHEAD[0] = not a.no_rebuild_ahead
    if a.trace:  # before anything loads the library
        os.environ.setdefault("WNW_B200_LIB", os.path.join(ROOT, "wnw_b200", "libwnw_b200_trace.so"))
    use_config(a.config, a.synthetic, a.depth)
    a.synth = a.config in SYNTH and (a.config != 2 or a.synthetic)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = world > 1
    if a.impl == "reference" and rank != 0:
        return
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    if dist and a.impl == "b200":
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                             device_id=dev)
    if a.mode != "step" and a.impl == "b200":
        try:
            if a.mode == "attn":
                if rank == 0:
                    mode_attn(a, dev)
            else:
                mode_sweep(a, dev, rank, world)
        finally:
            if dist:
                torch.distributed.destroy_process_group()
        return
    K, W = a.steps, a.warmup
    if a.synth:
        c = SYNTH[a.config]
        cfg_json = {"workload": f"{c['name']} wnw decode hot path (BASELINE config {a.config}): {c['note']}, "
                                f"{c['L']} layers", "config": a.config, "batch": c["B"], "layers": c["L"],
                    "q_heads": c["Hq"], "kv_heads": c["Hkv"], "head_dim": c["D"], "hidden": c["hidden"],
                    "class_a_kv_heads": list(c["class_a_kv"]), "retention": c["retention"],
                    "chunk_tokens": c["chunk"], "top_k": c["top_k"], "eviction_lag": c["lag"],
                    "inputs": "seeded synthetic prefill K/V and decode q/k/v ~ N(0, 1) (no model run)",
                    "l2": "per-step K/V working set > L2", "parallelism": f"request-sharded replicas x{world}"}
    else:
        workload = "voxtral-mini-3b wnw decode hot path, B=1, 15064-token prompt (15000 audio), 30 layers"
        cfg_json = {"workload": workload, "batch": 1, "prompt_tokens": 15064, "audio_tokens": 15000,
                    "layers": 30, "q_heads": 32, "kv_heads": 8, "head_dim": 128, "class_a_frac": WNW["frac_a"],
                    "chunk_tokens": WNW["chunk"], "top_k": WNW["top_k"], "eviction_lag": WNW["lag"],
                    "inputs": "q/k/v recorded from the random-init decoder, replayed",
                    "l2": "per-step K/V working set > L2 (30 layers x ~25 MB)",
                    "parallelism": f"request-sharded replicas x{world}"}
    tp = a.parallel == "tp" and a.impl == "b200"
    if tp:
        cfg_json["parallelism"] = f"tp{world} (kv heads sharded, o_proj all-reduce per layer)"
    if a.tier != "host":
        cfg_json["offload_tier"] = f"{a.tier} (class-B offloaded rows in device memory; not the headline)"
    # the clock sampler starts now so its start-up is long over by the timed
    # region; only the samples inside that region are reported
    clk = Clocks(local)
    if a.impl == "b200" and not a.profile:
        clk.__enter__()
    try:
        return _main(a, rank, world, local, dist, dev, K, W, cfg_json, tp, clk)
    finally:
        clk.__exit__(None, None, None)


def _main(a, rank, world, local, dist, dev, K, W, cfg_json, tp, clk):
    if a.impl == "reference":
        # the reference arm runs none of this package's code: its inputs are
        # recorded through the reference's own session and cache (on the
        # GPU, untimed), then the CPU restatement replays them
        n = max(1, K)
        try:
            if a.synth:
                rec = synthetic_record(dev, 1, a.config, cfg_cls=reference_modules()[2])
            else:
                rec = record(dev, W + n, seed=1000, reference=True)
        except Exception as e:  # report, exit 0
            print(json.dumps({"impl": "reference", "unavailable": f"{type(e).__name__}: {e}"[:300]}), flush=True)
            return
        if a.synth:  # a deep workload: one step of the first few layers, scaled to the full depth
            nl = min(MODEL["L"], 2 if a.config == 4 else 3)
            n, W = 1, 0
            sec = cpu_replay(rec, 1, start=0, layers=nl) * MODEL["L"] / nl
            sample = f"1 decode step of the first {nl} of {MODEL['L']} layers replayed by the CPU oracle, scaled"
        else:
            sec = cpu_replay(rec, n, start=W)
            sample = (f"{n} decode steps (all 30 layers, after {W} untimed) replayed by the CPU oracle; inputs "
                      "recorded through the reference's own session and cache")
        v = rec.get("batch", 1) / sec
        line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tokens/s",
                "n_gpus": a.gpus, "steps": n, "warmup": W, "ms_per_step": sec * 1e3, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": cfg_json,
                "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
                                 "sample": sample},
                "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    # replicas record their own request; tensor-parallel ranks share one
    if a.synth:
        rec = synthetic_record(dev, W + K, a.config)
    else:
        rec = record(dev, W + K, seed=1000 + (0 if tp else rank))
    B = rec.get("batch", 1)
    shard = Shard(dev, rank, world, tp=tp, seed=2000, exchange=a.tp_exchange, batch=B)
    if tp:
        cfg_json["parallelism"] += f", exchange {a.tp_exchange}"
    val = run_value(rec, dev, K, W, shard, tier=a.tier)
    clk.__exit__(None, None, None)
    e2e = run_e2e(rec, dev, K, W, shard, tier=a.tier)
    if shard.ex is not None:
        shard.ex.check()
    # the same step with the offloaded rows kept in HBM (offload_tier="hbm"),
    # for comparison only: the reference offloads to host memory
    hbm = (run_value(rec, dev, K, W, shard, tier="hbm") if not dist and not a.profile and a.tier == "host"
           else None)
    ref_gpu = (run_reference_gpu(rec, dev, K, W) if not dist and not a.profile and not tp and not a.synth
               else None)
    agreement = None
    if ref_gpu is not None and "_picks" in ref_gpu:
        agreement = selection_agreement(val["selections"], ref_gpu.pop("_picks"), ref_gpu.pop("_loaded"),
                                        WNW["top_k"])
    ms = val["ms"]
    if dist:
        t = torch.tensor([ms, e2e["ms"]], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, e2e_ms = float(t[0]), float(t[1])
        torch.distributed.barrier()
    else:
        e2e_ms = e2e["ms"]
    tokens = (1 if tp else world) * B * K
    peak, peak_kind = peaks()
    link, link_dma = h2d_link_probe(dev)
    fetch_bytes = val["fetched_rows"] / K * MODEL["D"] * 2 * 2
    achieved = val["attn_bytes"] / (val["attn_us"] * 1e-6) / 1e9
    line = {
        "metric": METRIC, "value": tokens / (ms * 1e-3),
        "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms / K,
        "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None, "dtype": "bf16",
        "data": ("synthetic (seeded N(0,1) K/V and q/k/v at the config's shapes)" if a.synth
                 else "synthetic (random-init decoder, N(0,0.02) audio embeddings)"), "config": cfg_json,
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": e2e["in_bytes"],
                "d2h_bytes_per_step": e2e["out_bytes"]},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": (achieved / peak) if achieved else None, "peak_source": peak_kind,
                     "traffic": traffic_per_launch(val["attn_bytes"]),
                     "kernel": f"wnw::decode_attn_mma_kernel<bf16,128,{MODEL['Hq'] // MODEL['Hkv']}>",
                     "bytes_per_launch": val["attn_bytes"], "us_per_launch": val["attn_us"],
                     "launches_timed": val["attn_n"],
                     "how": f"all {MODEL['L']} layers' launches back to back on the timed run's final state, CUDA events"},
        "gpu_launches": val["launches"],
        "clocks": clk.summary(val["window"]),
        "fetched_rows_per_step": val["fetched_rows"] / K,
        "host_link": {"fetch_bytes_per_step": fetch_bytes, "link_gbs": link,
                      "dma_contiguous_gbs": link_dma,
                      "fetch_kernel_frac_of_dma": link / link_dma if link and link_dma else None,
                      "fetch_ms_at_link": fetch_bytes / (link * 1e9) * 1e3 if link else None,
                      "step_frac_of_link_bound": (fetch_bytes / (link * 1e9) * 1e3) / (ms / K)
                      if link else None,
                      "how": "offloaded rows fetched per step over the host link (zero-copy kernel); link_gbs = "
                             "that kernel on 128 MB of random 128-row ranges, dma_contiguous_gbs = a copy-engine "
                             "copy of the same bytes from contiguous pinned memory (the link's practical "
                             "ceiling), both measured in this run"},
        "model_decode_ms_per_token": rec["model_ms"],
        "reference_gpu": ref_gpu,
        "selection_vs_reference_gpu": agreement,
        "host_wait_ms_per_step": val["host_wait_ms"] / K,
        "offload_tier_hbm": ({"value": tokens / (hbm["ms"] * 1e-3), "ms_per_step": hbm["ms"] / K,
                              "host_wait_ms_per_step": hbm["host_wait_ms"] / K,
                              "how": "same replay with offload_tier='hbm' (class-B rows in device memory, no "
                                     "host-link traffic); not the headline, which offloads to host memory as "
                                     "the reference does"} if hbm else None),
        "prefill_compress_ms": {"first": PREFILL_MS[0] if PREFILL_MS else None,
                                "warm": min(PREFILL_MS[1:]) if len(PREFILL_MS) > 1 else None,
                                "how": "prefill_after_attn x 30 layers + prefill_all_layers_done on the recorded "
                                       "prompt (15,064 tokens); first = including this process's first pinned "
                                       "allocation of the host store"},
    }
    if rank == 0 and not a.no_cpu and not a.profile:
        if a.synth:  # a deep workload: one step of the first few layers, scaled to the full depth
            nl = min(MODEL["L"], 2 if a.config == 4 else 3)
            sec = cpu_replay(rec, 1, start=0, layers=nl) * MODEL["L"] / nl
            sample = f"1 decode step of the first {nl} of {MODEL['L']} layers replayed by the CPU oracle, scaled"
        else:
            n = max(1, min(a.cpu_steps, K))
            sec = cpu_replay(rec, n, start=W)
            sample = f"{n} decode steps (all 30 layers) replayed by the CPU oracle"
        line["cpu_baseline"] = {"value": B / sec, "unit": "tokens/s", "cores": torch.get_num_threads(),
                                "kind": "port", "sample": sample}
    if rank == 0:
        print(json.dumps(line), flush=True)
    shard.close()
    if dist:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
