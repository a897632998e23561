"""Seeded scenarios shared by the golden generator and the tests.

Inputs are regenerated from fixed seeds (numpy PCG64, deterministic across
machines); only the reference's OUTPUTS are stored in the fixtures.
"""
from __future__ import annotations

import numpy as np

# ----------------------------------------------------------------- cache trace
CACHE_SCENARIO = dict(
    seed=7, L=3, Hkv=4, Hq=8, D=32, B=2, steps=8, S=325,
    audio_starts=[5, 55], audio_ends=[305, 305], pad=[0, 50],
    chunk_size_s=32.0, overlap_s=16.0, token_rate=1.0,          # stride 16, 2 segments / chunk
    class_a=[0, 1, 2, 3, 8 + 2],                                  # layer 0 kv0+kv1 (foldable), layer 1 q2 (not foldable)
    class_b=[2, 4, 7, 8, 9, 10],                                  # (l0,kv2) (l1,kv0) (l1,kv3) (l2,kv0..2)
    retention={(0, 2): 0.25, (0, 3): 0.5, (1, 0): 0.125, (1, 2): 0.25, (1, 3): 0.0,
               (2, 0): 0.25, (2, 1): 0.0625, (2, 2): 0.3, (2, 3): 0.5},
    top_k=3, lag=2, prefill_mode="last",
)


# the same scenario with the global per-head prefill top-k (cache.py:1141-1150)
GLOBAL_TOPK_SCENARIO = dict(CACHE_SCENARIO, global_topk=True)


def make_config_dict(sc):
    """Keyword arguments for the reference ``WnWConfig`` (config.py:6-30)."""
    L, H, Hq = sc["L"], sc["Hkv"], sc["Hq"]
    ret = []
    for l in range(L):
        for h in range(H):
            ret.append(sc["retention"].get((l, h)))
    return dict(chunk_size_s=sc["chunk_size_s"], overlap_s=sc["overlap_s"], token_rate=sc["token_rate"],
                class_a=list(sc["class_a"]), class_b=list(sc["class_b"]), retention_ratios=ret,
                top_k_chunks=sc["top_k"], eviction_lag=sc["lag"], prefill_score_mode=sc["prefill_mode"],
                prefill_global_topk=sc.get("global_topk", False),
                num_layers=L, num_kv_heads=H, num_q_heads=Hq)


def _class_a_kv(sc, l):
    G = sc["Hq"] // sc["Hkv"]
    return sorted({(g - l * sc["Hq"]) // G for g in sc["class_a"] if l * sc["Hq"] <= g < (l + 1) * sc["Hq"]})


def make_cache_inputs(sc):
    """Prefill K/V + scores and per-step decode q/k/v for ``CACHE_SCENARIO``."""
    import torch
    rng = np.random.default_rng(sc["seed"])
    L, H, Hq, D, B, S = sc["L"], sc["Hkv"], sc["Hq"], sc["D"], sc["B"], sc["S"]
    mask = np.ones((B, S), np.int64)
    for b in range(B):
        mask[b, :sc["pad"][b]] = 0
    n_audio = [e - s for s, e in zip(sc["audio_starts"], sc["audio_ends"])]
    inp = dict(audio_starts=list(sc["audio_starts"]), audio_ends=list(sc["audio_ends"]),
               attention_mask=mask, pad=list(sc["pad"]))
    if sc.get("torch_kv"):  # long contexts: torch's generator draws fp32 directly, ~10x faster
        g = torch.Generator().manual_seed(sc["seed"])
        inp["prefill_k"] = [torch.randn(B, H, S, D, generator=g).numpy() for _ in range(L)]
        inp["prefill_v"] = [torch.randn(B, H, S, D, generator=g).numpy() for _ in range(L)]
    else:
        inp["prefill_k"] = [rng.standard_normal((B, H, S, D)).astype(np.float32) for _ in range(L)]
        inp["prefill_v"] = [rng.standard_normal((B, H, S, D)).astype(np.float32) for _ in range(L)]
    cas, phs = [], []
    for l in range(L):
        ca_kv = _class_a_kv(sc, l)
        cas.append([torch.from_numpy(rng.random(n_audio[b]).astype(np.float32)) if ca_kv else None
                    for b in range(B)])
        phs.append([[None if h in ca_kv else torch.from_numpy(rng.random(n_audio[b]).astype(np.float32))
                     for h in range(H)] for b in range(B)])
    inp["class_a_scores"] = cas
    inp["per_head_scores"] = phs
    steps = sc["steps"]
    inp["dec_q"] = [[rng.standard_normal((B, Hq, 1, D)).astype(np.float32) for _ in range(L)] for _ in range(steps)]
    inp["dec_k"] = [[rng.standard_normal((B, H, 1, D)).astype(np.float32) for _ in range(L)] for _ in range(steps)]
    inp["dec_v"] = [[rng.standard_normal((B, H, 1, D)).astype(np.float32) for _ in range(L)] for _ in range(steps)]
    return inp


# -------------------------------------------------------------------- planner
PLANNER_SCENARIOS = [
    dict(seed=11, L=3, H=4, B=2, seg_count=[12, 9], spc=2, top_k=3, lag=1, steps=6),
    dict(seed=12, L=2, H=3, B=3, seg_count=[7, 15, 4], spc=1, top_k=4, lag=3, steps=8),
    dict(seed=13, L=4, H=2, B=1, seg_count=[20], spc=3, top_k=2, lag=2, steps=10),
]


def make_planner_inputs(ps):
    """Random but self-consistent planner state + a sequence of top-k choices."""
    rng = np.random.default_rng(ps["seed"])
    L, H, B = ps["L"], ps["H"], ps["B"]
    S = B * H
    sc = list(ps["seg_count"])
    c2s_flat, c2s_off = [], []
    for b in range(B):
        flat, off = [], [0]
        for c in range(sc[b]):
            flat.extend(range(c, min(c + ps["spc"], sc[b])))
            off.append(len(flat))
        c2s_flat.append(flat)
        c2s_off.append(off)
    class_b = [sorted(rng.choice(H, size=rng.integers(1, H + 1), replace=False).tolist()) for _ in range(L)]
    loaded = []
    for b in range(B):
        k = int(rng.integers(0, sc[b] + 1))
        loaded.append(sorted(rng.choice(sc[b], size=k, replace=False).tolist()))
    cpu_s, cpu_e, gpu_s, gpu_e, seq_lens = [], [], [], [], []
    cursor = 0
    for l in range(L):
        for fi in range(S):
            b, h = divmod(fi, H)
            base = int(rng.integers(3, 40))
            rel = base
            for si in range(sc[b]):
                n = int(rng.integers(0, 6)) if h in class_b[l] else 0
                if n == 0:
                    cpu_s.append(-1); cpu_e.append(-1); gpu_s.append(-1); gpu_e.append(-1)
                    continue
                cpu_s.append(cursor); cpu_e.append(cursor + n)
                cursor += n
                if si in loaded[b]:
                    gpu_s.append(rel); gpu_e.append(rel + n)
                    rel += n
                else:
                    gpu_s.append(-1); gpu_e.append(-1)
            seq_lens.append(rel)
    steps = []
    for _ in range(ps["steps"]):
        tk, off = [], [0]
        for b in range(B):
            k = min(ps["top_k"], sc[b])
            if rng.random() < 0.1:
                k = 0
            tk.extend(rng.choice(sc[b], size=k, replace=False).tolist())
            off.append(len(tk))
        steps.append((tk, off))
    return dict(seg_count=sc, c2s_flat=c2s_flat, c2s_off=c2s_off, class_b=class_b, loaded=loaded,
                cpu_s=cpu_s, cpu_e=cpu_e, gpu_s=gpu_s, gpu_e=gpu_e, seq_lens=seq_lens,
                steps=steps, n_cpu_rows=cursor)


# -------------------------------------------------------------------- session
SESSION_SCENARIO = dict(
    seed=3, L=2, Hkv=2, Hq=4, D=16, hidden=64, vocab=128, inter=128,
    prompt=120, audio_start=4, audio_end=100, new_tokens=6,
    chunk_size_s=16.0, overlap_s=0.0, token_rate=1.0,
    class_a=[0, 1],                    # layer 0, q heads 0-1 = kv 0 (foldable)
    class_b=[1, 2, 3],                 # (l0, kv1), (l1, kv0), (l1, kv1)
    retention={(0, 1): 0.25, (1, 0): 0.25, (1, 1): 0.125},
    top_k=2, lag=1, prefill_mode="last",
)


# the session scenario with the reference's default prefill score mode (the
# mean over the post-audio text queries, session.py:185-196)
MEAN_TEXT_SESSION_SCENARIO = dict(SESSION_SCENARIO, prefill_mode="mean_text")


def make_tiny_llama_config(ss):
    return dict(vocab_size=ss["vocab"], hidden_size=ss["hidden"], intermediate_size=ss["inter"],
                num_hidden_layers=ss["L"], num_attention_heads=ss["Hq"], num_key_value_heads=ss["Hkv"],
                head_dim=ss["D"], max_position_embeddings=512, rms_norm_eps=1e-6)


def session_inputs(ss):
    import torch
    g = torch.Generator().manual_seed(ss["seed"] + 100)
    return torch.randint(1, ss["vocab"], (1, ss["prompt"]), generator=g)
