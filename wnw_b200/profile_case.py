"""Small standalone decode-attention case for profiling (ncu) and timing.

Builds `--layers` independent layer states with the config-2 (Voxtral-Mini)
segment geometry -- batch 1, 8 kv heads: two class-A segments of 15,100 rows
and six class-B segments of 2,300 rows, bf16, head_dim 128, GQA 4 -- with
class-A scoring on, and launches the decode-attention kernel over the layers
round-robin (~180 MB for 8 layers: more than L2, so each launch reads HBM).

    python -m wnw_b200.profile_case [--layers 8] [--reps 20] [--cluster C --tiles T] [--reference]

Prints the mean launch time and the algorithmic-bytes bandwidth.  With
``--reference`` it also times, on the same layers packed into the reference's
flat layout, the reference's own GPU kernels from the offline install of the
reference in ``baseline/_ref`` (its Triton ``q1_decode_attn_score`` /
``q1_decode_attn``, src/common/kv/fused_attn.py, and the torch ``varlen_attn``
call of its default path, src/algorithms/wnw/code/session.py:90-106) -- for
comparison only.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

from wnw_b200 import kernels as Kx


def build_layer(dev, lens, a0, a1, G, D, cluster, seed, tiles=0):
    S = len(lens)
    dtype = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(seed)
    cap = np.asarray(lens, np.int64) + 64
    cap_al = (cap + 15) // 16 * 16
    base = np.concatenate([[0], np.cumsum(cap_al)[:-1]]).astype(np.int64)
    rows = int(cap_al.sum())
    ks = torch.randn(rows, D, device=dev, generator=g).to(dtype)
    vs = torch.randn(rows, D, device=dev, generator=g).to(dtype)
    q = torch.randn(S, G, D, device=dev, generator=g).to(dtype)
    if tiles <= 0 or cluster <= 0:  # the library's launch-shape choice
        split, cluster = Kx.attn_launch_shape(dtype, D, cap)
    else:
        split = Kx.split_rows(dtype, D) * tiles
    work = torch.from_numpy(Kx.build_work_table(cap, split, cluster)).to(dev)
    scratch = Kx.AttnScratch(dev, work.shape[0], G, D, S)
    ca = [s for s in range(S) if lens[s] >= a1]
    slot = torch.full((S,), -1, dtype=torch.int32)
    for i, s in enumerate(ca):
        slot[s] = i
    n_a = a1 - a0
    score = dict(slot=slot.to(dev), audio_start=torch.tensor([a0], dtype=torch.int32, device=dev),
                 audio_end=torch.tensor([a1], dtype=torch.int32, device=dev),
                 logits=torch.zeros(max(1, len(ca)) * n_a * G, device=dev),
                 logits_off=torch.tensor([i * n_a * G for i in range(max(1, len(ca)))], dtype=torch.int64,
                                         device=dev),
                 stats=torch.zeros(S * 2 * G, device=dev))
    args = Kx.make_attn_args(dtype, S, G, D, ks, vs, torch.from_numpy(base).to(dev),
                             torch.tensor(lens, dtype=torch.int32, device=dev), work, cluster, D ** -0.5,
                             scratch, seg_cap=torch.from_numpy(cap.astype(np.int32)).to(dev), num_kv_heads=S,
                             score=score, split=split)
    nbytes = int(np.sum(lens)) * D * 2 * 2 + S * G * D * 2 * 2 + 8 * len(ca) * n_a
    keep = (ks, vs, work, scratch, score, base, split, cluster)
    return args, q, torch.empty_like(q), nbytes, keep


def time_round_robin(fns, reps):
    """Mean time per call of fns called round-robin (CUDA events), us."""
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


def reference_timings(layers, lens, a0, a1, G, D, reps):
    """The reference's GPU kernels on the same layers in its packed layout."""
    ref = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
    if not os.path.isdir(ref):
        return {"reference": "unavailable: baseline/_ref (offline install of the reference) not present"}
    sys.path.insert(0, ref)
    from common.kv.fused_attn import q1_decode_attn, q1_decode_attn_score
    from torch.nn.attention.varlen import varlen_attn
    dev = layers[0][1].device
    S = len(lens)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=dev)
    n_audio = a1 - a0
    ca_mask = torch.tensor([1 if n >= a1 else 0 for n in lens], dtype=torch.int32, device=dev)
    a_s = torch.tensor([a0], dtype=torch.int32, device=dev)
    a_e = torch.tensor([a1], dtype=torch.int32, device=dev)
    acc = torch.zeros(n_audio, dtype=torch.float32, device=dev)
    offs = torch.tensor([0, n_audio], dtype=torch.int32, device=dev)
    packed = []
    for _, q, _, _, keep in layers:
        ks, vs, base = keep[0], keep[1], keep[5]
        pk = torch.cat([ks[int(b):int(b) + n] for b, n in zip(base, lens)])
        pv = torch.cat([vs[int(b):int(b) + n] for b, n in zip(base, lens)])
        packed.append((q, pk, pv))
    scale = D ** -0.5
    cu_q = torch.arange(S + 1, dtype=torch.int32, device=dev)
    max_k = int(max(lens))

    def varlen(q, pk, pv):
        T = pk.shape[0]
        ke = pk.unsqueeze(1).as_strided((T, G, D), (D, 0, 1))
        ve = pv.unsqueeze(1).as_strided((T, G, D), (D, 0, 1))
        return varlen_attn(q, ke, ve, cu_q, cu, max_q=1, max_k=max_k, scale=scale)

    out = {}
    out["q1_decode_attn_score_us"] = time_round_robin(
        [lambda p=p: q1_decode_attn_score(p[0], p[1], p[2], cu, scale, ca_mask, S, a_s, a_e, acc, offs)
         for p in packed], reps)
    out["q1_decode_attn_us"] = time_round_robin(
        [lambda p=p: q1_decode_attn(p[0], p[1], p[2], cu, scale) for p in packed], reps)
    try:
        out["varlen_attn_us"] = time_round_robin([lambda p=p: varlen(*p) for p in packed], reps)
    except Exception as e:  # the library kernel may not cover this layout
        out["varlen_attn_us"] = f"failed: {type(e).__name__}: {e}"[:200]
    # a check that both compute the same thing as ours on the first layer
    ref_o = q1_decode_attn(packed[0][0], packed[0][1], packed[0][2], cu, scale)
    out["max_abs_diff_vs_ours"] = float((ref_o.float() - layers[0][2].float()).abs().max())
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--cluster", type=int, default=0, help="CTAs per cluster (0: library choice)")
    ap.add_argument("--class-a", type=int, default=15100)
    ap.add_argument("--class-b", type=int, default=2300)
    ap.add_argument("--tiles", type=int, default=0, help="128-row tiles streamed per CTA (0: library choice)")
    ap.add_argument("--reference", action="store_true",
                    help="also time the reference's GPU kernels from baseline/_ref on the same layers")
    a = ap.parse_args()
    dev = torch.device("cuda:0")
    lens = [a.class_a, a.class_a] + [a.class_b] * 6
    layers = [build_layer(dev, lens, 4, 15004, 4, 128, a.cluster, seed=l, tiles=a.tiles) for l in range(a.layers)]
    st = torch.cuda.current_stream().cuda_stream
    for args, q, out, _, _ in layers:
        Kx.launch_attn(args, q, None, None, out, st)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.reps):
        for args, q, out, _, _ in layers:
            Kx.launch_attn(args, q, None, None, out, st)
    e1.record()
    torch.cuda.synchronize()
    n = a.reps * a.layers
    us = e0.elapsed_time(e1) * 1e3 / n
    nbytes = layers[0][3]
    print(json.dumps({"us_per_launch": us, "bytes_per_launch": nbytes, "gbs": nbytes / (us * 1e-6) / 1e9,
                      "launches": n, "cluster": layers[0][4][7], "split_rows": layers[0][4][6], "lens": lens}))
    if a.reference:
        r = reference_timings(layers, lens, 4, 15004, 4, 128, max(1, a.reps // 4))
        for k in ("q1_decode_attn_score_us", "q1_decode_attn_us", "varlen_attn_us"):
            if isinstance(r.get(k), float):
                r[k.replace("_us", "_gbs")] = nbytes / (r[k] * 1e-6) / 1e9
        print(json.dumps({"reference_kernels": r, "ours_us": us}))


if __name__ == "__main__":
    main()
