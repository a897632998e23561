"""Small standalone decode-attention case for profiling (ncu) and timing.

Builds `--layers` independent layer states with the config-2 (Voxtral-Mini)
segment geometry -- batch 1, 8 kv heads: two class-A segments of 15,100 rows
and six class-B segments of 2,300 rows, bf16, head_dim 128, GQA 4 -- with
class-A scoring on, and launches the decode-attention kernel over the layers
round-robin (~180 MB for 8 layers: more than L2, so each launch reads HBM).

    python -m wnw_b200.profile_case [--layers 8] [--reps 20] [--cluster C --tiles T]

Prints the mean launch time and the algorithmic-bytes bandwidth.
"""
from __future__ import annotations

import argparse
import json

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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--reps", type=int, default=20)
    ap.add_argument("--cluster", type=int, default=0, help="CTAs per cluster (0: library choice)")
    ap.add_argument("--class-a", type=int, default=15100)
    ap.add_argument("--class-b", type=int, default=2300)
    ap.add_argument("--tiles", type=int, default=0, help="128-row tiles streamed per CTA (0: library choice)")
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


if __name__ == "__main__":
    main()
