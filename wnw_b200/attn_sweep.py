"""Kernel-only decode-attention sweep (the BASELINE config-5 grid).

Random bf16 K/V/q ~ N(0, 1), 8 kv heads x head_dim 128, GQA 4.  Per sample,
the first round(frac_a * 8) kv heads are class A (the whole context) and the
rest class B (retained * context rows).  Each cell lays out one layer per
slot as the cache does, takes the library's launch shape, and times
back-to-back launches round-robin over enough layer copies that the working
set exceeds L2 (CUDA events).  Prints one JSON line per cell with the
algorithmic bytes (K + V rows + q in + o out) per launch and GB/s.

    python -m wnw_b200.attn_sweep [--batch 1,16,64,256] [--ctx 1024,8192,32768,131072]
                                  [--frac-a 0.1,0.3,0.5,1.0] [--retained 0.1,0.25,0.5,1.0]
                                  [--reps 10] [--max-gb 48] [--check]
"""
from __future__ import annotations

import argparse
import json
import math

import numpy as np
import torch

from wnw_b200 import kernels as Kx

H, D, G = 8, 128, 4
L2_BYTES = 126 << 20


def cell_lens(batch, ctx, frac_a, retained):
    n_a = min(H, max(0, round(frac_a * H)))
    lb = max(1, int(retained * ctx))
    return [ctx if h < n_a else lb for _ in range(batch) for h in range(H)]


def build(dev, lens, seed):
    dtype = torch.bfloat16
    S = len(lens)
    cap = np.asarray(lens, np.int64) + 16
    cap_al = (cap + 15) // 16 * 16
    base = np.concatenate([[0], np.cumsum(cap_al)[:-1]]).astype(np.int64)
    rows = int(cap_al.sum())
    g = torch.Generator(device=dev).manual_seed(seed)
    ks = torch.randn(rows, D, device=dev, generator=g, dtype=dtype)
    vs = torch.randn(rows, D, device=dev, generator=g, dtype=dtype)
    q = torch.randn(S, G, D, device=dev, generator=g, dtype=dtype)
    split, cs = Kx.attn_launch_shape(dtype, D, cap)
    work = torch.from_numpy(Kx.build_work_table(cap, split, cs)).to(dev)
    scratch = Kx.AttnScratch(dev, work.shape[0], G, D, S)
    args = Kx.make_attn_args(dtype, S, G, D, ks, vs, torch.from_numpy(base).to(dev),
                             torch.tensor(lens, dtype=torch.int32, device=dev), work, cs, D ** -0.5, scratch,
                             seg_cap=torch.from_numpy(cap.astype(np.int32)).to(dev), num_kv_heads=H, split=split)
    return args, q, torch.empty_like(q), (split, cs, int(work.shape[0]) * cs), (ks, vs, base)


def check_cell(lens, layer):
    """Max |error| of up to 4 segments (first / last class-A and class-B) of
    a launched layer against softmax(q K^T / sqrt(d)) V in fp32 (torch)."""
    _, q, out, _, (ks, vs, base) = layer
    S = len(lens)
    pick = sorted({0, S - 1, next((s for s in range(S) if lens[s] != lens[0]), 0),
                   max((s for s in range(S) if lens[s] != lens[-1]), default=S - 1)})
    err = 0.0
    for s in pick:
        k = ks[base[s]:base[s] + lens[s]].float()
        v = vs[base[s]:base[s] + lens[s]].float()
        p = torch.softmax(q[s].float() @ k.t() * D ** -0.5, dim=-1)
        err = max(err, float((p @ v - out[s].float()).abs().max()))
    return err


def run_cell(dev, batch, ctx, frac_a, retained, reps, max_gb, check=False):
    lens = cell_lens(batch, ctx, frac_a, retained)
    nbytes = int(np.sum(lens)) * D * 2 * 2 + len(lens) * G * D * 2 * 2
    store = (int(np.sum(lens)) + 16 * len(lens)) * D * 2 * 2
    if store > max_gb * 1e9:
        return {"batch": batch, "ctx": ctx, "frac_a": frac_a, "retained": retained, "skipped": "exceeds --max-gb"}
    # enough layer copies that consecutive launches cannot hit in L2 (one
    # copy once a layer is far larger than L2)
    n_layers = 1 if store > 8 * L2_BYTES else max(2, math.ceil(2 * L2_BYTES / store))
    layers = [build(dev, lens, seed=l) for l in range(n_layers)]
    st = torch.cuda.current_stream().cuda_stream
    for args, q, out, _, _ in layers:
        Kx.launch_attn(args, q, None, None, out, st)
    torch.cuda.synchronize()
    err = check_cell(lens, layers[0]) if check else None
    n = max(reps, math.ceil(20 / n_layers)) * n_layers
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(n):
        args, q, out, _, _ = layers[i % n_layers]
        Kx.launch_attn(args, q, None, None, out, st)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / n
    split, cs, ctas = layers[0][3]
    del layers
    torch.cuda.empty_cache()
    return {"batch": batch, "ctx": ctx, "frac_a": frac_a, "retained": retained, "bytes": nbytes,
            "us": us, "gbs": nbytes / (us * 1e-6) / 1e9, "split_rows": split, "cluster": cs, "ctas": ctas,
            "layers": n_layers, **({"max_abs_err": err} if check else {})}


def main():
    ap = argparse.ArgumentParser()
    f = lambda t: [float(x) for x in t.split(",")]
    i = lambda t: [int(x) for x in t.split(",")]
    ap.add_argument("--batch", type=i, default=[1, 16, 64, 256])
    ap.add_argument("--ctx", type=i, default=[1024, 8192, 32768, 131072])
    ap.add_argument("--frac-a", type=f, default=[0.1, 0.3, 0.5, 1.0])
    ap.add_argument("--retained", type=f, default=[0.1, 0.25, 0.5, 1.0])
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--max-gb", type=float, default=48.0)
    ap.add_argument("--check", action="store_true", help="compare sampled segments with a torch fp32 reference")
    a = ap.parse_args()
    dev = torch.device("cuda:0")
    for b in a.batch:
        for c in a.ctx:
            for fa in a.frac_a:
                for r in a.retained:
                    print(json.dumps(run_cell(dev, b, c, fa, r, a.reps, a.max_gb, a.check)), flush=True)


if __name__ == "__main__":
    main()
