"""Tensor parallelism by KV head for the decode hot path.

Every (sample, kv head) segment's attention is independent, so rank r of a
group of P owns kv heads ``[r*H/P, (r+1)*H/P)`` of every layer -- with their
query heads, their class-B host store, their planner state and their slice of
o_proj -- and runs an ordinary ``B200WnWCache`` over those heads with
``shard_config``'s re-indexed head classes.  Two exchanges remain:

* per step, the class-A score accumulator: each rank sums only its own
  class-A heads, and top-k must see the sum over all of them, so
  ``ScoreReducer`` gathers every rank's accumulator and adds them in rank
  order (the same fp32 additions on every rank, so every rank selects the
  same chunks and their planners stay in step);
* per layer, the o_proj partial sums of the attention output (the model's
  row-parallel projection), an all-reduce over NVLink.

The reference has no tensor-parallel mode; its multi-GPU runs are
independent per-request replicas (src/eval/launch_wnw.py), which
``bench.py --gpus N`` keeps as its default.
"""
from __future__ import annotations

import copy

import torch


def head_range(rank, world, num_kv_heads):
    """kv heads [h0, h1) owned by ``rank``."""
    if world < 1 or num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} kv heads do not split over {world} ranks")
    n = num_kv_heads // world
    return rank * n, (rank + 1) * n


def shard_config(cfg, rank, world, num_layers, num_kv_heads, num_q_heads):
    """The ``WnWConfig`` of one rank: class-A q heads, class-B kv heads and
    retention ratios of its kv heads, re-indexed to local head ids (global
    ids are layer * heads + head, as in the reference's config)."""
    h0, h1 = head_range(rank, world, num_kv_heads)
    g = num_q_heads // num_kv_heads
    hl, ql = h1 - h0, (h1 - h0) * g
    class_a, class_b, ratios = [], [], []
    for gid in cfg.class_a:
        l, q = divmod(gid, num_q_heads)
        if h0 * g <= q < h1 * g:
            class_a.append(l * ql + q - h0 * g)
    for gid in cfg.class_b:
        l, kv = divmod(gid, num_kv_heads)
        if h0 <= kv < h1:
            class_b.append(l * hl + kv - h0)
    for l in range(num_layers):
        ratios.extend(cfg.retention_ratios[l * num_kv_heads + h0:l * num_kv_heads + h1])
    out = copy.copy(cfg)
    out.class_a, out.class_b, out.retention_ratios = sorted(class_a), sorted(class_b), ratios
    out.num_layers, out.num_kv_heads, out.num_q_heads = num_layers, hl, ql
    out.__post_init__()
    return out


class ScoreReducer:
    """Sum of every rank's fp32 score accumulator, in rank order.

    ``all_gather`` then ``acc = x_0 + x_1 + ... + x_{P-1}`` elementwise, so
    the result is bit-identical on every rank (an all-reduce may sum in a
    different order per rank or per algorithm, and a one-ulp difference can
    flip a near-tie in the top-k)."""

    def __init__(self, group=None):
        self.group = group
        self.world = torch.distributed.get_world_size(group)

    def __call__(self, acc):
        if self.world == 1:
            return acc
        parts = [torch.empty_like(acc) for _ in range(self.world)]
        torch.distributed.all_gather(parts, acc.contiguous(), group=self.group)
        out = parts[0].clone()
        for p in parts[1:]:
            out += p
        return out


def slice_kv(x, h0, h1):
    """kv heads [h0, h1) of a [B, Hkv, ...] tensor."""
    return x[:, h0:h1]


def slice_flat(x, h0, h1, num_kv_heads):
    """kv heads [h0, h1) of a segment-major [B * Hkv, ...] tensor."""
    B = x.shape[0] // num_kv_heads
    return x.reshape(B, num_kv_heads, *x.shape[1:])[:, h0:h1].reshape(-1, *x.shape[1:])
