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
import ctypes as C

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
    flip a near-tie in the top-k).  The gather buffer and the result are
    allocated once per shape; the returned tensor is valid until the next
    call."""

    def __init__(self, group=None):
        self.group = group
        self.world = torch.distributed.get_world_size(group)
        self._buf = None  # [world, n] gather buffer and [n] result, kept from call to call

    def __call__(self, acc):
        if self.world == 1:
            return acc
        x = acc.contiguous().reshape(-1)
        if self._buf is None or self._buf[1].numel() != x.numel() or self._buf[1].dtype != x.dtype \
                or self._buf[1].device != x.device:
            self._buf = (torch.empty(self.world * x.numel(), dtype=x.dtype, device=x.device),
                         torch.empty(x.numel(), dtype=x.dtype, device=x.device))
        flat, out = self._buf
        torch.distributed.all_gather_into_tensor(flat, x, group=self.group)
        parts = flat.view(self.world, -1)
        torch.add(parts[0], parts[1], out=out)
        for r in range(2, self.world):
            out += parts[r]
        return out.reshape(acc.shape)


def slice_kv(x, h0, h1):
    """kv heads [h0, h1) of a [B, Hkv, ...] tensor."""
    return x[:, h0:h1]


def slice_flat(x, h0, h1, num_kv_heads):
    """kv heads [h0, h1) of a segment-major [B * Hkv, ...] tensor."""
    B = x.shape[0] // num_kv_heads
    return x.reshape(B, num_kv_heads, *x.shape[1:])[:, h0:h1].reshape(-1, *x.shape[1:])


class OprojAllReduce:
    """The per-layer tensor-parallel exchange as one kernel
    (``wnw_oproj_allreduce``): y = sum over ranks of x_r . W_r^T, the o_proj
    GEMV of this rank's query heads fused with an all-reduce over NVLink
    peer memory.  Receive buffers and flags are one CUDA-IPC allocation per
    rank, mapped into every other rank's process once, here.

    ``__call__`` must be issued by every rank of the group in the same
    order (each call is one epoch); a rank whose peers do not arrive within
    ``timeout_s`` gets zeros and ``check()`` raises."""

    def __init__(self, dev, n_out, batch=1, dtype=torch.bfloat16, group=None, timeout_s=2.0):
        from wnw_b200 import native as N
        self.N = N
        dev = torch.device(dev)
        self._dev_index = dev.index if dev.index is not None else torch.cuda.current_device()
        self.dev = torch.device("cuda", self._dev_index)
        dist = torch.distributed
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        if self.world > N.TP_MAX_RANKS:
            raise ValueError(f"at most {N.TP_MAX_RANKS} ranks")
        self.batch, self.n_out, self.dtype = batch, n_out, dtype
        nch = N.lib.wnw_oproj_allreduce_chunks(n_out)
        recv_bytes = (2 * self.world * batch * n_out * 4 + 255) // 256 * 256
        total = recv_bytes + self.world * nch * 4
        with torch.cuda.device(self.dev):
            own, handle = C.c_void_p(), (C.c_char * 64)()
            N.call("wnw_ipc_alloc", total, C.byref(own), handle)
            self._own = own.value
            self._peers = {}
            bases = [None] * self.world
            bases[self.rank] = self._own
            if self.world > 1:
                handles = [None] * self.world
                dist.all_gather_object(handles, bytes(handle), group=group)
                for p in range(self.world):
                    if p != self.rank:
                        ptr = C.c_void_p()
                        N.call("wnw_ipc_open", C.create_string_buffer(handles[p], 64), C.byref(ptr))
                        self._peers[p] = ptr.value
                        bases[p] = ptr.value
                dist.barrier(group=group)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.dev)
        a = self.args = N.OprojAllReduceArgs()
        a.dtype = N.dtype_code(dtype)
        a.batch, a.recv_batch, a.n_out, a.rank, a.world = batch, batch, n_out, self.rank, self.world
        for p in range(self.world):
            a.recv[p] = bases[p]
            a.flags[p] = bases[p] + recv_bytes
        a.timeout_ns = int(timeout_s * 1e9)
        a.err = self.err.data_ptr()
        self.epoch = 0

    def __call__(self, x, w, y=None, stream=None):
        """x [B, K] (this rank's heads), w [N, K] -> y [B, N], summed over ranks.

        B may not exceed the batch the receive buffers were built for (the
        kernel stores B rows into every peer's buffer); x, w and y must be
        contiguous device tensors of this exchange's dtype, with w [n_out,
        K] and y [B, n_out]."""
        self._check_shapes(x, w, y)
        a = self.args
        if y is None:
            y = torch.empty(x.shape[0], self.n_out, dtype=self.dtype, device=self.dev)
        self.epoch += 1
        a.epoch = self.epoch
        a.k_in = x.shape[-1]
        a.batch = x.shape[0]
        a.x, a.w, a.y = x.data_ptr(), w.data_ptr(), y.data_ptr()
        sp = stream.cuda_stream if stream is not None else torch._C._cuda_getCurrentRawStream(self._dev_index)
        st = self.N.lib.wnw_oproj_allreduce(C.byref(a), sp)
        if st:
            self.N.check(st, "wnw_oproj_allreduce")
        return y

    def _check_shapes(self, x, w, y):
        if x.dim() != 2 or w.dim() != 2:
            raise ValueError(f"x must be [B, K] and w [N, K]; got {tuple(x.shape)} and {tuple(w.shape)}")
        if not 1 <= x.shape[0] <= self.batch:
            raise ValueError(f"batch {x.shape[0]} not in 1..{self.batch} (the receive buffers' rows)")
        if tuple(w.shape) != (self.n_out, x.shape[1]):
            raise ValueError(f"w must be [{self.n_out}, {x.shape[1]}]; got {tuple(w.shape)}")
        if x.dtype != self.dtype or w.dtype != self.dtype:
            raise TypeError(f"x and w must be {self.dtype}; got {x.dtype} and {w.dtype}")
        if not (x.is_contiguous() and w.is_contiguous()):
            raise ValueError("x and w must be contiguous")
        if x.device != self.dev or w.device != self.dev:
            raise ValueError(f"x and w must live on {self.dev}")
        if y is not None and (tuple(y.shape) != (x.shape[0], self.n_out) or y.dtype != self.dtype
                              or not y.is_contiguous() or y.device != self.dev):
            raise ValueError(f"y must be a contiguous [{x.shape[0]}, {self.n_out}] {self.dtype} tensor on {self.dev}")

    def check(self):
        """Raise if a peer's partials ever failed to arrive (host sync)."""
        if int(self.err.item()) & self.N.DEVERR_PEER_TIMEOUT:
            raise RuntimeError("tensor-parallel o_proj exchange: a peer's partial sums did not arrive in time")

    def close(self):
        """Unmap the peers' buffers and free this rank's (after a device sync)."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.dev)
        for ptr in self._peers.values():
            self.N.call("wnw_ipc_close", ptr, 0)
        self._peers = {}
        if self.world > 1:
            torch.distributed.barrier(group=self.group)  # no peer still maps our buffer
        self.N.call("wnw_ipc_close", self._own, 1)
        self._own = None
