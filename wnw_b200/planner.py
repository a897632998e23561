"""``Planner``: the native decode planner behind the C ABI.

Same class name, constructor and method names as the reference's pybind11
``Planner`` (src/algorithms/wnw_cpp/code/planner.cpp:327-341); arguments may
be int32 CPU tensors (as the reference takes) or numpy arrays / lists.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from wnw_b200 import native as N


def _i32(x):
    if hasattr(x, "numpy"):
        x = x.detach().cpu().numpy()
    a = np.ascontiguousarray(np.asarray(x, dtype=np.int32))
    return a


class Planner:
    def __init__(self, num_layers, num_kv_heads, batch_size, num_kv_groups=1):
        h = C.c_void_p()
        N.call("wnw_planner_create", int(num_layers), int(num_kv_heads), int(batch_size),
               int(num_kv_groups), C.byref(h))
        self._h = h
        self.L, self.H, self.B = int(num_layers), int(num_kv_heads), int(batch_size)
        self.S = self.B * self.H

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            N.lib.wnw_planner_destroy(h)
            self._h = None

    # planner.cpp:29-102 --------------------------------------------------
    def set_config(self, top_k_chunks, eviction_lag):
        N.call("wnw_planner_set_config", self._h, int(top_k_chunks), int(eviction_lag))

    def set_seg_count(self, seg_count):
        a = _i32(seg_count)
        N.call("wnw_planner_set_seg_count", self._h, N.ptr(a), a.size)

    def set_chunk_to_segs(self, b, flat_segs, offsets):
        f, o = _i32(flat_segs), _i32(offsets)
        N.call("wnw_planner_set_chunk_to_segs", self._h, int(b), N.ptr(f), f.size, N.ptr(o), o.size)

    def set_class_b(self, layer, kv_heads):
        a = _i32(kv_heads)
        N.call("wnw_planner_set_class_b", self._h, int(layer), N.ptr(a), a.size)

    def set_restore_meta(self, cpu_s, cpu_e, gpu_s, gpu_e):
        a, b, c, d = (_i32(x) for x in (cpu_s, cpu_e, gpu_s, gpu_e))
        N.call("wnw_planner_set_restore_meta", self._h, N.ptr(a), N.ptr(b), N.ptr(c), N.ptr(d), a.size)

    def set_loaded(self, b, segs):
        a = _i32(segs)
        N.call("wnw_planner_set_loaded", self._h, int(b), N.ptr(a), a.size)

    def set_seq_lens(self, seq_lens_flat):
        a = _i32(seq_lens_flat)
        N.call("wnw_planner_set_seq_lens", self._h, N.ptr(a), a.size)

    def get_loaded_segments(self, b):
        n = C.c_int()
        N.call("wnw_planner_get_loaded_segments", self._h, int(b), None, 0, C.byref(n))
        out = np.zeros(max(1, n.value), np.int32)
        N.call("wnw_planner_get_loaded_segments", self._h, int(b), N.ptr(out), out.size, C.byref(n))
        return out[:n.value].tolist()

    # planner.cpp:124-306 -------------------------------------------------
    # planner.cpp:104-122 ----------------------------------------------
    def set_restore_buffers(self, cpu_k, cpu_v, stg_k, stg_v):
        """The host restore store and the staging buffers ``gather_restore``
        copies between; as in the reference, the caller keeps them alive
        (their addresses are used, not copies)."""
        if cpu_k.dim() != 2 or cpu_v.shape != cpu_k.shape or stg_k.shape[1:] != cpu_k.shape[1:] \
                or stg_v.shape != stg_k.shape:
            raise ValueError("restore buffers: [rows, head_dim] tensors of matching shapes expected")
        self._restore = (cpu_k, cpu_v, stg_k, stg_v)

    def gather_restore(self, n_threads=8):
        """Copy the last plan's host ranges, in planner order, to the front of
        the staging buffers."""
        cpu_k, cpu_v, stg_k, stg_v = getattr(self, "_restore", (None,) * 4)
        if cpu_k is None:
            raise RuntimeError("gather_restore before set_restore_buffers")
        r = self.cpu_ranges()
        need = int((r[:, 1] - r[:, 0]).sum()) if r.size else 0
        if need > stg_k.shape[0]:
            raise N.WnwError(3, "gather_restore", f"staging holds {stg_k.shape[0]} rows, the plan needs {need}")
        gather_rows(cpu_k, cpu_v, r, stg_k, stg_v, n_threads)

    def compute_and_prepare(self, topk_idx, topk_off, load_starts_2d, load_lens_2d, cu_new_2d,
                            new_lens_2d, evict_offsets_2d, evict_max, evict_layer_ptr):
        """Fills the caller's int32 output arrays (numpy or CPU tensors) in
        place and returns ``(any_change, total_tokens, ev_starts, ev_ends,
        cpu_ranges[nr, 2])`` like the reference (planner.cpp:124-306): int32
        CPU tensors when the top-k input is a tensor, as the reference's cache
        expects (wnw_cpp/code/cache.py:254-268), numpy arrays otherwise."""
        tk, to = _i32(topk_idx), _i32(topk_off)
        outs = [load_starts_2d, load_lens_2d, cu_new_2d, new_lens_2d, evict_offsets_2d, evict_max,
                evict_layer_ptr]
        for o in outs:
            arr = o.numpy() if hasattr(o, "numpy") else o
            if arr.dtype != np.int32 or not arr.flags["C_CONTIGUOUS"]:
                raise TypeError("planner outputs must be contiguous int32")
        ch, tot = C.c_int(), C.c_int()
        N.call("wnw_planner_compute_and_prepare", self._h, N.ptr(tk) if tk.size else None, N.ptr(to),
               *[N.ptr(o) for o in outs], C.byref(ch), C.byref(tot))
        ev_s, ev_e = self.evictions()
        ranges = self.cpu_ranges()
        if hasattr(topk_idx, "numpy"):
            import torch
            ev_s, ev_e, ranges = (torch.from_numpy(x) for x in (ev_s, ev_e, ranges))
        return ch.value, tot.value, ev_s, ev_e, ranges

    def compute(self, topk_idx, topk_off, out_ptrs):
        """``compute_and_prepare`` for callers that keep the plan on the
        planner (wnw_planner_issue_fetch): int32 numpy top-k input, the seven
        output arrays as pre-taken pointers; returns (any_change, total)."""
        ch, tot = C.c_int(), C.c_int()
        N.call("wnw_planner_compute_and_prepare", self._h, topk_idx.ctypes.data if topk_idx.size else None,
               topk_off.ctypes.data, *out_ptrs, C.byref(ch), C.byref(tot))
        return ch.value, tot.value

    def evictions(self):
        n = C.c_int()
        N.call("wnw_planner_get_evictions", self._h, None, None, 0, C.byref(n))
        s = np.zeros(n.value, np.int32)
        e = np.zeros(n.value, np.int32)
        N.call("wnw_planner_get_evictions", self._h, N.ptr(s) if n.value else None,
               N.ptr(e) if n.value else None, n.value, C.byref(n))
        return s, e

    def cpu_ranges(self):
        n = C.c_int()
        N.call("wnw_planner_get_cpu_ranges", self._h, None, 0, C.byref(n))
        r = np.zeros((n.value, 2), np.int32)
        if n.value:
            N.call("wnw_planner_get_cpu_ranges", self._h, N.ptr(r), n.value, C.byref(n))
        return r

    def layer_transfer_rows(self):
        return self.layer_transfer()[0]

    def layer_transfer(self):
        """(transfer-row offsets [L+1], cpu-range offsets [L+1]) of the last plan."""
        rows = np.zeros(self.L + 1, np.int32)
        rng = np.zeros(self.L + 1, np.int32)
        N.call("wnw_planner_get_layer_transfer", self._h, N.ptr(rows), N.ptr(rng))
        return rows, rng

    def changes(self, b):
        nl, ne = C.c_int(), C.c_int()
        N.call("wnw_planner_get_changes", self._h, int(b), None, 0, C.byref(nl), None, 0, C.byref(ne))
        a = np.zeros(max(1, nl.value), np.int32)
        e = np.zeros(max(1, ne.value), np.int32)
        N.call("wnw_planner_get_changes", self._h, int(b), N.ptr(a), a.size, C.byref(nl), N.ptr(e), e.size,
               C.byref(ne))
        return a[:nl.value].tolist(), e[:ne.value].tolist()

    def device_plan(self, out=None):
        """The rebuild plan blob (int32) for ``wnw_rebuild_segments``; written
        into ``out`` (numpy int32, e.g. a view of pinned memory) when given."""
        used = C.c_int64()
        N.call("wnw_planner_device_plan", self._h, None, 0, C.byref(used))
        if out is None:
            out = np.zeros(used.value, np.int32)
        elif out.size < used.value:
            raise N.WnwError(3, "device_plan", f"buffer of {out.size} ints < {used.value}")
        N.call("wnw_planner_device_plan", self._h, N.ptr(out), out.size, C.byref(used))
        return out[:used.value]


class DevicePlan:
    """Device mirror of a Planner's selection state (wnw_dplan_*): plans each
    step's fetch on the GPU from the device top-k and launches it on the copy
    stream with no host round trip; ``verify`` checks it against the host
    planner once that has planned the same step.  ``create`` returns None
    when the state does not fit the planning kernel (the host path is used)."""

    def __init__(self, h):
        self._h = h

    @classmethod
    def create(cls, planner):
        h = C.c_void_p()
        st = N.lib.wnw_dplan_create(planner._h, C.byref(h))
        if st == N.WNW_ERR_UNSUPPORTED:
            return None
        N.check(st, "wnw_dplan_create")
        return cls(h)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            N.lib.wnw_dplan_destroy(h)
            self._h = None

    def verify(self, planner):
        N.check(N.lib.wnw_dplan_verify(self._h, planner._h), "wnw_dplan_verify")


def gather_rows(src_k, src_v, ranges, dst_k, dst_v, n_threads=8):
    """planner.cpp:113-122: copy the rows of each planned CPU range, in order,
    into ``dst`` (host memory, e.g. pinned staging)."""
    r = _i32(ranges).reshape(-1, 2)
    row_bytes = src_k.shape[1] * src_k.element_size() if hasattr(src_k, "element_size") else \
        src_k.shape[1] * src_k.itemsize
    N.call("wnw_gather_rows", N.ptr(src_k), N.ptr(src_v), int(row_bytes), N.ptr(r) if r.size else None,
           r.shape[0], N.ptr(dst_k), N.ptr(dst_v), int(n_threads))
