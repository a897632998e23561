"""Pure-Python restatement of the WnW decode planner -- TEST INFRASTRUCTURE ONLY.

Follows ``src/algorithms/wnw_cpp/code/planner.cpp:19-325`` (class ``Planner``)
whose integer semantics equal the Python path
``src/algorithms/wnw/code/cache.py:609-630`` (selection diff with eviction lag)
and ``cache.py:756-866`` (per-layer evict / load / new-length planning).

Everything here is integer work; the rebuilt C++ planner must match it
bit-for-bit.
"""
from __future__ import annotations

import numpy as np


class OraclePlanner:
    """Same method names and argument meaning as the reference ``Planner``.

    Tensors are replaced by numpy int arrays / Python lists.
    """

    def __init__(self, num_layers, num_kv_heads, batch_size, num_kv_groups=0):
        # planner.cpp:21-27
        self.L = int(num_layers)
        self.H = int(num_kv_heads)
        self.B = int(batch_size)
        self.num_segs = self.B * self.H
        self.loaded = [set() for _ in range(self.B)]
        self.counters = [[] for _ in range(self.B)]
        self.c2s = [[] for _ in range(self.B)]
        self.class_b = [[] for _ in range(self.L)]
        self.top_k = 0
        self.evict_lag = 1
        self.prev_changed = False
        self.seg_count = []
        self.seq_lens = []
        self.cpu_s = self.cpu_e = self.gpu_s = self.gpu_e = None
        self.cpu_ranges = []

    # planner.cpp:29-32
    def set_config(self, top_k_chunks, eviction_lag):
        self.top_k = int(top_k_chunks)
        self.evict_lag = int(eviction_lag)

    # planner.cpp:34
    def set_seg_count(self, seg_count):
        self.seg_count = [int(x) for x in seg_count]

    # planner.cpp:36-45
    def set_chunk_to_segs(self, b, flat_segs, offsets):
        flat_segs = [int(x) for x in flat_segs]
        offsets = [int(x) for x in offsets]
        self.c2s[b] = [flat_segs[offsets[c]:offsets[c + 1]] for c in range(len(offsets) - 1)]

    # planner.cpp:47-51
    def set_class_b(self, layer, kv_heads):
        self.class_b[layer] = [int(x) for x in kv_heads]

    # planner.cpp:53-80 : flattened [L][nseg][seg_count[b]]
    def set_restore_meta(self, cpu_s, cpu_e, gpu_s, gpu_e):
        cs, ce, gs, ge = (list(map(int, a)) for a in (cpu_s, cpu_e, gpu_s, gpu_e))
        self.cpu_s = [[None] * self.num_segs for _ in range(self.L)]
        self.cpu_e = [[None] * self.num_segs for _ in range(self.L)]
        self.gpu_s = [[None] * self.num_segs for _ in range(self.L)]
        self.gpu_e = [[None] * self.num_segs for _ in range(self.L)]
        idx = 0
        for l in range(self.L):
            for fi in range(self.num_segs):
                sc = self.seg_count[fi // self.H]
                self.cpu_s[l][fi] = cs[idx:idx + sc]
                self.cpu_e[l][fi] = ce[idx:idx + sc]
                self.gpu_s[l][fi] = gs[idx:idx + sc]
                self.gpu_e[l][fi] = ge[idx:idx + sc]
                idx += sc

    # planner.cpp:82-87
    def set_loaded(self, b, segs):
        self.loaded[b] = set(int(x) for x in segs)

    # planner.cpp:89-98
    def set_seq_lens(self, seq_lens_flat):
        p = [int(x) for x in seq_lens_flat]
        self.seq_lens = [p[l * self.num_segs:(l + 1) * self.num_segs] for l in range(self.L)]
        self.counters = [[0] * self.seg_count[b] for b in range(self.B)]
        self.prev_changed = False

    # planner.cpp:100-102
    def get_loaded_segments(self, b):
        return sorted(self.loaded[b])

    def gather_restore(self, cpu_k, cpu_v):
        """planner.cpp:113-122 -- rows of every planned CPU range, in plan order."""
        from oracle.kernels import gather_restore
        pairs = [(self.cpu_ranges[i], self.cpu_ranges[i + 1])
                 for i in range(0, len(self.cpu_ranges) - 1, 2)]
        return gather_restore(cpu_k, cpu_v, pairs)

    def compute_and_prepare(self, topk_idx, topk_off):
        """planner.cpp:124-306.

        Returns a dict with the reference's outputs: ``any_change``, ``total``,
        ``load_starts`` [L,nseg], ``load_lens`` [L,nseg], ``cu_new`` [L,nseg+1],
        ``new_lens`` [L,nseg], ``evict_offsets`` [L,nseg+1] (per-layer relative),
        ``evict_max`` [L], ``evict_layer_ptr`` [L+1], ``ev_starts``, ``ev_ends``,
        ``cpu_ranges`` [nr,2] and, for checking the rebuilt planner's richer
        output, ``to_load`` / ``to_evict`` per sample.
        ``load_*``/``cu_new``/``new_lens``/``evict_*`` are only meaningful when
        ``any_change`` is 1 (the reference leaves them untouched otherwise).
        """
        L, S = self.L, self.num_segs
        if not self.prev_changed:
            for l in range(L):
                for fi in range(S):
                    self.seq_lens[l][fi] += 1

        tk = [int(x) for x in topk_idx]
        toff = [int(x) for x in topk_off]
        to_load = [set() for _ in range(self.B)]
        to_evict = [set() for _ in range(self.B)]
        any_change = False
        for b in range(self.B):
            lo, hi = toff[b], toff[b + 1]
            if hi == lo:
                continue
            needed = set()
            for j in range(lo, hi):
                needed.update(self.c2s[b][tk[j]])
            loaded = self.loaded[b]
            cnt = self.counters[b]
            tl_ = {si for si in needed if si not in loaded}
            te_ = set()
            for si in sorted(loaded):
                if si not in needed:
                    cnt[si] += 1
                    if cnt[si] >= self.evict_lag:
                        te_.add(si)
                else:
                    cnt[si] = 0
            loaded |= tl_
            for si in te_:
                loaded.discard(si)
                cnt[si] = 0
            to_load[b] = tl_
            to_evict[b] = te_
            if tl_ or te_:
                any_change = True

        self.cpu_ranges = []
        res = {"to_load": [sorted(x) for x in to_load],
               "to_evict": [sorted(x) for x in to_evict]}
        if not any_change:
            self.prev_changed = False
            res.update(any_change=0, total=0,
                       ev_starts=np.zeros(0, np.int32), ev_ends=np.zeros(0, np.int32),
                       cpu_ranges=np.zeros((0, 2), np.int32))
            return res

        changed = [b for b in range(self.B) if to_load[b] or to_evict[b]]
        layer_new_lens = [[0] * S for _ in range(L)]
        layer_load = [[] for _ in range(L)]
        layer_evict = [[[] for _ in range(S)] for _ in range(L)]
        gts = 0
        for l in range(L):
            for fi in range(S):
                layer_new_lens[l][fi] = self.seq_lens[l][fi] + 1
            for b in changed:
                for kv_h in self.class_b[l]:
                    fi = b * self.H + kv_h
                    seg_len = self.seq_lens[l][fi]
                    sc = self.seg_count[b]
                    gs, ge = self.gpu_s[l][fi], self.gpu_e[l][fi]
                    cs, ce = self.cpu_s[l][fi], self.cpu_e[l][fi]
                    evicted = 0
                    if to_evict[b]:
                        ev = []
                        for si in sorted(to_evict[b]):
                            if cs[si] >= 0 and gs[si] >= 0:
                                ev.append((gs[si], ge[si]))
                                gs[si] = ge[si] = -1
                        ev.sort()
                        evicted = sum(e - s for s, e in ev)
                        if ev:
                            for si in range(sc):
                                if cs[si] < 0 or gs[si] < 0 or si in to_evict[b]:
                                    continue
                                shift = sum(e - s for s, e in ev if e <= gs[si])
                                gs[si] -= shift
                                ge[si] -= shift
                        layer_evict[l][fi] = ev
                    rel = seg_len - evicted
                    loaded_n = 0
                    for si in sorted(to_load[b]):
                        if cs[si] < 0:
                            continue
                        n = ce[si] - cs[si]
                        self.cpu_ranges += [cs[si], ce[si]]
                        layer_load[l].append((fi, gts, n))
                        gs[si] = rel
                        ge[si] = rel + n
                        rel += n
                        loaded_n += n
                        gts += n
                    layer_new_lens[l][fi] = seg_len - evicted + loaded_n + 1

        load_starts = np.full((L, S), -1, np.int32)
        load_lens = np.zeros((L, S), np.int32)
        cu_new = np.zeros((L, S + 1), np.int32)
        new_lens = np.zeros((L, S), np.int32)
        evict_offsets = np.zeros((L, S + 1), np.int32)
        evict_max = np.zeros(L, np.int32)
        elp = np.zeros(L + 1, np.int32)
        ev_s, ev_e = [], []
        for l in range(L):
            for fi, ts, n in layer_load[l]:
                if load_starts[l, fi] < 0:
                    load_starts[l, fi] = ts
                load_lens[l, fi] += n
            for fi in range(S):
                new_lens[l, fi] = layer_new_lens[l][fi]
                cu_new[l, fi + 1] = cu_new[l, fi] + layer_new_lens[l][fi]
            emax = 0
            for fi in range(S):
                for s_, e_ in layer_evict[l][fi]:
                    ev_s.append(s_)
                    ev_e.append(e_)
                evict_offsets[l, fi + 1] = len(ev_s) - (0 if l == 0 else int(elp[l]))
                emax = max(emax, len(layer_evict[l][fi]))
            evict_max[l] = emax
            elp[l + 1] = len(ev_s)
        self.seq_lens = layer_new_lens
        self.prev_changed = True
        res.update(any_change=1, total=gts, load_starts=load_starts, load_lens=load_lens,
                   cu_new=cu_new, new_lens=new_lens, evict_offsets=evict_offsets,
                   evict_max=evict_max, evict_layer_ptr=elp,
                   ev_starts=np.asarray(ev_s, np.int32), ev_ends=np.asarray(ev_e, np.int32),
                   cpu_ranges=np.asarray(self.cpu_ranges, np.int32).reshape(-1, 2))
        return res


def device_fetch_plan(P, topk_rows):
    """Restates, in plain Python, what the device fetch plan kernel
    (wnw_b200/csrc/device_plan.cu) computes from one step's top-k, for the
    planner state ``P`` (an ``OraclePlanner``, whose loaded sets and counters
    are advanced in place as the kernel advances its device copy):

    * per sample with at least one top-k chunk: needed = union of the chunks'
      segments, loads = needed - loaded (ascending); a loaded, unneeded
      segment bumps its counter and is evicted at the lag (counter reset);
      a needed one resets its counter -- the selection diff of
      planner.cpp:124-160 / cache.py:609-630;
    * ranges in the planner's emission order (layer, sample, class-B kv head,
      loaded segment; (layer, head, segment)s without host rows skipped,
      planner.cpp:231-260), each landing at the running row count.

    Returns ``ranges`` [(start, end)], ``dst`` landing rows, ``layer_ranges``
    and ``layer_rows`` ([L+1] offsets)."""
    B, L, H = P.B, P.L, P.H
    loads = []
    for b in range(B):
        chunks = [int(c) for c in topk_rows[b] if int(c) >= 0]
        if not chunks:
            loads.append([])
            continue
        needed = set(s for c in chunks for s in P.c2s[b][c])
        before = set(P.loaded[b])
        cnt = P.counters[b]
        for s in range(P.seg_count[b]):
            if s in before:
                if s in needed:
                    cnt[s] = 0
                else:
                    cnt[s] += 1
                    if cnt[s] >= P.evict_lag:
                        P.loaded[b].discard(s)
                        cnt[s] = 0
        new = sorted(needed - before)
        P.loaded[b] |= set(new)
        loads.append(new)
    ranges, dst, layer_ranges, layer_rows = [], [], [], []
    row = 0
    for l in range(L):
        layer_ranges.append(len(ranges))
        layer_rows.append(row)
        for b in range(B):
            for h in P.class_b[l]:
                cs, ce = P.cpu_s[l][b * H + h], P.cpu_e[l][b * H + h]
                for s in loads[b]:
                    if cs[s] < 0:
                        continue
                    ranges.append((cs[s], ce[s]))
                    dst.append(row)
                    row += ce[s] - cs[s]
    layer_ranges.append(len(ranges))
    layer_rows.append(row)
    return dict(ranges=ranges, dst=dst, layer_ranges=layer_ranges, layer_rows=layer_rows)
