"""Runtime statistics with the reference ``InferenceStats`` schema
(src/common/monitoring/inference_stats.py:12-137, docs/data_format.md:110-128):
cache/GPU snapshots and per-step CPU<->GPU transfer events
``(step, c2g_tokens, g2c_tokens, c2g_bytes, g2c_bytes)``."""
from __future__ import annotations

from collections import defaultdict

import torch


_TOTAL = {}


def gpu_snapshot(index):
    """Device memory in the reference's GPUMonitor fields
    (src/common/monitoring/gpu_monitor.py:10-31), read without a driver
    query: total = the device's memory (looked up once), used = the bytes
    this process's allocator holds.  The reference calls cudaMemGetInfo
    (device-wide); that call took from 0.1 to ~55 ms on a shared B200 while
    another process queried the driver, and the snapshot sits inside the
    decode step every ``interval`` steps."""
    try:
        if index not in _TOTAL:
            _TOTAL[index] = int(torch.cuda.get_device_properties(index).total_memory)
        total = _TOTAL[index]
        used = int(torch.cuda.memory_reserved(index))
    except Exception:
        return {"gpu_index": index, "memory_total_bytes": None, "memory_free_bytes": None,
                "memory_used_bytes": None}
    return {"gpu_index": index, "memory_total_bytes": total, "memory_free_bytes": total - used,
            "memory_used_bytes": used}


class InferenceStats:
    def __init__(self, device, interval=5):
        self.device = torch.device(device)
        self.set_interval(interval)
        self.reset(0)

    def set_interval(self, interval):
        self.interval = interval
        self.enabled = interval > 0

    def reset(self, batch_size):
        self._batch_size = batch_size
        self._before, self._prefill, self._snaps = [], [], []
        self._events = defaultdict(list)
        self._step = defaultdict(lambda: [0, 0, 0, 0])
        self._before_done = False

    def _snap(self, fn, step):
        gpu = gpu_snapshot(self.device.index or 0)
        return [{**s, **gpu} for s in fn(step=step)]

    def record_prefill_before(self, fn):
        if self.enabled and not self._before_done:
            self._before = self._snap(fn, -1)
            self._before_done = True

    def record_prefill(self, fn):
        if self.enabled:
            self._prefill = self._snap(fn, -1)
            self.flush_decode_step(-1)

    def record_decode(self, step, fn):
        if self.enabled:
            self._snaps.append(self._snap(fn, step))

    def record_cpu_gpu_transfer(self, b, c2g_tokens=0, g2c_tokens=0, c2g_bytes=0, g2c_bytes=0):
        if self.enabled:
            acc = self._step[b]
            acc[0] += int(c2g_tokens)
            acc[1] += int(g2c_tokens)
            acc[2] += int(c2g_bytes)
            acc[3] += int(g2c_bytes)

    def flush_decode_step(self, step):
        if not self.enabled:
            return
        for b in sorted(self._step):
            a = self._step[b]
            if any(a):
                self._events[b].append((int(step), *a))
        self._step.clear()

    def get_all_stats(self):
        out = []
        for b in range(self._batch_size):
            snaps = [s[b] for s in self._snaps if b < len(s)]
            pre = self._prefill[b] if b < len(self._prefill) else {}
            out.append({"prefill_before": self._before[b] if b < len(self._before) else {},
                        "prefill": pre, "decode_snapshots": snaps,
                        "decode_final": snaps[-1] if snaps else pre,
                        "cpu_gpu_events": self._events.get(b, [])})
        return out
