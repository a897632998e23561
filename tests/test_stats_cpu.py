"""InferenceStats (wnw_b200.stats) against the reference's own, driven by the
same scripted call sequence (tests/golden/stats.json, recorded by executing
the reference's InferenceStats): snapshots, interval, once-only prefill
snapshot, per-sample transfer events, all-zero entries skipped."""
import json
import os

import torch

from tests.stats_compare import normalise
from wnw_b200.stats import InferenceStats


def test_scripted_stats_match_reference(golden_dir):
    with open(os.path.join(golden_dir, "stats.json")) as f:
        ref = json.load(f)["scripted"]
    st = InferenceStats(torch.device("cpu"), interval=2)
    st.reset(3)

    def snap(step=-1):
        return [{"step": step, "b": b, "x": b * 10 + max(step, 0)} for b in range(3)]

    st.record_prefill_before(snap)
    st.record_prefill_before(snap)
    st.record_cpu_gpu_transfer(0, g2c_tokens=7, g2c_bytes=70)
    st.record_cpu_gpu_transfer(2, c2g_tokens=3, c2g_bytes=30)
    st.record_prefill(snap)
    for step in range(1, 6):
        st.record_cpu_gpu_transfer(step % 3, c2g_tokens=step, c2g_bytes=step * 11)
        st.record_cpu_gpu_transfer(1, c2g_tokens=0)
        st.flush_decode_step(step)
        if step % st.interval == 0:
            st.record_decode(step, snap)
    got = st.get_all_stats()
    assert normalise(got) == normalise(ref)
    assert got[0]["prefill"]["memory_total_bytes"] is None  # no CUDA device: None, as the reference
