"""Compare InferenceStats outputs with the reference's recorded ones: the
GPU-memory fields (device-dependent, None where the reference ran without
CUDA) are dropped, transfer events compared as lists."""

MEMORY = ("gpu_index", "memory_total_bytes", "memory_free_bytes", "memory_used_bytes")


def _strip(d):
    return {k: v for k, v in d.items() if k not in MEMORY}


def normalise(stats):
    out = []
    for s in stats:
        out.append({"prefill_before": _strip(s["prefill_before"]), "prefill": _strip(s["prefill"]),
                    "decode_snapshots": [_strip(x) for x in s["decode_snapshots"]],
                    "decode_final": _strip(s["decode_final"]),
                    "cpu_gpu_events": [list(e) for e in s["cpu_gpu_events"]]})
    return out
