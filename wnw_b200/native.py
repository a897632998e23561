"""ctypes binding of ``libwnw_b200.so`` (declared in ``include/wnw_b200.h``).

Importing this module loads the library or raises ``ImportError`` -- there is
no fallback path.  Build it with ``python -m wnw_b200.build``.
"""
from __future__ import annotations

import ctypes as C
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("WNW_B200_LIB", os.path.join(_PKG, "libwnw_b200.so"))

if not os.path.exists(LIB_PATH):
    raise ImportError(f"libwnw_b200.so not found at {LIB_PATH}; build it with `python -m wnw_b200.build`")
lib = C.CDLL(LIB_PATH)

WNW_OK = 0
WNW_ERR_INVALID = 1
WNW_ERR_CAPACITY = 3
WNW_ERR_UNSUPPORTED = 6
STATUS_NAMES = {0: "ok", 1: "invalid argument", 2: "CUDA error", 3: "capacity exceeded",
                4: "invalid state", 5: "timed out", 6: "unsupported"}
DEVERR_MBAR_TIMEOUT = 1
DEVERR_LEN_MISMATCH = 2
DEVERR_CAPACITY = 4
DEVERR_PEER_TIMEOUT = 8
DEVERR_BAD_INDEX = 16

F32, F16, BF16 = 0, 1, 2


class WnwError(RuntimeError):
    """A C-ABI call returned a non-OK status."""

    def __init__(self, status, func, msg):
        self.status = status
        super().__init__(f"{func}: {STATUS_NAMES.get(status, status)}: {msg}")


P = C.c_void_p
I32P = C.POINTER(C.c_int32)
I64P = C.POINTER(C.c_int64)


class DecodeAttnArgs(C.Structure):
    _fields_ = [
        ("dtype", C.c_int), ("head_dim", C.c_int), ("group", C.c_int), ("num_segs", C.c_int),
        ("num_kv_heads", C.c_int),
        ("q", P), ("new_k", P), ("new_v", P), ("k_store", P), ("v_store", P),
        ("seg_base", P), ("seg_len", P), ("seg_cap", P), ("work", P),
        ("n_clusters", C.c_int), ("cluster_size", C.c_int), ("split_rows", C.c_int),
        ("out", P), ("scale", C.c_float),
        ("score_slot", P), ("audio_start", P), ("audio_end", P), ("logits", P), ("logits_off", P),
        ("stats", P), ("partials", P), ("counters", P), ("err", P), ("store_rows", C.c_int64),
        ("plan", P), ("plan_ctas", C.c_int), ("plan_parts", C.c_int), ("plan_combine", C.c_int),
        ("flags", C.c_int),
    ]


ATTN_ROWS_READY = 1


class AttnPlanInfo(C.Structure):
    _fields_ = [("ctas", C.c_int), ("cluster", C.c_int), ("parts", C.c_int), ("combine", C.c_int),
                ("ints", C.c_int64)]


TP_MAX_RANKS = 8


class OprojAllReduceArgs(C.Structure):
    _fields_ = [
        ("dtype", C.c_int), ("batch", C.c_int), ("n_out", C.c_int), ("k_in", C.c_int),
        ("recv_batch", C.c_int), ("rank", C.c_int), ("world", C.c_int), ("x", P), ("w", P), ("y", P),
        ("recv", P * TP_MAX_RANKS), ("flags", P * TP_MAX_RANKS), ("epoch", C.c_uint32),
        ("timeout_ns", C.c_uint64), ("err", P),
    ]


MASK_NONE, MASK_CAUSAL, MASK_ADDITIVE = 0, 1, 2


class PrefillTask(C.Structure):
    _fields_ = [("batch", C.c_int32), ("kv_head", C.c_int32), ("head_off", C.c_int32), ("n_heads", C.c_int32),
                ("row0", C.c_int32), ("n_rows", C.c_int32), ("audio_start", C.c_int32), ("audio_end", C.c_int32),
                ("out_off", C.c_int64)]


class PrefillScoresArgs(C.Structure):
    _fields_ = [
        ("dtype", C.c_int), ("head_dim", C.c_int), ("batch", C.c_int), ("num_q_heads", C.c_int),
        ("num_kv_heads", C.c_int), ("seq_len", C.c_int), ("num_tasks", C.c_int), ("num_heads", C.c_int),
        ("max_rows", C.c_int), ("max_audio", C.c_int),
        ("q", P), ("q_stride_b", C.c_int64), ("q_stride_h", C.c_int64), ("q_stride_s", C.c_int64),
        ("k", P), ("k_stride_b", C.c_int64), ("k_stride_h", C.c_int64), ("k_stride_s", C.c_int64),
        ("mask_kind", C.c_int), ("mask", P), ("mask_stride_b", C.c_int64), ("mask_stride_s", C.c_int64),
        ("scaling", C.c_float), ("tasks", P), ("heads", P), ("out", P), ("out_len", C.c_int64), ("scratch", P),
        ("scratch_bytes", C.c_int64), ("err", P),
    ]


class FetchInfo(C.Structure):
    _fields_ = [("plan_ints", C.c_int64), ("total_rows", C.c_int64), ("n_ranges", C.c_int64),
                ("max_moved_rows", C.c_int64), ("fetch_launches", C.c_int64), ("layer_changed", P)]


def _sig(name, restype, *argtypes):
    f = getattr(lib, name)
    f.restype = restype
    f.argtypes = list(argtypes)
    return f


_S = C.c_int  # wnw_status
_sig("wnw_abi_version", C.c_int)
_sig("wnw_status_string", C.c_char_p, _S)
_sig("wnw_last_error", C.c_char_p)
_sig("wnw_decode_attn", _S, C.POINTER(DecodeAttnArgs), P)
_sig("wnw_decode_attn_noalloc", _S, C.POINTER(DecodeAttnArgs), P)
_sig("wnw_split_rows", C.c_int, C.c_int, C.c_int)
_sig("wnw_attn_launch_shape", _S, C.c_int, C.c_int, P, C.c_int, C.POINTER(C.c_int), C.POINTER(C.c_int))
_sig("wnw_build_work_table", _S, P, C.c_int, C.c_int, C.c_int, P, C.c_int, C.POINTER(C.c_int))
_sig("wnw_attn_plan", _S, P, C.c_int, C.c_int, C.c_int, P, C.c_int64, C.POINTER(AttnPlanInfo))
_sig("wnw_advance_lengths", _S, P, C.c_int64, P)
_sig("wnw_score_finalize", _S, P, P, P, P, P, P, C.c_int, C.c_int, P, C.c_int, P, P)
_sig("wnw_chunk_topk", _S, P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P, P, P, P)
_sig("wnw_rebuild_segments", _S, C.c_int, C.c_int, P, P, P, P, P, C.c_int, P, P, C.c_int64, P, C.c_int64, C.c_int,
     P, P, C.c_int64, P, P, P)
_sig("wnw_copy_segments", _S, C.c_int, C.c_int, P, P, P, P, P, P, P, C.c_int, P)
_sig("wnw_interleave_append", _S, C.c_int, C.c_int, P, P, P, C.c_int, P, P)
_sig("wnw_planner_create", _S, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(P))
_sig("wnw_planner_destroy", None, P)
_sig("wnw_planner_set_config", _S, P, C.c_int, C.c_int)
_sig("wnw_planner_set_seg_count", _S, P, P, C.c_int)
_sig("wnw_planner_set_chunk_to_segs", _S, P, C.c_int, P, C.c_int, P, C.c_int)
_sig("wnw_planner_set_class_b", _S, P, C.c_int, P, C.c_int)
_sig("wnw_planner_set_restore_meta", _S, P, P, P, P, P, C.c_int64)
_sig("wnw_planner_set_loaded", _S, P, C.c_int, P, C.c_int)
_sig("wnw_planner_set_seq_lens", _S, P, P, C.c_int64)
_sig("wnw_planner_get_loaded_segments", _S, P, C.c_int, P, C.c_int, C.POINTER(C.c_int))
_sig("wnw_planner_compute_and_prepare", _S, P, P, P, P, P, P, P, P, P, P, C.POINTER(C.c_int),
     C.POINTER(C.c_int))
_sig("wnw_planner_get_evictions", _S, P, P, P, C.c_int, C.POINTER(C.c_int))
_sig("wnw_planner_get_cpu_ranges", _S, P, P, C.c_int, C.POINTER(C.c_int))
_sig("wnw_planner_get_layer_transfer", _S, P, P, P)
_sig("wnw_planner_get_changes", _S, P, C.c_int, P, C.c_int, C.POINTER(C.c_int), P, C.c_int,
     C.POINTER(C.c_int))
_sig("wnw_planner_device_plan", _S, P, P, C.c_int64, C.POINTER(C.c_int64))
_sig("wnw_gather_rows", _S, P, P, C.c_int64, P, C.c_int, P, P, C.c_int)
_sig("wnw_h2d_async", _S, P, P, P, P, C.c_int64, P, P)
_sig("wnw_stream_wait_event", _S, P, P)
_sig("wnw_copy_async", _S, P, P, C.c_int64, P)
_sig("wnw_copy_mapped", _S, P, P, C.c_int64, C.c_int, P)
_sig("wnw_decode_attn_step", _S, C.POINTER(DecodeAttnArgs), P, P, P, P, P)
_sig("wnw_planner_issue_fetch", _S, P, P, P, C.c_int64, P, P, P, P, C.c_int64, P, P, C.c_int64, P, P, C.c_int64,
     C.c_int, P, P, C.POINTER(FetchInfo))
_sig("wnw_planner_upload_plan", _S, P, P, P, C.c_int64, P, C.POINTER(FetchInfo))
_sig("wnw_dplan_create", _S, P, C.POINTER(C.c_void_p))
_sig("wnw_dplan_destroy", None, P)
_sig("wnw_dplan_step", _S, P, P, C.c_int, P, P, P, C.c_int64, P, P, C.c_int64, C.c_int, P, P, P)
_sig("wnw_dplan_verify", _S, P, P)
_sig("wnw_oproj_allreduce_chunks", C.c_int, C.c_int)
_sig("wnw_oproj_allreduce", _S, C.POINTER(OprojAllReduceArgs), P)
_sig("wnw_ipc_alloc", _S, C.c_int64, C.POINTER(C.c_void_p), P)
_sig("wnw_ipc_open", _S, P, C.POINTER(C.c_void_p))
_sig("wnw_ipc_close", _S, P, C.c_int)
_sig("wnw_host_device_pointer", _S, P, C.POINTER(P))
_sig("wnw_fetch_rows", _S, P, P, C.c_int64, P, P, C.c_int, P, P, C.c_int, P)
_sig("wnw_fetch_layers", _S, P, P, C.c_int64, P, P, P, C.c_int, P, P, C.c_int, P, P)
_sig("wnw_prefill_scores", _S, C.POINTER(PrefillScoresArgs), P)
_sig("wnw_attn_resident_clusters", _S, C.c_int, C.c_int, C.POINTER(C.c_int))
_sig("wnw_rebuild_layers", _S, C.c_int, C.c_int, C.c_int, P, P, P, P, P, P, P, P, P, C.c_int64, P, C.c_int64,
     P, P, C.c_int64, P, P, P, P, P)
_sig("wnw_rebuild_layers_fused", _S, C.c_int, C.c_int, C.c_int, P, P, P, P, P, P, P, P, P, C.c_int64, P,
     C.c_int64, P, P, C.c_int64, P, C.c_int64, P, P, P, P)
_sig("wnw_prefill_scores_scratch_bytes", _S, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int64))

#: every symbol the header declares (checked by the CPU test suite)
EXPORTS = [
    "wnw_abi_version", "wnw_status_string", "wnw_last_error", "wnw_decode_attn", "wnw_decode_attn_noalloc",
    "wnw_split_rows", "wnw_attn_launch_shape",
    "wnw_build_work_table", "wnw_attn_plan", "wnw_advance_lengths", "wnw_score_finalize", "wnw_chunk_topk",
    "wnw_rebuild_segments", "wnw_copy_segments", "wnw_interleave_append", "wnw_planner_create",
    "wnw_planner_destroy", "wnw_planner_set_config", "wnw_planner_set_seg_count",
    "wnw_planner_set_chunk_to_segs", "wnw_planner_set_class_b", "wnw_planner_set_restore_meta",
    "wnw_planner_set_loaded", "wnw_planner_set_seq_lens", "wnw_planner_get_loaded_segments",
    "wnw_planner_compute_and_prepare", "wnw_planner_get_evictions", "wnw_planner_get_cpu_ranges",
    "wnw_planner_get_layer_transfer", "wnw_planner_get_changes", "wnw_planner_device_plan",
    "wnw_gather_rows", "wnw_h2d_async", "wnw_stream_wait_event", "wnw_planner_issue_fetch", "wnw_copy_async", "wnw_copy_mapped", "wnw_decode_attn_step", "wnw_oproj_allreduce",
    "wnw_oproj_allreduce_chunks", "wnw_ipc_alloc", "wnw_ipc_open", "wnw_ipc_close", "wnw_host_device_pointer", "wnw_fetch_rows",
    "wnw_fetch_layers", "wnw_planner_upload_plan", "wnw_dplan_create", "wnw_dplan_destroy", "wnw_dplan_step",
    "wnw_dplan_verify", "wnw_prefill_scores", "wnw_prefill_scores_scratch_bytes", "wnw_attn_resident_clusters",
    "wnw_rebuild_layers", "wnw_rebuild_layers_fused",
]


def check(status, func="wnw"):
    """Raise ``WnwError`` for a non-OK status."""
    if status != WNW_OK:
        raise WnwError(status, func, lib.wnw_last_error().decode(errors="replace"))


def call(name, *args):
    check(getattr(lib, name)(*args), name)


def ptr(t):
    """Device or host address of a tensor / ndarray (None -> NULL)."""
    if t is None:
        return None
    if hasattr(t, "data_ptr"):
        return t.data_ptr()
    if hasattr(t, "ctypes"):
        return t.ctypes.data
    raise TypeError(f"cannot take the address of {type(t)}")


def dtype_code(torch_dtype):
    import torch
    codes = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}
    if torch_dtype not in codes:
        raise TypeError(f"unsupported dtype {torch_dtype}")
    return codes[torch_dtype]


def stream_ptr(stream=None):
    import torch
    s = torch.cuda.current_stream() if stream is None else stream
    return s.cuda_stream
