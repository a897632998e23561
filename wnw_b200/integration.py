"""Glue for running this package's cache under the reference's own session.

The reference's WnWSession checks every cache it drives against its own base
class (``assert isinstance(cache, FlatVarlenCache)``,
src/algorithms/wnw/code/session.py:43, with ``FlatVarlenCache`` imported at
session.py:11 from src/common/kv/flat_cache.py).  ``B200WnWCache`` implements
that base class's contract (hooks, HF ``Cache`` methods, attributes the session
reads) on its own base, so the check needs widening, not the cache.

Only the session's fused-attention branch is supported (``WNW_FUSED_ATTN=1``,
session.py:17, 85-88): the session then hands attention, append and class-A
scoring to ``cache.fused_decode_attention``.  Its default branch
(session.py:90-112) runs torch's ``varlen_attn`` over a packed copy of every
layer and scores in ``decode_after_attn``; this cache keeps per-segment slots
and builds no packed copy, so that branch is refused here, and
``B200WnWCache.decode_after_attn`` raises should a session reach it anyway.
"""
from __future__ import annotations


class NonFusedSessionError(RuntimeError):
    """The reference session is in its non-fused mode (WNW_FUSED_ATTN unset)."""


def accept_in_reference_session(session_module, *, enable_fused=False):
    """Let the reference session module (``algorithms.wnw.code.session``)
    accept ``wnw_b200`` caches as well as its own; idempotent.

    The module must be in fused-attention mode: it reads ``WNW_FUSED_ATTN``
    once, at import, into ``_FUSED_ATTN``.  When it is not, this raises
    ``NonFusedSessionError`` -- unless ``enable_fused=True``, which switches
    the module to its fused branch (for every cache it drives from then on).
    """
    if not getattr(session_module, "_FUSED_ATTN", False):
        if not enable_fused:
            raise NonFusedSessionError(
                "the reference session module is in its non-fused mode (WNW_FUSED_ATTN != '1' when it was "
                "imported): it would call varlen_attn on packed K/V that B200WnWCache does not build. Set "
                "WNW_FUSED_ATTN=1 before importing it, or pass enable_fused=True")
        session_module._FUSED_ATTN = True
    from wnw_b200.flat_cache import FlatVarlenCache
    cur = session_module.FlatVarlenCache
    classes = cur if isinstance(cur, tuple) else (cur,)
    if FlatVarlenCache not in classes:
        session_module.FlatVarlenCache = classes + (FlatVarlenCache,)
