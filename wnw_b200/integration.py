"""Glue for running this package's cache under the reference's own session.

The reference's WnWSession checks every cache it drives against its own base
class (``assert isinstance(cache, FlatVarlenCache)``,
src/algorithms/wnw/code/session.py:43, with ``FlatVarlenCache`` imported at
session.py:11 from src/common/kv/flat_cache.py).  ``B200WnWCache`` implements
that base class's contract (hooks, HF ``Cache`` methods, attributes the session
reads) on its own base, so the check needs widening, not the cache.
"""
from __future__ import annotations


def accept_in_reference_session(session_module):
    """Let the reference session module (``algorithms.wnw.code.session``)
    accept ``wnw_b200`` caches as well as its own; idempotent."""
    from wnw_b200.flat_cache import FlatVarlenCache
    cur = session_module.FlatVarlenCache
    classes = cur if isinstance(cur, tuple) else (cur,)
    if FlatVarlenCache not in classes:
        session_module.FlatVarlenCache = classes + (FlatVarlenCache,)
