"""CPU oracle for the WnW decode hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain numpy / CPU torch, the algorithms of the
XMUDeepLIT/WnW decode path (Triton kernels, the Python cache state machine and
the C++ planner).  Every function cites the reference file:line it follows.

It is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import
it.  The shipped ``wnw_b200`` package never imports anything from here and fails
loudly when its CUDA library is missing.

Pinning: the restatements are checked against golden vectors produced by
running the reference itself in the build container (``tests/golden``), and the
planner additionally against the reference's own ``planner.cpp`` compiled into
``oracle/_ref`` by ``oracle/build_ref.py``.
"""
