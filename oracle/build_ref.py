"""Compile the reference's own C++ planner into ``oracle/_ref`` -- TEST
INFRASTRUCTURE ONLY (the checker, never the product).

The source compiles in place from the reference checkout
(``src/algorithms/wnw_cpp/code/planner.cpp``; the checkout named by
``WNW_REFERENCE_ROOT``, by default a ``reference`` directory beside this
repository) with torch's
extension builder, exactly as the reference's ``_ext.py:18-47`` does (-O3),
but with the build directory under ``oracle/_ref`` so the module travels with
the repository snapshot and never lands in a user cache.  No reference source
is copied.

    python oracle/build_ref.py
"""
from __future__ import annotations

import glob
import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
NAME = "wnw_ref_planner"


def source_path():
    root = os.environ.get("WNW_REFERENCE_ROOT",
                          os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))
    return os.path.join(root, "src", "algorithms", "wnw_cpp", "code", "planner.cpp")


def build(verbose=False):
    src = source_path()
    if not os.path.exists(src):
        return None
    os.makedirs(OUT, exist_ok=True)
    from torch.utils.cpp_extension import load
    return load(name=NAME, sources=[src], extra_cflags=["-O3"], build_directory=OUT, verbose=verbose)


def load_prebuilt():
    """Import the compiled reference planner from oracle/_ref (None if absent)."""
    cands = glob.glob(os.path.join(OUT, NAME + "*.so"))
    if not cands:
        return None
    import torch  # noqa: F401  (the module links against libtorch)
    spec = importlib.util.spec_from_file_location(NAME, cands[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    m = build(verbose="-v" in sys.argv)
    print("built" if m is not None else "reference source not found", OUT)
