"""Build ``libwnw_b200.so`` in-tree with nvcc for sm_100a.

    python -m wnw_b200.build [--verbose] [--ptxas-info] [--trace]

Objects go to ``wnw_b200/_build/`` (rebuilt when a source or header is newer),
the library to ``wnw_b200/libwnw_b200.so``.  ``--trace`` builds
``wnw_b200/libwnw_b200_trace.so`` instead (objects in ``_build_trace/``):
the same code with the bf16 tensor-core attention kernel recording per-CTA
phase timestamps (``bench.py --mode attn --trace`` reads them); nothing else
changes and the product never loads it.  The CUDA runtime is linked
statically so the library does not depend on which ``libcudart`` the host
process (e.g. torch) loaded first.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libwnw_b200.so")
HEADERS = [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith((".cuh", ".h"))] + \
    [os.path.join(ROOT, "include", "wnw_b200.h")]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-DNDEBUG"]


def _nvcc():
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; set NVCC or put /usr/local/cuda/bin on PATH")
    return cand


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _stale(src, obj):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(x) > t for x in [src] + HEADERS)


TRACE_BUILD = os.path.join(PKG, "_build_trace")
TRACE_LIB = os.path.join(PKG, "libwnw_b200_trace.so")


def _compile(src, ptxas_info, trace=False):
    obj = os.path.join(TRACE_BUILD if trace else BUILD, os.path.basename(src) + ".o")
    if not _stale(src, obj):
        return obj, ""
    cmd = [_nvcc()] + ARCH + NVCC_FLAGS + (["-DWNW_ATTN_TRACE"] if trace else []) + ["-c", src, "-o", obj]
    if ptxas_info and src.endswith(".cu"):
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stderr}")
    return obj, r.stderr


def build(verbose=False, ptxas_info=False, trace=False):
    out_dir, lib = (TRACE_BUILD, TRACE_LIB) if trace else (BUILD, LIB)
    os.makedirs(out_dir, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        results = list(ex.map(lambda s: _compile(s, ptxas_info, trace), srcs))
    objs = [o for o, _ in results]
    if verbose or ptxas_info:
        for (_, log), s in zip(results, srcs):
            if log:
                print(f"--- {os.path.basename(s)}\n{log}")
    if not os.path.exists(lib) or any(os.path.getmtime(o) > os.path.getmtime(lib) for o in objs):
        cmd = [_nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", lib] + objs + ["-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    ap.add_argument("--trace", action="store_true", help="build libwnw_b200_trace.so (attention phase timestamps)")
    a = ap.parse_args()
    try:
        print(build(a.verbose, a.ptxas_info, a.trace))
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
