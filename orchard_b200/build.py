"""Ahead-of-time build of the native parts, in-tree.

* ``orchard_b200/lib/liborchard_b200.so`` -- every CUDA kernel and the C ABI declared in
  ``include/orchard_b200.h``, compiled for sm_100a only.
* ``orchard_b200/orchard_core<ext>`` -- the pybind11 module with the reference's
  operator surface (``MetalBackend``, ``Tensor``, ``DType``; src/bindings.cpp), linked
  against the library above with an ``$ORIGIN`` rpath.

Usage: ``python -m orchard_b200.build [--force] [-j N]``.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "liborchard_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = ["capi.cu", "qgemm.cu", "tcgemm.cu", "tcgemm_sk.cu", "gemv.cu", "attention.cu", "attention_prefill.cu", "elementwise.cu", "quantize.cu", "peer_allreduce.cu"]
CORE_SOURCES = ["core_backend.cpp", "core_bindings.cpp"]


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hs + [os.path.join(ROOT, "include", "orchard_b200.h")]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def nvcc_flags(extra=()):
    return [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
            "-Xcompiler", "-fPIC", "-I", os.path.join(ROOT, "include"), "-I", CSRC, *extra]


def build_lib(force=False, jobs=8, verbose=False, ptxas_info=False):
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    hdrs = _headers()
    todo = []
    objs = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ, src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + hdrs):
            extra = ["-Xptxas", "-v"] if ptxas_info else []
            todo.append(nvcc_flags(extra) + ["-c", s, "-o", o])
    with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        for out in ex.map(_run, todo):
            if verbose and out.strip():
                print(out)
    if force or todo or _stale(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart", "-Xlinker", "-soname=liborchard_b200.so"])
    return LIB


def core_ext_path():
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return os.path.join(PKG, "orchard_core" + suffix)


def build_core(force=False):
    """pybind11 module with the reference operator surface, linked to the C ABI."""
    import pybind11

    target = core_ext_path()
    srcs = [os.path.join(CSRC, s) for s in CORE_SOURCES]
    deps = srcs + _headers() + [LIB]
    if not force and not _stale(target, deps):
        return target
    py_inc = sysconfig.get_paths()["include"]
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
           "-I", pybind11.get_include(), "-I", py_inc, "-I", os.path.join(ROOT, "include"),
           "-I", CSRC, *srcs, "-o", target, "-L", LIBDIR, "-lorchard_b200",
           "-Wl,-rpath,$ORIGIN/lib"]
    _run(cmd)
    return target


def build_all(force=False, jobs=8, verbose=False):
    build_lib(force=force, jobs=jobs, verbose=verbose)
    build_core(force=force)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("-v", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    args = ap.parse_args()
    if args.ptxas_info:
        build_lib(force=True, jobs=args.j, verbose=True, ptxas_info=True)
    else:
        build_all(force=args.force, jobs=args.j, verbose=args.v)
    print(LIB)
    sys.exit(0)
