"""Build the native parts of torch_ans_b200 in-tree (no JIT cache, no pip install).

* ``libtorch_ans_b200.so`` -- the C ABI (include/torch_ans_b200.h): the CUDA kernels, compiled
  with nvcc for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``), CUDA runtime linked
  statically, no torch dependency.
* ``_C<ext>.so`` -- the torch extension module with the reference's op names
  (csrc/bindings.cpp), compiled with g++ against torch's headers and linked to the C ABI library
  through an ``$ORIGIN`` rpath.

Usage: ``python -m torch_ans_b200.build [--force] [--jobs N]``; ``__graft_entry__.build()``
calls :func:`build`.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD_DIR = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libtorch_ans_b200.so")
CU_SOURCES = ["rans_push.cu", "rans_pop.cu", "rans_aux.cu", "rans_pop_fast_v0.cu", "rans_pop_fast_v1.cu",
              "rans_pop_fast_v2.cu", "rans_push_fast_v0.cu", "rans_push_fast_v1.cu", "rans_push_fast_v2.cu",
              "rans_push_ws_v0.cu", "rans_push_ws_v1.cu", "rans_push_ws_v2.cu", "rans_pop_lean_v0.cu",
              "rans_pop_lean_v1.cu", "rans_pop_lean_v2.cu", "rans_noalloc.cu", "rans_ragged.cu", "rans_alias.cu",
              "rans_probe.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def ext_path() -> str:
    return os.path.join(PKG, "_C" + sysconfig.get_config_var("EXT_SUFFIX"))


def _nvcc() -> str:
    cand = [os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc"), shutil.which("nvcc") or ""]
    for c in cand:
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found (set CUDA_HOME)")


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hs + [os.path.join(INCLUDE, "torch_ans_b200.h")]


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print("[torch_ans_b200 build]", " ".join(cmd[:3]), "...", os.path.basename(cmd[-1]))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"command failed: {' '.join(cmd)}")
    return r.stdout + r.stderr


def build_lib(force=False, jobs=8, verbose=True, extra_nvcc=()):
    os.makedirs(BUILD_DIR, exist_ok=True)
    nvcc = _nvcc()
    hdrs = _headers()
    objs, todo = [], []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD_DIR, src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + hdrs):
            todo.append([nvcc, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                         "-Xptxas", "-v", *extra_nvcc, "-c", "-o", o, s])
    with cf.ThreadPoolExecutor(max(1, jobs)) as ex:
        for out in ex.map(lambda c: _run(c, verbose), todo):
            log = os.path.join(BUILD_DIR, "ptxas.log")
            with open(log, "a") as f:
                f.write(out)
    if force or todo or _stale(LIB, objs):
        _run([nvcc, *ARCH, "-shared", "-o", LIB + ".tmp", *objs, "-lpthread", "-ldl", "-lrt"], verbose)
        os.replace(LIB + ".tmp", LIB)
    return LIB


def build_ext(force=False, verbose=True):
    import torch
    from torch.utils import cpp_extension

    src = os.path.join(CSRC, "bindings.cpp")
    out = ext_path()
    if not (force or _stale(out, [src, LIB, os.path.join(INCLUDE, "torch_ans_b200.h")])):
        return out
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cmd = ["g++", "-O2", "-fPIC", "-shared", "-std=c++17", "-w",
           "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           *[f"-I{p}" for p in cpp_extension.include_paths()],
           f"-I{os.path.join(cuda_home, 'include')}", f"-I{sysconfig.get_paths()['include']}",
           "-o", out + ".tmp", src,
           f"-L{PKG}", "-ltorch_ans_b200", "-Wl,-rpath,$ORIGIN",
           f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
           f"-Wl,-rpath,{torch_lib}"]
    _run(cmd, verbose)
    os.replace(out + ".tmp", out)
    return out


def build(force=False, jobs=8, verbose=True):
    """Compile every native part for sm_100a (incremental unless force)."""
    build_lib(force=force, jobs=jobs, verbose=verbose)
    build_ext(force=force, verbose=verbose)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=8)
    a = ap.parse_args()
    build(force=a.force, jobs=a.jobs)
