"""Compile the reference torch_ans CPU path into ``oracle/_ref`` (test infrastructure only).

The reference's own CPU backend (``torch_ans/rans_cpu.cpp`` + ``torch_ans/rans_utils.hpp``),
its dispatch/serialisation glue (``torch_ans/rans.cpp``, ``torch_ans/rans.hpp``) and its pybind
module (``torch_ans/lib.cpp``) are compiled with g++ straight from the files where they lie in the
reference checkout -- the reference's setup.py is not run and no source is copied into this
repository.  The checkout is the folder named by the ``TORCH_ANS_REFERENCE`` environment variable,
else a folder ``reference`` beside this repository's root.  The result is ``oracle/_ref/torch_ans_ref/_C<ext>.so`` (git-ignored; it travels to the
GPU box next to the library's own built files).  It exposes exactly the reference ``_C`` surface
(``rans64_push`` ...) on CPU tensors and is used by:

* ``tests/golden/make_golden.py`` to write the golden vectors that pin ``oracle/rans_oracle.c``;
* the tests, as a second checker when it is present;
* ``bench.py --impl reference`` as the reference CPU implementation timed on the host cores.

Build flags follow the reference build (``setup.py:33-40``: ``-std=c++17 -O3 -fopenmp``) except
``-march=native``, replaced by ``-march=x86-64-v3`` so the binary built here also runs on the GPU
box's host CPU.  ``WITH_CUDA`` is not defined, so only the CPU path is built.

Usage: ``python oracle/build_ref.py [--reference PATH] [--force]``
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref", "torch_ans_ref")
SOURCES = ("torch_ans/lib.cpp", "torch_ans/rans.cpp", "torch_ans/rans_cpu.cpp")


def default_reference() -> str:
    """The reference checkout: $TORCH_ANS_REFERENCE, else ``reference`` beside the repository."""
    env = os.environ.get("TORCH_ANS_REFERENCE")
    if env:
        return env
    return os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")


def target_path() -> str:
    return os.path.join(OUT_DIR, "_C" + sysconfig.get_config_var("EXT_SUFFIX"))


def build(reference: str | None = None, force: bool = False, verbose: bool = True) -> str | None:
    """Compile the reference CPU extension; returns the .so path, or None when the sources are absent."""
    reference = reference or default_reference()
    out = target_path()
    srcs = [os.path.join(reference, s) for s in SOURCES]
    if not all(os.path.exists(s) for s in srcs):
        if verbose:
            print(f"[oracle/_ref] reference sources not found under {reference}; "
                  f"using prebuilt {out if os.path.exists(out) else '(none)'}")
        return out if os.path.exists(out) else None
    if os.path.exists(out) and not force:
        newest = max(os.path.getmtime(s) for s in srcs)
        if os.path.getmtime(out) >= newest:
            return out
    import torch
    from torch.utils import cpp_extension

    os.makedirs(OUT_DIR, exist_ok=True)
    with open(os.path.join(OUT_DIR, "__init__.py"), "w") as f:
        f.write("# compiled reference torch_ans CPU path (checker only); see oracle/build_ref.py\n")
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    inc = [f"-I{p}" for p in cpp_extension.include_paths()]
    inc += [f"-I{sysconfig.get_paths()['include']}", f"-I{os.path.join(reference, 'torch_ans')}"]
    objs = []
    build_dir = os.path.join(HERE, "_build")
    os.makedirs(build_dir, exist_ok=True)
    for s in srcs:
        o = os.path.join(build_dir, os.path.basename(s) + ".o")
        cmd = ["g++", "-c", s, "-o", o, "-fPIC", "-std=c++17", "-O3", "-fopenmp", "-march=x86-64-v3",
               "-DNDEBUG", "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H",
               f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-w"] + inc
        if verbose:
            print("[oracle/_ref]", " ".join(cmd[:4]), "...")
        subprocess.run(cmd, check=True)
        objs.append(o)
    link = ["g++", "-shared", "-o", out] + objs + [
        f"-L{torch_lib}", "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-fopenmp",
        f"-Wl,-rpath,{torch_lib}"]
    subprocess.run(link, check=True)
    if verbose:
        print("[oracle/_ref] built", out)
    return out


def load():
    """Import the compiled reference ``_C`` module (``torch_ans_ref._C``) or return None."""
    if not os.path.exists(target_path()):
        return None
    parent = os.path.dirname(OUT_DIR)
    if parent not in sys.path:
        sys.path.insert(0, parent)
    import importlib
    return importlib.import_module("torch_ans_ref._C")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help="reference checkout (default: $TORCH_ANS_REFERENCE or ../reference)")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    r = build(a.reference, a.force)
    sys.exit(0 if r else 1)
