"""ctypes binding of the C ABI library ``libtorch_ans_b200.so`` (include/torch_ans_b200.h).

This is the binding a non-torch host (or a test) uses: plain device pointers, sizes and a CUDA
stream handle.  ``SYMBOLS`` lists every entry point the header declares.
"""
from __future__ import annotations

import ctypes
import os
import re

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libtorch_ans_b200.so")
HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "torch_ans_b200.h")

RANS64, RANS32, RANS32_16 = 0, 1, 2
LOOKUP_SEARCH, LOOKUP_INVCDF, LOOKUP_ALIAS = 0, 1, 2
VARIANT = {"rans64": RANS64, "rans32": RANS32, "rans32_16": RANS32_16}
LOOKUP = {"search": LOOKUP_SEARCH, "invcdf": LOOKUP_INVCDF, "alias": LOOKUP_ALIAS}

OK = 0
DEV_BAD_INDEX, DEV_BAD_VALUE, DEV_OVERFLOW, DEV_UNDERFLOW, DEV_BAD_FREQ, DEV_BAD_ESCAPE = 1, 2, 4, 8, 16, 32
DEV_STALLED = 64

_P, _I64, _I, _SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
_SIGS = {
    "tans_version": ([], _I),
    "tans_status_string": ([_I], ctypes.c_char_p),
    "tans_launch_count": ([], ctypes.c_uint64),
    "tans_push_workspace_size": ([_I, _I64, _I64], _SZ),
    "tans_push": ([_I, _I, _I, _P, _I64, _I64, _P, _P, _I64, _P, _I64, _I64, _P, _P, _I, _I, _I, _P, _SZ, _P, _P], _I),
    "tans_push_noalloc": ([_I, _I, _I, _P, _I64, _I64, _P, _P, _I64, _P, _I64, _I64, _P, _P, _I, _I, _I, _P, _P], _I),
    "tans_pop_workspace_size": ([_I, _I, _I64, _I64, _I], _SZ),
    "tans_pop": ([_I, _I, _I, _P, _I64, _I64, _P, _P, _I64, _P, _I64, _I64, _P, _P, _I, _I, _I, _P, _SZ, _P, _P], _I),
    "tans_stream_max_length": ([_P, _I64, _I64, _P, _P], _I),
    "tans_init_stream": ([_I, _I, _P, _I64, _I64, _P], _I),
    "tans_gather_payloads": ([_P, _I64, _I64, _P, _I, _I64, _P, _P], _I),
    "tans_scatter_payloads": ([_P, _P, _P, _P, _I64, _I64, _P], _I),
    "tans_cdf_fix_zero_freqs": ([_P, _I64, _I64, _P, _P], _I),
    "tans_push_ragged_workspace_size": ([_I64], _SZ),
    "tans_alias_workspace_size": ([_I64, _I], _SZ),
    "tans_alias_build_table": ([_P, _I64, _I64, _P, _I, _I, _P, _P, _P, _SZ, _P], _I),
    "tans_push_ragged": ([_I, _P, _I64, _I64, _P, _P, _P, _I64, _P, _I64, _I64, _P, _P, _I, _I, _I, _P, _SZ, _P, _P],
                         _I),
    "tans_pop_ragged": ([_I, _P, _I64, _I64, _P, _P, _P, _I64, _P, _I64, _I64, _P, _P, _I, _I, _I, _P, _P], _I),
    "tans_probe": ([_I, _I64, ctypes.POINTER(ctypes.c_double)], _I),
}

PROBES = {"smem_chase": 0, "l2_chase": 1, "l2_chase_busy": 2, "pop32_step": 3, "push32_step": 4, "pop64_step": 5,
          "push64_step": 6}


def probe(kind: str, steps: int = 200000) -> float:
    """Cycles of one dependent step of a latency probe (tans_probe; needs a GPU)."""
    lib = load()
    out = ctypes.c_double(0.0)
    rc = lib.tans_probe(PROBES[kind], int(steps), ctypes.byref(out))
    if rc != OK:
        raise RuntimeError(f"tans_probe({kind}): {lib.tans_status_string(rc).decode()}")
    return out.value

_lib = None


def declared_symbols(header: str = HEADER):
    """Names of the functions declared in the C header."""
    text = open(header).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tans_\w+)\s*\(", text)))


def load():
    """Load libtorch_ans_b200.so and set argument types of every declared entry point."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is not built; run `python -m torch_ans_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in _SIGS.items():
            f = getattr(lib, name, None)
            if f is not None:
                f.argtypes = args
                f.restype = res
        _lib = lib
    return _lib


def ptr(t) -> int:
    return t.data_ptr() if t is not None else None
