"""torch_ans_b200 -- B200-native rANS entropy coding, a drop-in for torch_ans's coding path.

* ``torch_ans_b200._C``: the reference's op surface (``rans64_push`` / ``rans64_pop`` / ... , 30
  names, same arguments and in-place semantics) running on hand-written sm_100a kernels.
* ``torch_ans_b200.utils``: the CompressAI-like ``TorchANSInterface`` coder and its helpers.
* ``torch_ans_b200.capi``: ctypes access to the C ABI library (include/torch_ans_b200.h).

The native extension is loaded when ``_C`` (or a module that codes) is first used, not when the
package is imported: ``torch_ans_b200.workloads`` (seeded benchmark inputs) and
``torch_ans_b200.build`` need no native code, so a process that only generates inputs -- the
reference CPU leg of the benchmark, for one -- maps none of this library's shared objects.
There is no CPU coding path: using ``_C`` without the built extension raises ImportError, and
coding ops raise on CPU tensors.
"""
import importlib as _importlib

import torch as _torch  # noqa: F401  (loads libtorch before the extension)


def __getattr__(name):
    if name == "_C":
        try:
            mod = _importlib.import_module("._C", __name__)
        except ImportError as e:
            raise ImportError(
                "torch_ans_b200 native extension is not built; run `python -m torch_ans_b200.build` "
                f"(or __graft_entry__.build()). Original error: {e}") from e
        globals()["_C"] = mod
        return mod
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


__all__ = ["_C"]
