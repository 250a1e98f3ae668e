"""torch_ans_b200 -- B200-native rANS entropy coding, a drop-in for torch_ans's coding path.

* ``torch_ans_b200._C``: the reference's op surface (``rans64_push`` / ``rans64_pop`` / ... , 30
  names, same arguments and in-place semantics) running on hand-written sm_100a kernels.
* ``torch_ans_b200.utils``: the CompressAI-like ``TorchANSInterface`` coder and its helpers.
* ``torch_ans_b200.capi``: ctypes access to the C ABI library (include/torch_ans_b200.h).

There is no CPU coding path: using the package without its native extension fails loudly
(``torch_ans_b200._C`` and every module that codes raise ImportError), and coding ops raise on
CPU tensors.  Only ``torch_ans_b200.build`` works before the extension exists.
"""
import torch as _torch  # noqa: F401  (loads libtorch before the extension)

try:
    from . import _C  # noqa: F401
except ImportError as _e:  # the build step itself imports this package before _C exists
    _IMPORT_ERROR = _e

    def __getattr__(name):
        if name == "_C":
            raise ImportError(
                "torch_ans_b200 native extension is not built; run `python -m torch_ans_b200.build` "
                f"(or __graft_entry__.build()). Original error: {_IMPORT_ERROR}") from _IMPORT_ERROR
        raise AttributeError(name)

__all__ = ["_C"]
