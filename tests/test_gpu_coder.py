"""The high-level coder on the GPU against the reference's own TorchANSInterface.

``tests/golden/coder_cases.npz`` was written by running the reference's torch_ans/utils.py
(TorchANSInterface, utils.py:583-966) on the compiled reference CPU extension
(tests/golden/make_coder_golden.py).  Each case is replayed here through
``torch_ans_b200.utils.TorchANSInterface`` on CUDA with the same constructor arguments and call
sequence, and every returned byte string and decoded tensor must be identical:
encode_with_indexes / decode_with_indexes (rans64, rans32, "rans32_16" -> rans32, escapes on and
off, precisions 8 / 12 / 16, 2-byte prefixes, num_parallel_states), cached encodes + flush with
whole and streamed (set_stream + decode_stream) decodes, the tensor API's encode_flush with partial
decodes, encode_with_freqs / decode_with_freqs, set_cdfs and single-symbol tables.
"""
import json
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "coder_cases.npz")


def _cases():
    with np.load(PATH) as z:
        names = sorted({k.split("/")[0] for k in z.files})
    return names


def _load(name):
    with np.load(PATH) as z:
        d = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(name + "/")}
    d["meta"] = json.loads(str(d["meta"]))
    return d


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a))


def B(a):
    return np.ascontiguousarray(a, dtype=np.uint8).tobytes()


@pytest.mark.parametrize("name", _cases())
def test_coder_matches_reference_interface(name):
    from torch_ans_b200 import _C
    from torch_ans_b200.utils import TorchANSInterface
    _C.set_sync_check(False)
    _C.device_status(reset=True)
    d = _load(name)
    kind, kw = d["meta"]["kind"], d["meta"]["kwargs"]
    coder = TorchANSInterface(device="cuda", **kw)
    if kind == "indexes":
        coder.init_params(T(d["pmf"]), T(d["num_freqs"]), T(d["offsets"]))
        assert torch.equal(coder.cdfs.cpu(), T(d["cdfs"])), "quantised cdf tables differ from the reference coder's"
        assert torch.equal(coder.cdfs_sizes.cpu(), T(d["cdfs_sizes"]))
        enc = coder.encode_with_indexes(T(d["symbols"]), T(d["indexes"]))
        assert isinstance(enc, bytes) and enc == B(d["encoded"])
        dec = coder.decode_with_indexes(enc, T(d["indexes"]))
        assert dec.is_cuda and torch.equal(dec.cpu(), T(d["decoded"]))
    elif kind == "set_cdfs":
        coder.set_cdfs(T(d["cdfs"]), T(d["cdfs_sizes"]), T(d["offsets"]))
        enc = coder.encode_with_indexes(T(d["symbols"]), T(d["indexes"]))
        assert enc == B(d["encoded"])
        assert torch.equal(coder.decode_with_indexes(enc, T(d["indexes"])).cpu(), T(d["decoded"]))
    elif kind == "cache_flush":
        coder.init_params(T(d["pmf"]), T(d["num_freqs"]), T(d["offsets"]))
        assert coder.encode_with_indexes(T(d["s1"]), T(d["i1"]), cache=True) is None
        assert coder.encode_with_indexes(T(d["s2"]), T(d["i2"]), cache=True) is None
        enc = coder.flush()
        assert enc == B(d["encoded"])
        whole = coder.decode_with_indexes(enc, torch.cat([T(d["i1"]), T(d["i2"])], 1))
        assert torch.equal(whole.cpu(), T(d["whole"]))
        c2 = TorchANSInterface(device="cuda", **kw)
        c2.init_params(T(d["pmf"]), T(d["num_freqs"]), T(d["offsets"]))
        c2.set_stream(enc)
        assert torch.equal(c2.decode_stream(T(d["i1"])).cpu(), T(d["d1"]))
        assert torch.equal(c2.decode_stream(T(d["i2"])).cpu(), T(d["d2"]))
    elif kind == "encode_flush_tensor":
        coder.init_params(T(d["pmf"]), T(d["num_freqs"]), T(d["offsets"]))
        assert coder.encode(T(d["s1"]), dist_indexes=T(d["i1"]), cache=True) is None
        coder.encode(T(d["s2"]), dist_indexes=T(d["i2"]), cache=True)
        stream = coder.encode_flush()
        assert stream.is_cuda and stream.shape[1] == d["meta"]["width"]
        assert torch.equal(stream[:, 0].cpu(), T(d["lengths"]))
        assert b"".join(_C.rans_stream_to_byte_strings(stream)) == B(d["payload"])
        assert torch.equal(coder.decode(stream, dist_indexes=T(d["i1"])).cpu(), T(d["d1"]))
        assert torch.equal(coder.decode(stream, dist_indexes=T(d["i2"])).cpu(), T(d["d2"]))
    elif kind == "freqs":
        enc = coder.encode_with_freqs(T(d["symbols"]), T(d["freqs"]), T(d["num_freqs"]), T(d["offsets"]))
        assert enc == B(d["encoded"])
        c2 = TorchANSInterface(device="cuda", **kw)
        dec = c2.decode_with_freqs(enc, T(d["freqs"]), T(d["num_freqs"]), T(d["offsets"]))
        assert torch.equal(dec.cpu(), T(d["decoded"]))
    else:
        raise AssertionError(f"unknown case kind {kind}")
    assert _C.device_status() == 0


def test_num_parallel_states_and_impl_quirk_are_covered():
    names = _cases()
    assert "idx_rans64_parallel4" in names and "idx_rans32_16" in names
    d = _load("idx_rans32_16")
    from torch_ans_b200.utils import TorchANSInterface
    coder = TorchANSInterface(device="cuda", **d["meta"]["kwargs"])
    assert coder.ans_encode_func.__name__ == "rans32_push"  # "rans32_16" resolves to rans32, as in the reference
