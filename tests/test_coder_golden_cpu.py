"""The reference coder's bytes (tests/golden/coder_cases.npz, written by the reference's own
TorchANSInterface) rebuilt on the CPU from the oracle's coding and this library's container
functions: pins the container format, the quantised tables and the oracle at the coder level."""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O

PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "coder_cases.npz")


def _load(name):
    with np.load(PATH) as z:
        d = {k.split("/", 1)[1]: z[k] for k in z.files if k.startswith(name + "/")}
    d["meta"] = json.loads(str(d["meta"]))
    return d


def _index_cases():
    with np.load(PATH) as z:
        names = sorted({k.split("/")[0] for k in z.files})
    return [n for n in names if _load(n)["meta"]["kind"] == "indexes"]


@pytest.mark.parametrize("name", _index_cases())
def test_oracle_and_container_rebuild_reference_coder_bytes(name):
    from torch_ans_b200.utils import merge_bytes, split_merged_bytes
    d = _load(name)
    kw = d["meta"]["kwargs"]
    impl = kw["impl"]
    variant = "rans64" if impl.startswith("rans64") else "rans32"  # "rans32_16" -> rans32 (utils.py:615-625)
    fp = min(kw.get("freq_precision", 16), 31 if variant == "rans64" else 23)
    bypass = kw.get("bypass_coding", True)
    bp = kw.get("bypass_precision", 4)
    nps = kw.get("num_parallel_states")
    prefix = kw.get("num_bytes_code_length", 4)
    # the quantised tables: the oracle's pmf -> cdf (float32 arithmetic) against the reference coder's
    pmf = d["pmf"].astype(np.float32)
    if bypass:
        pmf = np.concatenate([pmf, np.full(pmf[:, :1].shape, 1e-10, np.float32)], 1)
    pmf = pmf / pmf.sum(-1, keepdims=True)
    cdfs = O.pmf_to_quantized_cdf(pmf, fp)
    assert np.array_equal(cdfs, d["cdfs"])
    sym, idx = d["symbols"], d["indexes"]
    # encode() makes its stream with _init_stream() and no argument (utils.py:368): without
    # num_parallel_states the whole batch is one stream
    rows = nps if nps is not None else 1
    st, err = O.push(variant, O.init_stream(variant, rows), sym.reshape(rows, -1), idx.reshape(rows, -1), cdfs,
                     d["cdfs_sizes"], d["offsets"], fp, bypass, bp)
    assert err == 0
    enc = merge_bytes(O.stream_to_byte_strings(st), num_bytes_length=prefix, num_segments=nps)
    assert enc == d["encoded"].tobytes()
    segs = split_merged_bytes(enc, num_bytes_length=prefix, num_segments=nps)
    dec, err = O.pop(variant, O.byte_strings_to_stream(segs), idx.reshape(rows, -1), cdfs, d["cdfs_sizes"],
                     d["offsets"], fp, bypass, bp)
    assert err == 0 and np.array_equal(dec.reshape(sym.shape), d["decoded"])
