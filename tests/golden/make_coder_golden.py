"""Write tests/golden/coder_cases.npz: the reference's high-level coder (TorchANSInterface,
torch_ans/utils.py:583-966) run on seeded inputs, for the GPU coder's byte-parity tests.

The reference's own ``torch_ans/utils.py`` is loaded from the reference checkout with the compiled
reference CPU extension (oracle/_ref, built by oracle/build_ref.py) standing in as its
``torch_ans._C``, so every byte comes from the reference's Python and C++ code.  The call patterns
follow the reference's tests/test_high_level_api.py:
  * encode_with_indexes / decode_with_indexes for impl rans64, rans32 and "rans32_16" (which the
    reference resolves to rans32, utils.py:615-625), escape coding on and off, several
    precisions, 2-byte length prefixes;
  * encode_with_indexes(cache=True) twice, flush, then decode_with_indexes of the whole and
    set_stream + two decode_stream calls (utils.py:378-393, LIFO order);
  * encode(cache=True) twice + encode_flush on the tensor API, then two partial decodes;
  * encode_with_freqs / decode_with_freqs with one frequency row per symbol (utils.py:911);
  * num_parallel_states (the last segment unprefixed), set_cdfs, single-symbol tables.
Each case stores its inputs, constructor arguments, the bytes every encode call returned and every
decode result, under keys "<case>/<name>"; "<case>/meta" is a JSON string.

Run where the reference checkout exists ($TORCH_ANS_REFERENCE, or ``reference`` beside this
repository):
    python oracle/build_ref.py && python tests/golden/make_coder_golden.py
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import build_ref  # noqa: E402

OUT = os.path.join(HERE, "coder_cases.npz")


def reference_utils():
    """The reference's torch_ans.utils module running on the compiled reference extension."""
    build_ref.build()
    ref = build_ref.load()
    if ref is None:
        raise SystemExit("compiled reference not available (run oracle/build_ref.py)")
    pkg = types.ModuleType("torch_ans")
    pkg.__path__ = []
    pkg._C = ref
    sys.modules["torch_ans"] = pkg
    sys.modules["torch_ans._C"] = ref
    path = os.path.join(build_ref.default_reference(), "torch_ans", "utils.py")
    spec = importlib.util.spec_from_file_location("torch_ans.utils", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["torch_ans.utils"] = mod
    spec.loader.exec_module(mod)
    return mod


ARR = {}


def put(case, name, value):
    if isinstance(value, (bytes, bytearray)):
        value = np.frombuffer(bytes(value), np.uint8)
    elif isinstance(value, torch.Tensor):
        value = value.numpy()
    ARR[f"{case}/{name}"] = np.asarray(value)


def meta(case, **kw):
    ARR[f"{case}/meta"] = np.array(json.dumps(kw))


def tables(g, num_dists=4, num_symbols=16):
    pmf = torch.randint(1, 100, (num_dists, num_symbols), generator=g, dtype=torch.int32)
    return pmf, torch.full((num_dists,), num_symbols, dtype=torch.int32), torch.zeros(num_dists, dtype=torch.int32)


def main():
    U = reference_utils()
    g = torch.Generator().manual_seed(20241202)

    # encode_with_indexes / decode_with_indexes over impls, escape coding, precisions, prefixes
    plain_cases = [
        ("idx_rans64", dict(impl="rans64", freq_precision=12), (-0, 16)),
        ("idx_rans64_fp16", dict(impl="rans64", freq_precision=16), (0, 16)),
        ("idx_rans32", dict(impl="rans32", freq_precision=12), (0, 16)),
        ("idx_rans32_fp8", dict(impl="rans32", freq_precision=8), (0, 16)),
        ("idx_rans32_16", dict(impl="rans32_16", freq_precision=12), (0, 16)),
        ("idx_rans64_escapes", dict(impl="rans64", freq_precision=12), (-40, 60)),
        ("idx_rans32_escapes_bp2", dict(impl="rans32", freq_precision=16, bypass_precision=2), (-300, 400)),
        ("idx_rans64_no_bypass", dict(impl="rans64", freq_precision=12, bypass_coding=False), (0, 16)),
        ("idx_rans64_prefix2", dict(impl="rans64", freq_precision=12, num_bytes_code_length=2), (0, 16)),
        ("idx_rans64_parallel4", dict(impl="rans64", freq_precision=12, num_parallel_states=4), (0, 16)),
    ]
    for name, kw, (lo, hi) in plain_cases:
        pmf, nf, offs = tables(g)
        if "escapes" in name:
            offs = torch.randint(-5, 5, (4,), generator=g, dtype=torch.int32)
        sym = torch.randint(lo, hi, (2, 64), generator=g, dtype=torch.int32)
        idx = torch.randint(0, 4, (2, 64), generator=g, dtype=torch.int32)
        coder = U.TorchANSInterface(device="cpu", **kw)
        coder.init_params(pmf, nf, offs)
        enc = coder.encode_with_indexes(sym, idx)
        dec = coder.decode_with_indexes(enc, idx)
        assert torch.equal(dec, sym), name
        meta(name, kind="indexes", kwargs=kw)
        for k, v in dict(pmf=pmf, num_freqs=nf, offsets=offs, symbols=sym, indexes=idx, encoded=enc, decoded=dec,
                         cdfs=coder.cdfs, cdfs_sizes=coder.cdfs_sizes).items():
            put(name, k, v)

    # cached encodes + flush (bytes), decode of the whole and streamed partial decodes
    name = "cache_flush"
    pmf, nf, offs = tables(g)
    s1 = torch.randint(-3, 20, (2, 32), generator=g, dtype=torch.int32)
    i1 = torch.randint(0, 4, (2, 32), generator=g, dtype=torch.int32)
    s2 = torch.randint(-3, 20, (2, 32), generator=g, dtype=torch.int32)
    i2 = torch.randint(0, 4, (2, 32), generator=g, dtype=torch.int32)
    coder = U.TorchANSInterface(impl="rans64", freq_precision=12, device="cpu")
    coder.init_params(pmf, nf, offs)
    assert coder.encode_with_indexes(s1, i1, cache=True) is None
    assert coder.encode_with_indexes(s2, i2, cache=True) is None
    enc = coder.flush()
    whole = coder.decode_with_indexes(enc, torch.cat([i1, i2], 1))
    c2 = U.TorchANSInterface(impl="rans64", freq_precision=12, device="cpu")
    c2.init_params(pmf, nf, offs)
    c2.set_stream(enc)
    d1 = c2.decode_stream(i1)
    d2 = c2.decode_stream(i2)
    assert torch.equal(d1, s1) and torch.equal(d2, s2) and torch.equal(whole, torch.cat([s1, s2], 1))
    meta(name, kind="cache_flush", kwargs=dict(impl="rans64", freq_precision=12))
    for k, v in dict(pmf=pmf, num_freqs=nf, offsets=offs, s1=s1, i1=i1, s2=s2, i2=i2, encoded=enc, whole=whole,
                     d1=d1, d2=d2).items():
        put(name, k, v)

    # tensor API: encode(cache=True) x 2, encode_flush, partial decodes on the stream tensor
    name = "encode_flush_tensor"
    pmf, nf, offs = tables(g)
    s1 = torch.randint(0, 16, (3, 8), generator=g, dtype=torch.int32)
    i1 = torch.randint(0, 4, (3, 8), generator=g, dtype=torch.int32)
    s2 = torch.randint(0, 16, (3, 5), generator=g, dtype=torch.int32)
    i2 = torch.randint(0, 4, (3, 5), generator=g, dtype=torch.int32)
    coder = U.TorchANSInterface(impl="rans32", freq_precision=12, device="cpu")
    coder.init_params(pmf, nf, offs)
    coder.encode(s1, dist_indexes=i1, cache=True)
    coder.encode(s2, dist_indexes=i2, cache=True)
    stream = coder.encode_flush()
    flushed_bytes = b"".join(U.rans_stream_to_byte_strings(stream))
    flushed_lengths = stream[:, 0].clone()
    flushed_width = stream.shape[1]
    d1 = coder.decode(stream, dist_indexes=i1)
    d2 = coder.decode(stream, dist_indexes=i2)
    assert torch.equal(d1, s1) and torch.equal(d2, s2)
    meta(name, kind="encode_flush_tensor", kwargs=dict(impl="rans32", freq_precision=12), width=int(flushed_width))
    for k, v in dict(pmf=pmf, num_freqs=nf, offsets=offs, s1=s1, i1=i1, s2=s2, i2=i2, payload=flushed_bytes,
                     lengths=flushed_lengths, d1=d1, d2=d2).items():
        put(name, k, v)

    # per-element frequencies
    for name, kw in [("freqs_rans64", dict(impl="rans64", freq_precision=12)),
                     ("freqs_rans32_no_bypass", dict(impl="rans32", freq_precision=16, bypass_coding=False))]:
        sym = torch.randint(0, 16, (2, 24), generator=g, dtype=torch.int32)
        freqs = torch.randint(1, 100, (2, 24, 16), generator=g, dtype=torch.int32)
        nfr = torch.full((2, 24), 16, dtype=torch.int32)
        offr = torch.zeros((2, 24), dtype=torch.int32)
        coder = U.TorchANSInterface(device="cpu", **kw)
        enc = coder.encode_with_freqs(sym, freqs, nfr, offr)
        c2 = U.TorchANSInterface(device="cpu", **kw)
        dec = c2.decode_with_freqs(enc, freqs, nfr, offr)
        assert torch.equal(dec, sym), name
        meta(name, kind="freqs", kwargs=kw)
        for k, v in dict(symbols=sym, freqs=freqs, num_freqs=nfr, offsets=offr, encoded=enc, decoded=dec).items():
            put(name, k, v)

    # set_cdfs directly (tests/test_high_level_api.py:243-266 pattern) and single-symbol tables
    name = "set_cdfs"
    cdfs = torch.stack([torch.linspace(0, 256, 18).to(torch.int32) for _ in range(4)])
    sizes = torch.full((4,), 17, dtype=torch.int32)
    offs = torch.zeros(4, dtype=torch.int32)
    sym = torch.randint(0, 16, (2, 32), generator=g, dtype=torch.int32)
    idx = torch.randint(0, 4, (2, 32), generator=g, dtype=torch.int32)
    coder = U.TorchANSInterface(impl="rans64", freq_precision=8, device="cpu")
    coder.set_cdfs(cdfs, sizes, offs)
    enc = coder.encode_with_indexes(sym, idx)
    dec = coder.decode_with_indexes(enc, idx)
    assert torch.equal(dec, sym)
    meta(name, kind="set_cdfs", kwargs=dict(impl="rans64", freq_precision=8))
    for k, v in dict(cdfs=cdfs, cdfs_sizes=sizes, offsets=offs, symbols=sym, indexes=idx, encoded=enc,
                     decoded=dec).items():
        put(name, k, v)

    name = "single_symbol"
    pmf = torch.ones(4, 1, dtype=torch.int32)
    nf = torch.ones(4, dtype=torch.int32)
    offs = torch.zeros(4, dtype=torch.int32)
    sym = torch.zeros(2, 8, dtype=torch.int32)
    idx = torch.randint(0, 4, (2, 8), generator=g, dtype=torch.int32)
    coder = U.TorchANSInterface(impl="rans64", freq_precision=12, device="cpu")
    coder.init_params(pmf, nf, offs)
    enc = coder.encode_with_indexes(sym, idx)
    dec = coder.decode_with_indexes(enc, idx)
    assert torch.equal(dec, sym)
    meta(name, kind="indexes", kwargs=dict(impl="rans64", freq_precision=12))
    for k, v in dict(pmf=pmf, num_freqs=nf, offsets=offs, symbols=sym, indexes=idx, encoded=enc, decoded=dec,
                     cdfs=coder.cdfs, cdfs_sizes=coder.cdfs_sizes).items():
        put(name, k, v)

    np.savez_compressed(OUT, **ARR)
    print("wrote", OUT, os.path.getsize(OUT), "bytes,", len({k.split('/')[0] for k in ARR}), "cases")


if __name__ == "__main__":
    main()
