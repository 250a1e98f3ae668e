"""CPU tests of the product's host side: the C ABI library loads and exports every declared
entry point, the `_C` module carries the reference's op surface, and the host-side helpers
(stream init, byte-string conversion, alias-table build, container format, high-level API
plumbing) match the reference's golden vectors.  No CUDA compute runs here."""
import struct

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import golden_cases as G

REFERENCE_NAMES = sorted(
    ["rans_stream_to_byte_strings", "rans_byte_strings_to_stream", "rans_alias_build_table", "rans_pmf_to_quantized_cdf"]
    + [f"{p}_{op}" for p in ("rans64", "rans32", "rans32_16")
       for op in ("init_stream", "push", "pop", "i4_push", "i4_pop", "alias_push", "alias_pop", "invcdf_pop")]
    + ["rans32_i4_invcdf_pop", "rans32_16_i4_invcdf_pop"])


def test_capi_exports_every_declared_symbol():
    from torch_ans_b200 import capi
    declared = capi.declared_symbols()
    assert len(declared) >= 11
    lib = capi.load()
    missing = [n for n in declared if not hasattr(lib, n)]
    assert not missing, missing
    assert lib.tans_version() > 0
    assert lib.tans_status_string(0) == b"ok"


def test_capi_rejects_bad_arguments_without_touching_the_device():
    import ctypes
    from torch_ans_b200 import capi
    lib = capi.load()
    # freq precision above the variant's limit, bad interleave, bad variant: rejected on the host
    args = [0, 0, 1, None, 0, 3, None, None, 0, None, 0, 0, None, None, 16, 0, 4, None, 0, None, None]
    assert lib.tans_push(*args) == 0  # empty batch is a no-op
    bad = list(args); bad[4] = 1; bad[14] = 40
    assert lib.tans_push(*bad) == 1
    bad = list(args); bad[4] = 1; bad[2] = 3
    assert lib.tans_push(*bad) == 1
    bad = list(args); bad[4] = 1; bad[0] = 7
    assert lib.tans_push(*bad) == 1
    assert lib.tans_gather_payloads(None, 1, 3, None, 3, 0, None, None) == 1  # 3-byte prefix invalid


def test_module_has_reference_op_surface():
    from torch_ans_b200 import _C
    names = sorted(n for n in dir(_C) if not n.startswith("_"))
    for n in REFERENCE_NAMES:
        assert n in names, n
    assert len(REFERENCE_NAMES) == 30


@pytest.mark.parametrize("variant,ilv,prealloc", [("rans64", 1, 0), ("rans32", 4, 16), ("rans32_16", 4, 16), ("rans64", 4, 7)])
def test_init_stream_matches_oracle(variant, ilv, prealloc):
    from torch_ans_b200 import _C
    s = getattr(_C, f"{variant}_init_stream")(3, ilv, prealloc)
    assert s.device.type == "cpu" and s.dtype == torch.int32
    assert np.array_equal(s.numpy(), O.init_stream(variant, 3, ilv, prealloc))


def test_byte_string_conversions_match_reference():
    from torch_ans_b200 import _C
    d = G.load("rans32_bypass")
    pushed = torch.from_numpy(d["pushed"])
    bs = _C.rans_stream_to_byte_strings(pushed)
    assert b"".join(bs) == d["pushed_bytes"].tobytes()
    back = _C.rans_byte_strings_to_stream(bs)
    assert np.array_equal(back.numpy(), O.byte_strings_to_stream(bs))


@pytest.mark.parametrize("variant", ["rans64", "rans32", "rans32_16"])
def test_alias_build_table_matches_reference(variant):
    from torch_ans_b200 import _C
    for name, sp in ((f"{variant}_alias", 5), (f"{variant}_alias_bypass", 4)):
        d = G.load(name)
        remap, table = _C.rans_alias_build_table(torch.from_numpy(d["cdfs"]), torch.from_numpy(d["sizes"]),
                                                 symbol_precision=sp, freq_precision=d["meta"]["fp"])
        assert np.array_equal(remap.numpy(), d["push_cdfs"]) and np.array_equal(table.numpy(), d["pop_cdfs"])
    d = G.load(f"{variant}_alias_rejected")
    remap, table = _C.rans_alias_build_table(torch.from_numpy(d["cdfs"]), torch.from_numpy(d["sizes"]),
                                             symbol_precision=d["meta"]["sp"], freq_precision=d["meta"]["fp"])
    assert np.array_equal(remap.numpy(), d["remap"]) and np.array_equal(table.numpy(), d["table"])


def test_push_on_cpu_stream_fails_loudly():
    from torch_ans_b200 import _C
    s = _C.rans64_init_stream(2)
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.rans64_push(s, torch.zeros(2, 4, dtype=torch.int32), torch.zeros(2, 4, dtype=torch.int32),
                       torch.tensor([[0, 1 << 16]], dtype=torch.int32), torch.tensor([2], dtype=torch.int32))
    with pytest.raises(ValueError, match="Symbols batch size mismatch!"):
        _C.rans64_push(s, torch.zeros(3, 4, dtype=torch.int32))
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.rans64_pop(s, torch.zeros(2, 4, dtype=torch.int32), torch.tensor([[0, 1 << 16]], dtype=torch.int32),
                      torch.tensor([2], dtype=torch.int32))
    assert _C.rans64_pop(s) is None  # no indexes: nothing decoded, as in the reference


def test_container_helpers_known_answers():
    from torch_ans_b200 import utils as U
    assert U._get_bytes_format(1) == "B" and U._get_bytes_format(8) == "<L"
    with pytest.raises(ValueError):
        U._get_bytes_format(3)
    assert U.merge_bytes([b"hello", b"world"]) == struct.pack("<I", 5) + b"hello" + struct.pack("<I", 5) + b"world"
    assert U.merge_bytes([b"hello", b"world", b"!"], num_segments=3) == (
        struct.pack("<I", 5) + b"hello" + struct.pack("<I", 5) + b"world" + b"!")
    assert U.split_merged_bytes(struct.pack("<H", 2) + b"hi" + struct.pack("<H", 2) + b"ok", 2) == [b"hi", b"ok"]
    orig = [b"test1", b"test2", b"test3"]
    assert U.split_merged_bytes(U.merge_bytes(orig, num_segments=3), num_segments=3) == orig
    assert U.split_merged_bytes(b"", num_segments=2) == [b"", b""]
    rng = np.random.default_rng(5)
    segs = [bytes(rng.integers(0, 256, rng.integers(0, 40)).astype(np.uint8)) for _ in range(9)]
    for nb in (1, 2, 4, 8):
        for ns in (None, 9):
            assert U.merge_bytes(segs, nb, ns) == O.merge_bytes(segs, nb, ns)
            if nb != 8:  # the reference's 8-byte mode packs "<L" (4 bytes) and cannot split back
                assert U.split_merged_bytes(U.merge_bytes(segs, nb, ns), nb, ns) == segs
    assert len(U.merge_bytes([b"ab"], 8)) == 4 + 2


def test_inverse_cdf_and_batched_quantiser_known_answers():
    from torch_ans_b200 import utils as U
    inv = U.inverse_quantized_cdf(torch.tensor([[0, 26, 77, 154, 256]], dtype=torch.int32), freq_precision=8)
    assert inv.shape == (1, 256)
    assert (inv[0, 0:26] == 0).all() and (inv[0, 26:77] == 1).all() and (inv[0, 154:256] == 3).all()
    rng = np.random.default_rng(0)
    c = np.sort(rng.integers(0, 4096, (3, 20)), axis=1).astype(np.int32)
    c[:, 0] = 0
    c[:, -1] = 4096
    assert np.array_equal(U.inverse_quantized_cdf(torch.from_numpy(c), 12).numpy(), O.inverse_quantized_cdf(c, 12))
    cdf = U.pmf_to_quantized_cdf_batched(torch.tensor([[0.25, 0.25, 0.25, 0.25]]), precision=8, add_tail=False)
    assert cdf.tolist() == [[0, 64, 128, 192, 256]]
    cdf = U.pmf_to_quantized_cdf_batched(torch.tensor([[0.3, 0.3, 0.3]]), precision=8, add_tail=True)
    assert cdf.shape == (1, 5) and cdf[0, -1] == 256


def test_high_level_impl_selection():
    from torch_ans_b200 import _C
    from torch_ans_b200.utils import TorchANSInterface
    with pytest.raises(NotImplementedError):
        TorchANSInterface(impl="invalid_impl")
    c = TorchANSInterface(impl="rans32_16", freq_precision=16)
    assert c.ans_encode_func is _C.rans32_push and c.freq_precision == 16  # prefix quirk of the reference
    c = TorchANSInterface(impl="rans64", freq_precision=40)
    assert c.freq_precision == 31 and c.ans_decode_func is _C.rans64_pop
    c = TorchANSInterface(impl="rans_byte", freq_precision=30, use_inverse_cdf=True)
    assert c.freq_precision == 23 and c.ans_decode_func is _C.rans32_invcdf_pop


def test_workload_tables_are_valid_and_seeded():
    from torch_ans_b200 import workloads as W
    a = W.laplace64(device="cpu", scale=1 / 16, length_scale=1 / 64)
    b = W.laplace64(device="cpu", scale=1 / 16, length_scale=1 / 64)
    assert torch.equal(a.symbols, b.symbols) and torch.equal(a.cdfs, b.cdfs)
    f = a.cdfs[:, 1:] - a.cdfs[:, :-1]
    assert (f >= 1).all() and (a.cdfs[:, -1] == 1 << 16).all()
    m = W.mixture_invcdf(device="cpu", scale=1 / 64, length_scale=1 / 256)
    inv = m.pop_cdfs[:, 1025:]
    assert inv.shape[1] == 1 << 16
    assert np.array_equal(inv.numpy(), O.inverse_quantized_cdf(m.cdfs.numpy(), 16))


@pytest.mark.parametrize("prefix", [1, 2, 4])
def test_parse_merged_matches_split_merged_bytes(prefix):
    """The host walk the pipeline decoder uses finds exactly the records split_merged_bytes finds
    (empty records, records past the end of the data, and a truncated prefix raising)."""
    import torch
    from torch_ans_b200 import _C
    from torch_ans_b200.utils import merge_bytes, split_merged_bytes
    rng = np.random.default_rng(prefix)
    cap = (1 << (8 * prefix)) - 1
    segs = [bytes(rng.integers(0, 256, int(n), dtype=np.uint8)) for n in rng.integers(0, min(cap, 700), 37)]
    segs[5] = b""
    data = merge_bytes(segs, num_bytes_length=prefix)
    t = torch.frombuffer(bytearray(data), dtype=torch.uint8)
    off, ln = _C.parse_merged(t, prefix, len(segs) + 3)
    want = split_merged_bytes(data, num_bytes_length=prefix)
    got = [data[o:o + n] for o, n in zip(off.tolist(), ln.tolist())]
    assert got[: len(want)] == want and all(g == b"" for g in got[len(want):])
    if prefix > 1:  # a data tail shorter than one prefix
        with pytest.raises(RuntimeError, match="truncated"):
            _C.parse_merged(torch.frombuffer(bytearray(b"\x01" * (prefix - 1)), dtype=torch.uint8), prefix, 1)


def _reference_bisection(row, size, cum, fp):
    """The search of rans_pop_step (rans_utils.hpp:424-450): first probe (size * cum) >> fp, then
    bisection on [0, size - 1]; returns s = idx - 1."""
    idx = (size * cum) >> fp
    low, high = 0, size - 1
    while high > low:
        if cum >= row[idx]:
            low = idx + 1
        else:
            high = idx
        idx = (low + high) // 2
    return idx - 1


def test_ballot_prefix_rule_equals_reference_bisection():
    """The ragged warp pop decodes s = popc(m) - 1 from the ballot m of row[j] <= cum (j < size)
    when bit 0 is set, bit size - 1 is clear and the set bits form a prefix; on every such mask the
    reference's bisection must end at the same s, for monotone and non-monotone rows alike."""
    import numpy as np
    rng = np.random.default_rng(7)
    fp = 8
    fired = 0
    for trial in range(300):
        size = int(rng.integers(2, 34))
        if trial % 3 == 0:
            row = np.sort(rng.integers(0, 1 << fp, size))
        else:  # non-monotone rows, values spread over the cum range
            row = rng.integers(0, 1 << fp, size)
        for cum in range(1 << fp):
            m = 0
            for j in range(size):
                if row[j] <= cum:
                    m |= 1 << j
            if (m & 1) and not (m >> (size - 1)) & 1 and (m & (m + 1)) == 0:
                fired += 1
                assert bin(m).count("1") - 1 == _reference_bisection(row, size, cum, fp), (row, size, cum)
    assert fired > 1000


def test_probe_rejects_bad_arguments_without_a_device():
    """tans_probe checks its arguments on the host before any CUDA call."""
    import ctypes
    from torch_ans_b200 import capi
    lib = capi.load()
    out = ctypes.c_double(0.0)
    assert lib.tans_probe(capi.PROBES["pop32_step"], 0, ctypes.byref(out)) == 1
    assert lib.tans_probe(99, 10, ctypes.byref(out)) == 1
    assert lib.tans_probe(0, 10, None) == 1
