"""CPU tests that pin the oracle (oracle/rans_oracle.c + oracle/oracle.py) to the reference.

Every golden case in tests/golden/ was produced by the compiled reference CPU path; the oracle
must reproduce each byte of each pushed stream, each decoded symbol and each popped stream row.
Also the reference's own known answers (tests/torch_ans_test.py:54-67 and
tests/test_utils.py:23-130 of the reference) for the table-prep and container helpers.
"""
import struct

import numpy as np
import pytest

from oracle import oracle as O
from tests import golden_cases as G


def _oracle_roundtrip(d):
    m = d["meta"]
    stream = d["stream_in"].copy()
    pushed, perr = O.push(m["variant"], stream, d["symbols"], d["indexes"], d["push_cdfs"], d["sizes"],
                          d["offsets"], m["fp"], bool(m["bypass"]), m["bp"], alias=bool(m["alias_push"]),
                          interleave=m["interleave"])
    st2 = O.byte_strings_to_stream(O.stream_to_byte_strings(pushed))
    dec, derr = O.pop(m["variant"], st2, d["indexes"], d["pop_cdfs"], d["sizes"], d["offsets"], m["fp"],
                      bool(m["bypass"]), m["bp"], lookup=m["lookup"], interleave=m["interleave"])
    return pushed, perr, dec, derr, st2


@pytest.mark.parametrize("name", G.coding_cases())
def test_oracle_matches_reference_bytes(name):
    d = G.load(name)
    pushed, perr, dec, derr, st2 = _oracle_roundtrip(d)
    assert perr == 0 and derr == 0
    assert pushed.shape == d["pushed"].shape  # same worst-case resize (rans.hpp:105-124)
    assert np.array_equal(pushed[:, 0], d["pushed"][:, 0])
    assert G.payload_bytes(pushed) == d["pushed_bytes"].tobytes()
    assert np.array_equal(dec, d["decoded"])
    assert np.array_equal(dec, d["symbols"])
    # after a full pop: length back to the state bytes and the state back to the lower bound
    assert np.array_equal(st2[:, 0], d["popped"][:, 0])
    assert G.payload_bytes(st2) == G.payload_bytes(d["popped"])


@pytest.mark.parametrize("variant", ["rans64", "rans32", "rans32_16"])
def test_oracle_streaming_matches_reference(variant):
    d = G.load(f"{variant}_streaming")
    fp = d["meta"]["fp"]
    st = O.init_stream(variant, 3)
    # the reference's resize_ leaves the bytes past each row's length uninitialised, so rows are
    # compared through (shape, length column, payload[0:len])
    same = lambda a, b: (a.shape == b.shape and np.array_equal(a[:, 0], b[:, 0])
                         and G.payload_bytes(a) == G.payload_bytes(b))
    st, e1 = O.push(variant, st, d["s2"], d["i2"], d["cdfs"], d["sizes"], d["offsets"], fp)
    assert same(st, d["after1"])
    st, e2 = O.push(variant, st, d["s1"], d["i1"], d["cdfs"], d["sizes"], d["offsets"], fp)
    assert same(st, d["after2"])
    d1, e3 = O.pop(variant, st, d["i1"], d["cdfs"], d["sizes"], d["offsets"], fp)
    assert np.array_equal(d1, d["s1"]) and same(st, d["mid"])
    d2, e4 = O.pop(variant, st, d["i2"], d["cdfs"], d["sizes"], d["offsets"], fp)
    assert np.array_equal(d2, d["s2"]) and same(st, d["final"])
    assert e1 == e2 == e3 == e4 == 0


@pytest.mark.parametrize("variant", ["rans64", "rans32", "rans32_16"])
def test_oracle_alias_tables_match_reference(variant):
    for name in (f"{variant}_alias", f"{variant}_alias_bypass"):
        d = G.load(name)
        m = d["meta"]
        sp = 5 if name.endswith("_alias") else 4
        remap, table, ok = O.alias_build_table(d["cdfs"], d["sizes"], sp, m["fp"])
        assert ok == d["cdfs"].shape[0]
        assert np.array_equal(remap, d["push_cdfs"]) and np.array_equal(table, d["pop_cdfs"])
    d = G.load(f"{variant}_alias_rejected")
    remap, table, ok = O.alias_build_table(d["cdfs"], d["sizes"], d["meta"]["sp"], d["meta"]["fp"])
    assert ok == 0
    assert np.array_equal(remap, d["remap"]) and np.array_equal(table, d["table"])


def test_oracle_pmf_to_quantized_cdf_matches_reference():
    d = G.load("pmf_to_quantized_cdf")
    for p in (8, 12, 16):
        assert np.array_equal(O.pmf_to_quantized_cdf(d["pmf"], p), d[f"cdf{p}"])


def test_oracle_pmf_known_answers():
    # reference tests/torch_ans_test.py:54-67
    assert O.pmf_to_quantized_cdf(np.array([0.25] * 4, np.float32), 8).tolist() == [0, 64, 128, 192, 256]
    assert O.pmf_to_quantized_cdf(np.array([0.1, 0.2, 0.3, 0.4], np.float32), 8).tolist() == [0, 26, 77, 154, 256]


def test_oracle_inverse_cdf_known_answers():
    # reference tests/test_utils.py:109-130
    inv = O.inverse_quantized_cdf(np.array([[0, 64, 128, 192, 256]], np.int32), 8)
    assert inv.shape == (1, 256)
    assert inv[0, 0] == 0 and inv[0, 64] == 1 and inv[0, 128] == 2 and inv[0, 192] == 3
    inv = O.inverse_quantized_cdf(np.array([[0, 26, 77, 154, 256]], np.int32), 8)
    assert (inv[0, 0:26] == 0).all() and (inv[0, 26:77] == 1).all()
    assert (inv[0, 77:154] == 2).all() and (inv[0, 154:256] == 3).all()


def test_oracle_container_known_answers():
    # reference tests/test_utils.py:22-70
    assert O.merge_bytes([b"hello", b"world"]) == struct.pack("<I", 5) + b"hello" + struct.pack("<I", 5) + b"world"
    assert O.merge_bytes([b"hello", b"world", b"!"], num_segments=3) == (
        struct.pack("<I", 5) + b"hello" + struct.pack("<I", 5) + b"world" + b"!")
    assert O.merge_bytes([b"hi", b"ok"], num_bytes_length=2) == struct.pack("<H", 2) + b"hi" + struct.pack("<H", 2) + b"ok"
    data = struct.pack("<I", 5) + b"hello" + struct.pack("<I", 5) + b"world" + b"!"
    assert O.split_merged_bytes(data, num_segments=3) == [b"hello", b"world", b"!"]
    assert O.split_merged_bytes(struct.pack("<H", 2) + b"hi" + struct.pack("<H", 2) + b"ok", 2) == [b"hi", b"ok"]
    orig = [b"test1", b"test2", b"test3"]
    assert O.split_merged_bytes(O.merge_bytes(orig, num_segments=3), num_segments=3) == orig


def test_oracle_init_stream_layout():
    # rans_cpu.cpp:22-41; value verified on the reference: rans32_16_init_stream(2,4,16)
    s = O.init_stream("rans32_16", 2, 4, 16)
    assert s.tolist() == [[16, 32768, 32768, 32768, 32768, 0, 0, 0, 0]] * 2
    s = O.init_stream("rans64", 1)
    assert s.tolist() == [[8, -(1 << 31), 0]]  # 2^31 stored in an int32 word


def test_oracle_flags_invalid_input_without_crashing():
    # out-of-range table index and out-of-range symbol without escape coding are flagged, not read
    cdfs = np.array([[0, 10, 20, 1 << 16]], np.int32)
    sizes = np.array([4], np.int32)
    st = O.init_stream("rans64", 1)
    _, err = O.push("rans64", st, np.array([[0, 5, 1]]), np.array([[0, 0, 3]]), cdfs, sizes,
                    freq_precision=16, bypass_coding=False)
    assert err & O.ERR_BAD_INDEX and err & O.ERR_BAD_VALUE
