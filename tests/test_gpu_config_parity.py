"""Byte parity of the CUDA path on every benchmark configuration's own tables.

The expected rows are the reference's (``tests/golden/config_cases.json``, made by the compiled
reference CPU path): cut-down batches of the five configurations with their exact tables (64
Laplace tables; 64 Gaussian scale tables with and without coded escapes; the 4,096-symbol Zipf
table at fp 15 with alias tables at symbol precision 12; the 256 mixture tables with 65,536-entry
inverse rows; ragged per-symbol rows).  Each case is pushed and popped through ``_C`` on the GPU
with every push kernel and every pop kernel / table layout forced in turn, and must give the
reference's row width, lengths, payload bytes (SHA-256 per row), decoded symbols and popped rows.
The alias tables are also built on the device and must equal the reference's.

When this host generates different inputs for a case than the host that made the file (the table
math is float64), the expected rows come from running the reference (oracle/_ref) on this host's
inputs, or the oracle when the reference is absent.
"""
import functools

import pytest
import torch

from tests import config_cases as CC

pytestmark = pytest.mark.gpu

FIX = CC.load_fixture()
RECT = [c.name for c in CC.CASES if c.builder != "ragged_adaptive"]
PUSH_KERNELS = ["default", "ws", "chunk", "generic"]
POP_VARIANTS = ["default", "lean_l1", "lean_l1_b10", "lean_bucket", "lean_bucket_plain_idx", "lean_split", "fast",
                "generic"]


@pytest.fixture(scope="module")
def C():
    from torch_ans_b200 import _C
    _C.set_sync_check(False)
    _C.device_status(reset=True)
    return _C


@functools.lru_cache(maxsize=None)
def expected(name):
    """(inputs, expected record) of a case; the fixture's record when this host's inputs match it."""
    case = CC.by_name(name)
    from oracle import build_ref
    ref = build_ref.load()
    if ref is not None:
        w = CC.build(case, alias_builder=ref.rans_alias_build_table)
    else:
        from tests.test_config_golden import _alias_builder
        w = CC.build(case, alias_builder=_alias_builder())
    rec = FIX[name]
    if CC.input_digest(w) != rec["input_sha256"]:
        if ref is not None:
            rec = CC.reference_record(case, ref)
        else:
            from tests.test_config_golden import oracle_record
            rec = dict(rec, **oracle_record(w))
    return w, rec


def _force(monkeypatch, push_kernel, pop_variant):
    if push_kernel != "default":
        monkeypatch.setenv("TORCH_ANS_B200_PUSH_KERNEL", push_kernel)
    if pop_variant in ("lean_l1", "lean_l1_b10"):
        monkeypatch.setenv("TORCH_ANS_B200_POP_KERNEL", "lean")
        monkeypatch.setenv("TORCH_ANS_B200_POP_LAYOUT", "bucket_global")
        monkeypatch.setenv("TORCH_ANS_B200_POP_L1", "1")
        if pop_variant == "lean_l1_b10":  # level-1 entries of 1,024 cum values
            monkeypatch.setenv("TORCH_ANS_B200_POP_L1_BITS", "10")
    elif pop_variant in ("lean_bucket", "lean_bucket_plain_idx"):
        monkeypatch.setenv("TORCH_ANS_B200_POP_KERNEL", "lean")
        monkeypatch.setenv("TORCH_ANS_B200_POP_LAYOUT", "bucket_global")
        monkeypatch.setenv("TORCH_ANS_B200_POP_L1", "0")
        if pop_variant == "lean_bucket_plain_idx":  # indexes on plain loads instead of the ring
            monkeypatch.setenv("TORCH_ANS_B200_POP_IRING", "0")
    elif pop_variant == "lean_split":
        monkeypatch.setenv("TORCH_ANS_B200_POP_KERNEL", "lean")
        monkeypatch.setenv("TORCH_ANS_B200_POP_LAYOUT", "split_global")
    elif pop_variant in ("fast", "generic"):
        monkeypatch.setenv("TORCH_ANS_B200_POP_KERNEL", pop_variant)


# every pop kernel / layout after the default push, every push kernel before the default pop
COMBOS = [("default", p) for p in POP_VARIANTS] + [(k, "default") for k in PUSH_KERNELS[1:]]


@pytest.mark.parametrize("push_kernel,pop_variant", COMBOS)
@pytest.mark.parametrize("name", RECT)
def test_config_rows_match_reference(C, name, push_kernel, pop_variant, monkeypatch):
    w, rec = expected(name)
    _force(monkeypatch, push_kernel, pop_variant)
    dev = torch.device("cuda")
    kw = dict(freq_precision=w.fp, bypass_coding=w.bypass, bypass_precision=w.bp)
    sym, idx = w.symbols.to(dev), w.indexes.to(dev)
    sizes, offs = w.cdfs_sizes.to(dev), w.offsets.to(dev)
    st = getattr(C, f"{w.variant}_init_stream")(sym.shape[0], device="cuda")
    getattr(C, w.push_op)(st, sym, idx, w.tables_for_push().to(dev), sizes, offs, **kw)
    assert C.device_status() == 0
    assert CC.rows_record(st.cpu().numpy()) == rec["pushed"]
    dec = getattr(C, w.pop_op)(st, idx, w.tables_for_pop().to(dev), sizes, offs, **kw)
    assert C.device_status() == 0
    assert torch.equal(dec.cpu(), w.symbols)
    assert CC.rows_record(st.cpu().numpy())["lengths"] == rec["popped"]["lengths"]
    assert CC.rows_record(st.cpu().numpy())["payload_sha256"] == rec["popped"]["payload_sha256"]


@pytest.mark.parametrize("name", RECT)
def test_config_rows_through_cpu_stream_tensor(C, name):
    """The reference's calling pattern: init_stream on the CPU, moved to the GPU, then push (the
    worst-case resize reads the device lengths), bytes out through rans_stream_to_byte_strings."""
    w, rec = expected(name)
    kw = dict(freq_precision=w.fp, bypass_coding=w.bypass, bypass_precision=w.bp)
    st = getattr(C, f"{w.variant}_init_stream")(w.symbols.shape[0]).cuda()
    getattr(C, w.push_op)(st, w.symbols.cuda(), w.indexes.cuda(), w.tables_for_push().cuda(), w.cdfs_sizes.cuda(),
                          w.offsets.cuda(), **kw)
    assert st.shape[1] == rec["pushed"]["width"]
    import hashlib
    got = [hashlib.sha256(b).hexdigest() for b in C.rans_stream_to_byte_strings(st)]
    assert got == rec["pushed"]["payload_sha256"]


def test_zipf_alias_tables_built_on_device_match_reference(C):
    """Device alias build (tans_alias_build_table) on the Zipf configuration's table."""
    w, rec = expected("zipf_alias")
    remap, table = C.rans_alias_build_table(w.cdfs.cuda(), w.cdfs_sizes.cuda(), symbol_precision=12,
                                            freq_precision=w.fp)
    assert torch.equal(remap.cpu(), w.tables_for_push()) and torch.equal(table.cpu(), w.tables_for_pop())
    assert CC._digest(remap.cpu(), table.cpu()) == FIX["zipf_alias"]["alias_tables_sha256"]


@pytest.mark.parametrize("pop_kernel", ["lean", "warp", "thread"])
def test_ragged_config_rows_match_per_stream_reference(C, pop_kernel, monkeypatch):
    monkeypatch.setenv("TORCH_ANS_B200_RAGGED_POP_WARP", "0" if pop_kernel == "thread" else "1")
    monkeypatch.setenv("TORCH_ANS_B200_RAGGED_POP_LEAN", "1" if pop_kernel == "lean" else "0")
    monkeypatch.setenv("TORCH_ANS_B200_RAGGED_PUSH_LEAN", "1" if pop_kernel == "lean" else "0")
    w, rec = expected("ragged_adaptive")
    dev = torch.device("cuda")
    kw = dict(freq_precision=w.fp, bypass_coding=w.bypass, bypass_precision=w.bp)
    B = w.num_streams
    st = getattr(C, f"{w.variant}_init_stream")(B, device="cuda")
    rs = w.row_starts.to(dev)
    getattr(C, f"{w.variant}_push_ragged")(st, w.symbols.to(dev), rs, w.cdfs.to(dev), w.cdfs_sizes.to(dev),
                                           offsets=w.offsets.to(dev), **kw)
    assert C.device_status() == 0
    got = CC.rows_record(st.cpu().numpy())
    assert got["lengths"] == [p["length"] for p in rec["per_stream"]]
    assert got["payload_sha256"] == [p["payload_sha256"] for p in rec["per_stream"]]
    dec = getattr(C, f"{w.variant}_pop_ragged")(st, rs, w.cdfs.to(dev), w.cdfs_sizes.to(dev),
                                                offsets=w.offsets.to(dev), **kw)
    assert C.device_status() == 0
    assert torch.equal(dec.cpu(), w.symbols)
    after = CC.rows_record(st.cpu().numpy())
    assert after["lengths"] == [p["length"] for p in rec["popped"]]
    assert after["payload_sha256"] == [p["payload_sha256"] for p in rec["popped"]]


def test_ragged_config_streams_alone_through_rectangular_ops(C):
    """Each ragged stream through the rectangular op alone (B = 1), the reference's own pattern,
    including the row width of each call."""
    w, rec = expected("ragged_adaptive")
    kw = dict(freq_precision=w.fp, bypass_coding=w.bypass, bypass_precision=w.bp)
    for b in range(w.num_streams):
        sym, idx, cdf, sz, off = CC.ragged_stream_inputs(w, b)
        st = getattr(C, f"{w.variant}_init_stream")(1, device="cuda")
        getattr(C, f"{w.variant}_push")(st, sym.cuda(), idx.cuda(), cdf.cuda(), sz.cuda(), off.cuda(), **kw)
        r = CC.rows_record(st.cpu().numpy())
        want = rec["per_stream"][b]
        assert (r["width"], r["lengths"][0], r["payload_sha256"][0]) == (want["width"], want["length"],
                                                                          want["payload_sha256"])
        dec = getattr(C, f"{w.variant}_pop")(st, idx.cuda(), cdf.cuda(), sz.cuda(), off.cuda(), **kw)
        assert torch.equal(dec.cpu(), sym)
    assert C.device_status() == 0
