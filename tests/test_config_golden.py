"""The oracle against the reference on every benchmark configuration's own tables (CPU).

``tests/golden/config_cases.json`` holds the reference's rows (made by the compiled reference CPU
path, tests/golden/make_config_golden.py) for cut-down batches of the five configurations with
their exact tables: 64 Laplace tables (A = 256), 64 Gaussian scale tables with escapes (rows up to
~3,100 entries), the Zipf table over 4,096 symbols with alias tables at symbol precision 12 / fp 15,
the 256 mixture tables with 65,536-entry inverse rows, and ragged per-symbol rows.  Here the C
oracle must reproduce every row width, length and payload byte and decode back to the symbols;
this library's host alias builder must reproduce the reference's alias tables.  When the compiled
reference is present it is run again and must still agree with the file.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import config_cases as CC

FIX = CC.load_fixture()


def _alias_builder():
    from oracle import build_ref
    ref = build_ref.load()
    if ref is not None:
        return ref.rans_alias_build_table

    def port(cdfs, sizes, symbol_precision=8, freq_precision=16):
        remap, table, _ = O.alias_build_table(cdfs.numpy(), sizes.numpy(), symbol_precision, freq_precision)
        return torch.from_numpy(remap), torch.from_numpy(table)
    return port


def _built(case):
    w = CC.build(case, alias_builder=_alias_builder())
    if CC.input_digest(w) != FIX[case.name]["input_sha256"]:
        pytest.skip("this host generates different inputs for the case (float64 table math); "
                    "the GPU tests fall back to running the reference here")
    return w


def oracle_record(w):
    """The oracle's rows for a case, in the fixture's format."""
    kw = dict(freq_precision=w.fp, bypass_coding=w.bypass, bypass_precision=w.bp)
    if hasattr(w, "row_starts"):
        per, popped = [], []
        for b in range(w.num_streams):
            sym, idx, cdf, sz, off = CC.ragged_stream_inputs(w, b)
            st, err = O.push(w.variant, O.init_stream(w.variant, 1), sym.numpy(), idx.numpy(), cdf.numpy(), sz.numpy(),
                             off.numpy(), **kw)
            assert err == 0
            r = CC.rows_record(st)
            per.append({"width": r["width"], "length": r["lengths"][0], "payload_sha256": r["payload_sha256"][0]})
            dec, err = O.pop(w.variant, st, idx.numpy(), cdf.numpy(), sz.numpy(), off.numpy(), **kw)
            assert err == 0 and np.array_equal(dec, sym.numpy())
            p = CC.rows_record(st)
            popped.append({"length": p["lengths"][0], "payload_sha256": p["payload_sha256"][0]})
        return {"per_stream": per, "popped": popped}
    B = w.symbols.shape[0]
    st, err = O.push(w.variant, O.init_stream(w.variant, B), w.symbols.numpy(), w.indexes.numpy(),
                     w.tables_for_push().numpy(), w.cdfs_sizes.numpy(), w.offsets.numpy(), alias=w.lookup == "alias",
                     threads=4, **kw)
    assert err == 0
    pushed = CC.rows_record(st)
    dec, err = O.pop(w.variant, st, w.indexes.numpy(), w.tables_for_pop().numpy(), w.cdfs_sizes.numpy(),
                     w.offsets.numpy(), lookup=w.lookup, threads=4, **kw)
    assert err == 0 and np.array_equal(dec, w.symbols.numpy())
    return {"pushed": pushed, "popped": CC.rows_record(st)}


@pytest.mark.parametrize("name", [c.name for c in CC.CASES])
def test_oracle_reproduces_reference_rows(name):
    case = CC.by_name(name)
    w = _built(case)
    got = oracle_record(w)
    want = FIX[name]
    for k in got:
        assert got[k] == want[k], (name, k)


def test_fixture_covers_every_configuration_and_escapes():
    builders = {FIX[n]["builder"] for n in FIX}
    assert builders == {"laplace64", "gaussian_latent", "zipf_alias", "mixture_invcdf", "ragged_adaptive"}
    assert FIX["gaussian_latent_escapes"]["escapes_coded"] is True
    assert FIX["mixture_invcdf"]["pop_op"] == "rans64_invcdf_pop"
    assert FIX["zipf_alias"]["pop_op"] == "rans32_16_alias_pop"


def test_library_host_alias_builder_matches_reference_at_config_size():
    """This library's rans_alias_build_table on CPU tensors (its host builder) against the
    reference's tables for the Zipf configuration (4,096 symbols, symbol precision 12, fp 15)."""
    from torch_ans_b200 import _C
    case = CC.by_name("zipf_alias")
    w = CC.build(case, alias_builder=_C.rans_alias_build_table)
    if CC.input_digest(w) != FIX["zipf_alias"]["input_sha256"]:
        ref_w = _built(case)  # skips when the inputs differ on this host
        assert torch.equal(w.tables_for_push(), ref_w.tables_for_push())
    assert CC._digest(w.tables_for_push(), w.tables_for_pop()) == FIX["zipf_alias"]["alias_tables_sha256"]


def test_compiled_reference_still_agrees_with_fixture():
    from oracle import build_ref
    ref = build_ref.load()
    if ref is None:
        pytest.skip("compiled reference (oracle/_ref) not present")
    for case in CC.CASES:
        rec = CC.reference_record(case, ref)
        if rec["input_sha256"] != FIX[case.name]["input_sha256"]:
            continue
        assert rec == FIX[case.name], case.name
